// Split-precision tcgen05 GEMM (see gemm_tc.cu).
#pragma once

#include "tt_common.cuh"

namespace tt {

struct TcGemmParams {
  // Operands as fp16 splits x = hi + lo (binary16 bit patterns, see f16_split):
  const uint16_t *A_hi, *A_lo;  // [M, K], leading dim lda (elements)
  int64_t lda;
  const uint16_t *W_hi, *W_lo;  // [N, K] (nn.Linear layout), scaled by 1 / *acc_scale
  const float *acc_scale;       // device pointer: the accumulator is multiplied by
                                // *acc_scale (a power of 2, written at pack time)
  const float *bias;            // [N]
  const float *R;               // residual [M, N] at ldc (may alias C)
  float *C;                     // fp32 output [M, N] at ldc, or null
  int64_t ldc;
  const uint8_t *row_mask;      // [M] or null
  DeviceStatus *status;         // device status word for bounded-wait timeouts
  int M, N, K;
  int epilogue;                 // GemmEpilogue
  // Outputs feeding another tensor-core kernel, as fp16 splits:
  //   columns [0, h_cols) to H_hi/H_lo [M, h_cols] (the next GEMM's A operand,
  //   or q|k for the attention);
  //   columns [vt_col0, N) (v) of row r = b*seq + s, head h, dim d transposed to
  //   vt_{hi,lo}[((b*heads + h)*head_dim + d)*seq_pad + s] (keys contiguous).
  // A value whose magnitude is beyond the fp16 range latches
  // TT_ERR_DEVICE_RANGE in the status word.
  uint16_t *H_hi, *H_lo;
  int h_cols;
  uint16_t *vt_hi, *vt_lo;
  int vt_col0, seq, seq_pad, heads, head_dim;
  // LayerNorm prologue (launch_gemm_ln_tc only): A = LayerNorm(ln_x) over K
  // features (nn.LayerNorm semantics, eps ln_eps), split in shared memory;
  // A_hi / A_lo / lda are then unused
  const float *ln_x;              // [M, K] fp32
  const float *ln_gamma, *ln_beta;
  float ln_eps;
  // Bounded waits give up after 2^wait_budget_log2 cycles (0: 2^28). The test
  // switch makes CTA 0's producer skip the loads of its first k-block (set by
  // the launcher when tt_test_arm_wait_timeout armed it, 0 otherwise).
  int wait_budget_log2;
  int test_skip_first_load;
  // Live row tiles (live_rows.cu), written by an earlier kernel of the
  // forward: the count and ascending list of the 128-row tiles to compute (the
  // CTA-pair kernel gives its two CTAs consecutive entries); the others are
  // skipped. Null: every tile.
  const int *live_count128, *live_list128;
  // Optional: an int that one thread of the kernel sets to zero once every
  // kernel before it has finished (after its griddepcontrol.wait) -- the work
  // counter of the persistent attention that follows the q|k|v projection.
  int *zero_word;
};

int launch_gemm_tc3(const TcGemmParams &p, cudaStream_t stream);

// Test support (tt_test_arm_wait_timeout): the next launch of the single-CTA
// kernel of launch_gemm_tc3 in this process runs with its test switch on and
// a wait budget of 2^budget_log2 cycles; whether such a launch is pending.
int arm_gemm_wait_timeout(int budget_log2);
bool gemm_wait_timeout_armed();

// Whether launch_gemm_ln_tc takes an M x N x K problem: K (the LayerNorm
// width) at most 128 and a problem small enough for the single-CTA schedule.
bool gemm_ln_fusable(int64_t M, int N, int K);
// The same GEMM with its A operand computed in the kernel as the fp16 split of
// LayerNorm(ln_x): one output tile per CTA, the whole A tile resident in
// shared memory. It replaces a LayerNorm launch and its round trip through
// memory for the small problems where each launch's latency is the cost.
int launch_gemm_ln_tc(const TcGemmParams &p, cudaStream_t stream);

}  // namespace tt
