// 3xTF32 tcgen05 GEMM (see gemm_tc.cu).
#pragma once

#include "tt_common.cuh"

namespace tt {

struct TcGemmParams {
  const float *A_hi, *A_lo;   // [M, K] TF32 split of the A operand, leading dim lda
  int64_t lda;
  const float *W_hi, *W_lo;   // [N, K] TF32 split of the weight (nn.Linear layout)
  const float *bias;          // [N]
  const float *R;             // residual [M, N] at ldc (may alias C)
  float *C;                   // fp32 output [M, N] at ldc, or null
  float *C_hi, *C_lo;         // TF32 split of the output, or null
  int64_t ldc;
  const uint8_t *row_mask;    // [M] or null
  DeviceStatus *status;       // device status word for bounded-wait timeouts
  int M, N, K;
  int epilogue;               // GemmEpilogue
  // Optional transposed copy of the value columns of a q|k|v projection, for
  // the tensor-core attention: columns [vt_col0, N) of row r = b*seq + s, head
  // h, dim d go to vt_{hi,lo}[((b*heads + h)*head_dim + d)*seq_pad + s]
  // (keys contiguous) instead of C_hi/C_lo.
  float *vt_hi, *vt_lo;
  int vt_col0, seq, seq_pad, heads, head_dim;
};

int launch_gemm_tc3(const TcGemmParams &p, cudaStream_t stream);

}  // namespace tt
