// Tensor-core (tcgen05) flash attention for head_dim 8, 16, 32, 64, 128 and
// 256 (see attention_tc.cu).
#pragma once

#include "tt_common.cuh"

namespace tt {

struct AttentionTcParams {
  const uint16_t *qk_hi, *qk_lo;  // [B*S, 2D] fp16 split of q | k (binary16 bits)
  const uint16_t *vt_hi, *vt_lo;  // [B*H, head_dim, seq_pad] fp16 split of v, keys contiguous
  uint16_t *ctx_hi, *ctx_lo;      // [B*S, D] fp16 split of the context
  const uint8_t *mask;            // [B, S] or null
  DeviceStatus *status;
  int64_t batch;
  int seq, seq_pad, d_model, num_heads, head_dim;
  int causal;
  float scale;
  // set by launch_attention_tc: (sequence, head) pairs per group of the grid
  // order (see the kernel); a divisor of batch * num_heads
  int bh_group;
  // work-item counter of the persistent form (head_dim up to 64): zero when
  // the kernel starts (the q|k|v GEMM before it zeroes it), taken with
  // atomicAdd; null selects the one-CTA-per-item form
  int *counter;
};

// Whether launch_attention_tc runs head_dim `hd` on the persistent form,
// which needs p.counter.
bool attention_tc_persistent(int head_dim);

bool attention_tc_supported(int head_dim, int d_model);
int launch_attention_tc(const AttentionTcParams &p, cudaStream_t stream);

}  // namespace tt
