// Tensor-core (tcgen05, 3xTF32) flash attention for head_dim 64 (see attention_tc.cu).
#pragma once

#include "tt_common.cuh"

namespace tt {

struct AttentionTcParams {
  const float *qkv_hi, *qkv_lo;  // [B*S, 3D] TF32 split of q | k (| v, unused)
  const float *vt_hi, *vt_lo;    // [B*H, 64, seq_pad] TF32 split of v, keys contiguous
  float *ctx_hi, *ctx_lo;        // [B*S, D] TF32 split of the context
  const uint8_t *mask;           // [B, S] or null
  DeviceStatus *status;
  int64_t batch;
  int seq, seq_pad, d_model, num_heads, head_dim;
  int causal;
  float scale;
};

bool attention_tc_supported(int head_dim, int d_model);
int launch_attention_tc(const AttentionTcParams &p, cudaStream_t stream);

}  // namespace tt
