// Layout of the packed model image and of the per-call workspace in HBM.
//
// Image (one per model, built by tt_pack_image):
//   [status word, 256 B]
//   per layer: ln1 w,b | Wqkv [3D,D] (q rows, then k, then v) | bqkv [3D] |
//              Wo [D,D] | bo | ln2 w,b | W1 [F,D] | b1 [F] | W2 [D,F] | b2 [D]
//              and, on the tensor-core path, the fp16 hi/lo split of each
//              weight scaled by a power of two, and the four scales
//   final_norm w,b
// Every array starts on a 256-byte boundary (TMA and float4 friendly).
//
// Workspace (per call, [T = batch*seq] tokens):
//   FFMA schedule:        qkv [T,3D] | ctx [T,D] | h [T,F]
//   tensor-core schedule: qkv [T,3D] (or, when the attention also runs on
//   tensor cores, any head_dim attention_tc_supported takes, the fp16 split of q|k qk_hi/qk_lo [T,2D]
//   and of v transposed vt_hi/vt_lo [B*H, hd, seq_pad]) | the fp16 splits of
//   the GEMM A operands: ln_hi/ln_lo [T,D], ctx_hi/ctx_lo [T,D], h_hi/h_lo [T,F].
#pragma once

#include <functional>

#include <vector>

#include "attention_tc.cuh"
#include "tt_common.cuh"

namespace tt {

enum ForwardPlan : int { PLAN_CLUSTER = 1, PLAN_OPS_FFMA = 2, PLAN_OPS_TC = 3, PLAN_TILE = 4 };

// Shapes the split-precision tensor-core schedule can run: every GEMM operand
// row (fp16) must be a whole number of 16-byte TMA units (d_model and ffn_dim
// multiples of 8). The packed image then carries the fp16 split of every
// weight.
inline bool uses_tensor_cores(const tt_config &cfg) {
  return cfg.d_model % 8 == 0 && cfg.ffn_dim % 8 == 0;
}

struct LayerOffsets {
  size_t ln1_w, ln1_b, wqkv, bqkv, wo, bo, ln2_w, ln2_b, w1, b1, w2, b2;
  size_t wqkv_hi, wqkv_lo, wo_hi, wo_lo, w1_hi, w1_lo, w2_hi, w2_lo;  // fp16 pieces
  // [0..3] accumulator scales of the q|k|v, out_proj, ffn_in, ffn_out GEMMs
  // (floats), [4..7] the weights' largest magnitudes (float bits, pack scratch)
  size_t wscale;
};

struct ImageLayout {
  size_t status = 0;
  std::vector<LayerOffsets> layer;
  size_t final_w = 0, final_b = 0, total = 0;
  bool tensor = false;

  explicit ImageLayout(const tt_config &cfg) {
    const size_t D = cfg.d_model, F = cfg.ffn_dim, f4 = sizeof(float);
    tensor = uses_tensor_cores(cfg);
    size_t cur = 0;
    auto take = [&](size_t n_floats) {
      const size_t off = cur;
      cur = align_up(cur + n_floats * f4, 256);
      return off;
    };
    status = take(256 / f4);
    layer.resize(cfg.num_layers);
    for (auto &o : layer) {
      o.ln1_w = take(D); o.ln1_b = take(D);
      o.wqkv = take(3 * D * D); o.bqkv = take(3 * D);
      o.wo = take(D * D); o.bo = take(D);
      o.ln2_w = take(D); o.ln2_b = take(D);
      o.w1 = take(F * D); o.b1 = take(F);
      o.w2 = take(D * F); o.b2 = take(D);
      if (tensor) {
        // fp16 pieces: two values per float of `take`
        o.wqkv_hi = take(3 * D * D / 2); o.wqkv_lo = take(3 * D * D / 2);
        o.wo_hi = take(D * D / 2); o.wo_lo = take(D * D / 2);
        o.w1_hi = take(F * D / 2); o.w1_lo = take(F * D / 2);
        o.w2_hi = take(D * F / 2); o.w2_lo = take(D * F / 2);
        o.wscale = take(8);
      } else {
        o.wqkv_hi = o.wqkv_lo = o.wo_hi = o.wo_lo = o.w1_hi = o.w1_lo = o.w2_hi = o.w2_lo = 0;
        o.wscale = 0;
      }
    }
    final_w = take(D);
    final_b = take(D);
    total = cur;
  }
};

// Live-row lists of a padded batch (live_rows.cu): ints in the workspace.
size_t live_rows_ints(int64_t batch, int64_t seq);
// The per-tile live flags inside the list that launch_live_rows writes.
const int *live_rows_flags(const int *ws_ints, int64_t batch, int64_t seq);
int launch_live_rows(const uint8_t *mask, int64_t batch, int seq, int *ws_ints,
                     cudaStream_t stream);

struct WorkspaceLayout {
  size_t qkv = 0, ctx = 0, h = 0, qk_hi = 0, qk_lo = 0, vt_hi = 0, vt_lo = 0;
  size_t live = 0;  // live-row lists (ints), tensor-core schedule
  size_t attn_counter = 0;  // work counter of the persistent attention (one int)
  int seq_pad = 0;  // row stride of the transposed value copy (multiple of 4)
  size_t ln_hi = 0, ln_lo = 0, ctx_hi = 0, ctx_lo = 0, h_hi = 0, h_lo = 0;
  size_t total = 0;
  bool tensor = false;        // buffers of the tensor-core schedule
  bool tc_attention = false;  // ... whose attention also runs on tensor cores

  WorkspaceLayout(const tt_config &cfg, int64_t batch, int64_t seq) {
    const size_t T = (size_t)batch * (size_t)seq, D = cfg.d_model, F = cfg.ffn_dim;
    const size_t f4 = sizeof(float);
    // the buffers of the schedule the call runs: forced, or what TT_PLAN_AUTO
    // picks when it does not take the single-launch one (which needs none)
    tensor = uses_tensor_cores(cfg) &&
             (cfg.plan == TT_PLAN_OPS_TC ||
              (cfg.plan == TT_PLAN_AUTO && (cfg.flags & TT_FLAG_FP32_ONLY) == 0));
    size_t cur = 0;
    auto take = [&](size_t n_floats) {
      const size_t off = cur;
      cur = align_up(cur + n_floats * f4, 256);
      return off;
    };
    const int hd = cfg.d_model / cfg.num_heads;
    tc_attention = tensor && attention_tc_supported(hd, cfg.d_model);
    if (tc_attention) {
      // q|k as an fp16 split, and v transposed per (sequence, head) with keys
      // contiguous (rows of seq_pad fp16 values, a multiple of 16 bytes), for
      // the tensor-core attention (sizes in floats: two fp16 values per float)
      seq_pad = (int)((seq + 7) / 8 * 8);
      qk_hi = take(T * D); qk_lo = take(T * D);
      vt_hi = take((size_t)batch * seq_pad * D / 2); vt_lo = take((size_t)batch * seq_pad * D / 2);
      attn_counter = take(1);
    } else {
      qkv = take(T * 3 * D);
    }
    if (tensor) {
      // A operands of the split-precision GEMMs, as fp16 hi/lo pairs
      ln_hi = take(T * D / 2); ln_lo = take(T * D / 2);
      ctx_hi = take(T * D / 2); ctx_lo = take(T * D / 2);
      h_hi = take(T * F / 2); h_lo = take(T * F / 2);
      live = take(live_rows_ints(batch, seq));
    } else {
      ctx = take(T * D);
      h = take(T * F);
    }
    total = cur;
  }
};

// Everything a per-op forward's launch sequence depends on (graph_cache.cu):
// compared bytewise, so only 64-bit fields (no padding) and zero-initialised.
struct ForwardKey {
  int64_t device, d_model, num_heads, ffn_dim, num_layers, causal, plan, batch, seq;
  uint64_t image, x, mask, y, scratch;
};
ForwardKey make_forward_key(const tt_config &cfg, int plan, const void *image, const float *x,
                            const uint8_t *mask, int64_t batch, int64_t seq, const float *y,
                            const void *scratch);
// Enqueues one forward on the given stream.
using ForwardLaunch = std::function<int(cudaStream_t)>;
// Runs launch on `stream`, directly or through a cached CUDA graph.
int run_forward_cached(const ForwardKey &key, cudaStream_t stream, const ForwardLaunch &launch);
// Whether the launch probe is timing the launches of this host thread.
bool launch_probe_active();

int validate_config(const tt_config *cfg);
int forward_plan(const tt_config *cfg, int64_t batch, int64_t seq);
// The per-op schedule TT_PLAN_AUTO uses (when the single-launch one does not
// apply): the tensor-core one unless the shape or TT_FLAG_FP32_ONLY rules it out.
int auto_ops_plan(const tt_config &cfg);
// Device address of tt_forward_noalloc's scratch array on the current device,
// looked up once per device and cached (noalloc.cu).
int noalloc_scratch_address(void **out);
int forward_ops(const tt_config &cfg, const ImageLayout &L, const char *image, const float *x,
                const uint8_t *mask, int64_t batch, int64_t seq, float *y,
                const WorkspaceLayout &W, char *ws, cudaStream_t stream);
// Whether the tensor-core schedule lists the live row tiles of the batch and
// lets its GEMMs skip the rest (one extra launch): GEMM-heavy shapes only.
bool ops_tc_skips_dead_rows(const tt_config &cfg, int64_t tokens);
int forward_ops_tc(const tt_config &cfg, const ImageLayout &L, const char *image, const float *x,
                   const uint8_t *mask, int64_t batch, int64_t seq, float *y,
                   const WorkspaceLayout &W, char *ws, cudaStream_t stream);

}  // namespace tt
