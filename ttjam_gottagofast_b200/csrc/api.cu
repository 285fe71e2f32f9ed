// C ABI of the forward pass: config validation, model-image packing and the
// forward schedule. Declared in include/ttjam_b200.h.
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "attention_tc.cuh"
#include "cluster_forward.cuh"
#include "gemm_tc.cuh"
#include "image.cuh"
#include "tile_forward.cuh"
#include "tt_common.cuh"

namespace tt {

static thread_local std::string g_last_error;

void set_last_error(const std::string &msg) { g_last_error = msg; }

bool pdl_enabled() {
  static const bool on = [] {
    const char *e = std::getenv("TT_PDL");
    return e == nullptr || std::strcmp(e, "0") != 0;
  }();
  return on;
}

namespace {

// Largest |w| of a weight matrix, as float bits (non-negative floats order
// like their bit patterns), into *out (zeroed by the caller).
__global__ void absmax_kernel(const float *__restrict__ src, int64_t n, unsigned *out) {
  float m = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(src[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0 && m > 0.f) atomicMax(out, __float_as_uint(m));
}

// fp16 split of w * 2^e with e chosen so the largest |w| * 2^e lies in
// [2^14, 2^15): the pieces keep their full relative precision and stay
// finite. Writes 2^-e (the GEMM's accumulator scale) to *acc_scale.
__global__ void weight_split_kernel(const float *__restrict__ src, uint16_t *__restrict__ hi,
                                    uint16_t *__restrict__ lo, int64_t n,
                                    const unsigned *__restrict__ maxbits,
                                    float *__restrict__ acc_scale) {
  const float mx = __uint_as_float(*maxbits);
  int e = 0;
  if (mx > 0.f && isfinite(mx)) {
    int ex;
    frexpf(mx, &ex);  // mx = f * 2^ex, f in [0.5, 1)
    e = min(max(15 - ex, -100), 100);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) *acc_scale = ldexpf(1.0f, -e);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    f16_split(ldexpf(src[i], e), hi[i], lo[i]);
}

int split_weight(const float *src, uint16_t *hi, uint16_t *lo, int64_t n, unsigned *maxbits,
                 float *acc_scale, cudaStream_t stream) {
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>(ceil_div(n, threads), 148 * 8);
  TT_CUDA_TRY(cudaMemsetAsync(maxbits, 0, sizeof(unsigned), stream));
  absmax_kernel<<<(unsigned)blocks, threads, 0, stream>>>(src, n, maxbits);
  TT_LAUNCH_CHECK("absmax");
  weight_split_kernel<<<(unsigned)blocks, threads, 0, stream>>>(src, hi, lo, n, maxbits,
                                                                 acc_scale);
  TT_LAUNCH_CHECK("weight_split");
  return TT_OK;
}

// Bound of one LayerNorm output element: a normalised row z of D elements has
// sum z = 0 and sum z^2 <= D, so |z_i| <= sqrt(D - 1); the affine map adds
// |gamma_i| * that + |beta_i|.
__device__ __forceinline__ float ln_bound(const float *gamma, const float *beta, int i,
                                          float zmax) {
  return fabsf(gamma[i]) * zmax + fabsf(beta[i]);
}

// One warp per weight row j: out = max over rows of
//   sum_i |W[j,i]| * ln_bound(i) + |b[j]|   (gelu: max with 0.17, the largest
// |gelu| of a negative argument), and of every ln_bound(i) itself. Results
// are non-negative floats combined with atomicMax on their bits (+inf and
// NaN bit patterns order above every finite value).
__global__ void operand_bound_kernel(const float *__restrict__ W, const float *__restrict__ b,
                                     const float *__restrict__ gamma,
                                     const float *__restrict__ beta, int rows, int D, int gelu,
                                     unsigned *out) {
  const float zmax = sqrtf((float)(D > 1 ? D - 1 : 0));
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  float m = 0.f;
  for (int j = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; j < rows; j += warps) {
    const float *w = W + (int64_t)j * D;
    float acc = 0.f;
    for (int i = lane; i < D; i += 32) acc = fmaf(fabsf(w[i]), ln_bound(gamma, beta, i, zmax), acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    acc += fabsf(b[j]);
    if (!(acc == acc)) acc = __int_as_float(0x7f800000);  // NaN -> +inf
    m = fmaxf(m, gelu ? fmaxf(acc, 0.17f) : acc);
  }
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
      float v = ln_bound(gamma, beta, i, zmax);
      if (!(v == v)) v = __int_as_float(0x7f800000);
      m = fmaxf(m, v);
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) atomicMax(out, __float_as_uint(m));
}

bool misaligned(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; }

// y[i] = gelu_erf(x[i]): the GELU every schedule applies, for its accuracy test.
__global__ void gelu_test_kernel(const float *__restrict__ x, float *__restrict__ y, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = gelu_erf(x[i]);
}

// Launch timing probe (tt_launch_probe_start / _read): per host thread, a
// pair of timing events around each kernel launch of the forward schedules.
struct LaunchProbe {
  std::vector<cudaEvent_t> events;  // 2 per launch: before, after
  std::vector<int32_t> kinds;
  int count = 0;
  int capacity() const { return (int)kinds.size(); }
};
thread_local LaunchProbe g_probe;

// Runs `launch` (which enqueues one kernel on `stream`), bracketed by the
// probe's events while the probe is on and has room.
template <class F>
int timed_launch(int kind, cudaStream_t stream, F &&launch) {
  LaunchProbe &pr = g_probe;
  const int i = pr.count;
  const bool on = i < pr.capacity();
  if (on) TT_CUDA_TRY(cudaEventRecord(pr.events[2 * i], stream));
  const int rc = launch();
  if (on && rc == TT_OK) {
    TT_CUDA_TRY(cudaEventRecord(pr.events[2 * i + 1], stream));
    pr.kinds[i] = kind;
    pr.count = i + 1;
  }
  return rc;
}

}  // namespace

bool launch_probe_active() {
  const LaunchProbe &pr = g_probe;
  return pr.count < pr.capacity();
}

ForwardKey make_forward_key(const tt_config &cfg, int plan, const void *image, const float *x,
                            const uint8_t *mask, int64_t batch, int64_t seq, const float *y,
                            const void *scratch) {
  ForwardKey k;
  std::memset(&k, 0, sizeof(k));
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    dev = -1;
  }
  k.device = dev;
  k.d_model = cfg.d_model;
  k.num_heads = cfg.num_heads;
  k.ffn_dim = cfg.ffn_dim;
  k.num_layers = cfg.num_layers;
  k.causal = cfg.causal;
  k.plan = plan;
  k.batch = batch;
  k.seq = seq;
  k.image = reinterpret_cast<uint64_t>(image);
  k.x = reinterpret_cast<uint64_t>(x);
  k.mask = reinterpret_cast<uint64_t>(mask);
  k.y = reinterpret_cast<uint64_t>(y);
  k.scratch = reinterpret_cast<uint64_t>(scratch);
  return k;
}

int validate_config(const tt_config *cfg) {
  if (cfg == nullptr) return fail(TT_ERR_INVALID_ARGUMENT, "config is NULL");
  // Same order and wording as TransformerConfig.validate
  // (torch_transformer_benchmark.py:39-56) for the fields this record holds.
  if (cfg->d_model <= 0) return fail(TT_ERR_INVALID_CONFIG, "d_model must be positive");
  if (cfg->num_heads <= 0) return fail(TT_ERR_INVALID_CONFIG, "num_heads must be positive");
  if (cfg->d_model % cfg->num_heads != 0)
    return fail(TT_ERR_INVALID_CONFIG, "d_model (" + std::to_string(cfg->d_model) +
                                           ") must be divisible by num_heads (" +
                                           std::to_string(cfg->num_heads) + ")");
  if (cfg->ffn_dim <= 0) return fail(TT_ERR_INVALID_CONFIG, "ffn_dim must be positive");
  if (cfg->num_layers <= 0) return fail(TT_ERR_INVALID_CONFIG, "num_layers must be positive");
  if (cfg->causal != 0 && cfg->causal != 1)
    return fail(TT_ERR_INVALID_CONFIG, "causal must be 0 or 1");
  if (cfg->plan < TT_PLAN_AUTO || cfg->plan > TT_PLAN_TILE)
    return fail(TT_ERR_INVALID_CONFIG, "plan must be one of TT_PLAN_*");
  if ((cfg->flags & ~TT_FLAG_FP32_ONLY) != 0)
    return fail(TT_ERR_INVALID_CONFIG, "flags holds an unknown TT_FLAG_* bit");
  if (cfg->reserved != 0) return fail(TT_ERR_INVALID_CONFIG, "reserved field must be 0");
  if (cfg->d_model / cfg->num_heads > 256)
    return fail(TT_ERR_UNSUPPORTED, "head_dim > 256 is not supported by this build");
  if (cfg->d_model > 65536 || cfg->ffn_dim > (1 << 20))
    return fail(TT_ERR_UNSUPPORTED, "d_model or ffn_dim too large for this build");
  return TT_OK;
}

int auto_ops_plan(const tt_config &cfg) {
  return uses_tensor_cores(cfg) && (cfg.flags & TT_FLAG_FP32_ONLY) == 0 ? PLAN_OPS_TC
                                                                        : PLAN_OPS_FFMA;
}

int forward_plan(const tt_config *cfg, int64_t batch, int64_t seq) {
  const int ops = uses_tensor_cores(*cfg) ? PLAN_OPS_TC : PLAN_OPS_FFMA;
  switch (cfg->plan) {
    case TT_PLAN_AUTO:
      if (choose_cluster(*cfg, batch, seq).cluster > 0) return PLAN_CLUSTER;
      // the tile forward holds activations as fp16 pieces, as the per-op
      // tensor-core schedule does. It runs a tile's four layers in about
      // 132 us whatever the number of tiles up to one per SM, and beats the
      // per-op schedule from one full tile on (measured on B200, d 128, 4
      // layers: 1 tile 132 us against 140, 8 tiles (workload A) 131.5 against
      // 148, 64 tiles 132 against 189, 10000 tiles 8.1 ms against 15.8). Below
      // 128 rows the cluster forward, or the per-op schedule, is faster.
      if ((cfg->flags & TT_FLAG_FP32_ONLY) == 0 && tile_forward_supported(*cfg, batch, seq) &&
          batch * seq >= 128)
        return PLAN_TILE;
      return auto_ops_plan(*cfg);
    case TT_PLAN_TILE:
      if (tile_forward_supported(*cfg, batch, seq)) return PLAN_TILE;
      return fail(TT_ERR_UNSUPPORTED, "tile schedule needs d_model = ffn_dim = 128, 4 heads "
                                      "and seq a divisor of 128");
    case TT_PLAN_CLUSTER:
      if (choose_cluster(*cfg, batch, seq).cluster > 0) return PLAN_CLUSTER;
      return fail(TT_ERR_UNSUPPORTED, "cluster schedule needs d_model = ffn_dim = 128, "
                                      "num_heads in {1,2,4,8,16} and a short sequence");
    case TT_PLAN_OPS_FFMA:
      return PLAN_OPS_FFMA;
    default:
      if (ops == PLAN_OPS_TC) return PLAN_OPS_TC;
      return fail(TT_ERR_UNSUPPORTED, "tensor-core schedule is not available for this shape");
  }
}

int forward_cluster(const tt_config &cfg, const ClusterChoice &cc, const ImageLayout &L,
                    const char *image, const float *x, const uint8_t *mask, int64_t batch,
                    int64_t seq, float *y, cudaStream_t stream) {
  ClusterArgs a{};
  a.image = image;
  a.layer_stride = L.layer.size() > 1 ? L.layer[1].ln1_w - L.layer[0].ln1_w : 0;
  a.off = L.layer[0];
  a.final_w = reinterpret_cast<const float *>(image + L.final_w);
  a.final_b = reinterpret_cast<const float *>(image + L.final_b);
  a.x = x;
  a.mask = mask;
  a.y = y;
  a.status = reinterpret_cast<DeviceStatus *>(const_cast<char *>(image) + L.status);
  a.seq = (int)seq;
  a.nseq = (int)batch;
  a.seq_per_cluster = cc.seq_per_cluster;
  a.num_layers = cfg.num_layers;
  a.causal = cfg.causal;
  a.scale = (float)(1.0 / std::sqrt((double)(cfg.d_model / cfg.num_heads)));
  a.eps = 1e-5f;
  return timed_launch(TT_KERNEL_WHOLE_FORWARD, stream,
                      [&] { return launch_cluster_forward(cc, a, cfg.num_heads, stream); });
}

int forward_tile(const tt_config &cfg, const ImageLayout &L, const char *image, const float *x,
                 const uint8_t *mask, int64_t batch, int64_t seq, float *y, cudaStream_t stream) {
  TileArgs a{};
  a.image = image;
  // bytes between layers: the same for every layer (and independent of their
  // number), so a two-layer layout gives it also for a one-layer model
  tt_config two = cfg;
  two.num_layers = 2;
  const ImageLayout L2(two);
  a.layer_stride = L2.layer[1].ln1_w - L2.layer[0].ln1_w;
  a.off = L.layer[0];
  a.final_w = reinterpret_cast<const float *>(image + L.final_w);
  a.final_b = reinterpret_cast<const float *>(image + L.final_b);
  a.x = x;
  a.mask = mask;
  a.y = y;
  a.status = reinterpret_cast<DeviceStatus *>(const_cast<char *>(image) + L.status);
  a.rows = batch * seq;
  a.seq = (int)seq;
  a.num_layers = cfg.num_layers;
  a.causal = cfg.causal;
  a.scale = (float)(1.0 / std::sqrt((double)(cfg.d_model / cfg.num_heads)));
  a.eps = 1e-5f;
  return timed_launch(TT_KERNEL_WHOLE_FORWARD, stream, [&] { return launch_tile_forward(a, stream); });
}

int forward_ops(const tt_config &cfg, const ImageLayout &L, const char *image, const float *x,
                const uint8_t *mask, int64_t batch, int64_t seq, float *y,
                const WorkspaceLayout &W, char *ws, cudaStream_t stream) {
  const int D = cfg.d_model, F = cfg.ffn_dim, H = cfg.num_heads, hd = D / H;
  const int64_t T = batch * seq;
  float *qkv = reinterpret_cast<float *>(ws + W.qkv);
  float *ctx = reinterpret_cast<float *>(ws + W.ctx);
  float *hbuf = reinterpret_cast<float *>(ws + W.h);
  const float eps = 1e-5f;
  for (int l = 0; l < cfg.num_layers; ++l) {
    const LayerOffsets &o = L.layer[l];
    auto P = [&](size_t off) { return reinterpret_cast<const float *>(image + off); };
    const float *xin = (l == 0) ? x : y;
    int rc;
    // q|k|v = LayerNorm1(x) . Wqkv^T + bqkv
    GemmParams g{};
    g.A = xin; g.lda = D; g.W = P(o.wqkv); g.bias = P(o.bqkv); g.C = qkv; g.ldc = 3LL * D;
    g.ln_gamma = P(o.ln1_w); g.ln_beta = P(o.ln1_b); g.ln_eps = eps;
    g.M = T; g.N = 3 * D; g.K = D; g.epilogue = EPI_BIAS;
    if ((rc = timed_launch(TT_KERNEL_QKV, stream, [&] { return launch_gemm_ffma(g, stream); })))
      return rc;
    // context = softmax(q k^T * scale + masks) v
    AttentionParams a{};
    a.qkv = qkv; a.ctx = ctx; a.mask = mask; a.batch = batch; a.seq = (int)seq;
    a.d_model = D; a.num_heads = H; a.head_dim = hd; a.causal = cfg.causal;
    a.scale = (float)(1.0 / std::sqrt((double)hd));
    if ((rc = timed_launch(TT_KERNEL_ATTENTION, stream,
                           [&] { return launch_attention_ffma(a, stream); })))
      return rc;
    // y = x + masked(context . Wo^T + bo)
    GemmParams go{};
    go.A = ctx; go.lda = D; go.W = P(o.wo); go.bias = P(o.bo); go.R = xin; go.C = y;
    go.ldc = D; go.row_mask = mask; go.M = T; go.N = D; go.K = D;
    go.epilogue = EPI_BIAS_RESIDUAL;
    if ((rc = timed_launch(TT_KERNEL_OUT_PROJ, stream, [&] { return launch_gemm_ffma(go, stream); })))
      return rc;
    // h = gelu(LayerNorm2(y) . W1^T + b1)
    GemmParams g1{};
    g1.A = y; g1.lda = D; g1.W = P(o.w1); g1.bias = P(o.b1); g1.C = hbuf; g1.ldc = F;
    g1.ln_gamma = P(o.ln2_w); g1.ln_beta = P(o.ln2_b); g1.ln_eps = eps;
    g1.M = T; g1.N = F; g1.K = D; g1.epilogue = EPI_BIAS_GELU;
    if ((rc = timed_launch(TT_KERNEL_FFN_IN, stream, [&] { return launch_gemm_ffma(g1, stream); })))
      return rc;
    // y = masked(y + h . W2^T + b2)
    GemmParams g2{};
    g2.A = hbuf; g2.lda = F; g2.W = P(o.w2); g2.bias = P(o.b2); g2.R = y; g2.C = y;
    g2.ldc = D; g2.row_mask = mask; g2.M = T; g2.N = D; g2.K = F;
    g2.epilogue = EPI_BIAS_RESIDUAL;
    if ((rc = timed_launch(TT_KERNEL_FFN_OUT, stream, [&] { return launch_gemm_ffma(g2, stream); })))
      return rc;
  }
  return timed_launch(TT_KERNEL_FINAL_NORM, stream, [&] {
    return launch_layernorm(y, y, nullptr, nullptr,
                            reinterpret_cast<const float *>(image + L.final_w),
                            reinterpret_cast<const float *>(image + L.final_b), mask, 1, T, D,
                            eps, stream);
  });
}

// Per-op schedule with split-precision tensor-core GEMMs: per layer LN1 ->
// fp16 split, q|k|v GEMM, attention (writes the split context), out_proj GEMM
// + residual, LN2 -> split, ffn_in GEMM + GELU (writes the split hidden),
// ffn_out GEMM + residual; then the final LayerNorm.
// Whether the tensor-core schedule folds both LayerNorms of a block into the
// GEMMs that read them (small problems with d_model <= 128: 5 launches per
// layer instead of 7).
bool ops_tc_fuses_ln(const tt_config &cfg, int64_t tokens) {
  return gemm_ln_fusable(tokens, 3 * cfg.d_model, cfg.d_model) &&
         gemm_ln_fusable(tokens, cfg.ffn_dim, cfg.d_model);
}

// GEMM-heavy shapes (d_model >= 256, at least 1024 rows) list the live row
// tiles of the batch first (live_rows.cu), and their GEMMs and LayerNorms
// skip the rest: one small launch that reads the mask, against projections
// whose cost per row tile is large. Without a mask every tile is live. (At
// d_model 128 the GEMMs are bound by their latency, not their rows: measured
// on B200, workload C 299 -> 305 us and official case 13 1113 -> 1147 us with
// the skip.)
bool ops_tc_skips_dead_rows(const tt_config &cfg, int64_t tokens) {
  return cfg.d_model >= 256 && tokens >= 4 * 256;
}

int forward_ops_tc(const tt_config &cfg, const ImageLayout &L, const char *image, const float *x,
                   const uint8_t *mask, int64_t batch, int64_t seq, float *y,
                   const WorkspaceLayout &W, char *ws, cudaStream_t stream) {
  const int D = cfg.d_model, F = cfg.ffn_dim, H = cfg.num_heads, hd = D / H;
  const int64_t T = batch * seq;
  if (T > INT32_MAX) return fail(TT_ERR_UNSUPPORTED, "tensor-core schedule: too many tokens");
  auto WS = [&](size_t off) { return reinterpret_cast<float *>(ws + off); };
  auto WH = [&](size_t off) { return reinterpret_cast<uint16_t *>(ws + off); };
  float *qkv = WS(W.qkv);
  uint16_t *qk_hi = WH(W.qk_hi), *qk_lo = WH(W.qk_lo), *vt_hi = WH(W.vt_hi), *vt_lo = WH(W.vt_lo);
  uint16_t *ln_hi = WH(W.ln_hi), *ln_lo = WH(W.ln_lo);
  uint16_t *ctx_hi = WH(W.ctx_hi), *ctx_lo = WH(W.ctx_lo);
  uint16_t *h_hi = WH(W.h_hi), *h_lo = WH(W.h_lo);
  DeviceStatus *status = reinterpret_cast<DeviceStatus *>(const_cast<char *>(image) + L.status);
  const float eps = 1e-5f;
  const bool fuse_ln = ops_tc_fuses_ln(cfg, T);
  const int *live = nullptr;  // live-row lists, or null: every tile
  if (ops_tc_skips_dead_rows(cfg, T)) {
    int *lv = reinterpret_cast<int *>(ws + W.live);
    int rc;
    if ((rc = timed_launch(TT_KERNEL_ROW_SCAN, stream, [&] {
           return launch_live_rows(mask, batch, (int)seq, lv, stream);
         })))
      return rc;
    live = lv;
  }
  // the persistent attention's work counter, zeroed by the q|k|v GEMM of each
  // layer before the attention takes items from it
  int *attn_counter = W.tc_attention && attention_tc_persistent(hd)
                          ? reinterpret_cast<int *>(ws + W.attn_counter)
                          : nullptr;
  // per-tile flags for the LayerNorms ahead of the GEMMs (the final one still
  // writes every row: it zeroes the padded rows of y)
  const int *live_tiles = live != nullptr ? live_rows_flags(live, batch, seq) : nullptr;
  auto set_live = [&](TcGemmParams &g) {
    if (live == nullptr) return;
    g.live_count128 = live;
    g.live_list128 = live + 1;
  };
  for (int l = 0; l < cfg.num_layers; ++l) {
    const LayerOffsets &o = L.layer[l];
    auto P = [&](size_t off) { return reinterpret_cast<const float *>(image + off); };
    auto PH = [&](size_t off) { return reinterpret_cast<const uint16_t *>(image + off); };
    const float *wsc = P(o.wscale);  // accumulator scales of the four GEMMs
    const float *xin = (l == 0) ? x : y;
    int rc;
    if (!fuse_ln &&
        (rc = timed_launch(TT_KERNEL_LAYERNORM, stream, [&] {
           return launch_layernorm(xin, nullptr, ln_hi, ln_lo, P(o.ln1_w), P(o.ln1_b), nullptr,
                                   0, T, D, eps, stream, live_tiles);
         })))
      return rc;
    TcGemmParams g{};
    g.A_hi = ln_hi; g.A_lo = ln_lo; g.lda = D; g.W_hi = PH(o.wqkv_hi); g.W_lo = PH(o.wqkv_lo);
    g.acc_scale = wsc;
    g.bias = P(o.bqkv); g.ldc = 3LL * D; g.status = status;
    g.M = (int)T; g.N = 3 * D; g.K = D; g.epilogue = EPI_BIAS;
    if (W.tc_attention) {
      g.H_hi = qk_hi; g.H_lo = qk_lo; g.h_cols = 2 * D;  // the attention reads the fp16 split
      g.vt_hi = vt_hi; g.vt_lo = vt_lo;                  // ... and v transposed
      g.vt_col0 = 2 * D; g.seq = (int)seq; g.seq_pad = W.seq_pad; g.heads = H; g.head_dim = hd;
      g.zero_word = attn_counter;
    } else {
      g.C = qkv;
    }
    if (fuse_ln) {
      g.ln_x = xin; g.ln_gamma = P(o.ln1_w); g.ln_beta = P(o.ln1_b); g.ln_eps = eps;
    } else {
      set_live(g);
    }
    if ((rc = timed_launch(TT_KERNEL_QKV, stream, [&] {
           return fuse_ln ? launch_gemm_ln_tc(g, stream) : launch_gemm_tc3(g, stream);
         })))
      return rc;
    const float scale = (float)(1.0 / std::sqrt((double)hd));
    if (W.tc_attention) {
      AttentionTcParams a{};
      a.qk_hi = qk_hi; a.qk_lo = qk_lo; a.vt_hi = vt_hi; a.vt_lo = vt_lo;
      a.ctx_hi = ctx_hi; a.ctx_lo = ctx_lo; a.mask = mask; a.status = status;
      a.batch = batch; a.seq = (int)seq; a.seq_pad = W.seq_pad; a.d_model = D; a.num_heads = H;
      a.head_dim = hd; a.causal = cfg.causal; a.scale = scale; a.counter = attn_counter;
      if ((rc = timed_launch(TT_KERNEL_ATTENTION, stream,
                             [&] { return launch_attention_tc(a, stream); })))
        return rc;
    } else {
      AttentionParams a{};
      a.qkv = qkv; a.ctx = nullptr; a.ctx_hi = ctx_hi; a.ctx_lo = ctx_lo; a.mask = mask;
      a.batch = batch; a.seq = (int)seq; a.d_model = D; a.num_heads = H; a.head_dim = hd;
      a.causal = cfg.causal; a.scale = scale;
      if ((rc = timed_launch(TT_KERNEL_ATTENTION, stream,
                             [&] { return launch_attention_ffma(a, stream); })))
        return rc;
    }
    TcGemmParams go{};
    go.A_hi = ctx_hi; go.A_lo = ctx_lo; go.lda = D; go.W_hi = PH(o.wo_hi); go.W_lo = PH(o.wo_lo);
    go.acc_scale = wsc + 1;
    go.bias = P(o.bo); go.R = xin; go.C = y; go.ldc = D; go.row_mask = mask; go.status = status;
    go.M = (int)T; go.N = D; go.K = D; go.epilogue = EPI_BIAS_RESIDUAL;
    set_live(go);
    if ((rc = timed_launch(TT_KERNEL_OUT_PROJ, stream, [&] { return launch_gemm_tc3(go, stream); })))
      return rc;
    if (!fuse_ln &&
        (rc = timed_launch(TT_KERNEL_LAYERNORM, stream, [&] {
           return launch_layernorm(y, nullptr, ln_hi, ln_lo, P(o.ln2_w), P(o.ln2_b), nullptr, 0,
                                   T, D, eps, stream, live_tiles);
         })))
      return rc;
    TcGemmParams g1{};
    g1.A_hi = ln_hi; g1.A_lo = ln_lo; g1.lda = D; g1.W_hi = PH(o.w1_hi); g1.W_lo = PH(o.w1_lo);
    g1.acc_scale = wsc + 2;
    g1.bias = P(o.b1); g1.H_hi = h_hi; g1.H_lo = h_lo; g1.h_cols = F; g1.ldc = F;
    g1.status = status;
    g1.M = (int)T; g1.N = F; g1.K = D; g1.epilogue = EPI_BIAS_GELU;
    if (fuse_ln) {
      g1.ln_x = y; g1.ln_gamma = P(o.ln2_w); g1.ln_beta = P(o.ln2_b); g1.ln_eps = eps;
    } else {
      set_live(g1);
    }
    if ((rc = timed_launch(TT_KERNEL_FFN_IN, stream, [&] {
           return fuse_ln ? launch_gemm_ln_tc(g1, stream) : launch_gemm_tc3(g1, stream);
         })))
      return rc;
    TcGemmParams g2{};
    g2.A_hi = h_hi; g2.A_lo = h_lo; g2.lda = F; g2.W_hi = PH(o.w2_hi); g2.W_lo = PH(o.w2_lo);
    g2.acc_scale = wsc + 3;
    g2.bias = P(o.b2); g2.R = y; g2.C = y; g2.ldc = D; g2.row_mask = mask; g2.status = status;
    g2.M = (int)T; g2.N = D; g2.K = F; g2.epilogue = EPI_BIAS_RESIDUAL;
    set_live(g2);
    if ((rc = timed_launch(TT_KERNEL_FFN_OUT, stream, [&] { return launch_gemm_tc3(g2, stream); })))
      return rc;
  }
  return timed_launch(TT_KERNEL_FINAL_NORM, stream, [&] {
    return launch_layernorm(y, y, nullptr, nullptr,
                            reinterpret_cast<const float *>(image + L.final_w),
                            reinterpret_cast<const float *>(image + L.final_b), mask, 1, T, D,
                            eps, stream);
  });
}

}  // namespace tt

using namespace tt;

extern "C" {

int tt_abi_version(void) { return TT_ABI_VERSION; }

int tt_validate_config(const tt_config *cfg) { return validate_config(cfg); }

size_t tt_image_bytes(const tt_config *cfg) {
  if (validate_config(cfg) != TT_OK) return 0;
  return ImageLayout(*cfg).total;
}

int tt_pack_image(const tt_config *cfg, const tt_layer_params *layers,
                  const float *final_norm_weight, const float *final_norm_bias, void *image,
                  size_t image_bytes, void *stream_) {
  return tt_pack_image_typed(cfg, TT_DTYPE_F32, layers, final_norm_weight, final_norm_bias,
                             image, image_bytes, stream_);
}

int tt_pack_image_typed(const tt_config *cfg, int dtype, const tt_layer_params *layers,
                        const void *final_norm_weight, const void *final_norm_bias, void *image,
                        size_t image_bytes, void *stream_) {
  int rc = validate_config(cfg);
  if (rc != TT_OK) return rc;
  if (dtype != TT_DTYPE_F32 && dtype != TT_DTYPE_F16 && dtype != TT_DTYPE_BF16)
    return fail(TT_ERR_INVALID_ARGUMENT, "tt_pack_image: dtype must be a TT_DTYPE_* value");
  if (layers == nullptr || final_norm_weight == nullptr || final_norm_bias == nullptr ||
      image == nullptr)
    return fail(TT_ERR_INVALID_ARGUMENT, "tt_pack_image: NULL pointer argument");
  const ImageLayout L(*cfg);
  if (image_bytes < L.total)
    return fail(TT_ERR_WORKSPACE, "tt_pack_image: image buffer smaller than tt_image_bytes");
  if (misaligned(image)) return fail(TT_ERR_INVALID_ARGUMENT, "image must be 16-byte aligned");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  char *img = static_cast<char *>(image);
  const size_t D = cfg->d_model, F = cfg->ffn_dim, f4 = sizeof(float);
  // fp32 parameters are copied; 16-bit ones widen exactly to fp32
  auto copy = [&](size_t off, const void *src, size_t n) -> int {
    if (src == nullptr) return fail(TT_ERR_INVALID_ARGUMENT, "tt_pack_image: NULL parameter");
    if (dtype != TT_DTYPE_F32)
      return launch_widen(dtype, src, reinterpret_cast<float *>(img + off), (int64_t)n, stream);
    TT_CUDA_TRY(cudaMemcpyAsync(img + off, src, n * f4, cudaMemcpyDeviceToDevice, stream));
    return TT_OK;
  };
  TT_CUDA_TRY(cudaMemsetAsync(img + L.status, 0, sizeof(DeviceStatus), stream));
  for (int l = 0; l < cfg->num_layers; ++l) {
    const tt_layer_params &p = layers[l];
    const LayerOffsets &o = L.layer[l];
    if ((rc = copy(o.ln1_w, p.norm1_weight, D)) || (rc = copy(o.ln1_b, p.norm1_bias, D)) ||
        (rc = copy(o.wqkv, p.q_weight, D * D)) ||
        (rc = copy(o.wqkv + D * D * f4, p.k_weight, D * D)) ||
        (rc = copy(o.wqkv + 2 * D * D * f4, p.v_weight, D * D)) ||
        (rc = copy(o.bqkv, p.q_bias, D)) || (rc = copy(o.bqkv + D * f4, p.k_bias, D)) ||
        (rc = copy(o.bqkv + 2 * D * f4, p.v_bias, D)) || (rc = copy(o.wo, p.out_weight, D * D)) ||
        (rc = copy(o.bo, p.out_bias, D)) || (rc = copy(o.ln2_w, p.norm2_weight, D)) ||
        (rc = copy(o.ln2_b, p.norm2_bias, D)) || (rc = copy(o.w1, p.ffn_in_weight, F * D)) ||
        (rc = copy(o.b1, p.ffn_in_bias, F)) || (rc = copy(o.w2, p.ffn_out_weight, D * F)) ||
        (rc = copy(o.b2, p.ffn_out_bias, D)))
      return rc;
    if (L.tensor) {
      auto F_ = [&](size_t off) { return reinterpret_cast<float *>(img + off); };
      auto H_ = [&](size_t off) { return reinterpret_cast<uint16_t *>(img + off); };
      float *sc = F_(o.wscale);
      unsigned *mx = reinterpret_cast<unsigned *>(sc + 4);
      if ((rc = split_weight(F_(o.wqkv), H_(o.wqkv_hi), H_(o.wqkv_lo), 3 * D * D, mx, sc, stream)) ||
          (rc = split_weight(F_(o.wo), H_(o.wo_hi), H_(o.wo_lo), D * D, mx + 1, sc + 1, stream)) ||
          (rc = split_weight(F_(o.w1), H_(o.w1_hi), H_(o.w1_lo), F * D, mx + 2, sc + 2, stream)) ||
          (rc = split_weight(F_(o.w2), H_(o.w2_hi), H_(o.w2_lo), D * F, mx + 3, sc + 3, stream)))
        return rc;
    }
  }
  if ((rc = copy(L.final_w, final_norm_weight, D)) || (rc = copy(L.final_b, final_norm_bias, D)))
    return rc;
  // set-up of tt_forward_noalloc on this device: looking up its scratch
  // array's address loads the module that holds it, so the array is reserved
  // now rather than inside a later no-alloc call
  void *scratch = nullptr;
  return noalloc_scratch_address(&scratch);
}

int tt_fp16_operand_bound(const tt_config *cfg, const void *image, float *bound, void *stream_) {
  int rc = validate_config(cfg);
  if (rc != TT_OK) return rc;
  if (image == nullptr || bound == nullptr)
    return fail(TT_ERR_INVALID_ARGUMENT, "tt_fp16_operand_bound: NULL argument");
  if (misaligned(image)) return fail(TT_ERR_INVALID_ARGUMENT, "image must be 16-byte aligned");
  const ImageLayout L(*cfg);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const char *img = static_cast<const char *>(image);
  auto P = [&](size_t off) { return reinterpret_cast<const float *>(img + off); };
  // the accumulator lives in the status block's spare words (pad[0])
  DeviceStatus *st = reinterpret_cast<DeviceStatus *>(const_cast<char *>(img) + L.status);
  unsigned *acc = reinterpret_cast<unsigned *>(&st->pad[0]);
  TT_CUDA_TRY(cudaMemsetAsync(acc, 0, sizeof(unsigned), stream));
  const int D = cfg->d_model, F = cfg->ffn_dim;
  for (int l = 0; l < cfg->num_layers; ++l) {
    const LayerOffsets &o = L.layer[l];
    const int blocks_qkv = (int)std::min<int64_t>(ceil_div(3LL * D, 8), 148 * 4);
    operand_bound_kernel<<<blocks_qkv, 256, 0, stream>>>(P(o.wqkv), P(o.bqkv), P(o.ln1_w),
                                                           P(o.ln1_b), 3 * D, D, 0, acc);
    TT_LAUNCH_CHECK("operand_bound (q|k|v)");
    const int blocks_f = (int)std::min<int64_t>(ceil_div((int64_t)F, 8), 148 * 4);
    operand_bound_kernel<<<blocks_f, 256, 0, stream>>>(P(o.w1), P(o.b1), P(o.ln2_w), P(o.ln2_b),
                                                         F, D, 1, acc);
    TT_LAUNCH_CHECK("operand_bound (ffn_in)");
  }
  unsigned bits = 0;
  TT_CUDA_TRY(cudaMemcpyAsync(&bits, acc, sizeof(unsigned), cudaMemcpyDeviceToHost, stream));
  TT_CUDA_TRY(cudaStreamSynchronize(stream));
  float v;
  std::memcpy(&v, &bits, sizeof v);
  *bound = v;
  return TT_OK;
}

size_t tt_workspace_bytes(const tt_config *cfg, int64_t batch, int64_t seq) {
  if (validate_config(cfg) != TT_OK || batch < 0 || seq < 0) return 0;
  const int plan = forward_plan(cfg, batch, seq);
  if (plan < 0 || plan == PLAN_CLUSTER || plan == PLAN_TILE) return 0;
  return WorkspaceLayout(*cfg, batch, seq).total;
}

int tt_forward_plan(const tt_config *cfg, int64_t batch, int64_t seq) {
  const int rc = validate_config(cfg);
  if (rc != TT_OK) return rc;
  return forward_plan(cfg, batch, seq);
}

int tt_forward_launch_count(const tt_config *cfg, int64_t batch, int64_t seq) {
  const int rc = validate_config(cfg);
  if (rc != TT_OK) return rc;
  if (batch <= 0 || seq <= 0) return 0;
  const int plan = forward_plan(cfg, batch, seq);
  if (plan < 0) return plan;
  if (plan == PLAN_CLUSTER || plan == PLAN_TILE) return 1;
  if (plan == PLAN_OPS_TC)
    return (ops_tc_fuses_ln(*cfg, batch * seq) ? 5 : 7) * cfg->num_layers + 1 +
           (ops_tc_skips_dead_rows(*cfg, batch * seq) ? 1 : 0);
  return 5 * cfg->num_layers + 1;
}

int tt_forward(const tt_config *cfg, const void *image, const float *x, const uint8_t *mask,
               int64_t batch, int64_t seq, float *y, void *workspace, size_t workspace_bytes,
               void *stream_) {
  int rc = validate_config(cfg);
  if (rc != TT_OK) return rc;
  if (batch < 0 || seq < 0) return fail(TT_ERR_INVALID_ARGUMENT, "batch and seq must be >= 0");
  if (batch == 0 || seq == 0) return TT_OK;
  if (image == nullptr || x == nullptr || y == nullptr)
    return fail(TT_ERR_INVALID_ARGUMENT, "tt_forward: NULL image, x or y");
  if (x == y) return fail(TT_ERR_INVALID_ARGUMENT, "tt_forward: y may not alias x");
  if (misaligned(image) || misaligned(x) || misaligned(y) || misaligned(workspace))
    return fail(TT_ERR_INVALID_ARGUMENT, "tt_forward: pointers must be 16-byte aligned");
  if (seq > (int64_t)INT32_MAX || batch * seq > ((int64_t)1 << 40))
    return fail(TT_ERR_UNSUPPORTED, "tt_forward: batch*seq too large");
  const ImageLayout L(*cfg);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const int plan = forward_plan(cfg, batch, seq);
  if (plan < 0) return plan;
  if (plan == PLAN_CLUSTER)
    return forward_cluster(*cfg, choose_cluster(*cfg, batch, seq), L,
                           static_cast<const char *>(image), x, mask, batch, seq, y, stream);
  if (plan == PLAN_TILE)
    return forward_tile(*cfg, L, static_cast<const char *>(image), x, mask, batch, seq, y, stream);
  const WorkspaceLayout W(*cfg, batch, seq);
  if (workspace_bytes < W.total || (W.total > 0 && workspace == nullptr))
    return fail(TT_ERR_WORKSPACE, "tt_forward: workspace smaller than tt_workspace_bytes (" +
                                      std::to_string(W.total) + " bytes)");
  const char *img = static_cast<const char *>(image);
  char *ws = static_cast<char *>(workspace);
  const tt_config c = *cfg;
  return run_forward_cached(
      make_forward_key(c, plan, image, x, mask, batch, seq, y, workspace), stream,
      [&](cudaStream_t s) {
        return plan == PLAN_OPS_TC ? forward_ops_tc(c, L, img, x, mask, batch, seq, y, W, ws, s)
                                   : forward_ops(c, L, img, x, mask, batch, seq, y, W, ws, s);
      });
}

size_t tt_typed_workspace_bytes(const tt_config *cfg, int dtype, int64_t batch, int64_t seq) {
  if (validate_config(cfg) != TT_OK || batch < 0 || seq < 0) return 0;
  if (dtype == TT_DTYPE_F32) return tt_workspace_bytes(cfg, batch, seq);
  if (dtype != TT_DTYPE_F16 && dtype != TT_DTYPE_BF16) return 0;
  const size_t io = align_up((size_t)batch * (size_t)seq * (size_t)cfg->d_model * sizeof(float), 256);
  return 2 * io + tt_workspace_bytes(cfg, batch, seq);
}

int tt_forward_typed(const tt_config *cfg, const void *image, int dtype, const void *x,
                     const uint8_t *mask, int64_t batch, int64_t seq, void *y, void *workspace,
                     size_t workspace_bytes, void *stream_) {
  if (dtype == TT_DTYPE_F32)
    return tt_forward(cfg, image, static_cast<const float *>(x), mask, batch, seq,
                      static_cast<float *>(y), workspace, workspace_bytes, stream_);
  int rc = validate_config(cfg);
  if (rc != TT_OK) return rc;
  if (dtype != TT_DTYPE_F16 && dtype != TT_DTYPE_BF16)
    return fail(TT_ERR_INVALID_ARGUMENT, "tt_forward_typed: dtype must be a TT_DTYPE_* value");
  if (batch < 0 || seq < 0) return fail(TT_ERR_INVALID_ARGUMENT, "batch and seq must be >= 0");
  if (batch == 0 || seq == 0) return TT_OK;
  if (image == nullptr || x == nullptr || y == nullptr || workspace == nullptr)
    return fail(TT_ERR_INVALID_ARGUMENT, "tt_forward_typed: NULL image, x, y or workspace");
  if (x == y) return fail(TT_ERR_INVALID_ARGUMENT, "tt_forward_typed: y may not alias x");
  if (misaligned(x) || misaligned(y) || misaligned(workspace))
    return fail(TT_ERR_INVALID_ARGUMENT, "tt_forward_typed: pointers must be 16-byte aligned");
  if (seq > (int64_t)INT32_MAX || batch * seq > ((int64_t)1 << 40))
    return fail(TT_ERR_UNSUPPORTED, "tt_forward_typed: batch*seq too large");
  const size_t need = tt_typed_workspace_bytes(cfg, dtype, batch, seq);
  if (workspace_bytes < need)
    return fail(TT_ERR_WORKSPACE, "tt_forward_typed: workspace smaller than "
                                  "tt_typed_workspace_bytes (" + std::to_string(need) + " bytes)");
  const int64_t n = batch * seq * (int64_t)cfg->d_model;
  const size_t io = align_up((size_t)n * sizeof(float), 256);
  char *ws = static_cast<char *>(workspace);
  float *x32 = reinterpret_cast<float *>(ws);
  float *y32 = reinterpret_cast<float *>(ws + io);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if ((rc = timed_launch(TT_KERNEL_CONVERT, stream,
                         [&] { return launch_widen(dtype, x, x32, n, stream); })))
    return rc;
  if ((rc = tt_forward(cfg, image, x32, mask, batch, seq, y32, ws + 2 * io,
                       workspace_bytes - 2 * io, stream_)))
    return rc;
  return timed_launch(TT_KERNEL_CONVERT, stream,
                      [&] { return launch_narrow(dtype, y32, y, n, stream); });
}

// Largest x (bytes) that tt_forward_host moves with copy kernels.
constexpr size_t kHostKernelCopyMax = (size_t)1 << 20;

// The device address of a page-locked host buffer mapped for the device, or
// null (pageable memory, device memory, or misaligned): read, not assumed.
static const void *mapped_host(const void *p) {
  if ((reinterpret_cast<uintptr_t>(p) & 15) != 0) return nullptr;
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (at.type != cudaMemoryTypeHost || at.devicePointer == nullptr) return nullptr;
  if ((reinterpret_cast<uintptr_t>(at.devicePointer) & 15) != 0) return nullptr;
  return at.devicePointer;
}

size_t tt_host_workspace_bytes(const tt_config *cfg, int64_t batch, int64_t seq) {
  if (validate_config(cfg) != TT_OK || batch < 0 || seq < 0) return 0;
  const size_t T = (size_t)batch * (size_t)seq;
  return 2 * align_up(T * (size_t)cfg->d_model * sizeof(float), 256) + align_up(T, 256) +
         tt_workspace_bytes(cfg, batch, seq);
}

int tt_forward_host(const tt_config *cfg, const void *image, const float *x_host,
                    const uint8_t *mask_host, int64_t batch, int64_t seq, float *y_host,
                    void *workspace, size_t workspace_bytes, void *stream_) {
  int rc = validate_config(cfg);
  if (rc != TT_OK) return rc;
  if (batch < 0 || seq < 0) return fail(TT_ERR_INVALID_ARGUMENT, "batch and seq must be >= 0");
  if (batch == 0 || seq == 0) return TT_OK;
  if (image == nullptr || x_host == nullptr || y_host == nullptr)
    return fail(TT_ERR_INVALID_ARGUMENT, "tt_forward_host: NULL image, x or y");
  if (x_host == y_host) return fail(TT_ERR_INVALID_ARGUMENT, "tt_forward_host: y may not alias x");
  if (misaligned(workspace))
    return fail(TT_ERR_INVALID_ARGUMENT, "tt_forward_host: workspace must be 16-byte aligned");
  if (seq > (int64_t)INT32_MAX || batch * seq > ((int64_t)1 << 40))
    return fail(TT_ERR_UNSUPPORTED, "tt_forward_host: batch*seq too large");
  const size_t need = tt_host_workspace_bytes(cfg, batch, seq);
  if (workspace_bytes < need || workspace == nullptr)
    return fail(TT_ERR_WORKSPACE, "tt_forward_host: workspace smaller than "
                                  "tt_host_workspace_bytes (" + std::to_string(need) + " bytes)");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const size_t T = (size_t)batch * (size_t)seq;
  const size_t xb = T * (size_t)cfg->d_model * sizeof(float), io = align_up(xb, 256);
  char *ws = static_cast<char *>(workspace);
  float *xs = reinterpret_cast<float *>(ws);
  float *ys = reinterpret_cast<float *>(ws + io);
  uint8_t *ms = reinterpret_cast<uint8_t *>(ws + 2 * io);
  const size_t used = 2 * io + align_up(T, 256);
  // Small steps whose buffers are page-locked and mapped for the device copy
  // with kernels (every 16-byte piece in flight at once, one round trip over
  // the host link) instead of DMA copies, whose fixed set-up cost dominates
  // a step of a few tens of microseconds.
  const void *xd = nullptr, *md = nullptr;
  void *yd = nullptr;
  const bool small = xb <= kHostKernelCopyMax && (xd = mapped_host(x_host)) != nullptr &&
                     (yd = const_cast<void *>(mapped_host(y_host))) != nullptr &&
                     (mask_host == nullptr || (md = mapped_host(mask_host)) != nullptr);
  if (small) {
    if ((rc = timed_launch(TT_KERNEL_CONVERT, stream,
                           [&] { return launch_small_copy(xd, xs, (int64_t)xb, stream); })))
      return rc;
    if (mask_host != nullptr &&
        (rc = timed_launch(TT_KERNEL_CONVERT, stream,
                           [&] { return launch_small_copy(md, ms, (int64_t)T, stream); })))
      return rc;
  } else {
    TT_CUDA_TRY(cudaMemcpyAsync(xs, x_host, xb, cudaMemcpyHostToDevice, stream));
    if (mask_host != nullptr)
      TT_CUDA_TRY(cudaMemcpyAsync(ms, mask_host, T, cudaMemcpyHostToDevice, stream));
  }
  if ((rc = tt_forward(cfg, image, xs, mask_host != nullptr ? ms : nullptr, batch, seq, ys,
                       ws + used, workspace_bytes - used, stream_)))
    return rc;
  if (small)
    return timed_launch(TT_KERNEL_CONVERT, stream,
                        [&] { return launch_small_copy(ys, yd, (int64_t)xb, stream); });
  TT_CUDA_TRY(cudaMemcpyAsync(y_host, ys, xb, cudaMemcpyDeviceToHost, stream));
  return TT_OK;
}

int tt_read_status(const tt_config *cfg, const void *image, int32_t *code, int32_t *detail,
                   void *stream_) {
  int rc = validate_config(cfg);
  if (rc != TT_OK) return rc;
  if (image == nullptr || code == nullptr)
    return fail(TT_ERR_INVALID_ARGUMENT, "tt_read_status: NULL argument");
  const ImageLayout L(*cfg);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  DeviceStatus st{};
  char *img = const_cast<char *>(static_cast<const char *>(image));
  TT_CUDA_TRY(cudaMemcpyAsync(&st, img + L.status, 2 * sizeof(int32_t), cudaMemcpyDeviceToHost,
                              stream));
  TT_CUDA_TRY(cudaStreamSynchronize(stream));
  TT_CUDA_TRY(cudaMemsetAsync(img + L.status, 0, sizeof(DeviceStatus), stream));
  *code = st.code;
  if (detail) *detail = st.detail;
  return TT_OK;
}

int tt_launch_probe_start(int capacity) {
  LaunchProbe &pr = g_probe;
  if (capacity < 0) return fail(TT_ERR_INVALID_ARGUMENT, "tt_launch_probe_start: capacity < 0");
  for (cudaEvent_t e : pr.events) cudaEventDestroy(e);
  pr.events.clear();
  pr.kinds.clear();
  pr.count = 0;
  std::vector<cudaEvent_t> ev((size_t)2 * capacity);
  for (size_t i = 0; i < ev.size(); ++i) {
    const cudaError_t err = cudaEventCreate(&ev[i]);
    if (err != cudaSuccess) {
      for (size_t j = 0; j < i; ++j) cudaEventDestroy(ev[j]);
      return fail(TT_ERR_CUDA, std::string("cudaEventCreate: ") + cudaGetErrorString(err));
    }
  }
  pr.events = std::move(ev);
  pr.kinds.assign((size_t)capacity, 0);
  return TT_OK;
}

int tt_launch_probe_read(float *ms, int32_t *kinds, int capacity) {
  LaunchProbe &pr = g_probe;
  const int n = pr.count;
  for (int i = 0; i < n && i < capacity; ++i) {
    TT_CUDA_TRY(cudaEventSynchronize(pr.events[2 * i + 1]));
    float t = 0.f;
    TT_CUDA_TRY(cudaEventElapsedTime(&t, pr.events[2 * i], pr.events[2 * i + 1]));
    if (ms) ms[i] = t;
    if (kinds) kinds[i] = pr.kinds[i];
  }
  pr.count = 0;
  return n;
}

int tt_test_arm_wait_timeout(int budget_log2) { return arm_gemm_wait_timeout(budget_log2); }

int tt_test_gelu(const float *x, float *y, int64_t n, void *stream_) {
  if (n < 0 || (n > 0 && (x == nullptr || y == nullptr)))
    return fail(TT_ERR_INVALID_ARGUMENT, "tt_test_gelu: NULL pointer or negative size");
  if (n == 0) return TT_OK;
  const int64_t blocks = std::min<int64_t>(ceil_div(n, 256), 148 * 8);
  gelu_test_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream_)>>>(x, y, n);
  TT_LAUNCH_CHECK("gelu_test");
  return TT_OK;
}

int tt_last_error(char *buf, size_t len) {
  const std::string &m = g_last_error;
  if (buf != nullptr && len > 0) {
    const size_t n = std::min(len - 1, m.size());
    std::memcpy(buf, m.data(), n);
    buf[n] = '\0';
  }
  return (int)m.size();
}

}  // extern "C"
