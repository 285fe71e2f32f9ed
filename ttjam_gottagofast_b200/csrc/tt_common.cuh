// Shared helpers for the sm_100a kernels of the pre-norm Transformer forward.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

#include "ttjam_b200.h"

namespace tt {

// Device status word layout inside the model image: [0] first error code,
// [1] detail code of the kernel that raised it.
struct DeviceStatus {
  int32_t code;
  int32_t detail;
  int32_t pad[62];
};

__device__ __forceinline__ void raise_status(DeviceStatus *st, int32_t code, int32_t detail) {
  if (st == nullptr) return;
  if (atomicCAS(&st->code, 0, code) == 0) atomicExch(&st->detail, detail);
}

// Host-side error latch (per thread), surfaced through tt_last_error.
void set_last_error(const std::string &msg);

inline int fail(int code, const std::string &msg) {
  set_last_error(msg);
  return code;
}

#define TT_CUDA_TRY(expr)                                                              \
  do {                                                                                 \
    cudaError_t err__ = (expr);                                                        \
    if (err__ != cudaSuccess)                                                          \
      return ::tt::fail(TT_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(err__)); \
  } while (0)

#define TT_LAUNCH_CHECK(what)                                                          \
  do {                                                                                 \
    cudaError_t err__ = cudaGetLastError();                                            \
    if (err__ != cudaSuccess)                                                          \
      return ::tt::fail(TT_ERR_CUDA, std::string("launch of ") + (what) + ": " +     \
                                         cudaGetErrorString(err__));                   \
  } while (0)

// Programmatic dependent launch. The kernels of the per-op schedules are
// launched with programmatic stream serialization (launch_kernel). Each calls
// pdl_trigger() first: once every CTA of its grid has started, the next
// kernel on the stream may be scheduled, so that kernel's set-up (barriers,
// tensor-memory allocation, reads of the weights and the mask, which no
// kernel of a forward writes) overlaps this grid's tail. Each calls pdl_wait()
// before its first read of data an earlier kernel wrote and before its first
// global write: it returns once every earlier grid of the stream has
// completed and its writes are visible. Without the launch attribute both are
// no-ops.
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Whether launch_kernel sets the attribute: on unless the environment sets
// TT_PDL=0 (read once).
bool pdl_enabled();

// cudaLaunchKernelEx with programmatic stream serialization (when enabled)
// and, for cluster_x > 1, a cluster of cluster_x CTAs along x.
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, unsigned cluster_x, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Exact GELU, F.gelu(approximate="none") = v * Phi(v), Phi(v) = 1 - erfc(v/sqrt2)/2,
// to fp32 accuracy. erfc(z), z = |v|/sqrt2, is the Chebyshev fit of Numerical
// Recipes (Press, Teukolsky, Vetterling & Flannery, 2nd ed., sec. 6.2, erfcc):
//   erfc(z) = t exp(-z^2 + P(t)),  t = 1 / (1 + z/2),  P a degree-9 polynomial,
// with a fractional error below 1.2e-7 for every z >= 0. Then
//   v >= 0:  GELU = v (1 - erfc(z)/2),     v < 0:  GELU = v erfc(z)/2,
// so both tails keep their relative accuracy (the negative tail's tiny outputs
// too). One reciprocal, one exp2 and twelve FMAs, with no branch on the value:
// the ffn_in epilogue runs it on every output (measured on B200, workload E's
// ffn_in 2221 -> 2123 us per launch against erff). Infinities map as the
// erf form maps them (+inf -> +inf, -inf -> NaN), NaN stays NaN.
__device__ __forceinline__ float gelu_erf(float v) {
  const float z = fabsf(v) * 0.70710678118654752f;
  float t;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(fmaf(0.5f, z, 1.0f)));
  float p = 0.17087277f;
  p = fmaf(p, t, -0.82215223f);
  p = fmaf(p, t, 1.48851587f);
  p = fmaf(p, t, -1.13520398f);
  p = fmaf(p, t, 0.27886807f);
  p = fmaf(p, t, -0.18628806f);
  p = fmaf(p, t, 0.09678418f);
  p = fmaf(p, t, 0.37409196f);
  p = fmaf(p, t, 1.00002368f);
  p = fmaf(p, t, -1.26551223f);
  const float a = fmaf(-z, z, p) * 1.4426950408889634f;  // exponent in log2 units
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(a));
  const float r = t * e;  // erfc(z)
  const float phi = v >= 0.f ? fmaf(-0.5f, r, 1.0f) : 0.5f * r;
  return v * phi;
}

// fp16 split used by the tensor-core path (binary16 bit patterns): hi = x
// rounded to the nearest fp16 (cvt.rn), lo = x - hi, exact in fp32 (hi is x
// rounded to 11 significant bits), rounded to fp16. hi + lo carries about 22
// significant bits while |x| <= 65504; a larger |x| gives an infinite hi. For
// a pair: one pack, two widenings, two subtractions and one pack.
__device__ __forceinline__ uint16_t f16_bits(float x) {
  uint16_t h;
  asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(x));
  return h;
}
__device__ __forceinline__ float f16_value(uint16_t h) {
  float x;
  asm("cvt.f32.f16 %0, %1;" : "=f"(x) : "h"(h));
  return x;
}
__device__ __forceinline__ void f16_split(float x, uint16_t &hi, uint16_t &lo) {
  hi = f16_bits(x);
  lo = f16_bits(__fsub_rn(x, f16_value(hi)));
}
// Two values at once: hi and lo pieces packed as fp16 pairs, the element
// with the lower index (a) in the low 16 bits.
__device__ __forceinline__ void f16_split2(float a, float b, uint32_t &hi, uint32_t &lo) {
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(b), "f"(a));
  float ha, hb;
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\tcvt.f32.f16 %0, l;\n\tcvt.f32.f16 %1, h;\n\t}"
      : "=f"(ha), "=f"(hb)
      : "r"(hi));
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(__fsub_rn(b, hb)), "f"(__fsub_rn(a, ha)));
}
// max(a, b, c) in one instruction (three-input max.f32, sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// ---------------------------------------------------------------------------
// Kernel launchers (defined in the per-kernel .cu files).
// ---------------------------------------------------------------------------

// Row LayerNorm, nn.LayerNorm(D) semantics (eps, biased variance). If
// `zero_rows_mask` is set, rows whose mask byte is 0 are written as 0.
// If y_hi/y_lo are given, also writes the fp16 split of the output (y may then
// be null). With live_tile (one int per 128-row tile, 0 = dead), the rows of
// dead tiles may be left unwritten.
int launch_layernorm(const float *x, float *y, uint16_t *y_hi, uint16_t *y_lo, const float *gamma,
                     const float *beta, const uint8_t *row_mask, int zero_masked_rows,
                     int64_t rows, int d, float eps, cudaStream_t stream,
                     const int *live_tile = nullptr);

enum GemmEpilogue : int {
  EPI_BIAS = 0,             // C = A W^T + b
  EPI_BIAS_GELU = 1,        // C = gelu(A W^T + b)
  EPI_BIAS_RESIDUAL = 2,    // C = valid ? R + (A W^T + b) : 0   (R may alias C)
};

struct GemmParams {
  const float *A;        // [M, K] row-major, leading dim lda
  int64_t lda;
  const float *W;        // [N, K] row-major (nn.Linear weight)
  const float *bias;     // [N]
  const float *R;        // residual [M, N], leading dim ldc (may alias C)
  float *C;              // [M, N], leading dim ldc
  int64_t ldc;
  const uint8_t *row_mask;  // [M] row validity, or null (all valid)
  const float *ln_gamma, *ln_beta;  // LayerNorm prologue on A when non-null
  float ln_eps;
  int64_t M;
  int N, K;
  int epilogue;
};

// FFMA register-tiled fp32 GEMM with LayerNorm prologue and fused epilogues.
int launch_gemm_ffma(const GemmParams &p, cudaStream_t stream);

struct AttentionParams {
  const float *qkv;      // [B*S, 3D]: q | k | v, head h at columns h*hd..h*hd+hd-1
  float *ctx;            // [B*S, D], or null when only the split is wanted
  uint16_t *ctx_hi, *ctx_lo;  // optional fp16 split copies
  const uint8_t *mask;   // [B, S] or null
  int64_t batch;
  int seq, d_model, num_heads, head_dim;
  int causal;
  float scale;
};

// Flash-style causal / key-padded attention with fp32 online softmax.
int launch_attention_ffma(const AttentionParams &p, cudaStream_t stream);

// Widening of `n` elements of TT_DTYPE_F16 / TT_DTYPE_BF16 to fp32, and the
// rounding (to nearest even) of fp32 to them (typed_io.cu). Any alignment.
int launch_widen(int dtype, const void *src, float *dst, int64_t n, cudaStream_t stream);
int launch_narrow(int dtype, const float *src, void *dst, int64_t n, cudaStream_t stream);
// Copy of n bytes by a kernel, every 16-byte piece in flight at once; for
// small transfers to or from page-locked host memory mapped for the device
// (typed_io.cu). Both addresses 16-byte aligned.
int launch_small_copy(const void *src, void *dst, int64_t n, cudaStream_t stream);

}  // namespace tt
