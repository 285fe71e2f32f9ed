// Row LayerNorm (nn.LayerNorm semantics: biased variance, eps inside the sqrt),
// one warp per row, float4 HBM access, warp-shuffle reductions.
//
// Follows nn.LayerNorm(d_model) as the reference uses it for norm1 / norm2 /
// final_norm (torch_transformer_benchmark.py:128,130,160; applied :140,:141,:169)
// and the padded-row zeroing of the final output (:170-171).
#include "tt_common.cuh"

namespace tt {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Register-resident variant: D % 4 == 0 and D <= 128 * NV.
template <int NV>
__global__ void __launch_bounds__(256) layernorm_vec_kernel(
    const float *__restrict__ x, float *__restrict__ y, uint16_t *__restrict__ y_hi,
    uint16_t *__restrict__ y_lo, const float *__restrict__ gamma, const float *__restrict__ beta,
    const uint8_t *__restrict__ row_mask, int zero_masked_rows, int64_t rows, int d, float eps,
    const int *__restrict__ live_tile) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  // rows of a dead 128-row tile: their outputs feed only GEMM tiles that are
  // skipped (a block's 8 rows lie in one tile)
  if (live_tile != nullptr && live_tile[row >> 7] == 0) return;
  const int d4 = d >> 2;
  const float4 *xr = reinterpret_cast<const float4 *>(x + row * d);
  float4 v[NV];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    if (c < d4) {
      v[i] = xr[c];
      s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    } else {
      v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  const float mean = warp_sum(s) / (float)d;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    if (c < d4) {
      const float a = v[i].x - mean, b = v[i].y - mean, e = v[i].z - mean, f = v[i].w - mean;
      ss += (a * a + b * b) + (e * e + f * f);
    }
  }
  const float rstd = rsqrtf(warp_sum(ss) / (float)d + eps);
  const bool zero = zero_masked_rows && row_mask != nullptr && row_mask[row] == 0;
  float4 *yr = y != nullptr ? reinterpret_cast<float4 *>(y + row * d) : nullptr;
  const float4 *g4 = reinterpret_cast<const float4 *>(gamma);
  const float4 *b4 = reinterpret_cast<const float4 *>(beta);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    if (c < d4) {
      float4 o;
      if (zero) {
        o = make_float4(0.f, 0.f, 0.f, 0.f);
      } else {
        const float4 g = g4[c], b = b4[c];
        o.x = (v[i].x - mean) * rstd * g.x + b.x;
        o.y = (v[i].y - mean) * rstd * g.y + b.y;
        o.z = (v[i].z - mean) * rstd * g.z + b.z;
        o.w = (v[i].w - mean) * rstd * g.w + b.w;
      }
      if (y != nullptr) yr[c] = o;
      if (y_hi != nullptr) {
        uint16_t h[4], l[4];
        f16_split(o.x, h[0], l[0]);
        f16_split(o.y, h[1], l[1]);
        f16_split(o.z, h[2], l[2]);
        f16_split(o.w, h[3], l[3]);
        reinterpret_cast<uint2 *>(y_hi + row * d)[c] =
            make_uint2(h[0] | ((uint32_t)h[1] << 16), h[2] | ((uint32_t)h[3] << 16));
        reinterpret_cast<uint2 *>(y_lo + row * d)[c] =
            make_uint2(l[0] | ((uint32_t)l[1] << 16), l[2] | ((uint32_t)l[3] << 16));
      }
    }
  }
}

// Generic variant for any D: two passes over the row in global memory.
__global__ void __launch_bounds__(256) layernorm_generic_kernel(
    const float *__restrict__ x, float *__restrict__ y, uint16_t *__restrict__ y_hi,
    uint16_t *__restrict__ y_lo, const float *__restrict__ gamma, const float *__restrict__ beta,
    const uint8_t *__restrict__ row_mask, int zero_masked_rows, int64_t rows, int d, float eps) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float *xr = x + row * d;
  float s = 0.f;
  for (int c = lane; c < d; c += 32) s += xr[c];
  const float mean = warp_sum(s) / (float)d;
  float ss = 0.f;
  for (int c = lane; c < d; c += 32) {
    const float a = xr[c] - mean;
    ss += a * a;
  }
  const float rstd = rsqrtf(warp_sum(ss) / (float)d + eps);
  const bool zero = zero_masked_rows && row_mask != nullptr && row_mask[row] == 0;
  // x may alias y: every lane has finished reading its own elements above, and
  // each element below is read and written by the same lane.
  for (int c = lane; c < d; c += 32) {
    const float o = zero ? 0.f : (xr[c] - mean) * rstd * gamma[c] + beta[c];
    if (y != nullptr) y[row * d + c] = o;
    if (y_hi != nullptr) f16_split(o, y_hi[row * d + c], y_lo[row * d + c]);
  }
}

}  // namespace

int launch_layernorm(const float *x, float *y, uint16_t *y_hi, uint16_t *y_lo, const float *gamma,
                     const float *beta, const uint8_t *row_mask, int zero_masked_rows,
                     int64_t rows, int d, float eps, cudaStream_t stream, const int *live_tile) {
  if (rows <= 0) return TT_OK;
  const int threads = 256, rows_per_block = threads / 32;
  const int64_t blocks = ceil_div(rows, rows_per_block);
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) |
                         reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(beta) |
                         reinterpret_cast<uintptr_t>(y_hi) | reinterpret_cast<uintptr_t>(y_lo)) &
                        15) == 0 &&
                       (y_hi == nullptr || d % 8 == 0);
  if (d % 4 == 0 && aligned && d <= 1024) {
    const int nv = (int)ceil_div(d, 128);
#define TT_LN_CASE(NV)                                                                     \
  TT_CUDA_TRY(launch_kernel(layernorm_vec_kernel<NV>, dim3((unsigned)blocks), dim3(threads), 0, \
                            stream, 1, x, y, y_hi, y_lo, gamma, beta, row_mask,             \
                            zero_masked_rows, rows, d, eps, live_tile))
    if (nv == 1) TT_LN_CASE(1);
    else if (nv == 2) TT_LN_CASE(2);
    else if (nv <= 4) TT_LN_CASE(4);
    else TT_LN_CASE(8);
#undef TT_LN_CASE
  } else {
    TT_CUDA_TRY(launch_kernel(layernorm_generic_kernel, dim3((unsigned)blocks), dim3(threads), 0,
                              stream, 1, x, y, y_hi, y_lo, gamma, beta, row_mask,
                              zero_masked_rows, rows, d, eps));
  }
  TT_LAUNCH_CHECK("layernorm");
  return TT_OK;
}

}  // namespace tt
