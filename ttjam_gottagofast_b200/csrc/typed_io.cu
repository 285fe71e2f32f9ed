// Element-type conversion at the edges of the forward for 16-bit models.
//
// The reference runs its benchmark in float16 or bfloat16 by moving the whole
// model and its input to that dtype (torch_transformer_benchmark.py:225-231,
// :698-699). This build computes every such forward at fp32 accuracy: the
// 16-bit parameters and inputs widen exactly to fp32 (every fp16 and bf16
// value is an fp32 value), the fp32 schedules run unchanged, and the output
// is rounded once, to nearest even, to the caller's dtype. These kernels are
// that widening and that rounding; both are HBM-bound streams (2 + 4 bytes
// per element each way).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "tt_common.cuh"

namespace tt {
namespace {

__device__ __forceinline__ float widen1(__half v) { return __half2float(v); }
__device__ __forceinline__ float widen1(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T narrow1(float v);
template <> __device__ __forceinline__ __half narrow1<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 narrow1<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// dst[i] = (float)src[i]. Eight elements per thread and step: one 16-byte
// load, two 16-byte stores; the n % 8 tail element by element. With vec = 0
// (src or dst not 16-byte aligned) every element goes the scalar way.
template <typename T>
__global__ void __launch_bounds__(256) widen_kernel(const T *__restrict__ src,
                                                    float *__restrict__ dst, int64_t n, int vec) {
  pdl_trigger();
  pdl_wait();
  const int64_t vecs = vec ? n >> 3 : 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (int64_t v = t0; v < vecs; v += stride) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(src) + v);
    const T *e = reinterpret_cast<const T *>(&raw);
    float4 a, b;
    a.x = widen1(e[0]); a.y = widen1(e[1]); a.z = widen1(e[2]); a.w = widen1(e[3]);
    b.x = widen1(e[4]); b.y = widen1(e[5]); b.z = widen1(e[6]); b.w = widen1(e[7]);
    reinterpret_cast<float4 *>(dst)[2 * v] = a;
    reinterpret_cast<float4 *>(dst)[2 * v + 1] = b;
  }
  for (int64_t i = (vecs << 3) + t0; i < n; i += stride) dst[i] = widen1(src[i]);
}

// dst[i] = src[i] rounded to nearest even in T (vec as for widen_kernel).
template <typename T>
__global__ void __launch_bounds__(256) narrow_kernel(const float *__restrict__ src,
                                                     T *__restrict__ dst, int64_t n, int vec) {
  pdl_trigger();
  pdl_wait();
  const int64_t vecs = vec ? n >> 3 : 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (int64_t v = t0; v < vecs; v += stride) {
    const float4 a = __ldg(reinterpret_cast<const float4 *>(src) + 2 * v);
    const float4 b = __ldg(reinterpret_cast<const float4 *>(src) + 2 * v + 1);
    uint4 raw;
    T *e = reinterpret_cast<T *>(&raw);
    e[0] = narrow1<T>(a.x); e[1] = narrow1<T>(a.y); e[2] = narrow1<T>(a.z); e[3] = narrow1<T>(a.w);
    e[4] = narrow1<T>(b.x); e[5] = narrow1<T>(b.y); e[6] = narrow1<T>(b.z); e[7] = narrow1<T>(b.w);
    reinterpret_cast<uint4 *>(dst)[v] = raw;
  }
  for (int64_t i = (vecs << 3) + t0; i < n; i += stride) dst[i] = narrow1<T>(src[i]);
}

// One wave of 256-thread blocks, 8 per SM, or fewer for small arrays.
unsigned convert_blocks(int64_t n) {
  const int64_t per_block = 256 * 8;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, per_block), 148 * 8));
}

int aligned16(const void *a, const void *b) {
  return ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15) == 0;
}

// dst[0 .. n) = src[0 .. n): one 16-byte load and store per thread and step
// (src and dst 16-byte aligned), the n % 16 tail bytes one by one.
__global__ void __launch_bounds__(256) small_copy_kernel(const uint8_t *__restrict__ src,
                                                         uint8_t *__restrict__ dst, int64_t n) {
  pdl_trigger();
  pdl_wait();
  const int64_t vecs = n >> 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (int64_t v = t0; v < vecs; v += stride)
    reinterpret_cast<uint4 *>(dst)[v] = reinterpret_cast<const uint4 *>(src)[v];
  for (int64_t i = (vecs << 4) + t0; i < n; i += stride) dst[i] = src[i];
}

}  // namespace

int launch_small_copy(const void *src, void *dst, int64_t n, cudaStream_t stream) {
  if (n <= 0) return TT_OK;
  if (!aligned16(src, dst))
    return fail(TT_ERR_INVALID_ARGUMENT, "small copy: addresses must be 16-byte aligned");
  const int64_t threads = std::max<int64_t>(1, ceil_div(n, 16));
  const dim3 grid((unsigned)std::min<int64_t>(ceil_div(threads, 256), 148 * 8)), block(256);
  const cudaError_t err = launch_kernel(small_copy_kernel, grid, block, 0, stream, 1,
                                        static_cast<const uint8_t *>(src),
                                        static_cast<uint8_t *>(dst), n);
  if (err != cudaSuccess)
    return fail(TT_ERR_CUDA, std::string("launch of small copy: ") + cudaGetErrorString(err));
  return TT_OK;
}

int launch_widen(int dtype, const void *src, float *dst, int64_t n, cudaStream_t stream) {
  if (n <= 0) return TT_OK;
  const dim3 grid(convert_blocks(n)), block(256);
  const int vec = aligned16(src, dst);
  cudaError_t err;
  if (dtype == TT_DTYPE_F16)
    err = launch_kernel(widen_kernel<__half>, grid, block, 0, stream, 1,
                        static_cast<const __half *>(src), dst, n, vec);
  else if (dtype == TT_DTYPE_BF16)
    err = launch_kernel(widen_kernel<__nv_bfloat16>, grid, block, 0, stream, 1,
                        static_cast<const __nv_bfloat16 *>(src), dst, n, vec);
  else
    return fail(TT_ERR_INVALID_ARGUMENT, "widen: dtype must be TT_DTYPE_F16 or TT_DTYPE_BF16");
  if (err != cudaSuccess)
    return fail(TT_ERR_CUDA, std::string("launch of widen: ") + cudaGetErrorString(err));
  return TT_OK;
}

int launch_narrow(int dtype, const float *src, void *dst, int64_t n, cudaStream_t stream) {
  if (n <= 0) return TT_OK;
  const dim3 grid(convert_blocks(n)), block(256);
  const int vec = aligned16(src, dst);
  cudaError_t err;
  if (dtype == TT_DTYPE_F16)
    err = launch_kernel(narrow_kernel<__half>, grid, block, 0, stream, 1, src,
                        static_cast<__half *>(dst), n, vec);
  else if (dtype == TT_DTYPE_BF16)
    err = launch_kernel(narrow_kernel<__nv_bfloat16>, grid, block, 0, stream, 1, src,
                        static_cast<__nv_bfloat16 *>(dst), n, vec);
  else
    return fail(TT_ERR_INVALID_ARGUMENT, "narrow: dtype must be TT_DTYPE_F16 or TT_DTYPE_BF16");
  if (err != cudaSuccess)
    return fail(TT_ERR_CUDA, std::string("launch of narrow: ") + cudaGetErrorString(err));
  return TT_OK;
}

}  // namespace tt
