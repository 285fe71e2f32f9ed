// Causal, key-padding-masked multi-head attention in fp32, flash style: K/V
// tiles staged in shared memory, fp32 online softmax, the [B,H,S,S] score
// tensor never exists.
//
// Restates the reference attention core (torch_transformer_benchmark.py:97-117):
// scores = (q . k) * head_dim^-0.5 (scale applied after the dot product, :97),
// -inf for keys after the query when causal (:99-103) and for padded keys
// (:105-108), softmax in fp32 (:111), context = probs . v written straight in
// [B, S, H*hd] order (the layout :113-117 produces by transposing back).
// Queries with no allowed key (possible only for padded query rows) get a zero
// context; the reference gets NaN there and then zeroes those rows (:120-121).
#include <math_constants.h>

#include "tt_common.cuh"

namespace tt {
namespace {

constexpr int kThreads = 128;

template <int HDT>
struct AttnShape {
  static constexpr int G = HDT >= 64 ? HDT / 32 : 1;  // threads per query row
  static constexpr int P = HDT / G;                   // head dims per thread
  static constexpr int PS = P + 4;                    // padded smem stride per part
  static constexpr int BQ = kThreads / G;             // query rows per block
  static constexpr int BKV = HDT <= 64 ? 64 : 32;     // keys per smem tile
  static constexpr int CH = 8;                        // keys per softmax chunk
  static constexpr size_t smem_bytes = (size_t)2 * BKV * G * PS * sizeof(float) + BKV * sizeof(float);
};

template <int HDT, bool VEC>
__global__ void __launch_bounds__(kThreads) attention_ffma_kernel(AttentionParams p) {
  using Sh = AttnShape<HDT>;
  constexpr int G = Sh::G, P = Sh::P, PS = Sh::PS, BQ = Sh::BQ, BKV = Sh::BKV, CH = Sh::CH;
  extern __shared__ __align__(16) float smem[];
  float *sK = smem;                       // [BKV][G][PS]
  float *sV = sK + BKV * G * PS;          // [BKV][G][PS]
  float *sOk = sV + BKV * G * PS;         // [BKV] key allowed by the padding mask
  __shared__ int s_kv_len;
  pdl_trigger();
  pdl_wait();

  const int S = p.seq, D = p.d_model, hd = p.head_dim;
  const int64_t ld = 3LL * D;
  const int h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int q0 = blockIdx.x * BQ;
  const int tid = threadIdx.x;
  const uint8_t *mrow = p.mask ? p.mask + b * S : nullptr;

  // kv_len = 1 + last valid key of this sequence; keys at or after it are all padding.
  if (tid == 0) s_kv_len = mrow ? 0 : S;
  __syncthreads();
  if (mrow) {
    int last = 0;
    for (int j = tid; j < S; j += kThreads)
      if (mrow[j]) last = j + 1;
    if (last) atomicMax(&s_kv_len, last);
    __syncthreads();
  }
  const int kv_len = s_kv_len;
  if (q0 >= kv_len) return;  // every query row of this block is padding

  const int row = q0 + tid / G;
  const int part = tid % G;
  const bool row_in = row < S;
  const int64_t tok = b * S + (row_in ? row : 0);

  float q[P], o[P];
#pragma unroll
  for (int d = 0; d < P; ++d) {
    const int dd = part * P + d;
    q[d] = (row_in && dd < hd) ? p.qkv[tok * ld + (int64_t)h * hd + dd] : 0.f;
    o[d] = 0.f;
  }
  float m = -CUDART_INF_F, l = 0.f;

  const int kv_end = p.causal ? min(kv_len, min(S, q0 + BQ)) : kv_len;
  for (int k0 = 0; k0 < kv_end; k0 += BKV) {
    const int nk = min(BKV, kv_end - k0);
    __syncthreads();  // previous tile fully consumed
    // Stage K and V rows [k0, k0+nk) of head h.
    if (VEC) {
      constexpr int F4 = HDT / 4;  // float4 slots per key in the template width
      for (int idx = tid; idx < BKV * F4; idx += kThreads) {
        const int j = idx / F4, d4 = (idx % F4) * 4;
        float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
        if (j < nk && d4 < hd) {
          const float *src = p.qkv + (b * S + k0 + j) * ld + (int64_t)h * hd + d4;
          kv = *reinterpret_cast<const float4 *>(src + D);
          vv = *reinterpret_cast<const float4 *>(src + 2 * D);
        }
        const int off = (j * G + d4 / P) * PS + d4 % P;
        *reinterpret_cast<float4 *>(sK + off) = kv;
        *reinterpret_cast<float4 *>(sV + off) = vv;
      }
    } else {
      for (int idx = tid; idx < BKV * HDT; idx += kThreads) {
        const int j = idx / HDT, dd = idx % HDT;
        float kv = 0.f, vv = 0.f;
        if (j < nk && dd < hd) {
          const float *src = p.qkv + (b * S + k0 + j) * ld + (int64_t)h * hd + dd;
          kv = src[D];
          vv = src[2 * D];
        }
        const int off = (j * G + dd / P) * PS + dd % P;
        sK[off] = kv;
        sV[off] = vv;
      }
    }
    for (int j = tid; j < BKV; j += kThreads)
      sOk[j] = (j < nk && (mrow == nullptr || mrow[k0 + j] != 0)) ? 1.f : 0.f;
    __syncthreads();

    for (int jc = 0; jc < nk; jc += CH) {
      float s[CH];
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const int j = jc + c;
        const float *kr = sK + ((j < BKV ? j : 0) * G + part) * PS;
        float dot = 0.f;
#pragma unroll
        for (int d = 0; d < P; d += 4) {
          const float4 kk = *reinterpret_cast<const float4 *>(kr + d);
          dot = fmaf(q[d + 0], kk.x, dot);
          dot = fmaf(q[d + 1], kk.y, dot);
          dot = fmaf(q[d + 2], kk.z, dot);
          dot = fmaf(q[d + 3], kk.w, dot);
        }
#pragma unroll
        for (int off = 1; off < G; off <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
        const int kj = k0 + j;
        const bool ok = j < nk && sOk[j < BKV ? j : 0] != 0.f && (!p.causal || kj <= row);
        s[c] = ok ? dot * p.scale : -CUDART_INF_F;
      }
      float cmax = s[0];
#pragma unroll
      for (int c = 1; c < CH; ++c) cmax = fmaxf(cmax, s[c]);
      const float m_new = fmaxf(m, cmax);
      if (m_new == -CUDART_INF_F) continue;  // nothing allowed yet for this row
      const float alpha = __expf(m - m_new);   // 0 when m is -inf
      l *= alpha;
#pragma unroll
      for (int d = 0; d < P; ++d) o[d] *= alpha;
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const float pc = __expf(s[c] - m_new);  // 0 for masked keys
        l += pc;
        const float *vr = sV + ((jc + c < BKV ? jc + c : 0) * G + part) * PS;
#pragma unroll
        for (int d = 0; d < P; d += 4) {
          const float4 vv = *reinterpret_cast<const float4 *>(vr + d);
          o[d + 0] = fmaf(pc, vv.x, o[d + 0]);
          o[d + 1] = fmaf(pc, vv.y, o[d + 1]);
          o[d + 2] = fmaf(pc, vv.z, o[d + 2]);
          o[d + 3] = fmaf(pc, vv.w, o[d + 3]);
        }
      }
      m = m_new;
    }
  }

  if (!row_in) return;
  const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
  for (int d = 0; d < P; ++d) {
    if (part * P + d < hd) {
      const float v = o[d] * inv;
      if (p.ctx != nullptr) p.ctx[tok * D + (int64_t)h * hd + part * P + d] = v;
      if (p.ctx_hi != nullptr) {
        f16_split(v, p.ctx_hi[tok * D + (int64_t)h * hd + part * P + d],
                  p.ctx_lo[tok * D + (int64_t)h * hd + part * P + d]);
      }
    }
  }
}

template <int HDT>
int launch_hd(const AttentionParams &p, bool vec, cudaStream_t stream) {
  using Sh = AttnShape<HDT>;
  dim3 grid((unsigned)ceil_div(p.seq, Sh::BQ), (unsigned)p.num_heads, (unsigned)p.batch);
  const size_t smem = Sh::smem_bytes;
  static bool attr_set = false;
  if (!attr_set && smem > 48 * 1024) {
    TT_CUDA_TRY(cudaFuncSetAttribute(attention_ffma_kernel<HDT, true>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    TT_CUDA_TRY(cudaFuncSetAttribute(attention_ffma_kernel<HDT, false>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  }
  attr_set = true;
  if (vec)
    TT_CUDA_TRY(launch_kernel(attention_ffma_kernel<HDT, true>, grid, dim3(kThreads), smem, stream,
                              1, p));
  else
    TT_CUDA_TRY(launch_kernel(attention_ffma_kernel<HDT, false>, grid, dim3(kThreads), smem, stream,
                              1, p));
  TT_LAUNCH_CHECK("attention_ffma");
  return TT_OK;
}

}  // namespace

int launch_attention_ffma(const AttentionParams &p, cudaStream_t stream) {
  if (p.batch <= 0 || p.seq <= 0) return TT_OK;
  if (p.batch > 65535 || p.num_heads > 65535)
    return fail(TT_ERR_UNSUPPORTED, "attention: batch and num_heads must be <= 65535");
  const bool vec = (p.head_dim % 4 == 0) && (p.d_model % 4 == 0) &&
                   ((reinterpret_cast<uintptr_t>(p.qkv) & 15) == 0);
  const int hd = p.head_dim;
  if (hd <= 8) return launch_hd<8>(p, vec, stream);
  if (hd <= 16) return launch_hd<16>(p, vec, stream);
  if (hd <= 32) return launch_hd<32>(p, vec, stream);
  if (hd <= 64) return launch_hd<64>(p, vec, stream);
  if (hd <= 128) return launch_hd<128>(p, vec, stream);
  if (hd <= 256) return launch_hd<256>(p, vec, stream);
  return fail(TT_ERR_UNSUPPORTED, "attention: head_dim > 256 is not supported");
}

}  // namespace tt
