// Single-launch split-precision tensor-core forward for the d_model = 128,
// ffn_dim = 128, 4-head model (head_dim 32) on batches of short sequences: the
// reference forward (torch_transformer_benchmark.py:134-172, every layer and
// the final LayerNorm) in one launch. One CTA owns a tile of 128 token rows
// holding whole sequences (seq divides 128, so a tile's rows never attend to
// another tile's), and runs every layer on it with no exchange between CTAs.
//
// Per CTA (320 threads): warps 0-7 are the row threads -- tile row r belongs to
// threads r and r + 128, each taking one half of the row's columns (and of its
// keys in the softmax), with partial row statistics exchanged through shared
// memory; warp 9 (one lane) issues every MMA once the row warps have arrived
// on the barrier of the step that feeds it; warp 8 (one lane) streams the
// weights through a 5-stage ring with
// TMA (3-D tensor maps over [layer, out rows, k] of the packed fp16 pieces, so
// one map per matrix covers all layers). Every product is split precision as
// in the per-op tensor-core schedule (gemm_tc.cu): operands as fp16 hi/lo
// pairs, three kind::f16 MMAs per product (hi.hi, hi.lo, lo.hi), fp32
// accumulation in tensor memory, the weights' power-of-two pack scale undone
// in the epilogue.
//
// Tensor memory (512 columns, lane = tile row): the residual stream x (fp32,
// 128 columns) for the whole forward, the projection accumulator (128), the
// scores S of one head over the tile's 128 keys, overwritten by the fp16 split
// of P (128), and the four heads' attention outputs O (128).
// Shared memory: the A operand of the next projection (LayerNorm output,
// context or GELU output; 128 rows x 128 k as four 32-wide k-blocks of 64-byte
// rows in the 64-byte swizzle the MMA reads), Q and K of the current head and
// V^T of two heads in the same layout (V^T as 32 dims x 128 keys), and the
// weight ring.
//
// One layer is twelve MMA groups: q|k|v of head 0 (N = 96: its q, k and v
// rows), then per head h the scores S = Q K^T (N = 128), issued together with
// the q|k|v projection of head h+1 (which then runs under head h's softmax,
// completing on a barrier of its own), and P.V (N = 32); then out_proj, ffn_in
// and ffn_out (N = 128); out_proj's first three k-blocks (heads 0-2's
// contexts) are issued under the last head's softmax, its last k-block once
// that head's context is in. V^T is double-buffered by head parity, so head
// h+1's q|k|v epilogue writes it while head h's P.V still reads the other one.
// The row threads between groups: the q|k|v epilogue (bias, range check,
// Q and K rows and the transposed V^T into shared memory), the softmax (the
// whole row at once: exact max, 2^7-scaled P split into tensor memory), the
// context (O / l per head into the A operand), the out_proj epilogue (bias,
// residual, padded-row zeroing) with LayerNorm 2, the GELU epilogue, and the
// ffn_out epilogue (bias, residual, padded-row zeroing) with the next
// LayerNorm 1 or, after the last layer, the final LayerNorm and the output row.
//
// Masks: key j is allowed for query row r when both lie in the same sequence
// of the tile, j <= r (causal), and row j is a valid token (inside the batch,
// mask byte set); padded rows are zeroed at out_proj and at the block end, as
// in the per-op schedules, so only valid rows feed later layers' keys.
// Every mbarrier wait is bounded; a wait that gives up latches
// TT_ERR_DEVICE_TIMEOUT, the CTA runs its remaining steps without issuing
// MMAs or loads, drains what it started and frees its tensor memory.
#include <cuda.h>
#include <math_constants.h>

#include "tile_forward.cuh"

namespace tt {
namespace {

constexpr int D = 128, H = 4, HD = 32, TR = 128;  // model width, heads, head dim, tile rows
constexpr int kRowThreads = 256;  // warps 0-7: two threads per tile row, one per column half
constexpr int kThreads = kRowThreads + 64;  // warp 8: weight loads; warp 9: MMA issue
constexpr int NST = 5;                             // weight ring stages

// shared memory, offsets from a 1024-byte aligned base
constexpr uint32_t KBLK = 16384;  // a 32-wide k-block of a 128-row split operand: hi | lo
constexpr uint32_t HALF = 8192;   // lo piece offset inside a k-block (and a weight stage)
constexpr uint32_t OFF_A = 0;                 // A operand: 4 k-blocks
constexpr uint32_t OFF_Q = 4 * KBLK;          // Q of one head (one k-block)
constexpr uint32_t OFF_K = OFF_Q + KBLK;      // K of one head (one k-block)
constexpr uint32_t OFF_VT = OFF_K + KBLK;     // V^T of two heads (h even, h odd): 4 k-blocks each
constexpr uint32_t VT_KB = 4096, VT_HALF = 2048;  // a V^T k-block: 32 dims x 64 B, hi | lo
constexpr uint32_t VT_BUF = 4 * VT_KB;            // one head's V^T
constexpr uint32_t OFF_W = OFF_VT + 2 * VT_BUF;   // weight ring
constexpr uint32_t WSTAGE = 16384;  // up to 128 weight rows x one k-block: hi | lo
constexpr uint32_t OFF_KW = OFF_W + NST * WSTAGE;  // 4 words: valid key rows of the tile
// partial row statistics of the two threads of a row: [2 arrays][2 halves][128]
constexpr uint32_t OFF_XCH = OFF_KW + 256;
// softmax sums per head and half: [4 heads][2 halves][128]
constexpr uint32_t OFF_XL = OFF_XCH + 2048;
constexpr uint32_t OFF_BAR = OFF_XL + 4096;
constexpr size_t SMEM_BYTES = (size_t)OFF_BAR + 256 + 1024;  // + alignment slack
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
static_assert(OFF_W % 1024 == 0 && OFF_VT % 1024 == 0, "operands on the swizzle period");

// tensor memory columns
constexpr uint32_t T_X = 0, T_ACC = 128, T_SP = 256, T_O = 384, TMEM_COLS = 512;

// instruction descriptor (kind::f16): D fp32, A/B fp16, both K-major, M 128, N n
constexpr uint32_t idesc(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
constexpr uint32_t IDESC_QKV = idesc(3 * HD), IDESC_128 = idesc(128), IDESC_PV = idesc(HD);

// ---- PTX helpers ------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}
// Bounded wait: false after ~2^28 cycles (latching TT_ERR_DEVICE_TIMEOUT with
// `detail` and setting this CTA's abort word), or within 32 polls once the
// abort word is set (another thread of this CTA gave up first).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort_w,
                                          DeviceStatus *st, int detail) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 31) == 0) {
      if (*abort_w != 0) return false;
      if (clock64() - t0 > (1LL << 28)) {
        *abort_w = 1;
        raise_status(st, TT_ERR_DEVICE_TIMEOUT, detail);
        return false;
      }
    }
  }
}
// Bounded wait for work this thread started itself (its TMA loads, its MMAs)
// before the CTA frees its resources: ignores the abort word.
__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity, DeviceStatus *st,
                                           int detail) {
  const long long t0 = clock64();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return;
    if ((i & 31) == 31 && clock64() - t0 > (1LL << 28)) {
      raise_status(st, TT_ERR_DEVICE_TIMEOUT, detail);
      return;
    }
  }
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *tm, int c0, int c1,
                                            int c2, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *tm) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}
// Shared-memory matrix descriptor: K-major, 64-byte swizzle, rows of 64 bytes,
// 8-row groups 512 bytes apart, version 1. A k-step of 16 fp16 inside a
// k-block adds 2 (32 bytes) to the start address field.
__device__ __forceinline__ uint64_t desc_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(512 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)4 << 61;
  return d;
}
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t id,
                                       uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(id), "r"(accum)
      : "memory");
}
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t id,
                                       uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(id), "r"(accum)
      : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void *p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}
__device__ __forceinline__ void prefetch_l1(const void *p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// named barrier of the eight row-thread warps
__device__ __forceinline__ void rows_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float *v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float *v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t *v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
      "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
      "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// 2^x with the hardware's approximate base-2 exponential; 2^-inf = 0
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- row helpers (thread r of the row threads) -------------------------------
// Row r's 32 values v of one k-block -> the fp16 split in the 64-byte swizzle
// (16-byte unit u of row r at unit u ^ ((r >> 1) & 3); lo piece `lo_off`
// further); returns the largest magnitude.
__device__ __forceinline__ float put_kblock_row(uint8_t *kb, uint32_t lo_off, int r,
                                                const float *v) {
  float amax = 0.f;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a = v[8 * u + 2 * i], b = v[8 * u + 2 * i + 1];
      amax = fmax3(amax, fabsf(a), fabsf(b));
      f16_split2(a, b, hw[i], lw[i]);
    }
    const uint32_t off = (uint32_t)r * 64u + ((uint32_t)(u ^ ((r >> 1) & 3)) << 4);
    *reinterpret_cast<uint4 *>(kb + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4 *>(kb + lo_off + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  }
  return amax;
}

// LayerNorm of row r, its 128 columns split between the row's two threads:
// this thread's half hf is chunks 2 hf and 2 hf + 1 (32 columns each) of the
// row in tensor memory at xaddr, which load(chunk, values) reads (and may
// update first: the residual add). The mean and the biased variance from the
// two halves' partial statistics, which meet in xch ([2 arrays][2 halves][128
// rows]) across a barrier of the row threads; then this thread's chunks
// normalised, scaled by g and shifted by b and handed to out(chunk, values). Loops over chunks are not unrolled: the kernel runs
// each phase once per head or layer, so short loop bodies (which stay in the
// instruction cache) matter more than the loop overhead.
template <typename Load, typename Out>
__device__ __forceinline__ void layer_norm_half(uint32_t xaddr, int r, int hf, float *xch,
                                                const float *g, const float *b, float eps,
                                                Load load, Out out) {
  // one pass over this thread's 64 columns: sums shifted by the half's first
  // element (no cancellation while that element lies within a few standard
  // deviations of the mean), then the two halves' means and squared-deviation
  // sums combined with Chan, Golub and LeVeque's pairwise formula
  float s = 0.f, q = 0.f, k0 = 0.f;
#pragma unroll 1
  for (int cc = 0; cc < 2; ++cc) {
    float v[32];
    // chunk c of the row: as it is in tensor memory, or (the residual add)
    // updated and written back there first
    load(2 * hf + cc, v);
    if (cc == 0) k0 = v[0];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float d = v[i] - k0;
      s += d;
      q = fmaf(d, d, q);
    }
  }
  tmem_wait_st();  // the rows written back above, before the second pass reads them
  constexpr float kHalf = 1.0f / (D / 2);
  xch[hf * TR + r] = fmaf(s, kHalf, k0);           // mean of the half
  xch[2 * TR + hf * TR + r] = fmaf(-s, s * kHalf, q);  // its squared deviations
  rows_sync();
  const float m0 = xch[r], m1 = xch[TR + r], dm = m1 - m0;
  const float mean = 0.5f * (m0 + m1);
  const float m2 = xch[2 * TR + r] + xch[3 * TR + r] + dm * dm * (0.25f * D);
  const float rs = rsqrtf(fmaxf(m2, 0.f) * (1.0f / D) + eps);
#pragma unroll 1
  for (int cc = 0; cc < 2; ++cc) {
    const int c = 2 * hf + cc;
    float v[32];
    tmem_ld32(xaddr + 32 * c, v);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float4 g4 = *reinterpret_cast<const float4 *>(g + 32 * c + i);
      const float4 b4 = *reinterpret_cast<const float4 *>(b + 32 * c + i);
      v[i] = (v[i] - mean) * rs * g4.x + b4.x;
      v[i + 1] = (v[i + 1] - mean) * rs * g4.y + b4.y;
      v[i + 2] = (v[i + 2] - mean) * rs * g4.z + b4.z;
      v[i + 3] = (v[i + 3] - mean) * rs * g4.w + b4.w;
    }
    out(c, v);
  }
}

// Allowed keys [lo, hi) of the 32-key word w as a bit mask.
__device__ __forceinline__ uint32_t range_word(int w, int lo, int hi) {
  const int a = max(lo - 32 * w, 0), b = min(hi - 32 * w, 32);
  if (b <= a) return 0u;
  const uint32_t upto_b = b >= 32 ? 0xffffffffu : ((1u << b) - 1u);
  const uint32_t below_a = a >= 32 ? 0xffffffffu : ((1u << a) - 1u);
  return upto_b & ~below_a;
}

// 32 consecutive floats of a bias vector (16-byte aligned), as float4 loads.
__device__ __forceinline__ void load32(const float *p, float *v) {
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    const float4 q = *reinterpret_cast<const float4 *>(p + i);
    v[i] = q.x; v[i + 1] = q.y; v[i + 2] = q.z; v[i + 3] = q.w;
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    tile_forward_kernel(const __grid_constant__ CUtensorMap tm_qkv_hi,
                        const __grid_constant__ CUtensorMap tm_qkv_lo,
                        const __grid_constant__ CUtensorMap tm_o_hi,
                        const __grid_constant__ CUtensorMap tm_o_lo,
                        const __grid_constant__ CUtensorMap tm_1_hi,
                        const __grid_constant__ CUtensorMap tm_1_lo,
                        const __grid_constant__ CUtensorMap tm_2_hi,
                        const __grid_constant__ CUtensorMap tm_2_lo, const TileArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t *bp = smem_raw + (base - raw);
  const uint32_t bars = base + OFF_BAR;
  auto full = [&](int s) { return bars + 8u * s; };
  auto empty = [&](int s) { return bars + 8u * (NST + s); };
  const uint32_t mma_bar = bars + 8u * (2 * NST);
  const uint32_t drain_bar = bars + 8u * (2 * NST + 1);
  const uint32_t qkv_bar = bars + 8u * (2 * NST + 2);
  const uint32_t tmem_slot = bars + 8u * (2 * NST + 3);
  static_assert(8 * (2 * NST + 4) + 8 <= 256, "barrier area");
  uint32_t *tmem_slot_ptr = reinterpret_cast<uint32_t *>(bp + OFF_BAR + 8 * (2 * NST + 3));
  volatile int *abort_w = reinterpret_cast<volatile int *>(bp + OFF_BAR + 8 * (2 * NST + 3) + 4);
  // row threads -> MMA thread: one arrive per row warp once a step's operands
  // are in place; one barrier per kind of step, so that the row threads are
  // never two phases of one barrier ahead of the MMA thread's waits
  const uint32_t rows_misc = bars + 8u * (2 * NST + 4);  // LayerNorm 1, context, LayerNorm 2, GELU
  const uint32_t rows_epi = bars + 8u * (2 * NST + 5);   // a head's q|k|v epilogue
  const uint32_t rows_sm = bars + 8u * (2 * NST + 6);    // a head's softmax
  const uint32_t rows_ctx = bars + 8u * (2 * NST + 7);   // heads 0-2's contexts
  static_assert(8 * (2 * NST + 8) <= 256, "barrier area");
  uint32_t *kword = reinterpret_cast<uint32_t *>(bp + OFF_KW);
  float *xch = reinterpret_cast<float *>(bp + OFF_XCH);
  float *xl = reinterpret_cast<float *>(bp + OFF_XL);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int L = a.num_layers;
  pdl_trigger();
  if (tid == kRowThreads) {
    prefetch_tmap(&tm_qkv_hi); prefetch_tmap(&tm_qkv_lo);
    prefetch_tmap(&tm_o_hi); prefetch_tmap(&tm_o_lo);
    prefetch_tmap(&tm_1_hi); prefetch_tmap(&tm_1_lo);
    prefetch_tmap(&tm_2_hi); prefetch_tmap(&tm_2_lo);
  }
  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    mbar_init(mma_bar, 1);
    mbar_init(drain_bar, 1);
    mbar_init(qkv_bar, 1);
    mbar_init(rows_misc, kRowThreads / 32);
    mbar_init(rows_epi, kRowThreads / 32);
    mbar_init(rows_sm, kRowThreads / 32);
    mbar_init(rows_ctx, kRowThreads / 32);
    *abort_w = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tmem_slot),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = *tmem_slot_ptr;

  if (warp == kRowThreads / 32) {
    // ---- weight loads: per layer q|k|v by head (q, k and v rows of the head:
    // three 32-row boxes), then Wo, W1, W2; one k-block per stage ------------
    // (the weights are packed before the forward and no kernel writes them,
    // so the loads start before the wait on the previous kernel)
    if (lane == 0) {
      int ws = 0;
      bool ok = true;
      for (int l = 0; ok && l < L; ++l) {
        for (int m = 0; ok && m < H + 3; ++m) {
          for (int kb = 0; kb < 4; ++kb, ++ws) {
            const int s = ws % NST;
            if (ws >= NST &&
                !mbar_wait(empty(s), ((ws / NST) - 1) & 1, abort_w, a.status, 0x6100)) {
              ok = false;
              break;
            }
            const uint32_t st = base + OFF_W + (uint32_t)s * WSTAGE;
            if (m < H) {
              mbar_expect_tx(full(s), 2u * 3u * HD * 64u);
#pragma unroll
              for (int part = 0; part < 3; ++part) {
                tma_load_3d(st + part * 2048u, &tm_qkv_hi, kb * 32, part * D + m * HD, l, full(s));
                tma_load_3d(st + HALF + part * 2048u, &tm_qkv_lo, kb * 32, part * D + m * HD, l,
                            full(s));
              }
            } else {
              const CUtensorMap *thi = m == H ? &tm_o_hi : m == H + 1 ? &tm_1_hi : &tm_2_hi;
              const CUtensorMap *tlo = m == H ? &tm_o_lo : m == H + 1 ? &tm_1_lo : &tm_2_lo;
              mbar_expect_tx(full(s), 2u * 128u * 64u);
              tma_load_3d(st, thi, kb * 32, 0, l, full(s));
              tma_load_3d(st + HALF, tlo, kb * 32, 0, l, full(s));
            }
          }
        }
      }
      // the loads of the last stages have landed before the CTA retires
      for (int k = ws > NST ? ws - NST : 0; k < ws; ++k)
        mbar_drain(full(k % NST), (k / NST) & 1, a.status, 0x6F00);
    }
  } else if (warp == kRowThreads / 32 + 1) {
    // the small per-layer vectors the row threads read from global memory
    // (LayerNorm gammas and betas, biases, accumulator scales), every layer's,
    // into L2 by the lanes that issue no MMAs: their first reads in a layer
    // then find them there, not in HBM
    if (lane != 0) {
      const int li = lane - 1;  // 0..30
      for (int l = 0; l < L; ++l) {
        const char *lbase = a.image + (size_t)l * a.layer_stride;
        if (li < 4) {  // the 512-byte vectors: four 128-byte lines each
          const int o = 128 * li;
          prefetch_l2(lbase + a.off.ln1_w + o);
          prefetch_l2(lbase + a.off.ln1_b + o);
          prefetch_l2(lbase + a.off.bo + o);
          prefetch_l2(lbase + a.off.ln2_w + o);
          prefetch_l2(lbase + a.off.ln2_b + o);
          prefetch_l2(lbase + a.off.b1 + o);
          prefetch_l2(lbase + a.off.b2 + o);
        }
        if (li < 12) prefetch_l2(lbase + a.off.bqkv + 128 * li);  // q|k|v bias, 1536 bytes
        if (li == 12) prefetch_l2(lbase + a.off.wscale);
      }
      if (li < 4) {
        prefetch_l2(reinterpret_cast<const char *>(a.final_w) + 128 * li);
        prefetch_l2(reinterpret_cast<const char *>(a.final_b) + 128 * li);
      }
    }
    // ---- MMA issue (one lane): each group once the row threads' step that
    // feeds it is done, in the order the row threads consume the results ----
    if (lane == 0) {
      bool ok = true;  // MMAs are issued while no wait has given up
      int ws = 0;      // weight stages consumed
      uint32_t pm = 0, pe = 0, ps = 0, pc = 0;  // phases waited on rows_misc, _epi, _sm, _ctx
      // one projection over k-blocks kb0 .. kb1 - 1 of the A operand into
      // tensor-memory column d_col (k-block 0 starts the sum), B rows from the
      // next weight stages
      auto gemm = [&](uint32_t d_col, uint32_t id, int kb0 = 0, int kb1 = 4) {
#pragma unroll 1
        for (int kb = kb0; kb < kb1; ++kb, ++ws) {
          const int s = ws % NST;
          if (!ok || !mbar_wait(full(s), (ws / NST) & 1, abort_w, a.status, 0x6200 + kb)) {
            ok = false;
            continue;
          }
          tc_fence_after();
          const uint32_t ab = base + OFF_A + (uint32_t)kb * KBLK;
          const uint32_t wb = base + OFF_W + (uint32_t)s * WSTAGE;
          const uint64_t ah = desc_sw64(ab), al = desc_sw64(ab + HALF);
          const uint64_t wh = desc_sw64(wb), wl = desc_sw64(wb + HALF);
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const uint64_t ko = (uint64_t)(2 * k);
            mma_ss(tm + d_col, ah + ko, wh + ko, id, (kb | k) != 0);
            mma_ss(tm + d_col, ah + ko, wl + ko, id, 1);
            mma_ss(tm + d_col, al + ko, wh + ko, id, 1);
          }
          mma_commit(empty(s));
        }
      };
      auto rows_wait = [&](uint32_t bar, uint32_t &ph, int detail) {
        if (!mbar_wait(bar, ph & 1, abort_w, a.status, detail)) ok = false;
        ++ph;
        tc_fence_after();
      };
#pragma unroll 1
      for (int l = 0; l < L; ++l) {
        rows_wait(rows_misc, pm, 0x6B00);  // LayerNorm 1 in the A operand
        gemm(T_ACC, IDESC_QKV);            // q|k|v of head 0
        mma_commit(mma_bar);
#pragma unroll 1
        for (int h = 0; h < H; ++h) {
          rows_wait(rows_epi, pe, 0x6B10 + h);  // Q, K and V^T of head h in shared memory
          if (ok) {
            // S = Q K^T over the tile's 128 keys (after P.V of the previous
            // head, which read the S/P cells it overwrites)
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk) {
              const uint64_t ko = (uint64_t)(2 * kk);
              const uint64_t qh = desc_sw64(base + OFF_Q) + ko, ql = desc_sw64(base + OFF_Q + HALF) + ko;
              const uint64_t kh = desc_sw64(base + OFF_K) + ko, kl = desc_sw64(base + OFF_K + HALF) + ko;
              mma_ss(tm + T_SP, qh, kh, IDESC_128, kk > 0);
              mma_ss(tm + T_SP, qh, kl, IDESC_128, 1);
              mma_ss(tm + T_SP, ql, kh, IDESC_128, 1);
            }
          }
          mma_commit(mma_bar);
          // q|k|v of the next head (the row threads have read the
          // accumulator): it runs under this head's softmax
          if (h + 1 < H) {
            gemm(T_ACC, IDESC_QKV);
            mma_commit(qkv_bar);
          } else {
            // heads 0-2's contexts in the A operand: out_proj's first three
            // k-blocks run under the last head's softmax
            rows_wait(rows_ctx, pc, 0x6B28);
            gemm(T_ACC, IDESC_128, 0, H - 1);
          }
          rows_wait(rows_sm, ps, 0x6B20 + h);  // P of head h in tensor memory
          if (ok) {
            // O_h = P V_h: keys 16 kk .. 16 kk + 15 are P_hi cells
            // 32 (kk / 2) + 8 (kk % 2) .. + 7 and P_lo 16 cells further
            const uint32_t od = tm + T_O + (uint32_t)(h * HD);
#pragma unroll
            for (int kk = 0; kk < TR / 16; ++kk) {
              const uint32_t vb = base + OFF_VT + (uint32_t)(h & 1) * VT_BUF + (uint32_t)(kk >> 1) * VT_KB;
              const uint64_t ko = (uint64_t)(2 * (kk & 1));
              const uint64_t vh = desc_sw64(vb) + ko, vl = desc_sw64(vb + VT_HALF) + ko;
              const uint32_t ph = tm + T_SP + 32u * (uint32_t)(kk >> 1) + 8u * (uint32_t)(kk & 1);
              mma_ts(od, ph, vh, IDESC_PV, kk > 0);
              mma_ts(od, ph, vl, IDESC_PV, 1);
              mma_ts(od, ph + 16u, vh, IDESC_PV, 1);
            }
          }
          // the last head's P.V completes the context; earlier ones complete
          // with the next head's scores, which are issued after them
          if (h + 1 == H) mma_commit(mma_bar);
        }
        rows_wait(rows_misc, pm, 0x6B30);  // the last head's context in the A operand
        gemm(T_ACC, IDESC_128, H - 1, H);  // out_proj's last k-block
        mma_commit(mma_bar);
        rows_wait(rows_misc, pm, 0x6B40);  // LayerNorm 2
        gemm(T_ACC, IDESC_128);            // ffn_in
        mma_commit(mma_bar);
        rows_wait(rows_misc, pm, 0x6B50);  // GELU output
        gemm(T_ACC, IDESC_128);            // ffn_out
        mma_commit(mma_bar);
      }
      // every MMA this thread issued has completed before the tensor memory
      // is freed
      mma_commit(drain_bar);
      mbar_drain(drain_bar, 0, a.status, 0x6F10);
    }
  } else {
    // ---- row threads: r = tile row (tensor-memory lane), hf = column half --
    const int r = tid & (TR - 1), hf = tid >> 7;
    const int64_t g = (int64_t)blockIdx.x * TR + r;
    const bool in = g < a.rows;
    const uint32_t lb = tm + ((uint32_t)((warp & 3) * 32) << 16);  // this warp's lanes
    const float sl = a.scale * 1.4426950408889634f;
    pdl_wait();  // x comes from the caller (or an earlier kernel)
    const bool valid = in && (a.mask == nullptr || a.mask[g] != 0);
    if (hf == 0) {
      const uint32_t w = __ballot_sync(0xffffffffu, valid);
      if (lane == 0) kword[warp] = w;
    }
    // allowed keys of row r: its sequence's rows of the tile, up to r (causal)
    const int j0 = (r / a.seq) * a.seq;
    const int jend = a.causal ? r + 1 : j0 + a.seq;
    uint32_t phase = 0;    // completed MMA groups on mma_bar
    uint32_t qphase = 0;   // completed q|k|v groups on qkv_bar (heads 1..3 of each layer)
    // all row threads: the last committed MMA group has completed
    auto wait_mma = [&](int detail) {
      mbar_wait(mma_bar, phase & 1, abort_w, a.status, detail);
      ++phase;
      tc_fence_after();
    };
    auto wait_qkv = [&](int detail) {
      mbar_wait(qkv_bar, qphase & 1, abort_w, a.status, detail);
      ++qphase;
      tc_fence_after();
    };
    // all row threads: this step's shared-memory operands and tensor-memory
    // writes are complete; the MMA thread waits for all eight row warps on
    // `bar` before it issues the next MMA group
    auto step_done = [&](uint32_t bar) {
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar);
    };
    auto to_a = [&](int c, float *v) { put_kblock_row(bp + OFF_A + c * KBLK, HALF, r, v); };
    // head h's context O_h / l -> k-block h of the A operand
    auto ctx_to_a = [&](int h) {
      float o[HD];
      tmem_ld32(lb + T_O + h * HD, o);
      tmem_wait_ld();
      const float lsum = xl[(h * 2) * TR + r] + xl[(h * 2 + 1) * TR + r];
      const float il = lsum > 0.f ? 1.0f / lsum : 0.f;
#pragma unroll
      for (int i = 0; i < HD; ++i) o[i] *= il;
      put_kblock_row(bp + OFF_A + h * KBLK, HALF, r, o);
    };
    // this thread's two 32-float chunks of a per-layer vector, into L1 ahead
    // of the step that reads them (issued before an MMA wait)
    auto pf_vec = [&](const float *v) {
      prefetch_l1(v + 64 * hf);
      prefetch_l1(v + 64 * hf + 32);
    };
    // this thread's chunks: x = valid ? x + acc * scale + bias : 0
    // chunk c of the residual stream as it is, for a LayerNorm
    auto x_as_is = [&](int c, float *v) {
      tmem_ld32(lb + T_X + 32 * c, v);
      tmem_wait_ld();
    };
    // chunk c of the residual stream after the residual add
    // x = valid ? x + acc * scale + bias : 0, written back to tensor memory:
    // the LayerNorm that follows takes its statistics in the same pass
    auto x_plus = [&](float scale, const float *bias) {
      return [&, scale, bias](int c, float *v) {
        float acc[32], bv[32];
        tmem_ld32(lb + T_ACC + 32 * c, acc);
        tmem_ld32(lb + T_X + 32 * c, v);
        load32(bias + 32 * c, bv);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = valid ? v[i] + fmaf(acc[i], scale, bv[i]) : 0.f;
        tmem_st32(lb + T_X + 32 * c, reinterpret_cast<uint32_t *>(v));
      };
    };

    // x row -> tensor memory (zeros past the batch), this thread's chunks
#pragma unroll 1
    for (int cc = 0; cc < 2; ++cc) {
      const int c = 2 * hf + cc;
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
        if (in) q = *reinterpret_cast<const float4 *>(a.x + g * D + 32 * c + i);
        v[i] = q.x; v[i + 1] = q.y; v[i + 2] = q.z; v[i + 3] = q.w;
      }
      tmem_st32(lb + T_X + 32 * c, reinterpret_cast<uint32_t *>(v));
    }
    tmem_wait_st();
    pf_vec(reinterpret_cast<const float *>(a.image + a.off.ln1_w));
    pf_vec(reinterpret_cast<const float *>(a.image + a.off.ln1_b));
    rows_sync();  // kword written
    // LayerNorm 1 of layer 0 -> A operand (later layers': after ffn_out)
    layer_norm_half(lb + T_X, r, hf, xch, reinterpret_cast<const float *>(a.image + a.off.ln1_w),
                    reinterpret_cast<const float *>(a.image + a.off.ln1_b), a.eps, x_as_is, to_a);
#pragma unroll 1
    for (int l = 0; l < L; ++l) {
      const char *lbase = a.image + (size_t)l * a.layer_stride;
      auto P = [&](size_t off) { return reinterpret_cast<const float *>(lbase + off); };
      const float *wsc = P(a.off.wscale);
      const float s_qkv = wsc[0], s_o = wsc[1], s_1 = wsc[2], s_2 = wsc[3];
      step_done(rows_misc);  // LayerNorm 1 in the A operand
      const float *bqkv = P(a.off.bqkv);
#pragma unroll 1
      for (int h = 0; h < H; ++h) {
        // ---- q|k|v epilogue of head h: half 0 takes q and value dims 0-15,
        // half 1 takes k and value dims 16-31 ------------------------------
        prefetch_l1(bqkv + hf * D + h * HD);
        prefetch_l1(bqkv + 2 * D + h * HD + 16 * hf);
        if (h == 0)
          wait_mma(0x6300);
        else
          wait_qkv(0x6300 + h);
        {
          float t[HD], bv[HD];
          tmem_ld32(lb + T_ACC + HD * hf, t);
          load32(bqkv + hf * D + h * HD, bv);
          float vv[16];
          tmem_ld16(lb + T_ACC + 2 * HD + 16 * hf, vv);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < HD; ++i) t[i] = fmaf(t[i], s_qkv, bv[i]);
          float amax = put_kblock_row(bp + (hf ? OFF_K : OFF_Q), HALF, r, t);
          // Q and K are in place (and every accumulator value is in registers):
          // the scores may start while V^T, which only P.V reads, is written
          // (the softmax's arrival, after it, publishes V^T)
          step_done(rows_epi);
          // V^T: dim i is row i of k-block r / 32, key r % 32 its element
          const float *bvv = bqkv + 2 * D + h * HD + 16 * hf;
          float bv16[16];
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            const float4 q = *reinterpret_cast<const float4 *>(bvv + i);
            bv16[i] = q.x; bv16[i + 1] = q.y; bv16[i + 2] = q.z; bv16[i + 3] = q.w;
          }
          uint8_t *vt = bp + OFF_VT + (uint32_t)(h & 1) * VT_BUF + (uint32_t)(r >> 5) * VT_KB;
          const int c = r & 31;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int d = 16 * hf + i;
            const float x = fmaf(vv[i], s_qkv, bv16[i]);
            uint16_t hi, lo;
            amax = fmaxf(amax, fabsf(x));
            f16_split(x, hi, lo);
            const uint32_t off = (uint32_t)d * 64u + ((uint32_t)((c >> 3) ^ ((d >> 1) & 3)) << 4) +
                                 (uint32_t)(c & 7) * 2u;
            *reinterpret_cast<uint16_t *>(vt + off) = hi;
            *reinterpret_cast<uint16_t *>(vt + VT_HALF + off) = lo;
          }
          if (!(amax <= 65504.f) && in) raise_status(a.status, TT_ERR_DEVICE_RANGE, 0x6400 + h);
        }
        // ---- softmax of row r, keys split by half: the row max (the halves'
        // maxima meet in xch), then 2^7-scaled P over S and the partial sums
        wait_mma(0x6500 + h);
        if (h + 1 == H) {
          // heads 0-2 are complete (their P.V ran before these scores, and
          // so did the last q|k|v read of the A operand): their contexts go
          // in now, half 0 taking heads 0 and 1, half 1 head 2
          ctx_to_a(2 * hf);
          if (hf == 0) ctx_to_a(1);
          step_done(rows_ctx);
        }
        {
          // a 32-key word no row of the warp may see (above the causal
          // diagonal, another sequence, padding) is skipped; one every row
          // sees in full needs no per-key test (both warp-uniform)
          float mx = -CUDART_INF_F;
#pragma unroll 1
          for (int cc = 0; cc < 2; ++cc) {
            const int c = 2 * hf + cc;
            const uint32_t al = range_word(c, j0, jend) & kword[c];
            if (!__any_sync(0xffffffffu, al != 0u)) continue;
            float t[32];
            tmem_ld32(lb + T_SP + 32 * c, t);
            tmem_wait_ld();
            if (__all_sync(0xffffffffu, al == 0xffffffffu)) {
#pragma unroll
              for (int j = 0; j < 32; j += 2) mx = fmax3(mx, t[j], t[j + 1]);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) mx = (al >> j) & 1u ? fmaxf(mx, t[j]) : mx;
            }
          }
          xch[hf * TR + r] = mx;
          rows_sync();
          mx = fmaxf(xch[r], xch[TR + r]);
          // 2^7 p = 2^(s sl - (m sl - 7)); 0 for masked keys and for rows
          // without an allowed key
          const bool live = mx != -CUDART_INF_F;
          const float noff = 7.0f - mx * sl;
          float lsum = 0.f;
#pragma unroll 1
          for (int cc = 0; cc < 2; ++cc) {
            const int c = 2 * hf + cc;
            const uint32_t al = live ? range_word(c, j0, jend) & kword[c] : 0u;
            uint32_t w[32];
            if (!__any_sync(0xffffffffu, al != 0u)) {
#pragma unroll
              for (int i = 0; i < 32; ++i) w[i] = 0u;  // P = 0: hi and lo pieces
            } else {
              float t[32];
              tmem_ld32(lb + T_SP + 32 * c, t);
              tmem_wait_ld();
              if (__all_sync(0xffffffffu, al == 0xffffffffu)) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  const float e0 = fast_exp2(fmaf(t[2 * i], sl, noff));
                  const float e1 = fast_exp2(fmaf(t[2 * i + 1], sl, noff));
                  lsum += e0 + e1;
                  f16_split2(e0, e1, w[i], w[16 + i]);
                }
              } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  const float e0 =
                      (al >> (2 * i)) & 1u ? fast_exp2(fmaf(t[2 * i], sl, noff)) : 0.f;
                  const float e1 =
                      (al >> (2 * i + 1)) & 1u ? fast_exp2(fmaf(t[2 * i + 1], sl, noff)) : 0.f;
                  lsum += e0 + e1;
                  f16_split2(e0, e1, w[i], w[16 + i]);
                }
              }
            }
            tmem_st32(lb + T_SP + 32 * c, w);
          }
          tmem_wait_st();
          xl[(h * 2 + hf) * TR + r] = lsum;
        }
        step_done(rows_sm);
      }
      // ---- the last head's context O / l -> A operand (half 1) -------------
      wait_mma(0x6600);
      if (hf == 1) ctx_to_a(H - 1);
      step_done(rows_misc);
      // ---- out_proj: x = valid ? x + ctx Wo^T + bo : 0, then LayerNorm 2 -----
      pf_vec(P(a.off.bo));
      pf_vec(P(a.off.ln2_w));
      pf_vec(P(a.off.ln2_b));
      wait_mma(0x6700);
      layer_norm_half(lb + T_X, r, hf, xch, P(a.off.ln2_w), P(a.off.ln2_b), a.eps,
                      x_plus(s_o, P(a.off.bo)), to_a);
      step_done(rows_misc);
      // ---- ffn_in + GELU -> A operand -----------------------------------------
      pf_vec(P(a.off.b1));
      wait_mma(0x6800);
      {
        const float *b1 = P(a.off.b1);
        float amax = 0.f;
#pragma unroll 1
        for (int cc = 0; cc < 2; ++cc) {
          const int c = 2 * hf + cc;
          float acc[32], bv[32];
          tmem_ld32(lb + T_ACC + 32 * c, acc);
          load32(b1 + 32 * c, bv);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[i] = gelu_erf(fmaf(acc[i], s_1, bv[i]));
          amax = fmaxf(amax, put_kblock_row(bp + OFF_A + c * KBLK, HALF, r, acc));
        }
        if (!(amax <= 65504.f) && in) raise_status(a.status, TT_ERR_DEVICE_RANGE, 0x6900);
      }
      step_done(rows_misc);
      // the ffn_out step's vectors, ahead of its wait
      pf_vec(P(a.off.b2));
      if (l + 1 < L) {
        const char *nbase = lbase + a.layer_stride;
        pf_vec(reinterpret_cast<const float *>(nbase + a.off.ln1_w));
        pf_vec(reinterpret_cast<const float *>(nbase + a.off.ln1_b));
        prefetch_l1(nbase + a.off.wscale);
      } else {
        pf_vec(a.final_w);
        pf_vec(a.final_b);
      }
      wait_mma(0x6A00);
      // ---- ffn_out: x = valid ? x + h W2^T + b2 : 0, with the next layer's
      // LayerNorm 1 -> A operand, or the final LayerNorm -> y (padded rows 0)
      if (l + 1 < L) {
        const char *nbase = lbase + a.layer_stride;
        layer_norm_half(lb + T_X, r, hf, xch, reinterpret_cast<const float *>(nbase + a.off.ln1_w),
                        reinterpret_cast<const float *>(nbase + a.off.ln1_b), a.eps,
                        x_plus(s_2, P(a.off.b2)), to_a);
      } else {
        layer_norm_half(lb + T_X, r, hf, xch, a.final_w, a.final_b, a.eps,
                        x_plus(s_2, P(a.off.b2)), [&](int c, float *v) {
                          if (!in) return;
                          float4 *dst = reinterpret_cast<float4 *>(a.y + g * D + 32 * c);
#pragma unroll
                          for (int i = 0; i < 8; ++i)
                            dst[i] = valid ? make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2],
                                                         v[4 * i + 3])
                                           : make_float4(0.f, 0.f, 0.f, 0.f);
                        });
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(TMEM_COLS)
                 : "memory");
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_fn(EncodeTiledFn *out) {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    TT_CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    if (ptr == nullptr || q != cudaDriverEntryPointSuccess)
      return fail(TT_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  *out = fn;
  return TT_OK;
}

// [layers, rows, 128] fp16 view of one packed weight piece of every layer
// (layer l at ptr + l * layer_stride bytes); box = 32 k x box_rows x 1,
// 64-byte swizzle.
int make_weight_map(CUtensorMap *tm, const void *ptr, int rows, int layers, size_t layer_stride,
                    int box_rows) {
  EncodeTiledFn encode;
  int rc = encode_fn(&encode);
  if (rc != TT_OK) return rc;
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)rows, (cuuint64_t)layers};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)layer_stride};
  cuuint32_t box[3] = {32, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = encode(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(ptr), dims,
                            strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TT_ERR_CUDA, "cuTensorMapEncodeTiled (tile forward weights) failed with CUresult " +
                                 std::to_string((int)r));
  return TT_OK;
}

}  // namespace

bool tile_forward_supported(const tt_config &cfg, int64_t batch, int64_t seq) {
  return cfg.d_model == D && cfg.ffn_dim == D && cfg.num_heads == H && batch > 0 && seq > 0 &&
         seq <= TR && TR % seq == 0 && (batch * seq + TR - 1) / TR <= INT32_MAX;
}

int launch_tile_forward(const TileArgs &a, cudaStream_t stream) {
  if (a.rows <= 0) return TT_OK;
  if (a.seq <= 0 || a.seq > TR || TR % a.seq != 0 || a.rows % a.seq != 0)
    return fail(TT_ERR_UNSUPPORTED, "tile forward: seq must divide 128");
  if (a.layer_stride % 16 != 0)
    return fail(TT_ERR_INVALID_ARGUMENT, "tile forward: layer stride must be a multiple of 16");
  CUtensorMap m[8];
  const LayerOffsets &o = a.off;
  const size_t offs[8] = {o.wqkv_hi, o.wqkv_lo, o.wo_hi, o.wo_lo, o.w1_hi, o.w1_lo, o.w2_hi, o.w2_lo};
  for (int i = 0; i < 8; ++i) {
    const bool qkv = i < 2;
    int rc = make_weight_map(&m[i], a.image + offs[i], qkv ? 3 * D : D, a.num_layers,
                             a.layer_stride, qkv ? HD : D);
    if (rc != TT_OK) return rc;
  }
  static bool attr_set = false;
  if (!attr_set) {
    TT_CUDA_TRY(cudaFuncSetAttribute(tile_forward_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES));
    attr_set = true;
  }
  const unsigned grid = (unsigned)((a.rows + TR - 1) / TR);
  TT_CUDA_TRY(launch_kernel(tile_forward_kernel, dim3(grid), dim3(kThreads), SMEM_BYTES, stream, 1,
                            m[0], m[1], m[2], m[3], m[4], m[5], m[6], m[7], a));
  TT_LAUNCH_CHECK("tile_forward");
  return TT_OK;
}

}  // namespace tt
