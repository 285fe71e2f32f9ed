// Causal / key-padded flash attention on tensor cores (tcgen05) for head_dim
// 8, 16, 32, 64, 128 and 256.
//
// Semantics as the reference attention (torch_transformer_benchmark.py:97-117):
// s = (q . k) * hd^-0.5, -inf for keys after the query (causal, :99-103) and
// for padded keys (:105-108), fp32 softmax (:111), ctx = p . v written in
// [B, S, H*hd] order. Queries without an allowed key (only padded queries)
// get a zero context; their rows are zeroed after out_proj as in :120-121.
//
// Precision: both products use a split x = x_hi + x_lo of each operand into
// two binary16 values (hi = x rounded to fp16, lo = the rest rounded to fp16:
// about 22 significant bits, as a TF32 pair) and three tensor-core products
// (hi.hi + hi.lo + lo.hi, tcgen05 kind::f16) accumulated in fp32. q, k, v
// arrive split by the q|k|v GEMM (which latches TT_ERR_DEVICE_RANGE for a
// value beyond the fp16 range); p = exp(s - m) is split by the softmax
// threads, scaled by 2^7 first so that its small values stay clear of the
// fp16 subnormals (the scale cancels in p.v / sum p; lazy rescaling keeps the
// scaled p below 2^15). The context accumulates in fp32 in tensor memory. A
// 16-bit MMA does twice the work of a TF32 one in the same cycles at N = 64
// and moves half the operand bytes.
//
// CTA = (query tile of 128 rows, head, sequence; and, at head_dim 256, half
// of the output dims). Up to head_dim 64 two CTAs share an SM (256
// tensor-memory columns each), so that one CTA's softmax runs while the
// other's MMAs use the tensor pipe; from head_dim 128 a CTA takes 512 columns
// and runs alone:
//   warp 0    TMA producer: per 64-key tile, K_hi K_lo (64 keys x HD dims) and
//             Vt_hi Vt_lo (HD dims x 64 keys, from the transposed copy of v the
//             q|k|v GEMM writes) into the ring;
//   warp 1    allocates / frees the tensor memory; then its lane 0 issues the
//             MMAs: S_j = Q.K^T (A = Q from tensor memory, B = K tile) into
//             S/P buffer j % NB (NB = 3 up to head_dim 32, else 2), NB tiles
//             ahead of the softmax, and O += P_j.V_j (A = P_j from the same
//             buffer, B = Vt tile) once the softmax has written P_j; both B
//             operands are K-major;
//   softmax   up to head_dim 64, warps 2-5 (192 threads per CTA): query row
//             q0+t (= tensor-memory lane t) belongs to one thread, which reads
//             the 64 scores of each tile, takes the row max on its own, and
//             writes P (split) over them; two CTAs per SM leave 128 registers
//             per thread. From head_dim 128, warps 2-9 (320 threads): two
//             threads per row, one per 32-key half, exchange the row max
//             through shared memory (one named barrier per tile). The P.V MMAs
//             accumulate the context in tensor memory, rescaled only when the
//             row max grows by more than 2^8.
// Every mbarrier wait is bounded; a wait that gives up latches
// TT_ERR_DEVICE_TIMEOUT, the producer and MMA roles stop and wait (bounded)
// for the loads and MMAs they started, and the kernel frees its tensor memory
// and returns. Every TMA load here fills only the issuing CTA's own shared
// memory.
#include <cuda.h>
#include <math_constants.h>

#include <algorithm>
#include <cstdlib>

#include "attention_tc.cuh"

namespace tt {
namespace {

constexpr int BQ = 128, BKV = 64;
constexpr int kThreads = 320;  // warp 0: TMA; warp 1: TMEM + MMA; warps 2-9: softmax
constexpr int kThreadsRow1 = 192;  // the same with softmax warps 2-5, one thread per row
constexpr int kSoftWarp0 = 2;  // first softmax warp

// Shapes for an MMA head dim HD (16, 32, 64, 128 or 256; head_dim 8 runs as
// 16). Shared-memory stage: K_hi, K_lo (64 keys x HD fp16 in boxes of up to
// 64 dims), then Vt_hi, Vt_lo (the CTA's output dims x 64 keys: 128-byte rows,
// 128-byte swizzle).
// Tensor-memory columns (32-bit cells; a 16-bit operand packs two values per
// cell): Q_hi, Q_lo (HD/2 each), two S/P buffers of 64 columns, O (HD). A
// buffer holds the fp32 scores S of a 64-key tile, then the fp16 split of P
// over the same columns: the softmax thread of key half kh writes P_hi of its
// 32 keys to cells [32 kh, 32 kh + 16) and P_lo to [32 kh + 16, 32 kh + 32),
// inside the scores it has read itself.
template <int HD>
struct AtShape {
  // A K operand is KSPLIT boxes of 64 keys x KBOX dims (one swizzle row of
  // 2*KBOX bytes: 32-byte swizzle at 16 dims, 64-byte at 32, 128-byte at 64);
  // head_dim 128 takes two 64-dim boxes. HD 16 also serves head_dim 8: the
  // Q dims 8..15 are zero in tensor memory, so the neighbouring head's k
  // values that the 16-dim box brings in add nothing, and V^T rows 8..15
  // (past the tensor, zero-filled) only feed O columns that are not stored.
  static constexpr int KBOX = HD < 64 ? HD : 64;
  static constexpr int KSPLIT = HD / KBOX;
  static constexpr uint32_t KROW = 2 * KBOX;            // bytes of one K row of a box
  static constexpr uint32_t KPART = 64 * KROW;          // one box
  static constexpr uint32_t OPK = KSPLIT * KPART;       // one K operand (hi or lo)
  // output dims per CTA: head_dim 256 splits O over two CTAs of 128 dims each
  // (both compute the full scores), so that Q, the S/P buffers and O fit 512
  // tensor-memory columns
  static constexpr int HDO = HD > 128 ? 128 : HD;
  static constexpr int NSPLIT = HD / HDO;
  static constexpr uint32_t OPV = HDO * 128;            // one V^T operand (hi or lo)
  static constexpr uint32_t STAGE = 2 * OPK + 2 * OPV;
  // S/P buffers in tensor memory: the scores of tile j + NB are issued after
  // P_j.V_j has read buffer j % NB, so NB tiles are in flight between the
  // MMAs and the softmax; three where the columns allow it (head_dim up to 32)
  static constexpr int NB = HD <= 32 ? 3 : 2;
  // ring stages: a stage holds tile j's K and V from their load until P_j.V_j
  // has read them, so one stage more than S/P buffers lets the next load start
  // a tile early
  static constexpr int NST = HD > 128 ? 2 : NB + 1;
  static constexpr size_t SMEM_BYTES = (size_t)NST * STAGE + 1024 + 256;
  static constexpr uint32_t T_QHI = 0, T_QLO = HD / 2, T_SP = HD, T_O = HD + 64 * NB;
  // two CTAs per SM up to head_dim 64 (256 columns each), one above
  static constexpr uint32_t TMEM_COLS = HD + 64 * NB + HDO <= 256 ? 256 : 512;
  static_assert(T_O + HDO <= TMEM_COLS, "tensor memory");
  static_assert(KPART % 1024 == 0 && OPV % 1024 == 0, "operands on the swizzle period");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
  // K operand descriptor fields: swizzle mode (6 = 32 B, 4 = 64 B, 2 = 128 B)
  // and the stride between 8-row groups
  static constexpr uint32_t K_SWZ = KBOX == 16 ? 6u : KBOX == 32 ? 4u : 2u;
  // O columns a softmax thread moves per tensor-memory access
  static constexpr int OC = HDO / 2 >= 16 ? 16 : 8;
  static constexpr uint32_t K_SBO = 8 * KROW;
  // instruction descriptors: kind::f16, D fp32, A/B fp16, both K-major, M = 128
  static constexpr uint32_t IDESC_S =
      (1u << 4) | ((uint32_t)(64 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
  static constexpr uint32_t IDESC_PV =
      (1u << 4) | ((uint32_t)(HDO >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
};

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
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
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
// abort word is set (another thread of this CTA gave up first). Other CTAs and
// launches do not look at the abort word. It is polled every 32nd poll only,
// so that a completed phase is seen without a round trip in the way.
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
// Bounded wait for work this thread started itself (TMA loads, MMAs) before
// the CTA frees its resources: ignores the abort word; latches the timeout and
// returns when it runs out.
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
// Shared-memory matrix descriptor, K-major, version 1: swizzle mode swz,
// 8-row groups sbo bytes apart.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t sbo, uint32_t swz) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)swz << 61;
  return d;
}
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accum)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
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
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t *v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t *v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
      : "memory");
}
__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t *v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr),
               "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3])
               : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float *v) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
// n = 16 or 8 fp32 cells of one lane's row
template <int N>
__device__ __forceinline__ void tmem_ld_n(uint32_t taddr, float *v) {
  if constexpr (N == 16) tmem_ld16(taddr, v);
  else tmem_ld8(taddr, v);
}
__device__ __forceinline__ void tmem_st8_f32(uint32_t taddr, const float *v) {  // fp32 cells
  uint32_t r[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) r[i] = __float_as_uint(v[i]);
  tmem_st8(taddr, r);
}
__device__ __forceinline__ void tmem_st16_f32(uint32_t taddr, const float *v) {  // fp32 cells
  uint32_t r[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(v[i]);
  tmem_st16(taddr, r);
}
// 2^x with the hardware's approximate base-2 exponential (ex2.approx.ftz);
// 2^-inf = 0.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// Two fp32 values -> their fp16 splits packed as (hi pair, lo pair), the
// element with the lower index in the low 16 bits.
__device__ __forceinline__ void split_pair(float a, float b, uint32_t &hi, uint32_t &lo) {
  f16_split2(a, b, hi, lo);
}
// The same split for two non-negative values below 65504 (the scaled
// probabilities P): hi = x rounded to fp16, lo = x - hi rounded to fp16, with
// hi widened back to fp32 by integer operations instead of conversions: the
// fp16 bit pattern shifted into the fp32 exponent field is 2^-112 times its
// value, for normal and subnormal fp16 alike, so one multiply by 2^112
// (without flush-to-zero) gives it exactly.
__device__ __forceinline__ float widen_f16_nonneg(uint32_t h16) {
  float r;
  asm("mul.rn.f32 %0, %1, 0f77800000;" : "=f"(r) : "f"(__uint_as_float(h16 << 13)));
  return r;
}
__device__ __forceinline__ void split_pair_nonneg(float a, float b, uint32_t &hi, uint32_t &lo) {
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(b), "f"(a));
  const float ha = widen_f16_nonneg(hi & 0xffffu), hb = widen_f16_nonneg(hi >> 16);
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(__fsub_rn(b, hb)), "f"(__fsub_rn(a, ha)));
}
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

// Named barrier of the two softmax warps that serve lane quarter q (ids 1-4,
// immediates: a register id would make the compiler reserve all 16 barriers,
// which leaves room for one CTA per SM).
__device__ __forceinline__ void pair_barrier(int q) {
  switch (q) {
    case 0: asm volatile("bar.sync 1, 64;" ::: "memory"); break;
    case 1: asm volatile("bar.sync 2, 64;" ::: "memory"); break;
    case 2: asm volatile("bar.sync 3, 64;" ::: "memory"); break;
    default: asm volatile("bar.sync 4, 64;" ::: "memory"); break;
  }
}

// ROW1 (head_dim up to 64): one softmax thread per query row, all 64 keys of
// a tile, 4 softmax warps and 192 threads per CTA -- no row-max exchange
// between threads, and two CTAs per SM leave 128 registers per thread.
// Otherwise two threads per row (one per 32-key half) exchange the row max
// through shared memory: 8 softmax warps, 320 threads.
template <int HD, bool GROUPED, bool ROW1>
__device__ __forceinline__ void attention_tc_body(const CUtensorMap &tm_hi,
                                                  const CUtensorMap &tm_lo,
                                                  const CUtensorMap &tm_vhi,
                                                  const CUtensorMap &tm_vlo,
                                                  const AttentionTcParams &p) {
  using Sh = AtShape<HD>;
  constexpr uint32_t STAGE = Sh::STAGE, OPK = Sh::OPK, OPV = Sh::OPV;
  constexpr int STAGES = Sh::NST, HDO = Sh::HDO, NB = Sh::NB;
  constexpr uint32_t T_QHI = Sh::T_QHI, T_QLO = Sh::T_QLO, T_O = Sh::T_O,
                     TMEM_COLS = Sh::TMEM_COLS;
  constexpr int NTHREADS = ROW1 ? kThreadsRow1 : kThreads;
  constexpr int NSOFT = ROW1 ? 4 : 8;  // softmax warps (one arrival each per barrier phase)
  static_assert(!ROW1 || HD <= 64, "one thread per row up to head_dim 64");
  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_kv_len, s_first_hole;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t bars = base + STAGES * STAGE;
  auto kv_full = [&](int s) { return bars + 8u * s; };
  auto kv_empty = [&](int s) { return bars + 8u * (STAGES + s); };
  // per S/P buffer b: S of its next tile written, P of that tile written, and
  // the P.V that read it finished
  auto s_full = [&](int b) { return bars + 8u * (2 * STAGES + b); };
  auto p_full = [&](int b) { return bars + 8u * (2 * STAGES + NB + b); };
  auto o_done = [&](int b) { return bars + 8u * (2 * STAGES + 2 * NB + b); };
  constexpr uint32_t XB = 2 * STAGES + 3 * NB;  // the barriers after those
  const uint32_t q_ready = bars + 8u * XB;
  const uint32_t o_final = bars + 8u * (XB + 1);  // every MMA finished
  const uint32_t tmem_slot = bars + 8u * (XB + 2);
  const uint32_t drain_bar = bars + 8u * (XB + 3);  // the MMA thread's last commit
  static_assert(8 * (XB + 4) <= 256, "barrier area");
  uint32_t *tmem_slot_ptr = reinterpret_cast<uint32_t *>(smem_raw + (tmem_slot - raw));
  volatile int *abort_w = reinterpret_cast<volatile int *>(smem_raw + (tmem_slot + 4 - raw));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.seq, D = p.d_model, hd = p.head_dim;  // hd < HD only for head_dim 8 (HD 16)
  // Grid: along x, query tiles latest (heaviest under the causal mask)
  // first, every (sequence, head) pair per tile, so that the longest CTAs
  // start first and the short ones fill the tail. GROUPED (very long
  // sequences, whose K/V far exceed the L2): blockIdx.y is a group of
  // bh_group pairs and x covers only the group's pairs; the groups run one
  // after another, so the CTAs running at one time share the K/V of a few
  // pairs through the L2. (Two instantiations: the group arithmetic costs
  // registers that the common case does not pay.)
  // head_dim 256: CTA pairs (consecutive) share a query tile and head, each
  // computing output dims [oh * HDO, oh * HDO + HDO)
  const int64_t group = GROUPED ? (int64_t)p.bh_group : p.batch * p.num_heads;
  const int64_t per_tile = group * Sh::NSPLIT;
  const int qt = (S + BQ - 1) / BQ - 1 - (int)(blockIdx.x / per_tile);
  const int64_t bh_idx = (GROUPED ? (int64_t)blockIdx.y * group : 0) +
                         (int64_t)((blockIdx.x % per_tile) / Sh::NSPLIT);
  const int oh = (int)(blockIdx.x % Sh::NSPLIT);
  const int h = (int)(bh_idx % p.num_heads);
  const int64_t b = bh_idx / p.num_heads;
  const int q0 = qt * BQ;
  const uint8_t *mrow = p.mask ? p.mask + b * S : nullptr;

  pdl_trigger();
  // kv_len = 1 + last valid key; keys at or after it are all padding.
  // first_hole = the first padded key; when it is at or past kv_len the valid
  // keys are a prefix and the tile loop takes them from kv_len alone,
  // without reading the mask again.
  if (threadIdx.x == 0) {
    s_kv_len = mrow ? 0 : S;
    s_first_hole = S;
  }
  __syncthreads();
  if (mrow) {
    int last = 0, hole = S;
    if ((reinterpret_cast<uintptr_t>(mrow) & 15) == 0 && S % 16 == 0) {
      for (int j = threadIdx.x; j < S / 16; j += NTHREADS) {
        const uint4 v = reinterpret_cast<const uint4 *>(mrow)[j];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (w[k]) last = 16 * j + 4 * k + (31 - __clz((int)w[k])) / 8 + 1;
          // lowest zero byte of w[k] (the lowest flagged byte of this test
          // is always a true zero)
          const uint32_t z = (w[k] - 0x01010101u) & ~w[k] & 0x80808080u;
          if (z) hole = min(hole, 16 * j + 4 * k + (__ffs((int)z) - 1) / 8);
        }
      }
    } else {
      for (int j = threadIdx.x; j < S; j += NTHREADS) {
        if (mrow[j]) last = j + 1;
        else hole = min(hole, j);
      }
    }
    if (last) atomicMax(&s_kv_len, last);
    if (hole < S) atomicMin(&s_first_hole, hole);
  }
  __syncthreads();
  const int kv_len = s_kv_len;
  // the mask the tile loop reads: none when the valid keys are a prefix
  const uint8_t *mtile = s_first_hole >= kv_len ? nullptr : mrow;
  if (q0 >= kv_len) return;  // every query of this tile is padding (uniform exit)
  const int kv_end = p.causal ? min(kv_len, q0 + BQ) : kv_len;
  const int nkv = (kv_end + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(kv_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    // the 8 softmax warps arrive once per warp (an elected lane after __syncwarp)
    for (int b = 0; b < NB; ++b) {
      mbar_init(s_full(b), 1);
      mbar_init(p_full(b), NSOFT);
      mbar_init(o_done(b), 1);
    }
    mbar_init(q_ready, NSOFT);
    mbar_init(o_final, 1);
    mbar_init(drain_bar, 1);
    *abort_w = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tmem_slot),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tm = *tmem_slot_ptr;
  pdl_wait();  // q|k and v^T come from the previous kernel (the mask is the caller's input)

  // A wait that gives up in the producer or the MMA thread stops that role (no
  // further loads, MMAs or commits, so no barrier phase is armed twice); the
  // producer then waits for the loads it started and the MMA thread for its
  // MMAs, bounded, before the CTA frees its tensor memory. The softmax threads
  // run on through their (then failing) waits with unchanged control flow, so
  // the pair barriers of their two warps always match.
  if (warp == 0 && lane == 0) {
    // ---- TMA producer: K/V tiles -------------------------------------------
    const int kcol = D + h * hd;  // first k column (fp16 elements) of this head
    const int bh = (int)b * p.num_heads + h;
    int j = 0;
    for (; j < nkv; ++j) {
      const int s = j % STAGES, n = j / STAGES;
      if (j >= STAGES && !mbar_wait(kv_empty(s), (n - 1) & 1, abort_w, p.status, 0x4100 + j))
        break;
      const uint32_t st = base + s * STAGE;
      mbar_expect_tx(kv_full(s), STAGE);
#pragma unroll
      for (int part = 0; part < Sh::KSPLIT; ++part) {
        tma_load_3d(st + part * Sh::KPART, &tm_hi, kcol + part * Sh::KBOX, j * BKV, (int)b,
                    kv_full(s));
        tma_load_3d(st + OPK + part * Sh::KPART, &tm_lo, kcol + part * Sh::KBOX, j * BKV, (int)b,
                    kv_full(s));
      }
      tma_load_3d(st + 2 * OPK, &tm_vhi, j * BKV, oh * HDO, bh, kv_full(s));
      tma_load_3d(st + 2 * OPK + OPV, &tm_vlo, j * BKV, oh * HDO, bh, kv_full(s));
    }
    // the last phase armed on each stage has landed before the CTA retires
    for (int k = j > STAGES ? j - STAGES : 0; k < j; ++k)
      mbar_drain(kv_full(k % STAGES), (k / STAGES) & 1, p.status, 0x4F00);
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer --------------------------------------------------------
    // S_j goes to buffer j % NB. The tensor pipe runs one thread's MMAs in
    // issue order, so S_{j+NB}, issued after P_j.V_j, overwrites P_j only after
    // that product has read it.
    auto issue_s = [&](int j) -> bool {
      const int s = j % STAGES;
      if (!mbar_wait(kv_full(s), (j / STAGES) & 1, abort_w, p.status, 0x4200 + j)) return false;
      const uint32_t kst = base + s * STAGE;
      const uint32_t sd = tm + Sh::T_SP + 64u * (uint32_t)(j % NB);
      // descriptors built once per box; a k-step of 16 dims advances the start
      // address by 32 bytes (2 units) inside its box
      constexpr int KK_BOX = Sh::KBOX / 16;  // k-steps per box
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        const uint32_t kpart = kst + (uint32_t)(kk / KK_BOX) * Sh::KPART;
        const uint64_t khi0 = sdesc(kpart, Sh::K_SBO, Sh::K_SWZ);
        const uint64_t klo0 = sdesc(kpart + OPK, Sh::K_SBO, Sh::K_SWZ);
        const uint64_t koff = (uint64_t)(2 * (kk % KK_BOX));
        mma_ts(sd, tm + T_QHI + 8u * kk, khi0 + koff, Sh::IDESC_S, kk > 0);
        mma_ts(sd, tm + T_QHI + 8u * kk, klo0 + koff, Sh::IDESC_S, 1);
        mma_ts(sd, tm + T_QLO + 8u * kk, khi0 + koff, Sh::IDESC_S, 1);
      }
      mma_commit(s_full(j % NB));
      return true;
    };
    bool ok = mbar_wait(q_ready, 0, abort_w, p.status, 0x4000);
    fence_after();
    for (int j = 0; j < NB && j < nkv; ++j) ok = ok && issue_s(j);
    for (int j = 0; ok && j < nkv; ++j) {
      const int s = j % STAGES, b = j % NB;
      if (!mbar_wait(p_full(b), (j / NB) & 1, abort_w, p.status, 0x4400 + j)) {
        ok = false;
        break;
      }
      fence_after();
      const uint32_t vst = base + s * STAGE + 2 * OPK;
      const uint64_t vhi0 = sdesc(vst, 1024, 2), vlo0 = sdesc(vst + OPV, 1024, 2);
      const uint32_t pb = tm + Sh::T_SP + 64u * b;
#pragma unroll
      for (int kk = 0; kk < BKV / 16; ++kk) {  // 16 keys per MMA
        const uint64_t voff = (uint64_t)(2 * kk);
        // keys 16 kk .. 16 kk + 15: P_hi at cells 32 (kk / 2) + 8 (kk % 2), P_lo 16 further
        const uint32_t phi = pb + 32u * (kk >> 1) + 8u * (kk & 1);
        mma_ts(tm + T_O, phi, vhi0 + voff, Sh::IDESC_PV, (j | kk) != 0);
        mma_ts(tm + T_O, phi, vlo0 + voff, Sh::IDESC_PV, 1);
        mma_ts(tm + T_O, phi + 16u, vhi0 + voff, Sh::IDESC_PV, 1);
      }
      mma_commit(o_done(b));
      mma_commit(kv_empty(s));
      if (j + NB < nkv) ok = issue_s(j + NB);  // into the buffer P_j.V_j has just read
    }
    if (ok) mma_commit(o_final);
    // every MMA issued above has completed before the tensor memory is freed
    mma_commit(drain_bar);
    mbar_drain(drain_bar, 0, p.status, 0x4F10);
  } else if (warp >= kSoftWarp0) {
   if constexpr (ROW1) {
    // ---- softmax, one thread per query row (warps 2-5) ----------------------
    const int t = (warp & 3) * 32 + lane;   // row within the tile = tensor-memory lane
    const int row = q0 + t;
    const bool row_in = row < S;
    const uint32_t lane_base = tm + ((uint32_t)((warp & 3) * 32) << 16);
    {
      // Q row -> tensor memory: HD dims as HD/2 packed cells of Q_hi and of
      // Q_lo; dims at or past hd (the padding of head_dim 8) are zero. Every
      // global load of the row is issued before the first tensor-memory store
      // (the stores are ordered against memory), so the row costs one memory
      // round trip rather than one per 16-byte chunk.
      const int64_t qoff = (b * S + (row_in ? row : 0)) * (int64_t)(2 * D) + (int64_t)h * hd;
      constexpr int QC = HD / 2 < 16 ? HD / 2 : 16;  // cells per store
      constexpr int NQ = HD / 8;                     // 16-byte chunks of hi (and of lo)
      uint4 qraw[2][NQ];
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint4 *src = reinterpret_cast<const uint4 *>((which ? p.qk_lo : p.qk_hi) + qoff);
#pragma unroll
        for (int u = 0; u < NQ; ++u)
          qraw[which][u] = (row_in && 8 * u < hd) ? src[u] : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint32_t tcol = lane_base + (which ? T_QLO : T_QHI);
#pragma unroll
        for (int c = 0; c < HD / 2; c += QC) {
          uint32_t qv[QC];
#pragma unroll
          for (int i = 0; i < QC / 4; ++i) {
            const uint4 v = qraw[which][c / 4 + i];  // dims 2c + 8i .. + 7
            qv[4 * i] = v.x; qv[4 * i + 1] = v.y; qv[4 * i + 2] = v.z; qv[4 * i + 3] = v.w;
          }
          if constexpr (QC == 16) tmem_st16(tcol + c, qv);
          else if constexpr (QC == 8) tmem_st8(tcol + c, qv);
          else tmem_st4(tcol + c, qv);
        }
      }
      tmem_wait_st();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
    }
    // log2-domain scores, lazy reference max and the 2^7 scale of P as in the
    // two-threads-per-row form below, with the whole row in this thread
    const float sl = p.scale * 1.4426950408889634f;
    constexpr float kLazy = 8.0f;
    constexpr float kPScale = 7.0f;
    float m_ref = -CUDART_INF_F, l = 0.f;
    for (int j = 0; j < nkv; ++j) {
      const int sb = j % NB;
      const int k0 = j * BKV;
      // allowed keys k0 .. k0 + 31 (ok0) and k0 + 32 .. k0 + 63 (ok1)
      uint32_t ok0, ok1;
      if (mtile == nullptr) {
        const int n = kv_end - k0, n1 = n - 32;
        ok0 = n >= 32 ? 0xffffffffu : (n <= 0 ? 0u : (1u << n) - 1u);
        ok1 = n1 >= 32 ? 0xffffffffu : (n1 <= 0 ? 0u : (1u << n1) - 1u);
      } else {
        const int ka = k0 + lane, kb2 = k0 + 32 + lane;
        ok0 = __ballot_sync(0xffffffffu, ka < kv_end && mtile[ka] != 0);
        ok1 = __ballot_sync(0xffffffffu, kb2 < kv_end && mtile[kb2] != 0);
      }
      const bool diag = p.causal && k0 + 63 > q0;  // tile reaches past the first query
      const bool open = !diag && (ok0 & ok1) == 0xffffffffu;  // warp-uniform
      const uint32_t sp = lane_base + Sh::T_SP + 64u * sb;
      mbar_wait(s_full(sb), (j / NB) & 1, abort_w, p.status, 0x4500 + j);
      fence_after();
      float sv[64];
      tmem_ld32(sp, sv);
      tmem_ld32(sp + 32, sv + 32);
      tmem_wait_ld();
      if (!open) {
        uint32_t a0 = ok0, a1 = ok1;
        if (diag) {
          const int lim = row - k0, lim1 = lim - 32;  // keys k0 + c <= row
          a0 &= lim >= 31 ? 0xffffffffu : (lim < 0 ? 0u : (2u << lim) - 1u);
          a1 &= lim1 >= 31 ? 0xffffffffu : (lim1 < 0 ? 0u : (2u << lim1) - 1u);
        }
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          sv[c] = (a0 >> c) & 1u ? sv[c] : -CUDART_INF_F;
          sv[32 + c] = (a1 >> c) & 1u ? sv[32 + c] : -CUDART_INF_F;
        }
      }
      // row max of the raw scores, eight chains of three-input maxima
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        mx8[i] = fmax3(sv[i], sv[i + 8], sv[i + 16]);
        mx8[i] = fmax3(mx8[i], sv[i + 24], sv[i + 32]);
        mx8[i] = fmax3(mx8[i], sv[i + 40], sv[i + 48]);
        mx8[i] = fmaxf(mx8[i], sv[i + 56]);
      }
      const float mx = fmaxf(fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]),
                                   mx8[6]),
                             mx8[7]) * sl;
      const bool raise = mx > m_ref + kLazy || (m_ref == -CUDART_INF_F && mx != -CUDART_INF_F);
      const float alpha = raise ? fast_exp2(m_ref - mx) : 1.f;  // 0 when m_ref is -inf
      // context rows of the warp rescaled together (warp-collective tensor-
      // memory access; alpha = 1 for the rows that need none), after
      // P_{j-1}.V_{j-1} has landed in them (the parity wait is exact as below)
      if (__any_sync(0xffffffffu, raise && m_ref != -CUDART_INF_F) && j > 0) {
        mbar_wait(o_done((j - 1) % NB), ((j - 1) / NB) & 1, abort_w, p.status, 0x4600 + j);
        fence_after();
        constexpr int OC = HDO >= 16 ? 16 : 8;
#pragma unroll
        for (int c = 0; c < HDO; c += OC) {
          float ov[OC];
          tmem_ld_n<OC>(lane_base + T_O + c, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < OC; ++i) ov[i] *= alpha;
          if constexpr (OC == 16) tmem_st16_f32(lane_base + T_O + c, ov);
          else tmem_st8_f32(lane_base + T_O + c, ov);
        }
      }
      if (raise) {
        l *= alpha;
        m_ref = mx;
      }
      // 2^7 p = 2^(s * sl - (m_ref - 7)), 0 for masked keys; each pair of
      // probabilities is split as soon as it exists, and P_j goes over S_j,
      // each 32-key half as 16 cells of P_hi then 16 of P_lo
      const bool live = m_ref != -CUDART_INF_F;
      const float noff = kPScale - m_ref;
      float ps4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t w[32];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const float e0 = live ? fast_exp2(fmaf(sv[32 * half + 2 * c], sl, noff)) : 0.f;
          const float e1 = live ? fast_exp2(fmaf(sv[32 * half + 2 * c + 1], sl, noff)) : 0.f;
          ps4[(2 * c) & 3] += e0;
          ps4[(2 * c + 1) & 3] += e1;
          split_pair_nonneg(e0, e1, w[c], w[16 + c]);
        }
        tmem_st32(sp + 32u * half, w);
      }
      l += (ps4[0] + ps4[1]) + (ps4[2] + ps4[3]);
      tmem_wait_st();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full(sb));
    }
    // context = O / l, written as an fp16 split (the out_proj GEMM's A operand)
    mbar_wait(o_final, 0, abort_w, p.status, 0x4700);
    fence_after();
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int64_t off = (b * S + (row_in ? row : 0)) * (int64_t)D + (int64_t)h * hd;
    // 8-dim chunks at HD 16, so that head_dim 8 (run as 16) stores only its own
    constexpr int OC = HDO >= 32 ? 16 : 8;
#pragma unroll
    for (int c = 0; c < HDO; c += OC) {
      float ov[OC];
      tmem_ld_n<OC>(lane_base + T_O + c, ov);
      tmem_wait_ld();
      if (row_in && c < hd) {  // the padding dims of head_dim 8 are not stored
        uint32_t hw[OC / 2], lw[OC / 2];
#pragma unroll
        for (int i = 0; i < OC / 2; ++i)
          split_pair(ov[2 * i] * inv, ov[2 * i + 1] * inv, hw[i], lw[i]);
        uint4 *dh = reinterpret_cast<uint4 *>(p.ctx_hi + off + c);
        uint4 *dl = reinterpret_cast<uint4 *>(p.ctx_lo + off + c);
#pragma unroll
        for (int u = 0; u < OC / 8; ++u) {
          dh[u] = make_uint4(hw[4 * u], hw[4 * u + 1], hw[4 * u + 2], hw[4 * u + 3]);
          dl[u] = make_uint4(lw[4 * u], lw[4 * u + 1], lw[4 * u + 2], lw[4 * u + 3]);
        }
      }
    }
   } else {
    // ---- softmax: rows split over two warpgroups by key half ----------------
    __shared__ float s_rowmax[2][2][128];  // [tile parity][key half][row]
    __shared__ float s_rowsum[2][128];
    const int t = (warp & 3) * 32 + lane;   // row within the tile = tensor-memory lane
    const int kh = (warp - kSoftWarp0) >> 2;  // which 32 keys (and HD/2 dims) of a tile
    const int row = q0 + t;
    const bool row_in = row < S;
    const uint32_t lane_base = tm + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t col_off = 32u * kh;                 // this thread's 32 scores of a tile
    const uint32_t dim_off = (uint32_t)(HDO / 2) * kh;  // ... and HDO/2 dims of O
    {
      // Q row -> tensor memory: this thread's dims [HD/2 kh, HD/2 kh + HD/2)
      // as HD/4 packed cells of Q_hi and of Q_lo (dims at or past hd, the
      // padding of head_dim 8, are zero), in chunks of at most 16 cells
      const bool q_in = row_in && (HD / 2) * kh < hd;
      const int64_t qoff = (b * S + (row_in ? row : 0)) * (int64_t)(2 * D) + (int64_t)h * hd +
                           (q_in ? (HD / 2) * kh : 0);
      const uint32_t qcol = (uint32_t)(HD / 4) * kh;
      constexpr int QC = HD / 4 < 16 ? HD / 4 : 16;
      // every global load of the half row before the first tensor-memory
      // store (the stores are ordered against memory): one round trip
      constexpr int NQ = HD / 16;  // 16-byte chunks of hi (and of lo)
      uint4 qraw[2][NQ];
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint4 *src = reinterpret_cast<const uint4 *>((which ? p.qk_lo : p.qk_hi) + qoff);
#pragma unroll
        for (int u = 0; u < NQ; ++u) qraw[which][u] = q_in ? src[u] : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint32_t tcol = lane_base + (which ? T_QLO : T_QHI) + qcol;
#pragma unroll
        for (int c = 0; c < HD / 4; c += QC) {
          uint32_t qv[QC];
#pragma unroll
          for (int i = 0; i < QC / 4; ++i) {
            const uint4 v = qraw[which][c / 4 + i];
            qv[4 * i] = v.x; qv[4 * i + 1] = v.y; qv[4 * i + 2] = v.z; qv[4 * i + 3] = v.w;
          }
          if constexpr (QC == 16) tmem_st16(tcol + c, qv);
          else if constexpr (QC == 8) tmem_st8(tcol + c, qv);
          else tmem_st4(tcol + c, qv);
        }
      }
      tmem_wait_st();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
    }
    // Scores live in the log2 domain: t = s * scale * log2(e). P is taken
    // relative to a reference max m_ref that is raised lazily: only when a
    // row's max exceeds it by more than 2^8 are the row's running context (in
    // tensor memory, accumulated by the P.V MMAs) and sum rescaled, so P <= 256
    // (2^15 after the 2^7 scale) and the usual case needs no tensor-memory
    // round trip. Both threads of a row see the same maxima, so they take the
    // same decisions.
    const float sl = p.scale * 1.4426950408889634f;
    constexpr float kLazy = 8.0f;
    constexpr float kPScale = 7.0f;  // log2 of the scale applied to P
    float m_ref = -CUDART_INF_F, l = 0.f;
    for (int j = 0; j < nkv; ++j) {
      const int sb = j % NB;
      const int k0 = j * BKV + 32 * kh;     // first key of this thread's half
      uint32_t ok;
      if (mtile == nullptr) {
        // keys k0 .. kv_end - 1 of this half
        const int n = kv_end - k0;
        ok = n >= 32 ? 0xffffffffu : (n <= 0 ? 0u : (1u << n) - 1u);
      } else {
        const int ka = k0 + lane;
        ok = __ballot_sync(0xffffffffu, ka < kv_end && mtile[ka] != 0);
      }
      const bool diag = p.causal && k0 + 31 > q0;  // half reaches past the first query
      // every key of this half allowed for every row of the warp (warp-uniform)
      const bool open = !diag && ok == 0xffffffffu;
      const uint32_t sp = lane_base + Sh::T_SP + 64u * sb + col_off;  // this thread's cells
      mbar_wait(s_full(sb), (j / NB) & 1, abort_w, p.status, 0x4500 + j);
      fence_after();
      float sv[32];
      tmem_ld16(sp, sv);
      tmem_ld16(sp + 16, sv + 16);
      tmem_wait_ld();
      if (!open) {
        // allowed keys of this half as one word: valid (ballot) and, on the
        // diagonal, key k0 + c <= row, i.e. bits 0 .. row - k0 (one select
        // per score; a per-score && / || compiles to branches)
        uint32_t allowed = ok;
        if (diag) {
          const int lim = row - k0;
          allowed &= lim >= 31 ? 0xffffffffu : (lim < 0 ? 0u : (2u << lim) - 1u);
        }
#pragma unroll
        for (int c = 0; c < 32; ++c) sv[c] = (allowed >> c) & 1u ? sv[c] : -CUDART_INF_F;
      }
      // row max of the raw scores (the log2-domain scale sl > 0 keeps the
      // order), four chains of three-input maxima
      float mx4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        mx4[i] = fmax3(sv[i], sv[i + 4], sv[i + 8]);
        mx4[i] = fmax3(mx4[i], sv[i + 12], sv[i + 16]);
        mx4[i] = fmax3(mx4[i], sv[i + 20], sv[i + 24]);
        mx4[i] = fmaxf(mx4[i], sv[i + 28]);
      }
      float mx = fmaxf(fmax3(mx4[0], mx4[1], mx4[2]), mx4[3]) * sl;
      s_rowmax[j & 1][kh][t] = mx;
      // the two warps that share these 32 rows (one per key half)
      pair_barrier(warp & 3);
      mx = fmaxf(mx, s_rowmax[j & 1][kh ^ 1][t]);
      const bool raise = mx > m_ref + kLazy || (m_ref == -CUDART_INF_F && mx != -CUDART_INF_F);
      const float alpha = raise ? fast_exp2(m_ref - mx) : 1.f;  // 0 when m_ref is -inf
      // The context rows of the warp are rescaled together when any of them
      // needs it (alpha = 1 for the others): the tensor-memory loads and
      // stores are warp-collective (.sync.aligned), so they run under a
      // warp-uniform condition. A row whose m_ref is -inf has a zero context
      // row, which alpha = 0 keeps.
      if (__any_sync(0xffffffffu, raise && m_ref != -CUDART_INF_F) && j > 0) {
        // the context in tensor memory must hold P_{j-1}.V_{j-1} before it
        // is rescaled. That product completes phase (j-1)/NB of buffer
        // (j-1) % NB's o_done; the phase before belongs to P_{j-1-NB}.V_{j-1-NB},
        // which completed before S_{j-1} (issued after it, and waited for
        // above), and no later phase can start before P_{j-1+NB} exists, so
        // the parity wait is exact.
        mbar_wait(o_done((j - 1) % NB), ((j - 1) / NB) & 1, abort_w, p.status, 0x4600 + j);
        fence_after();
        // this thread's HDO / 2 context columns (HDO = HD up to head_dim 128)
#pragma unroll
        for (int c = 0; c < HDO / 2; c += Sh::OC) {
          float ov[Sh::OC];
          tmem_ld_n<Sh::OC>(lane_base + T_O + dim_off + c, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < Sh::OC; ++i) ov[i] *= alpha;
          if constexpr (Sh::OC == 16) tmem_st16_f32(lane_base + T_O + dim_off + c, ov);
          else tmem_st8_f32(lane_base + T_O + dim_off + c, ov);
        }
      }
      if (raise) {
        l *= alpha;
        m_ref = mx;
      }
      float ps4[4] = {0.f, 0.f, 0.f, 0.f};
      if (m_ref != -CUDART_INF_F) {
        // 2^7 p = 2^(s * sl - (m_ref - 7)): one fused multiply-add and one
        // exponential per score; 0 for masked keys (s = -inf)
        const float noff = kPScale - m_ref;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          sv[c] = fast_exp2(fmaf(sv[c], sl, noff));
          ps4[c & 3] += sv[c];
        }
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) sv[c] = 0.f;
      }
      l += (ps4[0] + ps4[1]) + (ps4[2] + ps4[3]);
      uint32_t phi[16], plo[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) split_pair(sv[2 * c], sv[2 * c + 1], phi[c], plo[c]);
      // P_j over the scores S_j this thread has read
      tmem_st16(sp, phi);
      tmem_st16(sp + 16, plo);
      tmem_wait_st();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full(sb));
    }
    // row sum = both halves' partial sums
    s_rowsum[kh][t] = l;
    pair_barrier(warp & 3);
    l += s_rowsum[kh ^ 1][t];
    // context = O / l (this thread's HD/2 dims), written as an fp16 split (the
    // out_proj GEMM's A operand)
    // every P.V finished (o_done can be two phases behind here, so the
    // final commit has a barrier of its own)
    mbar_wait(o_final, 0, abort_w, p.status, 0x4700);
    fence_after();
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int64_t off = (b * S + (row_in ? row : 0)) * (int64_t)D + (int64_t)h * hd +
                        oh * HDO + dim_off;
    constexpr int OC = Sh::OC;
#pragma unroll
    for (int c = 0; c < HDO / 2; c += OC) {
      float ov[OC];
      tmem_ld_n<OC>(lane_base + T_O + dim_off + c, ov);
      tmem_wait_ld();
      // the padding dims of head_dim 8 are not stored
      if (row_in && oh * HDO + (int)dim_off + c < hd) {
        uint32_t hw[OC / 2], lw[OC / 2];
#pragma unroll
        for (int i = 0; i < OC / 2; ++i)
          split_pair(ov[2 * i] * inv, ov[2 * i + 1] * inv, hw[i], lw[i]);
        uint4 *dh = reinterpret_cast<uint4 *>(p.ctx_hi + off + c);
        uint4 *dl = reinterpret_cast<uint4 *>(p.ctx_lo + off + c);
#pragma unroll
        for (int u = 0; u < OC / 8; ++u) {
          dh[u] = make_uint4(hw[4 * u], hw[4 * u + 1], hw[4 * u + 2], hw[4 * u + 3]);
          dl[u] = make_uint4(lw[4 * u], lw[4 * u + 1], lw[4 * u + 2], lw[4 * u + 3]);
        }
      }
    }
   }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(TMEM_COLS)
                 : "memory");
  }
}

// ---- persistent form (head_dim up to 64) ------------------------------------
// One CTA per scheduling slot (two per SM), each running work items (query
// tile, head, sequence) one after another, taken heaviest first from a
// counter with atomicAdd; the tensor memory, the barriers and the K/V ring
// stay with the CTA across items. Roles as in the form above, with one
// softmax thread per row, plus:
//   warp 0    (all lanes) takes the next item, scans its sequence's mask for
//             the valid length, publishes the item's record in one of two
//             shared slots, then (lane 0) streams the item's K/V tiles into
//             the ring -- which it keeps doing while the other roles finish
//             the previous item, so the next item's first tiles are loaded
//             by the time its scores are issued;
//   softmax   after an item's last tile (every score of the item read, so
//             the Q columns are free), loads the next item's Q row and writes
//             it to tensor memory, then waits for the item's last P.V and
//             stores the context -- the MMA thread issues the next item's
//             first scores meanwhile.
// Ring stages and S/P buffers are indexed by a tile count that runs on across
// items; q_ready and o_final complete one phase per item that has work. The
// next item's first P.V overwrites the context only after the softmax has
// read it: that product waits for P of the item's first tile, which the
// softmax writes after the context store (program order). Work items are
// ordered as the grid of the form above: group of bh_group (sequence, head)
// pairs, then query tile latest first, then pair. The counter must be zero
// when the kernel starts (the q|k|v GEMM before it zeroes it); CTA c takes
// item c first, then gridDim.x + the counter's old value.
// Measured against the one-CTA-per-item form on B200 (forward attention,
// CUDA events): E (head_dim 64, 16384 items) 2007 -> 1761 us, D 94.7 -> 85.7,
// C (head_dim 32) 28.1 -> 26.2, official case 13 131.9 -> 114.5. The gain is
// the per-CTA start-up (barrier set-up, tensor-memory allocation, the mask
// scan and the first K/V loads) that the next item's hand-off hides.
template <int HD>
__device__ __forceinline__ void attention_tc_persist_body(const CUtensorMap &tm_hi,
                                                          const CUtensorMap &tm_lo,
                                                          const CUtensorMap &tm_vhi,
                                                          const CUtensorMap &tm_vlo,
                                                          const AttentionTcParams &p) {
  using Sh = AtShape<HD>;
  static_assert(HD <= 64, "persistent form up to head_dim 64");
  constexpr uint32_t STAGE = Sh::STAGE, OPK = Sh::OPK, OPV = Sh::OPV;
  constexpr int STAGES = Sh::NST, HDO = Sh::HDO, NB = Sh::NB;
  constexpr uint32_t T_QHI = Sh::T_QHI, T_QLO = Sh::T_QLO, T_O = Sh::T_O,
                     TMEM_COLS = Sh::TMEM_COLS;
  constexpr int NSOFT = 4;
  extern __shared__ uint8_t smem_raw[];
  // item records: valid (1 work, 0 all queries padded, -1 no more items),
  // sequence, head, first query, kv_len, kv_end, key tiles, mask has holes
  __shared__ int s_rec[2][8];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t bars = base + STAGES * STAGE;
  auto kv_full = [&](int s) { return bars + 8u * s; };
  auto kv_empty = [&](int s) { return bars + 8u * (STAGES + s); };
  auto s_full = [&](int b) { return bars + 8u * (2 * STAGES + b); };
  auto p_full = [&](int b) { return bars + 8u * (2 * STAGES + NB + b); };
  auto o_done = [&](int b) { return bars + 8u * (2 * STAGES + 2 * NB + b); };
  constexpr uint32_t XB = 2 * STAGES + 3 * NB;
  const uint32_t q_ready = bars + 8u * XB;
  const uint32_t o_final = bars + 8u * (XB + 1);
  auto info_ready = [&](int k) { return bars + 8u * (XB + 2 + k); };  // record k % 2 written
  auto info_free = [&](int k) { return bars + 8u * (XB + 4 + k); };   // record k % 2 read
  const uint32_t tmem_slot = bars + 8u * (XB + 6);
  const uint32_t drain_bar = bars + 8u * (XB + 7);
  static_assert(8 * (XB + 8) <= 256, "barrier area");
  uint32_t *tmem_slot_ptr = reinterpret_cast<uint32_t *>(smem_raw + (tmem_slot - raw));
  volatile int *abort_w = reinterpret_cast<volatile int *>(smem_raw + (tmem_slot + 4 - raw));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.seq, D = p.d_model, hd = p.head_dim;
  const int ntq = (S + BQ - 1) / BQ;
  const int64_t bh_all = p.batch * p.num_heads;
  const int64_t gsz = p.bh_group;  // pairs per group
  const int64_t n_items = (int64_t)ntq * bh_all;

  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(kv_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(s_full(b), 1);
      mbar_init(p_full(b), NSOFT);
      mbar_init(o_done(b), 1);
    }
    mbar_init(q_ready, NSOFT);
    mbar_init(o_final, 1);
    for (int k = 0; k < 2; ++k) {
      mbar_init(info_ready(k), 1);
      mbar_init(info_free(k), 1 + NSOFT);  // the MMA thread and the softmax warps
    }
    mbar_init(drain_bar, 1);
    *abort_w = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tmem_slot),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tm = *tmem_slot_ptr;
  // q|k, v^T and the zeroed item counter come from the previous kernel: each
  // role waits for it (griddepcontrol.wait) before its first read of them.
  // The first item's record needs only the mask, the caller's input, so the
  // producer publishes it before its wait.

  if (warp == 0) {
    // ---- items, mask scans and K/V tiles ------------------------------------
    int it = 0;  // K/V tiles loaded (ring index), over all items
    bool ok = true;
    for (int n = 0; ok; ++n) {
      int item = 0;
      if (lane == 0) item = n == 0 ? (int)blockIdx.x : atomicAdd(p.counter, 1) + (int)gridDim.x;
      item = __shfl_sync(0xffffffffu, item, 0);
      const int slot = n & 1;
      // record n - 2 (the same slot) has been read by every role
      if (n >= 2 && !__all_sync(0xffffffffu, mbar_wait(info_free(slot), ((n - 2) >> 1) & 1,
                                                       abort_w, p.status, 0x4800))) {
        ok = false;
        break;
      }
      int valid = -1, bb = 0, hh = 0, q0 = 0, kv_len = 0, kv_end = 0, nkv = 0, holes = 0;
      if (item < n_items) {
        const int64_t per_group = (int64_t)ntq * gsz;
        const int64_t grp = item / per_group, r = item % per_group;
        const int qt = ntq - 1 - (int)(r / gsz);
        const int64_t bh = grp * gsz + r % gsz;
        bb = (int)(bh / p.num_heads);
        hh = (int)(bh % p.num_heads);
        q0 = qt * BQ;
        int last = S, hole = S;
        if (p.mask != nullptr) {
          const uint8_t *mrow = p.mask + (int64_t)bb * S;
          last = 0;
          if ((reinterpret_cast<uintptr_t>(mrow) & 15) == 0 && S % 16 == 0) {
            for (int j = lane; j < S / 16; j += 32) {
              const uint4 v = reinterpret_cast<const uint4 *>(mrow)[j];
              const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                if (w[k]) last = 16 * j + 4 * k + (31 - __clz((int)w[k])) / 8 + 1;
                const uint32_t z = (w[k] - 0x01010101u) & ~w[k] & 0x80808080u;
                if (z) hole = min(hole, 16 * j + 4 * k + (__ffs((int)z) - 1) / 8);
              }
            }
          } else {
            for (int j = lane; j < S; j += 32) {
              if (mrow[j]) last = j + 1;
              else hole = min(hole, j);
            }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
            hole = min(hole, __shfl_xor_sync(0xffffffffu, hole, o));
          }
        }
        kv_len = last;
        holes = hole < kv_len ? 1 : 0;
        valid = q0 < kv_len ? 1 : 0;  // 0: every query of the tile is padding
        kv_end = p.causal ? min(kv_len, q0 + BQ) : kv_len;
        nkv = valid ? (kv_end + BKV - 1) / BKV : 0;
      }
      if (lane == 0) {
        int *rec = s_rec[slot];
        rec[0] = valid; rec[1] = bb; rec[2] = hh; rec[3] = q0;
        rec[4] = kv_len; rec[5] = kv_end; rec[6] = nkv; rec[7] = holes;
        mbar_arrive(info_ready(slot));  // release: the record is visible to its waiters
      }
      if (n == 0) pdl_wait();
      if (valid < 0) break;
      if (lane == 0) {
        const int kcol = D + hh * hd;
        const int bh = bb * p.num_heads + hh;
        for (int j = 0; j < nkv; ++j, ++it) {
          const int s = it % STAGES, ph = it / STAGES;
          if (it >= STAGES &&
              !mbar_wait(kv_empty(s), (ph - 1) & 1, abort_w, p.status, 0x4100 + (j & 0xff))) {
            ok = false;
            break;
          }
          const uint32_t st = base + s * STAGE;
          mbar_expect_tx(kv_full(s), STAGE);
#pragma unroll
          for (int part = 0; part < Sh::KSPLIT; ++part) {
            tma_load_3d(st + part * Sh::KPART, &tm_hi, kcol + part * Sh::KBOX, j * BKV, bb,
                        kv_full(s));
            tma_load_3d(st + OPK + part * Sh::KPART, &tm_lo, kcol + part * Sh::KBOX, j * BKV, bb,
                        kv_full(s));
          }
          tma_load_3d(st + 2 * OPK, &tm_vhi, j * BKV, 0, bh, kv_full(s));
          tma_load_3d(st + 2 * OPK + OPV, &tm_vlo, j * BKV, 0, bh, kv_full(s));
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      it = __shfl_sync(0xffffffffu, it, 0);
    }
    // the last phase armed on each stage has landed before the CTA retires
    if (lane == 0)
      for (int k = it > STAGES ? it - STAGES : 0; k < it; ++k)
        mbar_drain(kv_full(k % STAGES), (k / STAGES) & 1, p.status, 0x4F00);
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ---------------------------------------------------------
    pdl_wait();
    int g = 0, m = 0;  // tiles consumed over all items; items with work
    bool ok = true;
    auto issue_s = [&](int t) -> bool {  // S of tile t (over all items) into buffer t % NB
      const int s = t % STAGES;
      if (!mbar_wait(kv_full(s), (t / STAGES) & 1, abort_w, p.status, 0x4200)) return false;
      const uint32_t kst = base + s * STAGE;
      const uint32_t sd = tm + Sh::T_SP + 64u * (uint32_t)(t % NB);
      constexpr int KK_BOX = Sh::KBOX / 16;
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        const uint32_t kpart = kst + (uint32_t)(kk / KK_BOX) * Sh::KPART;
        const uint64_t khi0 = sdesc(kpart, Sh::K_SBO, Sh::K_SWZ);
        const uint64_t klo0 = sdesc(kpart + OPK, Sh::K_SBO, Sh::K_SWZ);
        const uint64_t koff = (uint64_t)(2 * (kk % KK_BOX));
        mma_ts(sd, tm + T_QHI + 8u * kk, khi0 + koff, Sh::IDESC_S, kk > 0);
        mma_ts(sd, tm + T_QHI + 8u * kk, klo0 + koff, Sh::IDESC_S, 1);
        mma_ts(sd, tm + T_QLO + 8u * kk, khi0 + koff, Sh::IDESC_S, 1);
      }
      mma_commit(s_full(t % NB));
      return true;
    };
    for (int n = 0; ok; ++n) {
      const int slot = n & 1;
      if (!mbar_wait(info_ready(slot), (n >> 1) & 1, abort_w, p.status, 0x4810)) break;
      const int valid = s_rec[slot][0], nkv = s_rec[slot][6];
      mbar_arrive(info_free(slot));
      if (valid < 0) break;
      if (valid == 0) continue;
      if (!mbar_wait(q_ready, m & 1, abort_w, p.status, 0x4000)) break;
      fence_after();
      for (int j = 0; j < NB && j < nkv; ++j) ok = ok && issue_s(g + j);
      for (int j = 0; ok && j < nkv; ++j) {
        const int t = g + j, s = t % STAGES, b = t % NB;
        if (!mbar_wait(p_full(b), (t / NB) & 1, abort_w, p.status, 0x4400)) {
          ok = false;
          break;
        }
        fence_after();
        const uint32_t vst = base + s * STAGE + 2 * OPK;
        const uint64_t vhi0 = sdesc(vst, 1024, 2), vlo0 = sdesc(vst + OPV, 1024, 2);
        const uint32_t pb = tm + Sh::T_SP + 64u * b;
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {
          const uint64_t voff = (uint64_t)(2 * kk);
          const uint32_t phi = pb + 32u * (kk >> 1) + 8u * (kk & 1);
          mma_ts(tm + T_O, phi, vhi0 + voff, Sh::IDESC_PV, (j | kk) != 0);
          mma_ts(tm + T_O, phi, vlo0 + voff, Sh::IDESC_PV, 1);
          mma_ts(tm + T_O, phi + 16u, vhi0 + voff, Sh::IDESC_PV, 1);
        }
        mma_commit(o_done(b));
        mma_commit(kv_empty(s));
        if (j + NB < nkv) ok = issue_s(t + NB);
      }
      if (ok) mma_commit(o_final);
      g += nkv;
      ++m;
    }
    mma_commit(drain_bar);
    mbar_drain(drain_bar, 0, p.status, 0x4F10);
  } else if (warp >= kSoftWarp0) {
    // ---- softmax, one thread per query row (warps 2-5) ----------------------
    const int t_row = (warp & 3) * 32 + lane;  // row within the tile = tensor-memory lane
    const uint32_t lane_base = tm + ((uint32_t)((warp & 3) * 32) << 16);
    const float sl = p.scale * 1.4426950408889634f;
    constexpr float kLazy = 8.0f;
    constexpr float kPScale = 7.0f;
    constexpr int NQ = HD / 8;  // 16-byte chunks of Q_hi (and of Q_lo)
    constexpr int QC = HD / 2 < 16 ? HD / 2 : 16;
    int n = 0;  // records read
    // the next record with work (or the end), read and released
    auto next_rec = [&](int *rec) -> bool {
      for (;;) {
        const int slot = n & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(info_ready(slot), (n >> 1) & 1, abort_w,
                                               p.status, 0x4820)))
          return false;
#pragma unroll
        for (int i = 0; i < 8; ++i) rec[i] = s_rec[slot][i];
        __syncwarp();
        if (lane == 0) mbar_arrive(info_free(slot));
        ++n;
        if (rec[0] != 0) return rec[0] > 0;
      }
    };
    // Q row of an item -> tensor memory, then q_ready (every global load of
    // the row is issued before the first store)
    auto put_q = [&](const int *rec) {
      uint4 qraw[2][NQ];
      const int row = rec[3] + t_row;
      const bool row_in = row < S;
      const int64_t qoff = ((int64_t)rec[1] * S + (row_in ? row : 0)) * (int64_t)(2 * D) +
                           (int64_t)rec[2] * hd;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint4 *src = reinterpret_cast<const uint4 *>((which ? p.qk_lo : p.qk_hi) + qoff);
#pragma unroll
        for (int u = 0; u < NQ; ++u)
          qraw[which][u] = (row_in && 8 * u < hd) ? src[u] : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint32_t tcol = lane_base + (which ? T_QLO : T_QHI);
#pragma unroll
        for (int c = 0; c < HD / 2; c += QC) {
          uint32_t qv[QC];
#pragma unroll
          for (int i = 0; i < QC / 4; ++i) {
            const uint4 v = qraw[which][c / 4 + i];
            qv[4 * i] = v.x; qv[4 * i + 1] = v.y; qv[4 * i + 2] = v.z; qv[4 * i + 3] = v.w;
          }
          if constexpr (QC == 16) tmem_st16(tcol + c, qv);
          else if constexpr (QC == 8) tmem_st8(tcol + c, qv);
          else tmem_st4(tcol + c, qv);
        }
      }
      tmem_wait_st();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
    };
    int cur[8];
    bool have = next_rec(cur);
    pdl_wait();
    if (have) put_q(cur);
    int g = 0, m = 0;
    while (have) {
      const int bb = cur[1], hh = cur[2], q0 = cur[3], kv_end = cur[5], nkv = cur[6];
      const uint8_t *mtile = cur[7] ? p.mask + (int64_t)bb * S : nullptr;
      const int row = q0 + t_row;
      const bool row_in = row < S;
      float m_ref = -CUDART_INF_F, l = 0.f;
      for (int j = 0; j < nkv; ++j) {
        const int t = g + j, sb = t % NB;
        const int k0 = j * BKV;
        uint32_t ok0, ok1;
        if (mtile == nullptr) {
          const int nn = kv_end - k0, n1 = nn - 32;
          ok0 = nn >= 32 ? 0xffffffffu : (nn <= 0 ? 0u : (1u << nn) - 1u);
          ok1 = n1 >= 32 ? 0xffffffffu : (n1 <= 0 ? 0u : (1u << n1) - 1u);
        } else {
          const int ka = k0 + lane, kb2 = k0 + 32 + lane;
          ok0 = __ballot_sync(0xffffffffu, ka < kv_end && mtile[ka] != 0);
          ok1 = __ballot_sync(0xffffffffu, kb2 < kv_end && mtile[kb2] != 0);
        }
        const bool diag = p.causal && k0 + 63 > q0;
        const bool open = !diag && (ok0 & ok1) == 0xffffffffu;
        const uint32_t sp = lane_base + Sh::T_SP + 64u * sb;
        mbar_wait(s_full(sb), (t / NB) & 1, abort_w, p.status, 0x4500);
        fence_after();
        float sv[64];
        tmem_ld32(sp, sv);
        tmem_ld32(sp + 32, sv + 32);
        tmem_wait_ld();
        if (!open) {
          uint32_t a0 = ok0, a1 = ok1;
          if (diag) {
            const int lim = row - k0, lim1 = lim - 32;
            a0 &= lim >= 31 ? 0xffffffffu : (lim < 0 ? 0u : (2u << lim) - 1u);
            a1 &= lim1 >= 31 ? 0xffffffffu : (lim1 < 0 ? 0u : (2u << lim1) - 1u);
          }
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            sv[c] = (a0 >> c) & 1u ? sv[c] : -CUDART_INF_F;
            sv[32 + c] = (a1 >> c) & 1u ? sv[32 + c] : -CUDART_INF_F;
          }
        }
        float mx8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          mx8[i] = fmax3(sv[i], sv[i + 8], sv[i + 16]);
          mx8[i] = fmax3(mx8[i], sv[i + 24], sv[i + 32]);
          mx8[i] = fmax3(mx8[i], sv[i + 40], sv[i + 48]);
          mx8[i] = fmaxf(mx8[i], sv[i + 56]);
        }
        const float mx = fmaxf(fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]),
                                     mx8[6]),
                               mx8[7]) * sl;
        const bool raise = mx > m_ref + kLazy || (m_ref == -CUDART_INF_F && mx != -CUDART_INF_F);
        const float alpha = raise ? fast_exp2(m_ref - mx) : 1.f;
        if (__any_sync(0xffffffffu, raise && m_ref != -CUDART_INF_F) && j > 0) {
          // P.V of the item's previous tile has landed in the context: phase
          // (t-1)/NB of buffer (t-1) % NB's o_done, exact as in the form above
          mbar_wait(o_done((t - 1) % NB), ((t - 1) / NB) & 1, abort_w, p.status, 0x4600);
          fence_after();
          constexpr int OC = HDO >= 16 ? 16 : 8;
#pragma unroll
          for (int c = 0; c < HDO; c += OC) {
            float ov[OC];
            tmem_ld_n<OC>(lane_base + T_O + c, ov);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < OC; ++i) ov[i] *= alpha;
            if constexpr (OC == 16) tmem_st16_f32(lane_base + T_O + c, ov);
            else tmem_st8_f32(lane_base + T_O + c, ov);
          }
        }
        if (raise) {
          l *= alpha;
          m_ref = mx;
        }
        const bool live = m_ref != -CUDART_INF_F;
        const float noff = kPScale - m_ref;
        float ps4[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t w[32];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const float e0 = live ? fast_exp2(fmaf(sv[32 * half + 2 * c], sl, noff)) : 0.f;
            const float e1 = live ? fast_exp2(fmaf(sv[32 * half + 2 * c + 1], sl, noff)) : 0.f;
            ps4[(2 * c) & 3] += e0;
            ps4[(2 * c + 1) & 3] += e1;
            split_pair_nonneg(e0, e1, w[c], w[16 + c]);
          }
          tmem_st32(sp + 32u * half, w);
        }
        l += (ps4[0] + ps4[1]) + (ps4[2] + ps4[3]);
        tmem_wait_st();
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full(sb));
      }
      // every score of this item has been read (each s_full waited above), so
      // the next item's Q may replace this one's while the last P.V runs
      int nxt[8];
      const bool more = next_rec(nxt);
      if (more) put_q(nxt);
      mbar_wait(o_final, m & 1, abort_w, p.status, 0x4700);
      fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int64_t off = ((int64_t)bb * S + (row_in ? row : 0)) * (int64_t)D + (int64_t)hh * hd;
      constexpr int OC = HDO >= 32 ? 16 : 8;
#pragma unroll
      for (int c = 0; c < HDO; c += OC) {
        float ov[OC];
        tmem_ld_n<OC>(lane_base + T_O + c, ov);
        tmem_wait_ld();
        if (row_in && c < hd) {
          uint32_t hw[OC / 2], lw[OC / 2];
#pragma unroll
          for (int i = 0; i < OC / 2; ++i)
            split_pair(ov[2 * i] * inv, ov[2 * i + 1] * inv, hw[i], lw[i]);
          uint4 *dh = reinterpret_cast<uint4 *>(p.ctx_hi + off + c);
          uint4 *dl = reinterpret_cast<uint4 *>(p.ctx_lo + off + c);
#pragma unroll
          for (int u = 0; u < OC / 8; ++u) {
            dh[u] = make_uint4(hw[4 * u], hw[4 * u + 1], hw[4 * u + 2], hw[4 * u + 3]);
            dl[u] = make_uint4(lw[4 * u], lw[4 * u + 1], lw[4 * u + 2], lw[4 * u + 3]);
          }
        }
      }
      // the context reads complete (tcgen05.wait::ld above) before the arrive
      // on p_full of the next item's first tile, which the P.V that
      // overwrites the context waits for
      g += nkv;
      ++m;
      have = more;
#pragma unroll
      for (int i = 0; i < 8; ++i) cur[i] = nxt[i];
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(TMEM_COLS)
                 : "memory");
  }
}

template <int HD>
__global__ void __maxnreg__(128)
    attention_tc_persist_kernel(const __grid_constant__ CUtensorMap tm_hi,
                                const __grid_constant__ CUtensorMap tm_lo,
                                const __grid_constant__ CUtensorMap tm_vhi,
                                const __grid_constant__ CUtensorMap tm_vlo,
                                const AttentionTcParams p) {
  attention_tc_persist_body<HD>(tm_hi, tm_lo, tm_vhi, tm_vlo, p);
}

// One softmax thread per row (head_dim up to 64): 6 warps fall 2, 2, 1, 1 on
// the four SM sub-partitions, so two CTAs per SM put 4 warps on one, whose 16K
// registers allow 128 per thread.
template <int HD, bool GROUPED>
__global__ void __maxnreg__(128)
    attention_tc_row_kernel(const __grid_constant__ CUtensorMap tm_hi,
                            const __grid_constant__ CUtensorMap tm_lo,
                            const __grid_constant__ CUtensorMap tm_vhi,
                            const __grid_constant__ CUtensorMap tm_vlo, const AttentionTcParams p) {
  attention_tc_body<HD, GROUPED, true>(tm_hi, tm_lo, tm_vhi, tm_vlo, p);
}
template <bool GROUPED>
__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel_hd128(const __grid_constant__ CUtensorMap tm_hi,
                              const __grid_constant__ CUtensorMap tm_lo,
                              const __grid_constant__ CUtensorMap tm_vhi,
                              const __grid_constant__ CUtensorMap tm_vlo,
                              const AttentionTcParams p) {
  attention_tc_body<128, GROUPED, false>(tm_hi, tm_lo, tm_vhi, tm_vlo, p);
}
template <bool GROUPED>
__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel_hd256(const __grid_constant__ CUtensorMap tm_hi,
                              const __grid_constant__ CUtensorMap tm_lo,
                              const __grid_constant__ CUtensorMap tm_vhi,
                              const __grid_constant__ CUtensorMap tm_vlo,
                              const AttentionTcParams p) {
  attention_tc_body<256, GROUPED, false>(tm_hi, tm_lo, tm_vhi, tm_vlo, p);
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

// [batch, seq, 2*d_model] fp16 view of a q|k buffer; box = kbox columns x 64
// rows x 1 sequence, kbox = min(hd_mma, 64) (rows of 32, 64 or 128 bytes with
// the matching swizzle; hd 128 loads two boxes), zero fill past the sequence
// end and past the last column.
int make_qk_map(CUtensorMap *tm, const uint16_t *ptr, int64_t batch, int seq, int d_model,
                int hd_mma) {
  EncodeTiledFn encode;
  int rc = encode_fn(&encode);
  if (rc != TT_OK) return rc;
  cuuint64_t dims[3] = {(cuuint64_t)(2 * d_model), (cuuint64_t)seq, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(2 * d_model) * 2, (cuuint64_t)seq * (2 * d_model) * 2};
  const int kbox = hd_mma < 64 ? hd_mma : 64;
  cuuint32_t box[3] = {(cuuint32_t)kbox, (cuuint32_t)BKV, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = encode(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<uint16_t *>(ptr),
                            dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            kbox == 16   ? CU_TENSOR_MAP_SWIZZLE_32B
                            : kbox == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                         : CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TT_ERR_CUDA, "cuTensorMapEncodeTiled (q|k) failed with CUresult " +
                                 std::to_string((int)r));
  return TT_OK;
}

// [batch*heads, hd, seq] fp16 view of a transposed value buffer (row stride
// seq_pad); box = 64 keys x rows dims x 1 (rows = the dims one CTA outputs:
// 128 of head_dim 256), 128-byte swizzle, zero fill past the sequence (and
// past hd when 16 rows serve head_dim 8).
int make_vt_map(CUtensorMap *tm, const uint16_t *ptr, int64_t bh, int seq, int seq_pad, int hd,
                int rows) {
  EncodeTiledFn encode;
  int rc = encode_fn(&encode);
  if (rc != TT_OK) return rc;
  cuuint64_t dims[3] = {(cuuint64_t)seq, (cuuint64_t)hd, (cuuint64_t)bh};
  cuuint64_t strides[2] = {(cuuint64_t)seq_pad * 2, (cuuint64_t)seq_pad * hd * 2};
  cuuint32_t box[3] = {(cuuint32_t)BKV, (cuuint32_t)rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = encode(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<uint16_t *>(ptr),
                            dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TT_ERR_CUDA, "cuTensorMapEncodeTiled (v^T) failed with CUresult " +
                                 std::to_string((int)r));
  return TT_OK;
}

template <int HD, bool GROUPED, bool ROW1>
constexpr auto attention_kernel_for() {
  static_assert(ROW1 == (HD <= 64), "one thread per row exactly up to head_dim 64");
  if constexpr (HD == 256) return &attention_tc_kernel_hd256<GROUPED>;
  else if constexpr (HD == 128) return &attention_tc_kernel_hd128<GROUPED>;
  else return &attention_tc_row_kernel<HD, GROUPED>;
}

template <int HD, bool GROUPED, bool ROW1>
int launch_hd_as(const AttentionTcParams &p, const CUtensorMap &thi, const CUtensorMap &tlo,
                 const CUtensorMap &tvhi, const CUtensorMap &tvlo, cudaStream_t stream) {
  using Sh = AtShape<HD>;
  constexpr auto fn = attention_kernel_for<HD, GROUPED, ROW1>();
  static bool attr_set = false;
  if (!attr_set) {
    TT_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)Sh::SMEM_BYTES));
    // two CTAs per SM need the largest shared-memory carveout
    TT_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     (int)cudaSharedmemCarveoutMaxShared));
    attr_set = true;
  }
  const int64_t ctas_x = (int64_t)((p.seq + BQ - 1) / BQ) * p.bh_group * Sh::NSPLIT;
  const int64_t groups = p.batch * p.num_heads / p.bh_group;
  dim3 grid((unsigned)ctas_x, (unsigned)groups);
  TT_CUDA_TRY(launch_kernel(fn, grid, dim3(ROW1 ? kThreadsRow1 : kThreads), Sh::SMEM_BYTES,
                            stream, 1, thi, tlo, tvhi, tvlo, p));
  TT_LAUNCH_CHECK("attention_tc");
  return TT_OK;
}

// CTAs of the persistent form that fit on the current device at once, from
// the SM's shared memory (each CTA also holds 64 static bytes and the
// per-block reservation): two per SM by design -- 128 registers x 192 threads
// and 256 tensor-memory columns each leave room for two. (The runtime's
// occupancy query answers one for this kernel on B200, whose launches run two
// per SM.)
template <int HD>
int persist_slots(int *slots_out) {
  using Sh = AtShape<HD>;
  static int slots_dev = -1, slots = 0;
  int dev = 0;
  TT_CUDA_TRY(cudaGetDevice(&dev));
  if (dev != slots_dev) {
    int smem_sm = 0, reserved = 0, sms = 0;
    TT_CUDA_TRY(cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev));
    TT_CUDA_TRY(cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev));
    TT_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int per_sm = std::min(2, smem_sm / ((int)Sh::SMEM_BYTES + 64 + reserved));
    if (per_sm <= 0 || sms <= 0)
      return fail(TT_ERR_CUDA, "attention_tc: the persistent kernel fits no SM");
    slots = per_sm * sms;
    slots_dev = dev;
  }
  *slots_out = slots;
  return TT_OK;
}

// The persistent form: one CTA per slot, each running work items until none
// are left.
template <int HD>
int launch_persist(const AttentionTcParams &p, const CUtensorMap &thi, const CUtensorMap &tlo,
                   const CUtensorMap &tvhi, const CUtensorMap &tvlo, int slots,
                   cudaStream_t stream) {
  using Sh = AtShape<HD>;
  constexpr auto fn = &attention_tc_persist_kernel<HD>;
  static bool attr_set = false;
  if (!attr_set) {
    TT_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)Sh::SMEM_BYTES));
    TT_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     (int)cudaSharedmemCarveoutMaxShared));
    attr_set = true;
  }
  TT_CUDA_TRY(launch_kernel(fn, dim3((unsigned)slots), dim3(kThreadsRow1), Sh::SMEM_BYTES,
                            stream, 1, thi, tlo, tvhi, tvlo, p));
  TT_LAUNCH_CHECK("attention_tc_persist");
  return TT_OK;
}

template <int HD>
int launch_hd(const AttentionTcParams &p, const CUtensorMap &thi, const CUtensorMap &tlo,
              const CUtensorMap &tvhi, const CUtensorMap &tvlo, cudaStream_t stream) {
  if constexpr (HD <= 64) {
    // persistent when the items outnumber the slots (with one item per CTA it
    // only adds the item hand-off, measured 1 us per launch slower)
    if (p.counter != nullptr) {
      int slots = 0, rc;
      if ((rc = persist_slots<HD>(&slots))) return rc;
      const int64_t items = (int64_t)((p.seq + BQ - 1) / BQ) * p.batch * p.num_heads;
      if (items > slots) return launch_persist<HD>(p, thi, tlo, tvhi, tvlo, slots, stream);
    }
  }
  // one softmax thread per row up to head_dim 64, two (one per key half) above
  constexpr bool ROW1 = HD <= 64;
  if (p.bh_group < p.batch * p.num_heads)
    return launch_hd_as<HD, true, ROW1>(p, thi, tlo, tvhi, tvlo, stream);
  return launch_hd_as<HD, false, ROW1>(p, thi, tlo, tvhi, tvlo, stream);
}

}  // namespace

bool attention_tc_persistent(int head_dim) {
  // TT_ATTENTION_PERSISTENT=0 selects the one-CTA-per-item form throughout
  static const bool off = [] {
    const char *e = std::getenv("TT_ATTENTION_PERSISTENT");
    return e != nullptr && e[0] == '0';
  }();
  return head_dim <= 64 && !off;
}

bool attention_tc_supported(int head_dim, int d_model) {
  return (head_dim == 8 || head_dim == 16 || head_dim == 32 || head_dim == 64 ||
          head_dim == 128 || head_dim == 256) &&
         d_model % 8 == 0;
}

int launch_attention_tc(const AttentionTcParams &p, cudaStream_t stream) {
  if (p.batch <= 0 || p.seq <= 0) return TT_OK;
  if (!attention_tc_supported(p.head_dim, p.d_model))
    return fail(TT_ERR_UNSUPPORTED, "attention_tc: head_dim must be 8, 16, 32, 64, 128 or 256");
  if ((int64_t)((p.seq + BQ - 1) / BQ) * p.num_heads * p.batch * 2 > INT32_MAX)
    return fail(TT_ERR_UNSUPPORTED, "attention_tc: more than 2^31 query tiles");
  if (((reinterpret_cast<uintptr_t>(p.qk_hi) | reinterpret_cast<uintptr_t>(p.qk_lo) |
        reinterpret_cast<uintptr_t>(p.ctx_hi) | reinterpret_cast<uintptr_t>(p.ctx_lo) |
        reinterpret_cast<uintptr_t>(p.vt_hi) | reinterpret_cast<uintptr_t>(p.vt_lo)) & 15) != 0)
    return fail(TT_ERR_INVALID_ARGUMENT, "attention_tc: buffers must be 16-byte aligned");
  if (p.seq_pad < p.seq || p.seq_pad % 8 != 0)
    return fail(TT_ERR_INVALID_ARGUMENT, "attention_tc: seq_pad must be >= seq and a multiple of 8");
  // head_dim 8 runs as 16 (zero Q padding, see AtShape)
  const int hd_mma = p.head_dim < 16 ? 16 : p.head_dim;
  CUtensorMap thi, tlo, tvhi, tvlo;
  int rc;
  const int64_t bh = p.batch * p.num_heads;
  if ((rc = make_qk_map(&thi, p.qk_hi, p.batch, p.seq, p.d_model, hd_mma)) ||
      (rc = make_qk_map(&tlo, p.qk_lo, p.batch, p.seq, p.d_model, hd_mma)) ||
      (rc = make_vt_map(&tvhi, p.vt_hi, bh, p.seq, p.seq_pad, p.head_dim, hd_mma > 128 ? 128 : hd_mma)) ||
      (rc = make_vt_map(&tvlo, p.vt_lo, bh, p.seq, p.seq_pad, p.head_dim, hd_mma > 128 ? 128 : hd_mma)))
    return rc;
  // Grid order. Each CTA streams its pair's K/V from key 0 to its diagonal;
  // CTAs running at one time reuse each other's K/V through the L2 only if
  // few pairs are in flight. When all pairs' K/V exceed 64 MB and sequences
  // have 8 query tiles or more, the grid runs groups of pairs whose K/V
  // total at most 32 MB (at least one pair), one group after another.
  AttentionTcParams q = p;
  q.bh_group = (int)bh;
  const int64_t kv_pair = (int64_t)p.seq * p.head_dim * 8;  // k, v x hi, lo x 2 B
  const int ntq = (p.seq + BQ - 1) / BQ;
  if (bh * kv_pair > (64LL << 20) && ntq >= 8) {
    const int64_t gmax = std::max<int64_t>(1, (32LL << 20) / kv_pair);
    for (int64_t g = std::min(gmax, bh); g >= 1; --g)
      if (bh % g == 0) {
        // the groups go on grid y (at most 65535)
        if (bh / g <= 65535) q.bh_group = (int)g;
        break;
      }
  }
  if (hd_mma == 16) return launch_hd<16>(q, thi, tlo, tvhi, tvlo, stream);
  if (p.head_dim == 32) return launch_hd<32>(q, thi, tlo, tvhi, tvlo, stream);
  if (p.head_dim == 64) return launch_hd<64>(q, thi, tlo, tvhi, tvlo, stream);
  if (p.head_dim == 128) return launch_hd<128>(q, thi, tlo, tvhi, tvlo, stream);
  return launch_hd<256>(q, thi, tlo, tvhi, tvlo, stream);
}

}  // namespace tt

