// Which row tiles of a padded batch the projection GEMMs must compute.
//
// The reference computes every projection over all batch x seq rows and then
// zeroes the padded rows (torch_transformer_benchmark.py:118-121, :143-144,
// :170-171); their values never reach a valid output. Rows past the last valid
// key of a sequence are only ever read by row-local work of their own rows --
// every GEMM row depends on its own A row, the epilogues zero invalid rows by
// select, the final LayerNorm zeroes them -- with one exception: the
// attention loads key/value tiles of 64 keys up to the one that holds the last
// valid key, so value rows up to that tile's end must be finite (they meet
// probability 0, and 0 times a stale NaN would not be 0). So a row is dead
// when its position in its sequence is at or past the last valid key rounded
// up to a multiple of 64; a 128-row tile of the batch is dead when all its
// rows are. Every GEMM of the forward skips the dead tiles (the single-CTA
// kernel takes one live tile per CTA, the CTA-pair kernel two consecutive
// entries of the list, adjacent or not), so every row of a live tile is
// written by every GEMM and no computed tile reads a row of a dead one.
//
// One launch, one CTA of 1024 threads: each warp finds the valid length of
// its sequences (the last non-zero mask byte, 16-byte loads), then the CTA
// lists the live tiles in order with a block-wide prefix count.
// Output (ints): [0] live 128-row tiles, [1 ..] their list; then the
// per-sequence lengths (`kvlen`) and one flag per 128-row tile (1 live, 0
// dead; the LayerNorms ahead of the GEMMs skip dead tiles with it). HBM
// traffic is the mask (B x S bytes) plus a few KB.
#include "image.cuh"
#include "tt_common.cuh"

namespace tt {
namespace {

constexpr int kScanThreads = 1024;

__global__ void __launch_bounds__(kScanThreads) live_rows_kernel(const uint8_t *__restrict__ mask,
                                                                 int64_t batch, int seq,
                                                                 int *__restrict__ kvlen,
                                                                 int *__restrict__ flags,
                                                                 int *__restrict__ out) {
  pdl_trigger();
  pdl_wait();  // the previous forward on this stream may still read the lists
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int kWarps = kScanThreads / 32;
  // ---- valid length of each sequence: 1 + index of its last valid key ------
  for (int64_t b = warp; b < batch; b += kWarps) {
    int last = 0;
    if (mask == nullptr) {
      last = seq;
    } else {
      const uint8_t *row = mask + b * seq;
      if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) {
        const int n16 = seq / 16;
        for (int j = lane; j < n16; j += 32) {
          const uint4 v = reinterpret_cast<const uint4 *>(row)[j];
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (w[k]) last = max(last, 16 * j + 4 * k + (31 - __clz((int)w[k])) / 8 + 1);
        }
        for (int j = 16 * n16 + lane; j < seq; j += 32)
          if (row[j]) last = max(last, j + 1);
      } else {
        for (int j = lane; j < seq; j += 32)
          if (row[j]) last = max(last, j + 1);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
    }
    if (lane == 0) kvlen[b] = last;
  }
  __syncthreads();  // kvlen (global, written by this CTA) visible to the CTA
  // ---- live 128-row tiles, listed in order --------------------------------------
  __shared__ int warp_count[kWarps];
  const int64_t rows = batch * (int64_t)seq;
  const int64_t nmt = (rows + 127) / 128;
  int *list = out + 1;
  int base = 0;
  for (int64_t s0 = 0; s0 < nmt; s0 += kScanThreads) {
    const int64_t s = s0 + tid;
    bool live = false;
    if (s < nmt) {
      const int64_t r0 = 128 * s, r1 = min(r0 + 128, rows);
      for (int64_t b = r0 / seq; !live && b * seq < r1; ++b) {
        const int64_t lo = max(r0, b * seq) - b * seq;
        const int lim = min(seq, (kvlen[b] + 63) / 64 * 64);
        live = lo < lim;
      }
    }
    if (s < nmt) flags[s] = live ? 1 : 0;
    const uint32_t bal = __ballot_sync(0xffffffffu, live);
    if (lane == 0) warp_count[warp] = __popc(bal);
    __syncthreads();
    int before = 0, sum = 0;
    for (int w = 0; w < kWarps; ++w) {
      before += w < warp ? warp_count[w] : 0;
      sum += warp_count[w];
    }
    if (live) list[base + before + __popc(bal & ((1u << lane) - 1u))] = (int)s;
    base += sum;
    __syncthreads();  // warp_count is reused by the next chunk
  }
  if (tid == 0) out[0] = base;
}

}  // namespace

size_t live_rows_ints(int64_t batch, int64_t seq) {
  const int64_t rows = batch * seq;
  return (size_t)(1 + 2 * ((rows + 127) / 128) + batch);
}

const int *live_rows_flags(const int *ws_ints, int64_t batch, int64_t seq) {
  return ws_ints + 1 + (batch * seq + 127) / 128 + batch;
}

int launch_live_rows(const uint8_t *mask, int64_t batch, int seq, int *ws_ints,
                     cudaStream_t stream) {
  const int64_t rows = batch * (int64_t)seq;
  int *out = ws_ints;
  int *kvlen = ws_ints + 1 + (rows + 127) / 128;
  int *flags = kvlen + batch;
  TT_CUDA_TRY(launch_kernel(live_rows_kernel, dim3(1), dim3(kScanThreads), 0, stream, 1, mask,
                            batch, seq, kvlen, flags, out));
  TT_LAUNCH_CHECK("live_rows");
  return TT_OK;
}

}  // namespace tt
