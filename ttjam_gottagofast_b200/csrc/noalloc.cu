// tt_forward_noalloc: the per-op forward pass with its scratch in a fixed
// device array inside this library, for callers that cannot allocate device
// memory at the point where they run the forward pass.
//
// Who needs it: a host that owns the whole device-memory budget and does not
// let a plugin allocate (the plugin must work in memory it was given), a
// serving loop that must never call cudaMalloc because the call can
// synchronise the device and stall other work, or a process that has handed
// all of its device memory to its own pool. Such a caller still passes the
// packed image, the input, the mask and the output, all of which it already
// holds; only the per-call scratch (the q|k|v, context and ffn-hidden rows of
// tt_workspace_bytes) comes from here.
//
// The array is TT_NOALLOC_SCRATCH_BYTES (16 MiB) of static device memory, so
// every GPU on which this library's module is loaded holds it until the
// process exits. The module is loaded on a device when the array's address is
// first looked up there; tt_pack_image does that (set-up time, the image's
// device current), so the no-alloc calls that follow find the address cached
// and neither load anything nor reserve memory. The calls launch their kernels
// directly on the caller's stream: they never go through the graph cache of
// tt_forward, whose capture stream and instantiated graphs the driver backs
// with memory of its own.
//
// All calls share the array: two calls whose work overlaps on the GPU
// (different streams without ordering, or different host threads) race on it
// and corrupt each other's results. Each call overwrites every scratch element
// it reads before reading it, so nothing in the array has to start at zero and
// the previous call's leftovers never reach an output.
#include <mutex>

#include "image.cuh"
#include "tt_common.cuh"

namespace tt {
namespace {

__device__ __align__(256) unsigned char g_noalloc_scratch[TT_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void *g_scratch_ptr[kMaxDevices] = {};

}  // namespace

// The device address of the scratch array on the current device. The array's
// name in host code is only a host-side handle, never a device address; the
// address is looked up once per device (with that device current) and cached.
int noalloc_scratch_address(void **out) {
  int dev = 0;
  TT_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices)
    return fail(TT_ERR_UNSUPPORTED, "tt_forward_noalloc: device index out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void *p = nullptr;
    TT_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    if (p == nullptr) return fail(TT_ERR_CUDA, "tt_forward_noalloc: scratch address is NULL");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return TT_OK;
}

}  // namespace tt

using namespace tt;

extern "C" int tt_forward_noalloc(const tt_config *cfg, const void *image, const float *x,
                                  const uint8_t *mask, int64_t batch, int64_t seq, float *y,
                                  void *stream_) {
  int rc = validate_config(cfg);
  if (rc != TT_OK) return rc;
  if (batch < 0 || seq < 0) return fail(TT_ERR_INVALID_ARGUMENT, "batch and seq must be >= 0");
  if (batch == 0 || seq == 0) return TT_OK;
  if (image == nullptr || x == nullptr || y == nullptr)
    return fail(TT_ERR_INVALID_ARGUMENT, "tt_forward_noalloc: NULL image, x or y");
  if (x == y) return fail(TT_ERR_INVALID_ARGUMENT, "tt_forward_noalloc: y may not alias x");
  if (((reinterpret_cast<uintptr_t>(image) | reinterpret_cast<uintptr_t>(x) |
        reinterpret_cast<uintptr_t>(y)) & 15) != 0)
    return fail(TT_ERR_INVALID_ARGUMENT, "tt_forward_noalloc: pointers must be 16-byte aligned");
  if (cfg->plan == TT_PLAN_CLUSTER || cfg->plan == TT_PLAN_TILE)
    return fail(TT_ERR_UNSUPPORTED,
                "tt_forward_noalloc runs the per-op schedule; TT_PLAN_CLUSTER and TT_PLAN_TILE "
                "need no scratch and are served by tt_forward");
  if (seq > (int64_t)INT32_MAX || batch > ((int64_t)1 << 40) / seq)
    return fail(TT_ERR_UNSUPPORTED, "tt_forward_noalloc: batch*seq too large");
  // the per-op schedule this call runs: forced by cfg->plan, else the one
  // tt_forward would use when it does not take the single-launch path
  tt_config ops = *cfg;
  if (ops.plan == TT_PLAN_AUTO) ops.plan = auto_ops_plan(*cfg);
  const int plan = forward_plan(&ops, batch, seq);
  if (plan < 0) return plan;
  const WorkspaceLayout W(ops, batch, seq);
  if (W.total > TT_NOALLOC_SCRATCH_BYTES)
    return fail(TT_ERR_WORKSPACE,
                "tt_forward_noalloc: this call needs " + std::to_string(W.total) +
                    " bytes of scratch but the library's fixed array holds " +
                    std::to_string((size_t)TT_NOALLOC_SCRATCH_BYTES) +
                    "; use tt_forward with a caller workspace, or a smaller batch*seq");
  void *scratch = nullptr;
  if ((rc = noalloc_scratch_address(&scratch)) != TT_OK) return rc;
  const ImageLayout L(ops);
  const char *img = static_cast<const char *>(image);
  char *ws = static_cast<char *>(scratch);
  cudaStream_t s = static_cast<cudaStream_t>(stream_);
  return plan == PLAN_OPS_TC ? forward_ops_tc(ops, L, img, x, mask, batch, seq, y, W, ws, s)
                             : forward_ops(ops, L, img, x, mask, batch, seq, y, W, ws, s);
}
