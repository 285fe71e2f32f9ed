// Replay of the per-op forward schedules through instantiated CUDA graphs.
//
// A per-op forward is 5 or 7 launches per layer plus one, each preceded on the
// host by tensor-map encoding and launch-attribute set-up. For small shapes
// (d_model 128, a few thousand tokens) the GPU finishes a kernel faster than
// the host issues the next, so the forward is bound by the host. A CUDA graph
// holds the whole launch sequence with its parameters; one cudaGraphLaunch
// replays it, and the kernels keep their programmatic-dependent-launch edges.
//
// The graph bakes in every pointer and size of the call, so it is cached under
// a key of all of them (device, the schedule-relevant config fields, image,
// x, mask, y, scratch, batch, seq). A call is replayed from a graph only when
// its key was seen before: the first call with a key launches directly (which
// also performs every one-time host set-up, such as kernel attributes, outside
// any capture), the second captures the launches on a private stream,
// instantiates the graph and launches it, later ones replay it. A key whose
// capture failed launches directly from then on. The cache keeps the 16 most
// recently used keys. Replaying a graph is the same work as launching it
// directly: the kernels read their inputs when they run.
//
// Direct launches are used instead when TT_GRAPHS=0 is set in the
// environment, while the launch probe is timing individual launches, while a
// test switch is armed (tt_test_arm_wait_timeout), and when the caller's
// stream is itself being captured (the launches then go into the caller's
// graph).
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "gemm_tc.cuh"
#include "image.cuh"
#include "tt_common.cuh"

namespace tt {
namespace {

struct GraphEntry {
  ForwardKey key;
  cudaGraphExec_t exec = nullptr;  // null: seen once, not captured yet
  bool capture_failed = false;     // launch directly from now on
  uint64_t last_use = 0;
};

constexpr size_t kMaxEntries = 16;
constexpr int kMaxDevices = 64;

std::mutex g_mutex;
std::vector<GraphEntry> g_entries;
uint64_t g_clock = 0;
cudaStream_t g_capture_stream[kMaxDevices] = {};

bool graphs_enabled() {
  static const bool on = [] {
    const char *e = std::getenv("TT_GRAPHS");
    return e == nullptr || std::strcmp(e, "0") != 0;
  }();
  return on;
}

bool same_key(const ForwardKey &a, const ForwardKey &b) {
  return std::memcmp(&a, &b, sizeof(ForwardKey)) == 0;
}

// Captures launch(cap) into a graph and instantiates it. On any failure the
// capture is ended, partial objects are released and *exec stays null.
int capture(const ForwardLaunch &launch, cudaStream_t cap, cudaGraphExec_t *exec) {
  *exec = nullptr;
  TT_CUDA_TRY(cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal));
  const int rc = launch(cap);
  cudaGraph_t graph = nullptr;
  const cudaError_t end = cudaStreamEndCapture(cap, &graph);
  if (rc != TT_OK || end != cudaSuccess || graph == nullptr) {
    if (graph != nullptr) cudaGraphDestroy(graph);
    cudaGetLastError();
    return rc != TT_OK ? rc : fail(TT_ERR_CUDA, "forward graph capture failed");
  }
  const cudaError_t inst = cudaGraphInstantiate(exec, graph, 0);
  cudaGraphDestroy(graph);
  if (inst != cudaSuccess) {
    *exec = nullptr;
    cudaGetLastError();
    return fail(TT_ERR_CUDA, std::string("cudaGraphInstantiate: ") + cudaGetErrorString(inst));
  }
  return TT_OK;
}

}  // namespace

int run_forward_cached(const ForwardKey &key, cudaStream_t stream, const ForwardLaunch &launch) {
  // an armed test switch must reach exactly one launch, never a cached graph
  if (!graphs_enabled() || launch_probe_active() || gemm_wait_timeout_armed())
    return launch(stream);
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  TT_CUDA_TRY(cudaStreamIsCapturing(stream, &cs));
  if (cs != cudaStreamCaptureStatusNone) return launch(stream);
  if (key.device < 0 || key.device >= kMaxDevices) return launch(stream);

  std::lock_guard<std::mutex> lock(g_mutex);
  GraphEntry *hit = nullptr;
  for (GraphEntry &e : g_entries)
    if (same_key(e.key, key)) hit = &e;
  if (hit == nullptr) {
    // first sighting: remember the key, launch directly
    if (g_entries.size() >= kMaxEntries) {
      size_t lru = 0;
      for (size_t i = 1; i < g_entries.size(); ++i)
        if (g_entries[i].last_use < g_entries[lru].last_use) lru = i;
      if (g_entries[lru].exec != nullptr) cudaGraphExecDestroy(g_entries[lru].exec);
      g_entries.erase(g_entries.begin() + (std::ptrdiff_t)lru);
    }
    GraphEntry e;
    e.key = key;
    e.last_use = ++g_clock;
    g_entries.push_back(e);
    return launch(stream);
  }
  hit->last_use = ++g_clock;
  if (hit->capture_failed) return launch(stream);
  if (hit->exec == nullptr) {
    cudaStream_t &cap = g_capture_stream[key.device];
    if (cap == nullptr) TT_CUDA_TRY(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking));
    cudaGraphExec_t exec = nullptr;
    if (capture(launch, cap, &exec) != TT_OK || exec == nullptr) {
      hit->capture_failed = true;
      return launch(stream);
    }
    hit->exec = exec;
  }
  TT_CUDA_TRY(cudaGraphLaunch(hit->exec, stream));
  return TT_OK;
}

}  // namespace tt
