// The whole Lloyd loop as one CUDA graph: a WHILE conditional node whose body
// is one in-place iteration (assign -> counting sort -> gather-accumulate ->
// finalize) followed by a one-thread control kernel that counts the iteration
// and clears the loop condition when max_iters is reached or the centroid
// shift fell below tol. One graph launch runs every iteration with no host
// round trip (the reference's loop synchronises on shift.item() every
// iteration when tol > 0, flash_kmeans_cuda/kmeans.py:186-190).
//
// Instantiated graphs are cached per (device, buffers, shape): a second call on
// the same buffers replays the graph. max_iters and tol live in a control
// block in device memory, written by a kernel before each launch, so they are
// not part of the key.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "fkc_internal.h"

namespace fkc {
namespace {

__global__ void loop_init_kernel(LoopCtl* ctl, int max_iters, float tol) {
  ctl->iter = 0;
  ctl->max_iters = max_iters;
  ctl->tol = tol;
  ctl->n_iters = 0;
}

// After iteration ctl->iter + 1: continue while iterations remain and, when
// tol > 0, the shift of this iteration is not below tol (kmeans.py:188-191).
__global__ void loop_ctl_kernel(cudaGraphConditionalHandle handle, LoopCtl* ctl,
                                const float* shift) {
  const int it = ctl->iter + 1;
  ctl->iter = it;
  ctl->n_iters = it;
  bool more = it < ctl->max_iters;
  if (ctl->tol > 0.f && *shift < ctl->tol) more = false;
  cudaGraphSetConditional(handle, more ? 1u : 0u);
}

struct Entry {
  LloydGraphKey key;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int kernels_per_iter = 0;
  uint64_t last_use = 0;
};

constexpr size_t kMaxGraphs = 8;
std::mutex g_mu;
std::vector<Entry> g_cache;
uint64_t g_tick = 0;
thread_local bool t_capturing = false;
thread_local uint64_t t_captured = 0;  // kernel launches recorded while capturing

bool same_key(const LloydGraphKey& a, const LloydGraphKey& b) {
  return std::memcmp(&a, &b, sizeof(LloydGraphKey)) == 0;
}

void destroy(Entry& e) {
  if (e.exec != nullptr) cudaGraphExecDestroy(e.exec);
  if (e.graph != nullptr) cudaGraphDestroy(e.graph);
  e.exec = nullptr;
  e.graph = nullptr;
}

// Builds the graph: WHILE(handle) { body(stream); loop_ctl_kernel }.
int build(const LloydGraphKey& key, const LoopBody& body, LoopCtl* ctl, const float* shift,
          Entry* out) {
  cudaGraph_t g = nullptr;
  FKC_CUDA_TRY(cudaGraphCreate(&g, 0));
  Entry e;
  e.key = key;
  e.graph = g;
  cudaGraphConditionalHandle handle;
  cudaError_t err = cudaGraphConditionalHandleCreate(&handle, g, 1u, cudaGraphCondAssignDefault);
  if (err != cudaSuccess) {
    destroy(e);
    return set_error(FKC_ECUDA, "cudaGraphConditionalHandleCreate: %s", cudaGetErrorString(err));
  }
  // cudaGraphNodeParams has no default constructor in C++ (a union member);
  // zero-initialised storage, as the API requires for unused fields.
  alignas(cudaGraphNodeParams) unsigned char params_mem[sizeof(cudaGraphNodeParams)] = {};
  cudaGraphNodeParams& params = *reinterpret_cast<cudaGraphNodeParams*>(params_mem);
  params.type = cudaGraphNodeTypeConditional;
  params.conditional.handle = handle;
  params.conditional.type = cudaGraphCondTypeWhile;
  params.conditional.size = 1;
  cudaGraphNode_t node;
  err = cudaGraphAddNode(&node, g, nullptr, 0, &params);
  if (err != cudaSuccess) {
    destroy(e);
    return set_error(FKC_ECUDA, "cudaGraphAddNode(while): %s", cudaGetErrorString(err));
  }
  cudaGraph_t loop_body = params.conditional.phGraph_out[0];

  cudaStream_t cs = nullptr;
  err = cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking);
  if (err != cudaSuccess) {
    destroy(e);
    return set_error(FKC_ECUDA, "cudaStreamCreateWithFlags: %s", cudaGetErrorString(err));
  }
  err = cudaStreamBeginCaptureToGraph(cs, loop_body, nullptr, nullptr, 0,
                                      cudaStreamCaptureModeRelaxed);
  int rc = FKC_OK;
  if (err != cudaSuccess) {
    rc = set_error(FKC_ECUDA, "cudaStreamBeginCaptureToGraph: %s", cudaGetErrorString(err));
  } else {
    t_capturing = true;
    const uint64_t before = capture_launch_count();
    rc = body(cs);
    if (rc == FKC_OK) {
      loop_ctl_kernel<<<1, 1, 0, cs>>>(handle, ctl, shift);
      err = cudaGetLastError();
      if (err != cudaSuccess)
        rc = set_error(FKC_ECUDA, "loop control launch: %s", cudaGetErrorString(err));
    }
    e.kernels_per_iter = static_cast<int>(capture_launch_count() - before) + 1;
    t_capturing = false;
    cudaGraph_t captured = nullptr;
    err = cudaStreamEndCapture(cs, &captured);
    if (rc == FKC_OK && err != cudaSuccess)
      rc = set_error(FKC_ECUDA, "cudaStreamEndCapture: %s", cudaGetErrorString(err));
  }
  cudaStreamDestroy(cs);
  if (rc == FKC_OK) {
    err = cudaGraphInstantiate(&e.exec, g, 0);
    if (err != cudaSuccess)
      rc = set_error(FKC_ECUDA, "cudaGraphInstantiate: %s", cudaGetErrorString(err));
  }
  if (rc != FKC_OK) {
    cudaGetLastError();
    destroy(e);
    return rc;
  }
  *out = e;
  return FKC_OK;
}

}  // namespace

bool count_captured_launch(int n) {
  if (!t_capturing) return false;
  t_captured += static_cast<uint64_t>(n);
  return true;
}

uint64_t capture_launch_count() { return t_captured; }

int run_lloyd_graph(const LloydGraphKey& key, const LoopBody& body, LoopCtl* ctl,
                    const float* shift, int max_iters, float tol, int32_t* n_iters_out,
                    cudaStream_t stream) {
  std::lock_guard<std::mutex> lk(g_mu);
  Entry* hit = nullptr;
  for (Entry& e : g_cache)
    if (same_key(e.key, key)) hit = &e;
  if (hit == nullptr) {
    Entry e;
    FKC_TRY(build(key, body, ctl, shift, &e));
    if (g_cache.size() >= kMaxGraphs) {
      size_t lru = 0;
      for (size_t i = 1; i < g_cache.size(); ++i)
        if (g_cache[i].last_use < g_cache[lru].last_use) lru = i;
      destroy(g_cache[lru]);
      g_cache.erase(g_cache.begin() + static_cast<std::ptrdiff_t>(lru));
    }
    g_cache.push_back(e);
    hit = &g_cache.back();
  }
  hit->last_use = ++g_tick;
  loop_init_kernel<<<1, 1, 0, stream>>>(ctl, max_iters, tol);
  FKC_CUDA_TRY(cudaGetLastError());
  FKC_CUDA_TRY(cudaGraphLaunch(hit->exec, stream));
  if (n_iters_out != nullptr)
    FKC_CUDA_TRY(cudaMemcpyAsync(n_iters_out, &ctl->n_iters, sizeof(int32_t),
                                 cudaMemcpyDeviceToDevice, stream));
  // Kernels run by this launch: at most max_iters iterations (fewer when tol stops
  // the loop early) plus the control-block initialisation.
  count_launches(1 + hit->kernels_per_iter * max_iters);
  return FKC_OK;
}

}  // namespace fkc
