// Row work sized by a count that only the device knows, inside one captured CUDA graph.
//
// After the loop's first passes most tokens have halted, so the per-token work of a later pass
// (the feed-forward block) touches a few percent of the rows. The active rows are packed at the
// front of a buffer of `cap` rows (the compaction kernels) and their number is an int32 on the
// device. The buffer's prefixes [0, end_k) with
//   end_0 = first, end_k = 2 end_{k-1}   (the last one clamped to cap)
// are the buckets: while a stream is being captured, one SWITCH conditional node is added whose
// body k holds the work over rows [0, end_k), and a kernel captured just before it sets the node's
// value when the graph runs: the smallest k with end_k >= count, or no body at all for a count of
// zero. A replay therefore runs the work of at most twice the active rows (at least `first` rows)
// with one launch per operation. Rows between the count and end_k must hold finite values (the
// gather kernels zero them); rows past end_k are never read.
#include "common.cuh"

namespace vb {
namespace {

constexpr int MAX_BUCKETS = 24;

int bucket_count(int cap, int first) {
  if (cap <= 0 || first <= 0) return 0;
  int n = 1;
  for (long long end = first; end < cap; end *= 2) ++n;
  return n;
}

__global__ void bucket_select_kernel(const int* __restrict__ count, cudaGraphConditionalHandle handle, int n,
                                     int first, int cap) {
  const int c = *count;
  unsigned value = (unsigned)n;  // no body: nothing is active
  if (c > 0) {
    long long end = first;
    unsigned k = 0;
    while (end < c && end < cap) {
      end *= 2;
      ++k;
    }
    value = k;
  }
  cudaGraphSetConditional(handle, value);
}

}  // namespace
}  // namespace vb

using namespace vb;

extern "C" int vb_slab_count(int cap, int first) { return bucket_count(cap, first); }

extern "C" int vb_slab_switch(const int* count, int cap, int first, void* stream, void** bodies) {
  const int n = bucket_count(cap, first);
  VB_REQUIRE(n > 0 && n <= MAX_BUCKETS, "slab_switch: %d buckets for cap=%d first=%d (1..%d)", n, cap, first,
             MAX_BUCKETS);
  VB_REQUIRE(count != nullptr && bodies != nullptr, "slab_switch: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  cudaStreamCaptureStatus status;
  cudaGraph_t graph = nullptr;
  VB_CUDA_CHECK(cudaStreamGetCaptureInfo(st, &status, nullptr, &graph), "slab_switch: capture info");
  VB_REQUIRE(status == cudaStreamCaptureStatusActive && graph != nullptr, "slab_switch: the stream is not being captured");
  cudaGraphConditionalHandle handle;
  VB_CUDA_CHECK(cudaGraphConditionalHandleCreate(&handle, graph, (unsigned)n, cudaGraphCondAssignDefault),
                "slab_switch: handle");
  bucket_select_kernel<<<1, 1, 0, st>>>(count, handle, n, first, cap);
  VB_LAUNCH_CHECK("slab_switch");
  const cudaGraphNode_t* deps = nullptr;
  size_t ndeps = 0;
  VB_CUDA_CHECK(cudaStreamGetCaptureInfo(st, &status, nullptr, &graph, &deps, &ndeps), "slab_switch: capture info");
  cudaGraphNodeParams p{};
  p.type = cudaGraphNodeTypeConditional;
  p.conditional.handle = handle;
  p.conditional.type = cudaGraphCondTypeSwitch;
  p.conditional.size = (unsigned)n;
  cudaGraphNode_t node;
  VB_CUDA_CHECK(cudaGraphAddNode(&node, graph, deps, ndeps, &p), "slab_switch: conditional node");
  VB_CUDA_CHECK(cudaStreamUpdateCaptureDependencies(st, &node, 1, cudaStreamSetCaptureDependencies),
                "slab_switch: dependencies");
  for (int k = 0; k < n; ++k) bodies[k] = (void*)p.conditional.phGraph_out[k];
  return VB_OK;
}

extern "C" int vb_slab_begin(void* body, void* body_stream) {
  VB_REQUIRE(body != nullptr && body_stream != nullptr, "slab_begin: null body or stream");
  VB_CUDA_CHECK(cudaStreamBeginCaptureToGraph((cudaStream_t)body_stream, (cudaGraph_t)body, nullptr, nullptr, 0,
                                              cudaStreamCaptureModeRelaxed),
                "slab_begin: body capture");
  return VB_OK;
}

extern "C" int vb_slab_close(void* body_stream) {
  cudaGraph_t body = nullptr;
  VB_CUDA_CHECK(cudaStreamEndCapture((cudaStream_t)body_stream, &body), "slab_close: body capture");
  return VB_OK;
}
