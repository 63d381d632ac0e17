// Conditional sections of a captured CUDA graph.
//
// A device-managed expert cache plans ceil(E / S) waves per layer, but a
// layer whose routed experts fit its slots needs only the first: the later
// waves' fill and grouped-SwiGLU launches find nothing to do and return.
// Inside a captured verify pass those empty launches still cost ~3 us per
// wave (measured on a B200), so the later waves of each layer are captured
// into the body of an IF node whose condition the layer's plan kernel sets
// (cudaGraphSetConditional) to "some wave after the first has experts".
//
//   sf_capture_body_stream  the stream bodies are captured on (one per device)
//   sf_capture_cond_handle  a handle of the graph `stream` is capturing into
//   sf_capture_if_begin     adds the IF node behind the stream's current
//                           dependencies, makes it the stream's dependency and
//                           starts capturing `body_stream` into its body
//   sf_capture_if_end       ends the body capture and adds a plain join kernel
//                           on `stream`, so a following kernel launched with
//                           programmatic serialization depends on a kernel node
//
// Outside a capture none of this is used: every wave is launched.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "common.cuh"

namespace sf {
namespace {

__global__ void capture_join_kernel() {}

int capturing_graph(cudaStream_t s, cudaGraph_t* graph, const cudaGraphNode_t** deps, size_t* n) {
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  const cudaGraphEdgeData* edges = nullptr;
  SF_CHECK_CUDA(cudaStreamGetCaptureInfo_v3(s, &st, nullptr, graph, deps, &edges, n));
  if (st != cudaStreamCaptureStatusActive) return set_error(SF_ERR_STATE, "the stream is not capturing");
  return SF_OK;
}

}  // namespace
}  // namespace sf

// A stream of the current device that only conditional bodies are captured
// on: created once per device (non-blocking) and kept until exit, so it can
// never be the stream whose capture it is nested in.
extern "C" int sf_capture_body_stream(void** stream) {
  using namespace sf;
  SF_CHECK_ARG(stream, "null pointer argument");
  static std::mutex mu;
  static cudaStream_t streams[64] = {};
  int dev = 0;
  SF_CHECK_CUDA(cudaGetDevice(&dev));
  SF_CHECK_ARG(dev >= 0 && dev < 64, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (streams[dev] == nullptr) SF_CHECK_CUDA(cudaStreamCreateWithFlags(&streams[dev], cudaStreamNonBlocking));
  *stream = streams[dev];
  return SF_OK;
}

extern "C" int sf_capture_cond_handle(void* stream, uint64_t* handle) {
  using namespace sf;
  SF_CHECK_ARG(handle, "null pointer argument");
  cudaGraph_t graph = nullptr;
  const cudaGraphNode_t* deps = nullptr;
  size_t n = 0;
  if (int rc = capturing_graph(as_stream(stream), &graph, &deps, &n)) return rc;
  cudaGraphConditionalHandle h = 0;
  // Reset to 0 at every launch of the graph; the plan kernel sets it.
  SF_CHECK_CUDA(cudaGraphConditionalHandleCreate(&h, graph, 0, cudaGraphCondAssignDefault));
  *handle = (uint64_t)h;
  return SF_OK;
}

extern "C" int sf_capture_if_begin(void* stream, void* body_stream, uint64_t handle) {
  using namespace sf;
  SF_CHECK_ARG(handle != 0, "no conditional handle");
  SF_CHECK_ARG(body_stream != stream && body_stream != nullptr, "the body needs its own stream");
  cudaStream_t s = as_stream(stream);
  cudaGraph_t graph = nullptr;
  const cudaGraphNode_t* deps = nullptr;
  size_t n = 0;
  if (int rc = capturing_graph(s, &graph, &deps, &n)) return rc;
  cudaGraphNodeParams p = {};
  p.type = cudaGraphNodeTypeConditional;
  p.conditional.handle = (cudaGraphConditionalHandle)handle;
  p.conditional.type = cudaGraphCondTypeIf;
  p.conditional.size = 1;
  cudaGraphNode_t node = nullptr;
  // Full (not programmatic) dependencies on what the stream has captured so far.
  SF_CHECK_CUDA(cudaGraphAddNode(&node, graph, deps, n, &p));
  cudaGraph_t body = p.conditional.phGraph_out[0];
  SF_CHECK_CUDA(cudaStreamUpdateCaptureDependencies(s, &node, 1, cudaStreamSetCaptureDependencies));
  SF_CHECK_CUDA(cudaStreamBeginCaptureToGraph(as_stream(body_stream), body, nullptr, nullptr, 0,
                                              cudaStreamCaptureModeRelaxed));
  return SF_OK;
}

extern "C" int sf_capture_if_end(void* stream, void* body_stream) {
  using namespace sf;
  cudaGraph_t body = nullptr;
  SF_CHECK_CUDA(cudaStreamEndCapture(as_stream(body_stream), &body));
  capture_join_kernel<<<1, 32, 0, as_stream(stream)>>>();
  SF_CHECK_LAUNCH();
  return SF_OK;
}
