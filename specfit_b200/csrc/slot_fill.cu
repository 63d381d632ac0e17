// K5: expert-slot fill from pinned host memory.
//
// Replaces `slot.tensor.copy_(source, non_blocking=True)` on the cache's copy
// stream (src/specfit/runtime/gpu_expert_cache.py:556-561).  The copy engines
// do this work; no SM kernel is involved.  One cudaMemcpyAsync per copy, in
// submission order, so the caller's event recorded after the batch orders
// every copy in it.
#include "common.cuh"

extern "C" int sf_slot_fill_batch(void* const* dst, const void* const* src, const size_t* bytes,
                                  int n, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(n >= 0, "n must be non-negative");
  if (n == 0) return SF_OK;
  SF_CHECK_ARG(dst && src && bytes, "null pointer argument");
  cudaStream_t s = as_stream(stream);
  for (int i = 0; i < n; ++i) {
    SF_CHECK_ARG(dst[i] && src[i], "null pointer in copy %d", i);
    if (bytes[i] == 0) continue;
    SF_CHECK_CUDA(cudaMemcpyAsync(dst[i], src[i], bytes[i], cudaMemcpyHostToDevice, s));
  }
  return SF_OK;
}
