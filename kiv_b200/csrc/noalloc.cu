// Allocation-free retrieval attention: kiv_retrieve_attend with its scratch
// in a fixed, file-scope device array instead of a caller-provided workspace.
//
// Who needs it: callers that cannot allocate device memory at the point where
// they run a decode step -- e.g. a serving engine that hands out all GPU memory
// to its own KV-block pool at start-up and forbids cudaMalloc afterwards, a
// plugin host (an inference runtime's custom-op interface) that gives a plugin
// no allocator and no workspace hook, or a latency-critical loop where a
// cudaMalloc would synchronize the device.  Such callers still own the store,
// the query, the selection and the output buffers; only the scratch is
// provided here.
//
// Limits and sharing:
// * the scratch is KIV_NOALLOC_SCRATCH_BYTES (32 MiB) per GPU, reserved in
//   every GPU that loads the library until the process exits; a store/query
//   shape whose workspace exceeds it is rejected with KIV_ERR_CAPACITY;
// * every call on a device uses the same array, which keeps the last call's
//   contents.  Each call therefore first clears, on its stream, the span of
//   the scratch that must start at zero (page marks through the select
//   histograms and statistics) -- whatever shape, failure or interruption the
//   previous call left behind.  The clear is part of every call, so it is
//   also recorded when the call is captured into a CUDA graph;
// * two calls whose work overlaps on the GPU (different streams with no
//   ordering between them, or graph replays running beside eager calls) race
//   on the array and give wrong results;
// * the first call on a device looks up the array's device address
//   (cudaGetSymbolAddress, with that device current); make that first call
//   before any stream capture.
#include <mutex>

#include "internal.h"

namespace kiv {

static __device__ __align__(256) unsigned char g_noalloc_scratch[KIV_NOALLOC_SCRATCH_BYTES];

static constexpr int kMaxDevices = 64;
static void *g_scratch_addr[kMaxDevices] = {};
static std::mutex g_scratch_mu;

// Device address of the scratch array for the current device (host-side
// `g_noalloc_scratch` is only a stand-in symbol, never a device address).
static kiv_status scratch_address(void **out) {
  int dev = -1;
  kiv_status rc = cuda_status(cudaGetDevice(&dev), "noalloc: cudaGetDevice");
  if (rc != KIV_OK) return rc;
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("noalloc: device %d out of range", dev);
    return KIV_ERR_ARG;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void *p = nullptr;
    rc = cuda_status(cudaGetSymbolAddress(&p, g_noalloc_scratch), "noalloc: cudaGetSymbolAddress");
    if (rc != KIV_OK) return rc;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return KIV_OK;
}

}  // namespace kiv

extern "C" kiv_status kiv_retrieve_attend_noalloc(const kiv_store *st, const kiv_query *q,
                                                  const kiv_mask *mask, int32_t *sel, void *out,
                                                  void *stream) {
  using namespace kiv;
  const size_t need = kiv_workspace_bytes(st, q);
  if (need == 0) {
    set_error("noalloc: invalid store or query descriptor");
    return KIV_ERR_ARG;
  }
  if (need > KIV_NOALLOC_SCRATCH_BYTES) {
    set_error("noalloc: this shape needs %zu bytes of scratch, more than the fixed %zu bytes; "
              "use kiv_retrieve_attend with a caller-provided workspace",
              need, (size_t)KIV_NOALLOC_SCRATCH_BYTES);
    return KIV_ERR_CAPACITY;
  }
  void *scratch = nullptr;
  kiv_status rc = scratch_address(&scratch);
  if (rc != KIV_OK) return rc;
  int64_t lay[10];
  rc = kiv_workspace_layout(st, q, lay);
  if (rc != KIV_OK) return rc;
  // the regions that must start at zero lie between the page marks and the
  // attention partials: clear that span on every call
  rc = cuda_status(cudaMemsetAsync(static_cast<unsigned char *>(scratch) + lay[1], 0, (size_t)(lay[5] - lay[1]),
                                   (cudaStream_t)stream),
                   "noalloc: clear zero-start regions");
  if (rc != KIV_OK) return rc;
  return kiv_retrieve_attend(st, q, mask, scratch, KIV_NOALLOC_SCRATCH_BYTES, 0, sel, out, stream);
}
