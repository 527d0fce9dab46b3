// qic_decode_attention_noalloc: decode attention whose split-KV scratch lives in a
// fixed array inside this library instead of memory the caller allocates.
//
// Who needs it: callers written against the reference's kernel interface
// (include/kernels.cuh), such as a per-token decode loop, have no workspace to hand
// over, and some of them must not call cudaMalloc: the allocation synchronises the
// device in the middle of the token loop, and hosts that reserve all HBM up front
// for their own page pool or allocator leave nothing for the library to allocate.
//
// The scratch is a file-scope __device__ array of kScratchBytes (2 MiB) that every
// GPU loading this library holds until the process exits. Its device address is
// looked up with cudaGetSymbolAddress once per device, on the first call made with
// that device current; make that first call before starting any stream capture.
// Every call uses the same array: the status word and merge counters are cleared at
// the start of each call, and calls that overlap on the GPU (different streams, or
// different host threads on one device) race on it.
#include <cuda_runtime.h>

#include <mutex>

#include "qic_internal.h"

namespace {

constexpr size_t kScratchBytes = size_t(2) << 20;  // status word + counters + partial slots

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

struct ScratchAddress {
  void* ptr = nullptr;
  bool ready = false;
};
std::mutex g_scratch_mutex;
ScratchAddress g_scratch[64];

// Device address of g_noalloc_scratch on the current device (set up once per device).
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return QIC_ERROR_CUDA;
  if (dev < 0 || dev >= 64) return QIC_ERROR_NOT_SUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch[dev].ready) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return QIC_ERROR_CUDA;
    g_scratch[dev].ptr = p;
    g_scratch[dev].ready = true;
  }
  *out = g_scratch[dev].ptr;
  return QIC_SUCCESS;
}

}  // namespace

extern "C" size_t qic_noalloc_scratch_bytes(void) { return kScratchBytes; }

extern "C" int qic_decode_attention_noalloc(const qic_decode_args* args, qic_stream_t stream) {
  if (args == nullptr) return QIC_ERROR_INVALID_VALUE;
  void* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc != QIC_SUCCESS) return rc;
  // The status word and the merge counters must start at zero; partial slots are
  // always written before they are read.
  cudaError_t e = cudaMemsetAsync(scratch, 0, qic::kWsPartialOffset, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return QIC_ERROR_CUDA;
  qic_decode_args a = *args;
  a.workspace = scratch;
  a.workspace_bytes = kScratchBytes;
  // shapes whose partials do not fit the fixed array come back as QIC_ERROR_WORKSPACE
  return qic_decode_attention(&a, stream);
}
