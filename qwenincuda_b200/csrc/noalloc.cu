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
// looked up with cudaGetSymbolAddress once per device and CUDA context, on the first
// call made with that device current (again after a cudaDeviceReset, which gives the
// device a new context); make that first call before starting any stream capture.
// Every call uses the same array: the merge counters are cleared at the start of each
// call, and calls that overlap on the GPU (different streams, or different host
// threads on one device) race on it. The device status word (byte 0) is not cleared
// by a call: bad-page, bad-length and timeout bits accumulate until
// qic_noalloc_status reads and clears them.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "qic_internal.h"

namespace {

constexpr size_t kScratchBytes = size_t(2) << 20;  // status word + counters + partial slots

// zero-initialised when the module loads: the status word starts clear
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn g_ctx_get_current = nullptr;
std::once_flag g_ctx_once;

// The CUDA context current on this thread (nullptr if the driver entry point is missing).
CUcontext current_context() {
  std::call_once(g_ctx_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
  });
  CUcontext c = nullptr;
  if (g_ctx_get_current == nullptr || g_ctx_get_current(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

struct ScratchAddress {
  void* ptr = nullptr;
  CUcontext ctx = nullptr;  // context the address belongs to
  bool ready = false;
};
std::mutex g_scratch_mutex;
ScratchAddress g_scratch[64];

// Device address of g_noalloc_scratch on the current device, looked up once per
// device and context. A thread with no context bound yet (its first CUDA call) looks
// the address up again; cudaGetSymbolAddress binds the device's primary context, whose
// handle is then recorded with the address.
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return QIC_ERROR_CUDA;
  if (dev < 0 || dev >= 64) return QIC_ERROR_NOT_SUPPORTED;
  const CUcontext ctx = current_context();
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  ScratchAddress& s = g_scratch[dev];
  if (!s.ready || ctx == nullptr || s.ctx != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return QIC_ERROR_CUDA;
    s.ptr = p;
    s.ctx = current_context();
    s.ready = true;
  }
  *out = s.ptr;
  return QIC_SUCCESS;
}

}  // namespace

extern "C" size_t qic_noalloc_scratch_bytes(void) { return kScratchBytes; }

extern "C" int qic_decode_attention_noalloc(const qic_decode_args* args, qic_stream_t stream) {
  if (args == nullptr) return QIC_ERROR_INVALID_VALUE;
  void* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc != QIC_SUCCESS) return rc;
  // The merge counters must start at zero (a call that timed out can leave them
  // set); the status word keeps earlier bits until qic_noalloc_status reads it, and
  // partial slots are always written before they are read.
  cudaError_t e = cudaMemsetAsync(static_cast<char*>(scratch) + qic::kWsHeader, 0,
                                  qic::kWsPartialOffset - qic::kWsHeader, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return QIC_ERROR_CUDA;
  qic_decode_args a = *args;
  a.workspace = scratch;
  a.workspace_bytes = kScratchBytes;
  // shapes whose partials do not fit the fixed array come back as QIC_ERROR_WORKSPACE
  return qic_decode_attention(&a, stream);
}

extern "C" int qic_noalloc_status(qic_stream_t stream, int* dev_status) {
  if (dev_status == nullptr) return QIC_ERROR_INVALID_VALUE;
  void* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc != QIC_SUCCESS) return rc;
  // read and clear word 0, in stream order after the calls made on `stream`
  return qic_workspace_status(scratch, stream, dev_status);
}
