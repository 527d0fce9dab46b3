// C-ABI entry points of include/qic.h: argument checks, TMA descriptor encoding,
// workspace layout and dispatch to the sm_100a kernels.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "qic_internal.h"

namespace {

thread_local int g_last_cuda_error = 0;

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return QIC_SUCCESS;
  g_last_cuda_error = static_cast<int>(e);
  return QIC_ERROR_CUDA;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool aligned2(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 1u) == 0; }

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
using AddrRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

EncodeTiledFn g_encode = nullptr;
AddrRangeFn g_addr_range = nullptr;
std::once_flag g_driver_once;

void load_driver_entry_points() {
  std::call_once(g_driver_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_addr_range = reinterpret_cast<AddrRangeFn>(fn);
  });
}

int sm_count() {
  static int counts[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (counts[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    counts[dev] = n;
  }
  return counts[dev];
}

uint64_t timeout_ns() {
  static uint64_t t = []() -> uint64_t {
    const char* s = std::getenv("QIC_TIMEOUT_MS");
    if (s != nullptr) {
      long v = std::strtol(s, nullptr, 10);
      if (v > 0) return static_cast<uint64_t>(v) * 1000000ull;
    }
    return qic::kDefaultTimeoutNs;
  }();
  return t;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Bytes of the allocation containing `p` from p to its end, 0 if unknown.
size_t bytes_to_allocation_end(const void* p) {
  load_driver_entry_points();
  if (g_addr_range == nullptr || p == nullptr) return 0;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (g_addr_range(&base, &size, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS) return 0;
  const uintptr_t end = static_cast<uintptr_t>(base) + size;
  const uintptr_t at = reinterpret_cast<uintptr_t>(p);
  return end > at ? static_cast<size_t>(end - at) : 0;
}

int encode_kv_map(CUtensorMap* map, int dtype, const void* base, int64_t tokens, int kv_dim, int box_h) {
  load_driver_entry_points();
  if (g_encode == nullptr) return QIC_ERROR_CUDA;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kv_dim), static_cast<cuuint64_t>(tokens)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(kv_dim) * 2};
  cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_h)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = g_encode(map, dtype == QIC_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QIC_SUCCESS : QIC_ERROR_INVALID_VALUE;
}

bool valid_dtype(int d) { return d == QIC_DTYPE_F16 || d == QIC_DTYPE_BF16; }
bool supported_head_dim(int d) { return d == 64 || d == 128 || d == 256; }

}  // namespace

extern "C" {

const char* qic_status_string(int status) {
  switch (status) {
    case QIC_SUCCESS: return "success";
    case QIC_ERROR_INVALID_VALUE: return "invalid value";
    case QIC_ERROR_NOT_SUPPORTED: return "shape not supported by the compiled kernels";
    case QIC_ERROR_MISALIGNED: return "pointer or stride not 16-byte aligned";
    case QIC_ERROR_WORKSPACE: return "workspace missing or too small";
    case QIC_ERROR_CUDA: return "CUDA error";
    case QIC_ERROR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case QIC_ERROR_BAD_PAGE: return "page-table entry outside the cache";
    case QIC_ERROR_PEER: return "peer exchange set-up failed";
    default: return "unknown status";
  }
}

int qic_last_cuda_error(void) { return g_last_cuda_error; }

int qic_version(void) { return 100; }

int qic_head_rmsnorm(int dtype, const void* x, const void* weight, int num_heads, int head_dim, float eps, void* out,
                     qic_stream_t stream) {
  if (!valid_dtype(dtype) || !x || !weight || !out || num_heads <= 0 || head_dim <= 0 || head_dim > 8192)
    return QIC_ERROR_INVALID_VALUE;
  return cuda_status(qic::launch_head_rmsnorm(dtype, x, weight, num_heads, head_dim, eps, out,
                                              reinterpret_cast<cudaStream_t>(stream)));
}

int qic_rope_inplace(int dtype, void* x, int num_heads, int head_dim, int position, float rope_theta,
                     qic_stream_t stream) {
  if (!valid_dtype(dtype) || !x || num_heads <= 0 || head_dim <= 0 || (head_dim & 1)) return QIC_ERROR_INVALID_VALUE;
  return cuda_status(qic::launch_rope_inplace(dtype, x, num_heads, head_dim, position, rope_theta,
                                              reinterpret_cast<cudaStream_t>(stream)));
}

int qic_sigmoid_mul_inplace(int dtype, void* x, const void* gate, int n, qic_stream_t stream) {
  if (!valid_dtype(dtype) || !x || !gate || n < 0) return QIC_ERROR_INVALID_VALUE;
  if (n == 0) return QIC_SUCCESS;
  return cuda_status(qic::launch_sigmoid_mul_inplace(dtype, x, gate, n, reinterpret_cast<cudaStream_t>(stream)));
}

int qic_kv_append(int dtype, const void* k_new, const void* v_new, const void* k_norm_w, float eps, float rope_theta,
                  int position, void* k_cache, void* v_cache, const int32_t* page_table, int page_size,
                  int64_t cache_tokens, int num_kv_heads, int head_dim, qic_stream_t stream) {
  if (!valid_dtype(dtype) || !k_new || !v_new || !k_norm_w || !k_cache || !v_cache || num_kv_heads <= 0 ||
      position < 0 || cache_tokens <= 0)
    return QIC_ERROR_INVALID_VALUE;
  if (!supported_head_dim(head_dim)) return QIC_ERROR_NOT_SUPPORTED;
  if (page_table != nullptr && page_size <= 0) return QIC_ERROR_INVALID_VALUE;
  if (page_table == nullptr && position >= cache_tokens) return QIC_ERROR_INVALID_VALUE;
  if (!aligned16(k_new) || !aligned16(v_new) || !aligned16(k_norm_w) || !aligned16(k_cache) || !aligned16(v_cache))
    return QIC_ERROR_MISALIGNED;
  return cuda_status(qic::launch_kv_append(dtype, k_new, v_new, k_norm_w, eps, rope_theta, position, page_table,
                                           page_size, cache_tokens, k_cache, v_cache, num_kv_heads, head_dim,
                                           reinterpret_cast<cudaStream_t>(stream)));
}

size_t qic_decode_workspace_bytes(int num_heads, int num_kv_heads, int head_dim, int max_seq_len) {
  if (num_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || max_seq_len < 0) return 0;
  const int G = num_heads / num_kv_heads;
  const int n_stages = (max_seq_len + qic::kStageTokens - 1) / qic::kStageTokens;
  const int splits = std::max(1, std::min(qic::kMaxSplits, n_stages));
  return qic::kWsHeader + align256(static_cast<size_t>(num_kv_heads) * sizeof(int)) +
         static_cast<size_t>(num_kv_heads) * splits * qic::partial_floats(G, head_dim) * sizeof(float);
}

int qic_workspace_init(void* workspace, size_t bytes, qic_stream_t stream) {
  if (workspace == nullptr || bytes < qic::kWsHeader) return QIC_ERROR_INVALID_VALUE;
  return cuda_status(cudaMemsetAsync(workspace, 0, bytes, reinterpret_cast<cudaStream_t>(stream)));
}

int qic_workspace_status(void* workspace, qic_stream_t stream, int* dev_status) {
  if (workspace == nullptr || dev_status == nullptr) return QIC_ERROR_INVALID_VALUE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemsetAsync(workspace, 0, sizeof(int), s);
  if (e != cudaSuccess) return cuda_status(e);
  *dev_status = v;
  return QIC_SUCCESS;
}

int qic_decode_attention(const qic_decode_args* a, qic_stream_t stream) {
  if (a == nullptr || !valid_dtype(a->dtype)) return QIC_ERROR_INVALID_VALUE;
  const int H = a->num_heads, Hkv = a->num_kv_heads, D = a->head_dim, S = a->seq_len;
  if (H <= 0 || Hkv <= 0 || H % Hkv != 0 || S < 0 || !a->q || !a->out || !a->k_cache || !a->v_cache)
    return QIC_ERROR_INVALID_VALUE;
  const int G = H / Hkv;
  if (!supported_head_dim(D) || G > qic::kMaxGroup) return QIC_ERROR_NOT_SUPPORTED;
  const bool paged = a->page_table != nullptr;
  if (paged && (a->page_size <= 0 || a->page_size % 8 != 0)) return QIC_ERROR_NOT_SUPPORTED;
  const bool fuse_q = (a->flags & QIC_FUSE_Q_PROLOGUE) != 0;
  const bool fuse_app = (a->flags & QIC_FUSE_APPEND) != 0;
  if (fuse_q && !a->q_norm_w) return QIC_ERROR_INVALID_VALUE;
  if (fuse_app && (!a->k_new || !a->v_new || !a->k_norm_w || S < 1)) return QIC_ERROR_INVALID_VALUE;
  if (!aligned16(a->q) || !aligned16(a->k_cache) || !aligned16(a->v_cache) || !aligned2(a->out) ||
      (a->gate && !aligned2(a->gate)) || (fuse_q && !aligned16(a->q_norm_w)) ||
      (fuse_app && (!aligned16(a->k_new) || !aligned16(a->v_new) || !aligned16(a->k_norm_w))) ||
      (a->workspace && !aligned16(a->workspace)))
    return QIC_ERROR_MISALIGNED;
  const int kv_dim = Hkv * D;
  const size_t row_bytes = static_cast<size_t>(kv_dim) * 2;
  int64_t cache_tokens = a->cache_tokens;
  if (cache_tokens <= 0) {
    const size_t kb = bytes_to_allocation_end(a->k_cache), vb = bytes_to_allocation_end(a->v_cache);
    cache_tokens = static_cast<int64_t>(std::min(kb, vb) / row_bytes);
    if (cache_tokens <= 0 && !paged) cache_tokens = S;
  }
  if (cache_tokens <= 0 || cache_tokens > (int64_t(1) << 31) - 1) return QIC_ERROR_INVALID_VALUE;
  if (!paged && S > cache_tokens) return QIC_ERROR_INVALID_VALUE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (S == 0) {  // no tokens: the reference writes acc * 1e12 = 0
    return cuda_status(cudaMemsetAsync(a->out, 0, static_cast<size_t>(H) * D * 2, st));
  }

  qic::AttnParams p;
  std::memset(&p, 0, sizeof(p));
  int box_h = qic::kStageTokens;
  if (paged) {
    box_h = a->page_size & (-a->page_size);  // largest power of two dividing P
    if (box_h > qic::kStageTokens) box_h = qic::kStageTokens;
  }
  int lbh = 0;
  while ((1 << lbh) < box_h) ++lbh;
  int rc = encode_kv_map(&p.tm_k, a->dtype, a->k_cache, cache_tokens, kv_dim, box_h);
  if (rc == QIC_SUCCESS) rc = encode_kv_map(&p.tm_v, a->dtype, a->v_cache, cache_tokens, kv_dim, box_h);
  if (rc != QIC_SUCCESS) return rc;

  const int n_stages = (S + qic::kStageTokens - 1) / qic::kStageTokens;
  int n_splits = a->num_splits;
  if (n_splits <= 0) n_splits = std::max(1, sm_count() / Hkv);
  n_splits = std::max(1, std::min(std::min(n_splits, n_stages), qic::kMaxSplits));
  int* status = nullptr;
  int* counters = nullptr;
  float* part = nullptr;
  if (a->workspace == nullptr) {
    n_splits = 1;
  } else {
    const size_t need = qic::kWsHeader + align256(static_cast<size_t>(Hkv) * sizeof(int)) +
                        static_cast<size_t>(Hkv) * n_splits * qic::partial_floats(G, D) * sizeof(float);
    if (a->workspace_bytes < need) return QIC_ERROR_WORKSPACE;
    char* ws = static_cast<char*>(a->workspace);
    status = reinterpret_cast<int*>(ws);
    counters = reinterpret_cast<int*>(ws + qic::kWsHeader);
    part = reinterpret_cast<float*>(ws + qic::kWsHeader + align256(static_cast<size_t>(Hkv) * sizeof(int)));
  }

  p.q = a->q;
  p.gate = a->gate;
  p.out = a->out;
  p.k_cache = a->k_cache;
  p.v_cache = a->v_cache;
  p.page_table = a->page_table;
  p.q_norm_w = a->q_norm_w;
  p.k_norm_w = a->k_norm_w;
  p.k_new = a->k_new;
  p.v_new = a->v_new;
  p.part = part;
  p.counters = counters;
  p.status = status;
  p.cache_tokens = cache_tokens;
  p.H = H;
  p.Hkv = Hkv;
  p.G = G;
  p.head_dim = D;
  p.seq_len = S;
  p.page_size = paged ? a->page_size : 0;
  p.box_h = box_h;
  p.log2_box_h = lbh;
  p.n_stages = n_stages;
  p.n_splits = n_splits;
  p.flags = static_cast<int>(a->flags & (QIC_FUSE_Q_PROLOGUE | QIC_FUSE_APPEND));
  p.eps = a->eps;
  p.theta = a->rope_theta;
  p.scale_log2 = static_cast<float>((1.0 / std::sqrt(static_cast<double>(D))) * 1.4426950408889634);
  p.timeout_ns = timeout_ns();
  return cuda_status(qic::launch_decode_attention(a->dtype, D, p, st));
}

int qic_gated_delta_decode(const qic_gdn_args* a, qic_stream_t stream) {
  if (a == nullptr || !valid_dtype(a->dtype)) return QIC_ERROR_INVALID_VALUE;
  if (a->num_k_heads <= 0 || a->num_v_heads <= 0 || a->num_v_heads % a->num_k_heads != 0)
    return QIC_ERROR_INVALID_VALUE;
  const int rep = a->num_v_heads / a->num_k_heads;
  if (a->k_head_dim != 128 || a->v_head_dim != 128 || (rep != 1 && rep != 2 && rep != 4) || a->conv_kernel < 1 ||
      a->conv_kernel > 8)
    return QIC_ERROR_NOT_SUPPORTED;
  if (!a->qkv || !a->z || !a->b || !a->a || !a->conv_w || !a->dt_bias || !a->a_log || !a->norm_w ||
      !a->conv_state || !a->recurrent_state || !a->out)
    return QIC_ERROR_INVALID_VALUE;
  if (!aligned16(a->recurrent_state) || !aligned2(a->qkv) || !aligned2(a->z) || !aligned2(a->out) ||
      (reinterpret_cast<uintptr_t>(a->conv_state) & 3u))
    return QIC_ERROR_MISALIGNED;
  return cuda_status(qic::launch_gated_delta(*a, reinterpret_cast<cudaStream_t>(stream)));
}

}  // extern "C"
