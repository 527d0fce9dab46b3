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
#include <vector>

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

// K/V cache view for TMA: a 3D tensor {64 elements, tokens, kv_dim/64 chunks} whose
// chunk dimension has a 128-byte stride, so one box {64, box_h, head_dim/64} copies
// every 64-element chunk of one head for box_h token rows. Shared memory receives the
// box chunk-major ([chunk][token][128 B], 128-byte swizzle), the layout the consumer
// warps index.
int encode_kv_map_uncached(CUtensorMap* map, int dtype, const void* base, int64_t tokens, int kv_dim, int head_dim,
                           int box_h) {
  load_driver_entry_points();
  if (g_encode == nullptr) return QIC_ERROR_CUDA;
  cuuint64_t dims[3] = {64u, static_cast<cuuint64_t>(tokens), static_cast<cuuint64_t>(kv_dim / 64)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(kv_dim) * 2, 128u};
  cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(box_h), static_cast<cuuint32_t>(head_dim / 64)};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = g_encode(map, dtype == QIC_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QIC_SUCCESS : QIC_ERROR_INVALID_VALUE;
}

// Encoded maps of recent calls, per host thread: a decode loop encodes the same
// (cache, shape) maps at every step. The key holds every argument of the encoding, so
// a hit is the map that encoding would produce (also after the memory at `base` was
// freed and allocated again).
struct MapKey {
  int kind;  // 0: K/V cache map, 1: GEMV weight map
  const void* base;
  int64_t tokens;
  int dtype, kv_dim, head_dim, box_h;
  bool operator==(const MapKey& o) const {
    return kind == o.kind && base == o.base && tokens == o.tokens && dtype == o.dtype && kv_dim == o.kv_dim &&
           head_dim == o.head_dim && box_h == o.box_h;
  }
};

template <typename Encode>
int encode_cached(CUtensorMap* map, const MapKey& key, Encode encode) {
  constexpr int kEntries = 256;  // e.g. K and V of 64 layers plus their projections
  struct Entry {
    MapKey key;
    CUtensorMap map;
    bool used;
  };
  thread_local std::vector<Entry> cache(kEntries);
  const size_t h = (reinterpret_cast<uintptr_t>(key.base) >> 8) ^ static_cast<size_t>(key.tokens) * 31u ^
                   static_cast<size_t>(key.box_h * 7 + key.head_dim + key.dtype + key.kind * 131 + key.kv_dim);
  Entry& e = cache[h % kEntries];
  if (e.used && e.key == key) {
    *map = e.map;
    return QIC_SUCCESS;
  }
  const int rc = encode(map);
  if (rc == QIC_SUCCESS) {
    e.key = key;
    e.map = *map;
    e.used = true;
  }
  return rc;
}

int encode_kv_map(CUtensorMap* map, int dtype, const void* base, int64_t tokens, int kv_dim, int head_dim, int box_h) {
  return encode_cached(map, MapKey{0, base, tokens, dtype, kv_dim, head_dim, box_h}, [&](CUtensorMap* m) {
    return encode_kv_map_uncached(m, dtype, base, tokens, kv_dim, head_dim, box_h);
  });
}

// GEMV weights [K rows, N columns] (N contiguous) as a 2D tensor {N, K}; one box is
// kGemvTile columns of kGemvRowsPerSlot rows, row-major in shared memory, zeros past
// either edge.
int encode_weight_map_uncached(CUtensorMap* map, int dtype, const void* w, int K, int N) {
  load_driver_entry_points();
  if (g_encode == nullptr) return QIC_ERROR_CUDA;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(K)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(N) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(qic::kGemvTile), static_cast<cuuint32_t>(qic::kGemvRowsPerSlot)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = g_encode(map, dtype == QIC_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        2, const_cast<void*>(w), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QIC_SUCCESS : QIC_ERROR_INVALID_VALUE;
}

int encode_weight_map(CUtensorMap* map, int dtype, const void* w, int K, int N) {
  return encode_cached(map, MapKey{1, w, K, dtype, N, 0, 0},
                       [&](CUtensorMap* m) { return encode_weight_map_uncached(m, dtype, w, K, N); });
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
      position < 0 || position >= QIC_MAX_SEQ_LEN || cache_tokens <= 0)
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
  if (num_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || max_seq_len < 0 || max_seq_len > QIC_MAX_SEQ_LEN)
    return 0;
  const int G = num_heads / num_kv_heads;
  const int tok = qic::stage_tokens(head_dim);
  const int n_stages = (max_seq_len + tok - 1) / tok;
  const int splits = std::max(1, std::min(qic::kMaxSplits, n_stages));  // bounds cluster partial slots too
  return qic::kWsPartialOffset +
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

}  // extern "C"

namespace {

// Shared checks of the single and batched decode entry points.
int check_attention_common(int dtype, int H, int Hkv, int D, uint32_t flags, const void* q, const void* out,
                           const void* k_cache, const void* v_cache, const void* gate, const void* q_norm_w,
                           const void* k_norm_w, const void* k_new, const void* v_new, const void* workspace) {
  if (!valid_dtype(dtype)) return QIC_ERROR_INVALID_VALUE;
  if (H <= 0 || Hkv <= 0 || H % Hkv != 0 || !q || !out || !k_cache || !v_cache) return QIC_ERROR_INVALID_VALUE;
  if (!supported_head_dim(D) || H / Hkv > qic::kMaxGroup) return QIC_ERROR_NOT_SUPPORTED;
  const bool fuse_q = (flags & QIC_FUSE_Q_PROLOGUE) != 0;
  const bool fuse_app = (flags & QIC_FUSE_APPEND) != 0;
  if (fuse_q && !q_norm_w) return QIC_ERROR_INVALID_VALUE;
  if (fuse_app && (!k_new || !v_new || !k_norm_w)) return QIC_ERROR_INVALID_VALUE;
  if ((flags & QIC_Q_GATE_INTERLEAVED) && gate) return QIC_ERROR_INVALID_VALUE;  // the gate is inside q
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned2(out) || (gate && !aligned2(gate)) ||
      (fuse_q && !aligned16(q_norm_w)) ||
      (fuse_app && (!aligned16(k_new) || !aligned16(v_new) || !aligned16(k_norm_w))) ||
      (workspace && !aligned16(workspace)))
    return QIC_ERROR_MISALIGNED;
  return QIC_SUCCESS;
}

void fill_common(qic::AttnParams& p, int H, int Hkv, int D, const void* q, const void* gate, void* out,
                 void* k_cache, void* v_cache, uint32_t flags, float eps, float theta, const void* q_norm_w,
                 const void* k_norm_w, const void* k_new, const void* v_new) {
  const bool interleaved = (flags & QIC_Q_GATE_INTERLEAVED) != 0;
  p.q = q;
  p.gate = interleaved ? static_cast<const void*>(static_cast<const char*>(q) + static_cast<size_t>(D) * 2) : gate;
  p.q_hstride = interleaved ? 2 * D : D;
  p.q_bstride = static_cast<long long>(H) * p.q_hstride;
  p.out_bstride = static_cast<long long>(H) * D;
  p.out = out;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.q_norm_w = q_norm_w;
  p.k_norm_w = k_norm_w;
  p.k_new = k_new;
  p.v_new = v_new;
  p.H = H;
  p.Hkv = Hkv;
  p.G = H / Hkv;
  p.head_dim = D;
  p.flags = static_cast<int>(flags & (QIC_FUSE_Q_PROLOGUE | QIC_FUSE_APPEND | QIC_PDL));
  p.rope_pos = -1;
  p.eps = eps;
  p.theta = theta;
  p.scale_log2 = static_cast<float>((1.0 / std::sqrt(static_cast<double>(D))) * 1.4426950408889634);
  p.timeout_ns = timeout_ns();
}

int box_height(bool paged, int page_size, int tok, int* log2) {
  int bh = tok;
  if (paged) {
    bh = page_size & (-page_size);  // largest power of two dividing P
    if (bh > tok) bh = tok;
  }
  int l = 0;
  while ((1 << l) < bh) ++l;
  *log2 = l;
  return bh;
}

}  // namespace

extern "C" {

}  // extern "C"

namespace {

// Stages a single-sequence call copies through the attention kernel's ring: with a fused
// append whose token is alone in the last stage (S - 1 a multiple of the stage size),
// that token's contribution comes from registers and its stage is not copied.
int copied_stages(int S, int tok, uint32_t flags) {
  const int n = (S + tok - 1) / tok;
  return n - (((flags & QIC_FUSE_APPEND) && S > 1 && (S - 1) % tok == 0) ? 1 : 0);
}

// Splits per kv head and CTAs per cluster of a single-sequence launch over n_stages
// pipeline stages: the caller's choice, else one wave of resident 8-CTA clusters
// (five sixths of it with QIC_PDL), fewer for shorter sequences.
int launch_shape(const qic_decode_args* a, bool cp, int n_stages, int* n_splits_out, int* cluster_out) {
  const int D = a->head_dim, Hkv = a->num_kv_heads;
  int n_splits = a->num_splits, cluster = a->cluster_size;
  if (cluster < 0 || cluster > qic::kMaxCluster) return QIC_ERROR_INVALID_VALUE;
  if (cp) cluster = qic::kCpSlices;
  if (n_splits <= 0) {
    // As many CTAs as can be resident in one wave: clusters of 8 (measured best on B200),
    // as many clusters per kv head as the GPU holds at once; fewer for short sequences.
    // With programmatic dependent launch (layers chained back to back) a sixth of the
    // resident slots is left free, so the next launch's CTAs start their copies while
    // this one merges its splits (measured on 36 chained S=8192 layers: 13.6 -> 12.8
    // us per layer; 8 chained d=256 S=32769 layers: 31.3 -> 30.2 us).
    const bool auto_cluster = cluster == 0;
    if (cluster == 0) cluster = 8;
    int max_clusters = qic::decode_attention_max_active_clusters(a->dtype, D, cluster, a->num_heads / Hkv);
    if (max_clusters <= 0) max_clusters = (3 * sm_count()) / cluster;  // three CTAs per SM
    if (a->flags & QIC_PDL) max_clusters = std::max(1, max_clusters * 5 / 6);
    // at most kMaxSplits splits per kv head: with one or two kv heads the wave is larger
    int nclust = std::max(1, std::min(max_clusters / Hkv, qic::kMaxSplits / cluster));
    n_splits = cluster * nclust;
    if (auto_cluster) {
      // Shorter sequences: about 6 stages per CTA (8 at d=256; 12 at d=64, the same
      // bytes as d=128, not swept), in multiples of 8 CTAs, and a single cluster per
      // kv head up to 16 CTAs, so the merge needs no cross-cluster step. Measured on
      // 8 chained layers: d=128 S=1025 10.0 -> 8.9 us, S=2049 10.5 -> 9.5, S=4097
      // 12.0 -> 11.5; d=256 S=2049 14.0 -> 12.1, S=8193 16.7 -> 15.6.
      const int per_split = D >= 256 ? 8 : (D >= 128 ? 6 : 12);
      int want = std::max(8, n_stages / per_split / 8 * 8);
      // Past 8 CTAs' rings (4 stages each, 8 at d=64) a kv head takes 16 CTAs, so no CTA
      // waits a second round trip for a fifth stage (36 chained Qwen3-8B layers, us per
      // layer, 8 -> 16 CTAs: S=1025 7.72 -> 6.29, S=2048 7.95 -> 6.08, S=2049 8.71 -> 8.23;
      // d=256 S=1025 9.74 -> 9.49).
      const int ring = D == 64 ? 8 : 4;
      if (n_stages > 8 * ring && want < 16) want = 16;
      if (want < n_splits) {
        n_splits = want;
        if (want <= qic::kMaxCluster) cluster = want;
      }
    }
    if (n_splits > n_stages) {
      nclust = std::max(1, n_stages / cluster);
      if (n_stages < cluster) cluster = n_stages;
      n_splits = cluster * nclust;
    }
  }
  if (cluster == 0) cluster = std::min(n_splits, qic::kMaxCluster);
  while (cluster > 1 && n_splits % cluster != 0) --cluster;
  if (n_splits > qic::kMaxSplits) return QIC_ERROR_INVALID_VALUE;
  if (a->workspace == nullptr) {
    n_splits = std::min(n_splits, qic::kMaxCluster);  // merged on chip only, no workspace needed
    cluster = n_splits;
  }
  *n_splits_out = n_splits;
  *cluster_out = cluster;
  return QIC_SUCCESS;
}

// Single-sequence decode attention; cp != nullptr adds the context-parallel exchange.
int decode_attention_impl(const qic_decode_args* a, const qic_cp_args* cp, qic_stream_t stream) {
  if (a == nullptr) return QIC_ERROR_INVALID_VALUE;
  const int H = a->num_heads, Hkv = a->num_kv_heads, D = a->head_dim, S = a->seq_len;
  int rc = check_attention_common(a->dtype, H, Hkv, D, a->flags, a->q, a->out, a->k_cache, a->v_cache, a->gate,
                                  a->q_norm_w, a->k_norm_w, a->k_new, a->v_new, a->workspace);
  if (rc != QIC_SUCCESS) return rc;
  if (S < 0 || S > QIC_MAX_SEQ_LEN) return QIC_ERROR_INVALID_VALUE;
  // device-resident length: seq_len is its upper bound and sizes the launch
  const bool dev_len = (a->flags & QIC_DEVICE_SEQ_LEN) != 0;
  if (dev_len && (a->seq_len_dev == nullptr || (reinterpret_cast<uintptr_t>(a->seq_len_dev) & 3u) != 0 || S < 1 ||
                  a->workspace == nullptr))
    return QIC_ERROR_INVALID_VALUE;
  if (dev_len && cp != nullptr) return QIC_ERROR_NOT_SUPPORTED;
  const int G = H / Hkv;
  const bool paged = a->page_table != nullptr;
  if (paged && (a->page_size <= 0 || a->page_size % 8 != 0)) return QIC_ERROR_NOT_SUPPORTED;
  if ((a->flags & QIC_FUSE_APPEND) && S < 1) return QIC_ERROR_INVALID_VALUE;
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
  const bool partial_out = (a->flags & QIC_PARTIAL_OUT) != 0;
  if (partial_out && (cp != nullptr || !aligned16(a->out))) return QIC_ERROR_INVALID_VALUE;
  if ((a->flags & QIC_EXPLICIT_POSITION) && (a->position < 0 || a->position >= QIC_MAX_SEQ_LEN))
    return QIC_ERROR_INVALID_VALUE;
  if (cp != nullptr) {
    if (cp->world < 1 || cp->world > qic::kMaxRanks || cp->rank < 0 || cp->rank >= cp->world ||
        cp->exchange == nullptr || cp->peer_exchange[cp->rank] != cp->exchange || a->workspace == nullptr ||
        a->workspace_bytes < qic::kWsPartialOffset || cp->timeout_ms < 0)
      return QIC_ERROR_INVALID_VALUE;
    for (int r = 0; r < cp->world; ++r)
      if (cp->peer_exchange[r] == nullptr || !aligned16(cp->peer_exchange[r])) return QIC_ERROR_INVALID_VALUE;
    if (cp->exchange_bytes < qic::cp_exchange_bytes(G, D, Hkv, cp->world)) return QIC_ERROR_WORKSPACE;
    if (a->cluster_size != 0 && a->cluster_size != qic::kCpSlices) return QIC_ERROR_NOT_SUPPORTED;
    if (a->num_splits != 0 && a->num_splits % qic::kCpSlices != 0) return QIC_ERROR_NOT_SUPPORTED;
    // every rank must reach the exchange: a shard shorter than one cluster of stages is not supported
    if (S < qic::kCpSlices * qic::stage_tokens(D)) return QIC_ERROR_NOT_SUPPORTED;
  }
  if (S == 0) {  // no tokens: the reference writes acc * 1e12 = 0
    if (partial_out) {  // o = 0 and lse = -inf for every head
      const int G0 = H / Hkv, pf = qic::partial_floats(G0, D);
      std::vector<float> host(static_cast<size_t>(Hkv) * pf, 0.0f);
      for (int k = 0; k < Hkv; ++k)
        for (int h = 0; h < G0; ++h) host[static_cast<size_t>(k) * pf + G0 * D + h] = -INFINITY;
      cudaError_t e = cudaMemcpyAsync(a->out, host.data(), host.size() * sizeof(float), cudaMemcpyHostToDevice, st);
      if (e == cudaSuccess) e = cudaStreamSynchronize(st);
      return cuda_status(e);
    }
    return cuda_status(cudaMemsetAsync(a->out, 0, static_cast<size_t>(H) * D * 2, st));
  }

  qic::AttnParams p;
  std::memset(&p, 0, sizeof(p));
  const int tok = qic::stage_tokens(D);
  int lbh = 0;
  const int box_h = box_height(paged, a->page_size, tok, &lbh);
  rc = encode_kv_map(&p.tm_k, a->dtype, a->k_cache, cache_tokens, kv_dim, a->head_dim, box_h);
  if (rc == QIC_SUCCESS) rc = encode_kv_map(&p.tm_v, a->dtype, a->v_cache, cache_tokens, kv_dim, a->head_dim, box_h);
  if (rc != QIC_SUCCESS) return rc;

  const int n_stages = copied_stages(S, tok, a->flags);
  int n_splits = 0, cluster = 0;
  rc = launch_shape(a, cp != nullptr, n_stages, &n_splits, &cluster);
  if (rc != QIC_SUCCESS) return rc;
  if (cp != nullptr && (cluster != qic::kCpSlices || n_splits % qic::kCpSlices != 0)) return QIC_ERROR_NOT_SUPPORTED;
  const int n_clusters = n_splits / cluster;
  if (n_clusters > 1) {
    const size_t need = qic::kWsPartialOffset +
                        static_cast<size_t>(Hkv) * n_clusters * qic::partial_floats(G, D) * sizeof(float);
    if (a->workspace_bytes < need || Hkv * cluster > qic::kMaxCounters - qic::kMaxStageCounters)
      return QIC_ERROR_WORKSPACE;
  }
  if (a->workspace != nullptr) {
    char* ws = static_cast<char*>(a->workspace);
    p.status = reinterpret_cast<int*>(ws);
    if (a->workspace_bytes >= qic::kWsPartialOffset) {
      p.counters = reinterpret_cast<int*>(ws + qic::kWsHeader);
      p.part = reinterpret_cast<float*>(ws + qic::kWsPartialOffset);
      p.num_counters = std::min(Hkv * cluster, qic::kMaxCounters - qic::kMaxStageCounters);
      if (Hkv <= qic::kMaxStageCounters && !(a->flags & QIC_DETERMINISTIC))
        p.stage_ctr = p.counters + (qic::kMaxCounters - qic::kMaxStageCounters);
      p.part_slots = static_cast<int>(std::min<size_t>(
          INT32_MAX, (a->workspace_bytes - qic::kWsPartialOffset) / (qic::partial_floats(G, D) * sizeof(float))));
    }
  }
  p.cluster = cluster;
  fill_common(p, H, Hkv, D, a->q, a->gate, a->out, a->k_cache, a->v_cache, a->flags, a->eps, a->rope_theta,
              a->q_norm_w, a->k_norm_w, a->k_new, a->v_new);
  p.page_table = a->page_table;
  p.cache_tokens = cache_tokens;
  p.seq_len = S;
  p.page_size = paged ? a->page_size : 0;
  p.box_h = box_h;
  p.log2_box_h = lbh;
  p.n_splits = n_splits;
  p.seq_len_dev = dev_len ? a->seq_len_dev : nullptr;
  p.rope_pos = (a->flags & QIC_EXPLICIT_POSITION) ? a->position : -1;
  if (partial_out) p.part_out = static_cast<float*>(a->out);
  if (cp != nullptr) {
    char* ws = static_cast<char*>(a->workspace);
    p.cp_rank = cp->rank;
    p.cp_world = cp->world;
    p.cp_mergers = Hkv * qic::kCpSlices;
    p.cp_epoch = reinterpret_cast<unsigned*>(ws + qic::kWsCpEpoch);
    p.cp_done = reinterpret_cast<unsigned*>(ws + qic::kWsCpDone);
    for (int r = 0; r < cp->world; ++r) p.cp_peer[r] = cp->peer_exchange[r];
    if (cp->timeout_ms > 0) p.timeout_ns = static_cast<uint64_t>(cp->timeout_ms) * 1000000ull;
  }
  return cuda_status(qic::launch_decode_attention(a->dtype, D, p, st));
}

}  // namespace

extern "C" {

int qic_decode_attention(const qic_decode_args* a, qic_stream_t stream) {
  return decode_attention_impl(a, nullptr, stream);
}

int qic_decode_launch_shape(const qic_decode_args* a, int* num_splits, int* cluster_size) {
  if (a == nullptr || num_splits == nullptr || cluster_size == nullptr) return QIC_ERROR_INVALID_VALUE;
  const int H = a->num_heads, Hkv = a->num_kv_heads, D = a->head_dim, S = a->seq_len;
  if (!valid_dtype(a->dtype) || H <= 0 || Hkv <= 0 || H % Hkv != 0 || S < 0 || S > QIC_MAX_SEQ_LEN)
    return QIC_ERROR_INVALID_VALUE;
  if (!supported_head_dim(D) || H / Hkv > qic::kMaxGroup) return QIC_ERROR_NOT_SUPPORTED;
  *num_splits = 0;
  *cluster_size = 0;
  if (S == 0) return QIC_SUCCESS;  // no launch
  const int tok = qic::stage_tokens(D);
  return launch_shape(a, false, copied_stages(S, tok, a->flags), num_splits, cluster_size);
}

int qic_cp_decode_attention(const qic_decode_args* a, const qic_cp_args* cp, qic_stream_t stream) {
  if (cp == nullptr) return QIC_ERROR_INVALID_VALUE;
  return decode_attention_impl(a, cp, stream);
}

size_t qic_cp_exchange_bytes(int num_heads, int num_kv_heads, int head_dim, int world) {
  if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0 || head_dim <= 0 || world < 1 ||
      world > qic::kMaxRanks)
    return 0;
  return qic::cp_exchange_bytes(num_heads / num_kv_heads, head_dim, num_kv_heads, world);
}

size_t qic_partial_floats(int num_heads, int num_kv_heads, int head_dim) {
  if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0 || head_dim <= 0) return 0;
  return static_cast<size_t>(qic::partial_floats(num_heads / num_kv_heads, head_dim));
}

int qic_attention_merge(int dtype, const float* partials, int num_partials, int num_heads, int num_kv_heads,
                        int head_dim, const void* gate, void* out, qic_stream_t stream) {
  if (!valid_dtype(dtype) || partials == nullptr || out == nullptr || num_partials < 1 || num_heads <= 0 ||
      num_kv_heads <= 0 || num_heads % num_kv_heads != 0)
    return QIC_ERROR_INVALID_VALUE;
  if (!supported_head_dim(head_dim) || num_heads / num_kv_heads > qic::kMaxGroup) return QIC_ERROR_NOT_SUPPORTED;
  if (!aligned2(out) || (gate && !aligned2(gate)) || (reinterpret_cast<uintptr_t>(partials) & 3u))
    return QIC_ERROR_MISALIGNED;
  return cuda_status(qic::launch_attention_merge(dtype, head_dim, partials, num_partials, num_heads, num_kv_heads, gate,
                                                 out, reinterpret_cast<cudaStream_t>(stream)));
}

int qic_device_alloc(size_t bytes, void** ptr) {
  if (ptr == nullptr || bytes == 0) return QIC_ERROR_INVALID_VALUE;
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
  if (e != cudaSuccess && *ptr != nullptr) {
    cudaFree(*ptr);
    *ptr = nullptr;
  }
  return cuda_status(e);
}

int qic_device_free(void* ptr) { return ptr == nullptr ? QIC_SUCCESS : cuda_status(cudaFree(ptr)); }

int qic_ipc_get_handle(const void* ptr, void* handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) <= QIC_IPC_HANDLE_BYTES, "IPC handle size");
  if (ptr == nullptr || handle == nullptr) return QIC_ERROR_INVALID_VALUE;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) return cuda_status(e);
  std::memset(handle, 0, QIC_IPC_HANDLE_BYTES);
  std::memcpy(handle, &h, sizeof(h));
  return QIC_SUCCESS;
}

int qic_ipc_open_handle(const void* handle, void** ptr) {
  if (handle == nullptr || ptr == nullptr) return QIC_ERROR_INVALID_VALUE;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return QIC_ERROR_PEER;
  return QIC_SUCCESS;
}

int qic_ipc_close_handle(void* ptr) {
  if (ptr == nullptr) return QIC_ERROR_INVALID_VALUE;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? QIC_SUCCESS : QIC_ERROR_PEER;
}

int qic_batch_plan(const int32_t* seq_lens, int batch, int num_heads, int num_kv_heads, int head_dim,
                   int target_ctas, void* plan, int max_items, int* items, size_t* workspace_bytes) {
  if (!seq_lens || batch <= 0 || num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0 || !items ||
      !workspace_bytes || max_items < 0 || (max_items > 0 && !plan))
    return QIC_ERROR_INVALID_VALUE;
  if (!supported_head_dim(head_dim)) return QIC_ERROR_NOT_SUPPORTED;
  const int tok = qic::stage_tokens(head_dim);
  long long total = 0;
  for (int b = 0; b < batch; ++b) {
    if (seq_lens[b] < 1 || seq_lens[b] > QIC_MAX_SEQ_LEN) return QIC_ERROR_INVALID_VALUE;
    total += static_cast<long long>((seq_lens[b] + tok - 1) / tok) * num_kv_heads;
  }
  if (target_ctas <= 0) {
    // Whole waves of resident CTAs with at least ~1 MiB of K/V per work item (a CTA's
    // set-up and merge cost a few microseconds), at most 16 items per SM.
    int resident = qic::decode_attention_max_active_clusters(QIC_DTYPE_BF16, head_dim, 1, num_heads / num_kv_heads);
    if (resident <= 0) resident = 3 * sm_count();
    const double bytes = static_cast<double>(total) * tok * head_dim * 2 * 2;
    const int max_waves = std::max(1, (16 * sm_count()) / resident);
    const int waves = static_cast<int>(
        std::min<double>(max_waves, std::max(1.0, std::round(bytes / (static_cast<double>(resident) * (1 << 20))))));
    target_ctas = resident * waves;
  }
  // stages per item: the smallest chunk whose item count (every (sequence, kv head)
  // cut into pieces of at most `chunk` stages, ragged last pieces included) fits the
  // target, so the ragged pieces do not spill into a nearly empty extra wave
  long long chunk = std::max<long long>(1, (total + target_ctas - 1) / target_ctas);
  auto items_for = [&](long long c) {
    long long n_items = 0;
    for (int b = 0; b < batch; ++b) {
      const long long n = (seq_lens[b] + tok - 1) / tok;
      n_items += std::min<long long>(std::min<long long>(n, qic::kMaxSplits), (n + c - 1) / c) * num_kv_heads;
    }
    return n_items;
  };
  if (items_for(chunk) > target_ctas) {
    // items_for falls as the chunk grows; at the longest sequence's stage count every
    // (sequence, kv head) is one item, the fewest possible
    long long lo = chunk, hi = 1;
    for (int b = 0; b < batch; ++b) hi = std::max<long long>(hi, (seq_lens[b] + tok - 1) / tok);
    hi = std::max(hi, lo);
    while (lo < hi) {
      const long long mid = lo + (hi - lo) / 2;
      if (items_for(mid) > target_ctas) lo = mid + 1; else hi = mid;
    }
    chunk = lo;
  }
  std::vector<qic::WorkItem> out;
  int part_base = 0;
  for (int b = 0; b < batch; ++b) {
    const int n = (seq_lens[b] + tok - 1) / tok;
    const int ns = static_cast<int>(std::min<long long>(std::min(n, qic::kMaxSplits), (n + chunk - 1) / chunk));
    for (int h = 0; h < num_kv_heads; ++h) {
      for (int s = 0; s < ns; ++s) {
        qic::WorkItem w;
        w.b = b;
        w.kvh = h;
        w.split = s;
        w.nsplit = ns;
        w.st_lo = static_cast<int>(static_cast<long long>(s) * n / ns);
        w.st_hi = static_cast<int>(static_cast<long long>(s + 1) * n / ns);
        w.seq_len = seq_lens[b];
        w.part_base = part_base;
        out.push_back(w);
      }
      part_base += ns;
    }
  }
  // longest first, so the last wave is made of the shortest items
  std::stable_sort(out.begin(), out.end(), [](const qic::WorkItem& x, const qic::WorkItem& y) {
    return (x.st_hi - x.st_lo) > (y.st_hi - y.st_lo);
  });
  const int G = num_heads / num_kv_heads;
  *items = static_cast<int>(out.size());
  if (static_cast<long long>(batch) * num_kv_heads > qic::kMaxCounters) return QIC_ERROR_NOT_SUPPORTED;
  *workspace_bytes = qic::kWsPartialOffset +
                     static_cast<size_t>(part_base) * qic::partial_floats(G, head_dim) * sizeof(float);
  if (static_cast<int>(out.size()) > max_items) return max_items == 0 ? QIC_SUCCESS : QIC_ERROR_INVALID_VALUE;
  std::memcpy(plan, out.data(), out.size() * sizeof(qic::WorkItem));
  return QIC_SUCCESS;
}

int qic_batch_decode_attention(const qic_batch_decode_args* a, qic_stream_t stream) {
  if (a == nullptr) return QIC_ERROR_INVALID_VALUE;
  const int H = a->num_heads, Hkv = a->num_kv_heads, D = a->head_dim;
  int rc = check_attention_common(a->dtype, H, Hkv, D, a->flags, a->q, a->out, a->k_cache, a->v_cache, a->gate,
                                  a->q_norm_w, a->k_norm_w, a->k_new, a->v_new, a->workspace);
  if (rc != QIC_SUCCESS) return rc;
  if (a->batch <= 0 || !a->block_tables || a->max_pages_per_seq <= 0 || !a->plan || a->plan_items <= 0 ||
      a->cache_tokens <= 0 || a->cache_tokens > (int64_t(1) << 31) - 1)
    return QIC_ERROR_INVALID_VALUE;
  if (a->page_size <= 0 || a->page_size % 8 != 0) return QIC_ERROR_NOT_SUPPORTED;
  if ((reinterpret_cast<uintptr_t>(a->plan) & 15u) != 0) return QIC_ERROR_MISALIGNED;
  const int G = H / Hkv;
  if (static_cast<long long>(a->batch) * Hkv > qic::kMaxCounters) return QIC_ERROR_NOT_SUPPORTED;
  const size_t head = qic::kWsPartialOffset;
  if (a->workspace == nullptr || a->workspace_bytes < head) return QIC_ERROR_WORKSPACE;
  const size_t slots = (a->workspace_bytes - head) / (qic::partial_floats(G, D) * sizeof(float));
  qic::AttnParams p;
  std::memset(&p, 0, sizeof(p));
  const int tok = qic::stage_tokens(D);
  int lbh = 0;
  const int box_h = box_height(true, a->page_size, tok, &lbh);
  const int kv_dim = Hkv * D;
  rc = encode_kv_map(&p.tm_k, a->dtype, a->k_cache, a->cache_tokens, kv_dim, a->head_dim, box_h);
  if (rc == QIC_SUCCESS) rc = encode_kv_map(&p.tm_v, a->dtype, a->v_cache, a->cache_tokens, kv_dim, a->head_dim, box_h);
  if (rc != QIC_SUCCESS) return rc;
  char* ws = static_cast<char*>(a->workspace);
  p.status = reinterpret_cast<int*>(ws);
  p.counters = reinterpret_cast<int*>(ws + qic::kWsHeader);
  p.part = reinterpret_cast<float*>(ws + head);
  p.num_counters = a->batch * Hkv;  // <= kMaxCounters
  p.part_slots = static_cast<int>(std::min<size_t>(slots, INT32_MAX));
  fill_common(p, H, Hkv, D, a->q, a->gate, a->out, a->k_cache, a->v_cache, a->flags, a->eps, a->rope_theta,
              a->q_norm_w, a->k_norm_w, a->k_new, a->v_new);
  p.page_table = a->block_tables;
  p.table_bstride = a->max_pages_per_seq;
  p.kv_new_bstride = static_cast<long long>(Hkv) * D;
  p.plan = static_cast<const qic::WorkItem*>(a->plan);
  p.cache_tokens = a->cache_tokens;
  p.page_size = a->page_size;
  p.box_h = box_h;
  p.log2_box_h = lbh;
  p.n_splits = a->plan_items;  // grid size
  p.cluster = 1;
  return cuda_status(qic::launch_decode_attention(a->dtype, D, p, reinterpret_cast<cudaStream_t>(stream)));
}

}  // extern "C"

namespace {

bool ranges_overlap(const void* a, size_t an, const void* b, size_t bn) {
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(a), b0 = reinterpret_cast<uintptr_t>(b);
  return a0 < b0 + bn && b0 < a0 + an;
}

// Checks a GEMV call and fills the kernel parameters (without the split count).
int gemv_prepare(const qic_gemv_args* a, qic::GemvParams* p, bool* pair, bool* norm) {
  if (a == nullptr || !valid_dtype(a->dtype)) return QIC_ERROR_INVALID_VALUE;
  const int K = a->in_dim, ns = a->num_segments;
  const uint32_t known = QIC_GEMV_RMSNORM | QIC_GEMV_SWIGLU | QIC_GEMV_RESIDUAL | QIC_PDL;
  if (K <= 0 || ns < 1 || ns > qic::kGemvMaxSegments || (a->flags & ~known) != 0 || a->x == nullptr)
    return QIC_ERROR_INVALID_VALUE;
  if (K > qic::kGemvMaxSplits * qic::kGemvMaxRowsPerSplit) return QIC_ERROR_NOT_SUPPORTED;
  if (a->splits < 0 || a->splits > qic::kGemvMaxSplits) return QIC_ERROR_INVALID_VALUE;
  *pair = (a->flags & QIC_GEMV_SWIGLU) != 0;
  *norm = (a->flags & QIC_GEMV_RMSNORM) != 0;
  const bool res = (a->flags & QIC_GEMV_RESIDUAL) != 0;
  if (*pair && (ns != 2 || res || a->seg[0].out_dim != a->seg[1].out_dim)) return QIC_ERROR_INVALID_VALUE;
  if (*norm && a->norm_w == nullptr) return QIC_ERROR_INVALID_VALUE;
  if (!aligned2(a->x) || (*norm && !aligned2(a->norm_w)) || (reinterpret_cast<uintptr_t>(a->status) & 3u))
    return QIC_ERROR_MISALIGNED;
  std::memset(p, 0, sizeof(*p));
  long long tiles = 0;
  for (int k = 0; k < ns; ++k) {
    const qic_gemv_segment& g = a->seg[k];
    if (g.w == nullptr || g.out_dim <= 0 || (g.out_dim % 8) != 0 || (g.out == nullptr && !(*pair && k == 1)) ||
        (res && g.residual == nullptr))
      return QIC_ERROR_INVALID_VALUE;
    if (!aligned16(g.w) || (g.out != nullptr && !aligned2(g.out)) || (res && !aligned2(g.residual)))
      return QIC_ERROR_MISALIGNED;
    // every CTA reads the whole input while others write their outputs
    if (g.out != nullptr && ranges_overlap(a->x, static_cast<size_t>(K) * 2, g.out, static_cast<size_t>(g.out_dim) * 2))
      return QIC_ERROR_INVALID_VALUE;
    p->seg[k].w = g.w;
    p->seg[k].out = g.out;
    p->seg[k].res = res ? g.residual : nullptr;
    p->seg[k].N = g.out_dim;
    p->seg[k].tile0 = static_cast<int>(tiles);
    if (!(*pair && k == 1)) tiles += (g.out_dim + qic::kGemvTile - 1) / qic::kGemvTile;
  }
  if (*pair) p->seg[1].tile0 = INT32_MAX;  // both halves of the pair share the tiles of segment 0
  if (tiles > 65535) return QIC_ERROR_NOT_SUPPORTED;
  p->x = a->x;
  p->norm_w = *norm ? a->norm_w : nullptr;
  p->eps = a->eps;
  p->K = K;
  p->flags = static_cast<int>(a->flags & QIC_PDL);
  p->nseg = ns;
  p->n_tiles = static_cast<int>(tiles);
  return QIC_SUCCESS;
}

// Rows of a tile per CTA when `splits` CTAs share them (multiple of 8).
int gemv_rows_per_split(int K, int splits) { return ((K + splits - 1) / splits + 7) / 8 * 8; }

// Split count: the caller's, else the largest cluster size from {16, 12, 8, 6, 5, 4, 3,
// 2, 1} (at least 64 rows per CTA, rows fitting shared memory) that keeps the grid at
// most 2 CTAs per SM with every tile's cluster resident at once. Swept on the
// Qwen3-8B projections (8 chained launches each, GB/s): q/k/v 24 tiles, splits 8 /
// 10 / 12 -> 4619 / 4361 / 3638; o 16 tiles, 12 / 13 / 16 -> 4000 / 3862 / 3023;
// gate/up 48 tiles, 5 / 6 -> 6152 / 4528; down 16 tiles, 12 / 13 -> 5446 / 4693. More
// CTAs (odd cluster sizes, or 2 per SM everywhere) left some clusters to a second
// wave behind the preceding launch's CTAs. The cap of 2 CTAs per SM (5/3 before)
// changes only smaller projections (Qwen3.5-4B widths): the whole decode step, A/B on
// one box, 521-523 -> 525-526 tokens/s.
int gemv_splits(const qic_gemv_args* a, int n_tiles) {
  const int K = a->in_dim;
  const int min_c = (K + qic::kGemvMaxRowsPerSplit - 1) / qic::kGemvMaxRowsPerSplit;
  if (a->splits > 0) return std::max(a->splits, min_c);
  static const int kSizes[] = {16, 12, 8, 6, 5, 4, 3, 2, 1};
  const long long cap = std::max<long long>(n_tiles, static_cast<long long>(sm_count()) * 2);
  for (int c : kSizes) {
    if (c < min_c) break;
    if (c > 1 && K < 64 * c) continue;
    if (static_cast<long long>(n_tiles) * c > cap) continue;
    const int m = qic::gemv_max_active_clusters(a->dtype, c, gemv_rows_per_split(K, c));
    if (m > 0 && n_tiles <= m) return c;
  }
  return std::max(1, min_c);  // more tiles than one wave holds: several waves
}

}  // namespace

extern "C" {

int qic_gemv_launch_shape(const qic_gemv_args* a, int* splits, int* tiles) {
  if (splits == nullptr || tiles == nullptr) return QIC_ERROR_INVALID_VALUE;
  qic::GemvParams p;
  bool pair = false, norm = false;
  const int rc = gemv_prepare(a, &p, &pair, &norm);
  if (rc != QIC_SUCCESS) return rc;
  *splits = gemv_splits(a, p.n_tiles);
  *tiles = p.n_tiles;
  return QIC_SUCCESS;
}

int qic_gemv(const qic_gemv_args* a, qic_stream_t stream) {
  qic::GemvParams p;
  bool pair = false, norm = false;
  int rc = gemv_prepare(a, &p, &pair, &norm);
  if (rc != QIC_SUCCESS) return rc;
  for (int k = 0; k < a->num_segments; ++k) {
    rc = encode_weight_map(&p.tm[k], a->dtype, a->seg[k].w, a->in_dim, a->seg[k].out_dim);
    if (rc != QIC_SUCCESS) return rc;
  }
  p.status = static_cast<int*>(a->status);
  p.timeout_ns = timeout_ns();
  p.splits = gemv_splits(a, p.n_tiles);
  if (p.splits > qic::kGemvMaxSplits) return QIC_ERROR_NOT_SUPPORTED;
  p.rows_per_split = gemv_rows_per_split(a->in_dim, p.splits);
  if (p.rows_per_split > qic::kGemvMaxRowsPerSplit) return QIC_ERROR_NOT_SUPPORTED;
  p.xs_floats = p.rows_per_split;  // a multiple of 8
  return cuda_status(qic::launch_gemv(a->dtype, p, pair, norm, reinterpret_cast<cudaStream_t>(stream)));
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
