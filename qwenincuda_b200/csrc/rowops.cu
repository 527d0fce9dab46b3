// Standalone head RMSNorm, RoPE, sigmoid gate and fused K/V append kernels.
//
// They keep the reference's call semantics (head_rmsnorm_kernel, rope_inplace_kernel,
// sigmoid_mul_inplace_kernel in src/kernels.cu:78-183 of the QweninCuda project, and
// the append at src/model.cpp:634-641) and produce the same bytes as the reference
// build, which is compiled with --use_fast_math; so is this translation unit.
#include "qic_internal.h"
#include "rowops.cuh"

namespace qic {

// One warp per head, any head_dim. The sum of squares follows the reference's
// thread mapping (thread i accumulates elements i, i+256, ...; the per-thread sums
// are added in ascending thread order), evaluated serially by lane 0.
template <typename T>
__global__ void head_rmsnorm_kernel(const T* x, const T* w, int num_heads, int head_dim, float eps, T* out) {
  extern __shared__ float xs[];
  const int h = blockIdx.x;
  const int lane = threadIdx.x;
  if (h >= num_heads) return;
  const T* xh = x + static_cast<size_t>(h) * head_dim;
  T* oh = out + static_cast<size_t>(h) * head_dim;
  for (int i = lane; i < head_dim; i += 32) xs[i] = to_f32<T>(xh[i]);
  __syncwarp();
  float ssum = 0.0f;
  if (lane == 0) {
    const int nthr = head_dim < 256 ? head_dim : 256;
    for (int t = 0; t < nthr; ++t) {
      float local = 0.0f;
      for (int i = t; i < head_dim; i += 256) local = fmaf(xs[i], xs[i], local);
      ssum = __fadd_rn(ssum, local);
    }
  }
  ssum = __shfl_sync(kFullMask, ssum, 0);
  const float inv_rms = rsqrtf(ssum / static_cast<float>(head_dim) + eps);
  for (int i = lane; i < head_dim; i += 32) {
    const float xv = xs[i];
    const float wv = to_f32<T>(w[i]);
    oh[i] = from_f32<T>(xv * inv_rms * wv);
  }
}

// One thread per rotated pair (i, i + head_dim/2).
template <typename T>
__global__ void rope_inplace_kernel(T* x, int num_heads, int head_dim, int position, float rope_theta) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const int half_dim = head_dim / 2;
  if (idx >= num_heads * half_dim) return;
  const int h = idx / half_dim;
  const int d = idx % half_dim;
  T* xh = x + static_cast<size_t>(h) * head_dim;
  const float x0 = to_f32<T>(xh[d]);
  const float x1 = to_f32<T>(xh[d + half_dim]);
  const float inv_freq = powf(rope_theta, -2.0f * static_cast<float>(d) / static_cast<float>(head_dim));
  const float angle = static_cast<float>(position) * inv_freq;
  const float c = cosf(angle);
  const float s = sinf(angle);
  const float y0 = x0 * c - x1 * s;
  const float y1 = x1 * c + x0 * s;
  xh[d] = from_f32<T>(y0);
  xh[d + half_dim] = from_f32<T>(y1);
}

template <typename T>
__global__ void sigmoid_mul_kernel(T* x, const T* gate, int n) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n) return;
  const float g = to_f32<T>(gate[idx]);
  const float sig = 1.0f / (1.0f + expf(-g));
  x[idx] = from_f32<T>(to_f32<T>(x[idx]) * sig);
}

// One warp per kv head: k row -> head RMSNorm -> RoPE -> cache slot; v row copied.
// The slot is the row paged_attention reads for token `position`
// (page_table[position/page_size]*page_size + position%page_size), or `position`
// itself without a page table. A slot outside [0, cache_tokens) is not written.
template <typename T, int D>
__global__ void kv_append_kernel(const T* k_new, const T* v_new, const T* k_norm_w, float eps, float theta,
                                 int position, const int32_t* page_table, int page_size, long long cache_tokens,
                                 T* k_cache, T* v_cache, int num_kv_heads) {
  const int kvh = blockIdx.x;
  const int lane = threadIdx.x;
  const size_t kv_dim = static_cast<size_t>(num_kv_heads) * D;
  long long slot = position;
  if (page_table != nullptr) {
    const int e = position / page_size;
    slot = static_cast<long long>(page_table[e]) * page_size + (position - e * page_size);
  }
  if (slot < 0 || slot >= cache_tokens) return;
  float v[D / 32];
  row_load<T, D>(k_new + static_cast<size_t>(kvh) * D, v, lane);
  row_rmsnorm<T, D>(v, k_norm_w, D, eps, lane);
  row_rope<T, D>(v, D, position, theta, lane);
  row_store<T, D>(k_cache + static_cast<size_t>(slot) * kv_dim + static_cast<size_t>(kvh) * D, v, lane);
  float vv[D / 32];
  row_load<T, D>(v_new + static_cast<size_t>(kvh) * D, vv, lane);
  row_store<T, D>(v_cache + static_cast<size_t>(slot) * kv_dim + static_cast<size_t>(kvh) * D, vv, lane);
}

// ---------------------------------------------------------------------------
template <typename T>
static cudaError_t head_rmsnorm_t(const void* x, const void* w, int H, int hd, float eps, void* out,
                                  cudaStream_t s) {
  head_rmsnorm_kernel<T><<<H, 32, hd * sizeof(float), s>>>(static_cast<const T*>(x), static_cast<const T*>(w), H,
                                                           hd, eps, static_cast<T*>(out));
  return cudaGetLastError();
}

cudaError_t launch_head_rmsnorm(int dtype, const void* x, const void* w, int num_heads, int head_dim, float eps,
                                void* out, cudaStream_t stream) {
  if (dtype == QIC_DTYPE_BF16) return head_rmsnorm_t<__nv_bfloat16>(x, w, num_heads, head_dim, eps, out, stream);
  return head_rmsnorm_t<__half>(x, w, num_heads, head_dim, eps, out, stream);
}

cudaError_t launch_rope_inplace(int dtype, void* x, int num_heads, int head_dim, int position, float theta,
                                cudaStream_t stream) {
  const int total = num_heads * (head_dim / 2);
  const int blocks = (total + 255) / 256;
  if (dtype == QIC_DTYPE_BF16)
    rope_inplace_kernel<__nv_bfloat16>
        <<<blocks, 256, 0, stream>>>(static_cast<__nv_bfloat16*>(x), num_heads, head_dim, position, theta);
  else
    rope_inplace_kernel<__half><<<blocks, 256, 0, stream>>>(static_cast<__half*>(x), num_heads, head_dim, position, theta);
  return cudaGetLastError();
}

cudaError_t launch_sigmoid_mul_inplace(int dtype, void* x, const void* gate, int n, cudaStream_t stream) {
  const int blocks = (n + 255) / 256;
  if (dtype == QIC_DTYPE_BF16)
    sigmoid_mul_kernel<__nv_bfloat16>
        <<<blocks, 256, 0, stream>>>(static_cast<__nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(gate), n);
  else
    sigmoid_mul_kernel<__half><<<blocks, 256, 0, stream>>>(static_cast<__half*>(x), static_cast<const __half*>(gate), n);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t kv_append_t(const void* k_new, const void* v_new, const void* w, float eps, float theta, int pos,
                               const int32_t* pt, int P, long long ct, void* kc, void* vc, int Hkv, cudaStream_t s) {
  kv_append_kernel<T, D><<<Hkv, 32, 0, s>>>(static_cast<const T*>(k_new), static_cast<const T*>(v_new),
                                            static_cast<const T*>(w), eps, theta, pos, pt, P, ct,
                                            static_cast<T*>(kc), static_cast<T*>(vc), Hkv);
  return cudaGetLastError();
}

cudaError_t launch_kv_append(int dtype, const void* k_new, const void* v_new, const void* k_norm_w, float eps,
                             float theta, int position, const int32_t* page_table, int page_size, int64_t cache_tokens,
                             void* k_cache, void* v_cache, int num_kv_heads, int head_dim, cudaStream_t stream) {
  const long long ct = static_cast<long long>(cache_tokens);
  if (dtype == QIC_DTYPE_BF16) {
    switch (head_dim) {
      case 64: return kv_append_t<__nv_bfloat16, 64>(k_new, v_new, k_norm_w, eps, theta, position, page_table, page_size, ct, k_cache, v_cache, num_kv_heads, stream);
      case 128: return kv_append_t<__nv_bfloat16, 128>(k_new, v_new, k_norm_w, eps, theta, position, page_table, page_size, ct, k_cache, v_cache, num_kv_heads, stream);
      case 256: return kv_append_t<__nv_bfloat16, 256>(k_new, v_new, k_norm_w, eps, theta, position, page_table, page_size, ct, k_cache, v_cache, num_kv_heads, stream);
    }
  } else {
    switch (head_dim) {
      case 64: return kv_append_t<__half, 64>(k_new, v_new, k_norm_w, eps, theta, position, page_table, page_size, ct, k_cache, v_cache, num_kv_heads, stream);
      case 128: return kv_append_t<__half, 128>(k_new, v_new, k_norm_w, eps, theta, position, page_table, page_size, ct, k_cache, v_cache, num_kv_heads, stream);
      case 256: return kv_append_t<__half, 256>(k_new, v_new, k_norm_w, eps, theta, position, page_table, page_size, ct, k_cache, v_cache, num_kv_heads, stream);
    }
  }
  return cudaErrorInvalidValue;
}

}  // namespace qic
