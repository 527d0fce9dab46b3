// Small kernels of the decode-step runner (model_runner.cpp): the embedding row of the
// current token and the greedy token of the logits, both reading their scalar inputs
// from device memory so that one captured CUDA graph serves every token.
//
// embed_kernel restates launch_embedding_lookup (src/kernels.cu:29-48 of the
// QweninCuda project: token clamped to [0, vocab)); argmax_kernel restates
// argmax_host (src/model.cpp:78-89: the first index of the largest logit) on the
// device.
#include <cuda_runtime.h>

#include "qic_internal.h"
#include "rowops.cuh"

namespace qic {

template <typename T>
__global__ void __launch_bounds__(256) embed_kernel(const T* __restrict__ table, int vocab, int hidden,
                                                    const int32_t* __restrict__ token, T* __restrict__ out) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  int t = *token;
  t = t < 0 ? 0 : (t >= vocab ? vocab - 1 : t);
  const uint4* src = reinterpret_cast<const uint4*>(table + static_cast<size_t>(t) * hidden);
  uint4* dst = reinterpret_cast<uint4*>(out);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden / 8; i += gridDim.x * blockDim.x) dst[i] = src[i];
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// One CTA: the first index of the largest value, starting from -1e30 like
// argmax_host (NaN never wins: comparisons are false). n is a multiple of 8: every
// thread reads 16-byte vectors, four in flight, in increasing index order.
template <typename T>
__global__ void __launch_bounds__(1024) argmax_kernel(const T* __restrict__ x, int n, int32_t* __restrict__ out) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ float sv[32];
  __shared__ int si[32];
  constexpr int U = 4;
  const int nv = n / 8;
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  float best = -1e30f;
  int bi = 0x7fffffff;
  for (int base = threadIdx.x; base < nv; base += blockDim.x * U) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * blockDim.x;
      v[u] = i < nv ? xv[i] : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * blockDim.x;
      if (i < nv) {
        const T* e = reinterpret_cast<const T*>(&v[u]);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float f = to_f32<T>(e[k]);
          if (f > best) {  // ascending index within the thread: the first of equal values stays
            best = f;
            bi = i * 8 + k;
          }
        }
      }
    }
  }
  auto better = [](float v, int i, float w, int j) { return w > v || (w == v && j < i); };
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(kFullMask, best, o);
    const int j = __shfl_xor_sync(kFullMask, bi, o);
    if (better(best, bi, w, j)) {
      best = w;
      bi = j;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : -1e30f;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float w = __shfl_xor_sync(kFullMask, best, o);
      const int j = __shfl_xor_sync(kFullMask, bi, o);
      if (better(best, bi, w, j)) {
        best = w;
        bi = j;
      }
    }
    if (lane == 0) *out = bi == 0x7fffffff ? 0 : bi;
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

namespace {

template <typename K, typename... A>
cudaError_t launch_pdl(K kern, dim3 grid, dim3 block, cudaStream_t stream, A... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  return e == cudaSuccess ? cudaGetLastError() : e;
}

}  // namespace

cudaError_t launch_embed(int dtype, const void* table, int vocab, int hidden, const int32_t* token, void* out,
                         cudaStream_t stream) {
  const int blocks = (hidden / 8 + 255) / 256;
  if (dtype == QIC_DTYPE_BF16)
    return launch_pdl(embed_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), stream,
                      static_cast<const __nv_bfloat16*>(table), vocab, hidden, token, static_cast<__nv_bfloat16*>(out));
  return launch_pdl(embed_kernel<__half>, dim3(blocks), dim3(256), stream, static_cast<const __half*>(table), vocab,
                    hidden, token, static_cast<__half*>(out));
}

cudaError_t launch_argmax(int dtype, const void* x, int n, int32_t* out, cudaStream_t stream) {
  if (dtype == QIC_DTYPE_BF16)
    return launch_pdl(argmax_kernel<__nv_bfloat16>, dim3(1), dim3(1024), stream, static_cast<const __nv_bfloat16*>(x),
                      n, out);
  return launch_pdl(argmax_kernel<__half>, dim3(1), dim3(1024), stream, static_cast<const __half*>(x), n, out);
}

}  // namespace qic
