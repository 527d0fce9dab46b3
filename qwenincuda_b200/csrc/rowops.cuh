// Warp-per-row device ops shared by the fused decode kernel and the standalone
// append / norm kernels: head RMSNorm and rotate-half RoPE of one head row.
//
// These must produce the same bytes as the reference kernels built with
// --use_fast_math (head_rmsnorm_kernel src/kernels.cu:78-112, rope_inplace_kernel
// src/kernels.cu:150-183 of the QweninCuda project), so every translation unit that
// includes this header is compiled with --use_fast_math too and writes the same
// expressions: rsqrtf(sum/hd + eps), x*inv*w, powf/cosf/sinf for the rotation, and
// rounding to the storage type after the norm and after the rotation. The sum of
// squares is accumulated in ascending index order with one rounding per square and
// per add, the order the reference's per-thread shared-memory atomicAdd takes.
#pragma once

#include "ptx.cuh"

namespace qic {

constexpr unsigned kFullMask = 0xffffffffu;

// Lane L holds elements [L*E, L*E+E) of a row of D elements, E = D/32.
template <typename T, int D>
__device__ __forceinline__ void row_load(const T* __restrict__ src, float (&v)[D / 32], int lane) {
  constexpr int E = D / 32;
  const T* p = src + lane * E;
  if constexpr (E == 8) {
    uint4 raw = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = to_f32<T>(e[i]);
  } else if constexpr (E == 4) {
    uint2 raw = *reinterpret_cast<const uint2*>(p);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = to_f32<T>(e[i]);
  } else {
    static_assert(E == 2, "head_dim must be 64, 128 or 256");
    uint32_t raw = *reinterpret_cast<const uint32_t*>(p);
    const T* e = reinterpret_cast<const T*>(&raw);
    v[0] = to_f32<T>(e[0]);
    v[1] = to_f32<T>(e[1]);
  }
}

// Stores the row rounded to T (values in v are already representable in T).
template <typename T, int D>
__device__ __forceinline__ void row_store(T* __restrict__ dst, const float (&v)[D / 32], int lane) {
  constexpr int E = D / 32;
  T* p = dst + lane * E;
  if constexpr (E == 8) {
    uint4 raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) e[i] = from_f32<T>(v[i]);
    *reinterpret_cast<uint4*>(p) = raw;
  } else if constexpr (E == 4) {
    uint2 raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) e[i] = from_f32<T>(v[i]);
    *reinterpret_cast<uint2*>(p) = raw;
  } else {
    uint32_t raw;
    T* e = reinterpret_cast<T*>(&raw);
    e[0] = from_f32<T>(v[0]);
    e[1] = from_f32<T>(v[1]);
    *reinterpret_cast<uint32_t*>(p) = raw;
  }
}

// Ascending-order fp32 sum of squares over the whole row, identical in every lane.
template <int D>
__device__ __forceinline__ float row_sumsq_ordered(const float (&v)[D / 32]) {
  constexpr int E = D / 32;
  float s = 0.0f;
#pragma unroll
  for (int src = 0; src < 32; ++src) {
#pragma unroll
    for (int e = 0; e < E; ++e) {
      float x = __shfl_sync(kFullMask, v[e], src);
      s = __fadd_rn(s, __fmul_rn(x, x));
    }
  }
  return s;
}

// In place: v = T(v * rsqrt(mean(v^2) + eps) * w), with this lane's weights wv
// already loaded (row_load layout).
template <typename T, int D>
__device__ __forceinline__ void row_rmsnorm_w(float (&v)[D / 32], const float (&wv)[D / 32], int head_dim,
                                              float eps) {
  constexpr int E = D / 32;
  float ssum = row_sumsq_ordered<D>(v);
  float inv_rms = rsqrtf(ssum / static_cast<float>(head_dim) + eps);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    float xv = v[e];
    v[e] = to_f32<T>(from_f32<T>(xv * inv_rms * wv[e]));
  }
}

// row_rmsnorm_w with the same ascending-order sum computed by lane 0 from the squares
// staged in shared memory (`scratch`: D floats, 16-byte aligned, free for this warp):
// the same bits, without the 32*E shuffles feeding the chain.
template <typename T, int D>
__device__ __forceinline__ void row_rmsnorm_w_staged(float (&v)[D / 32], const float (&wv)[D / 32], int head_dim,
                                                     float eps, float* scratch, int lane) {
  constexpr int E = D / 32;
#pragma unroll
  for (int e = 0; e < E; ++e) scratch[lane * E + e] = __fmul_rn(v[e], v[e]);
  __syncwarp();
  float ssum = 0.0f;
  if (lane == 0) {
    const float4* s4 = reinterpret_cast<const float4*>(scratch);
#pragma unroll 8
    for (int q = 0; q < D / 4; ++q) {
      const float4 t = s4[q];
      ssum = __fadd_rn(ssum, t.x);
      ssum = __fadd_rn(ssum, t.y);
      ssum = __fadd_rn(ssum, t.z);
      ssum = __fadd_rn(ssum, t.w);
    }
  }
  ssum = __shfl_sync(kFullMask, ssum, 0);
  __syncwarp();  // scratch may be reused after this
  float inv_rms = rsqrtf(ssum / static_cast<float>(head_dim) + eps);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    float xv = v[e];
    v[e] = to_f32<T>(from_f32<T>(xv * inv_rms * wv[e]));
  }
}

// row_rmsnorm_w with the sum of squares reduced as a butterfly (5 shuffle steps instead
// of the 32*E-step ordered chain): for rows whose bytes only feed tolerance-checked
// results (q), not rows stored for byte comparison (the appended k).
template <typename T, int D>
__device__ __forceinline__ void row_rmsnorm_w_tree(float (&v)[D / 32], const float (&wv)[D / 32], int head_dim,
                                                   float eps) {
  constexpr int E = D / 32;
  float ssum = 0.0f;
#pragma unroll
  for (int e = 0; e < E; ++e) ssum = __fadd_rn(ssum, __fmul_rn(v[e], v[e]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ssum += __shfl_xor_sync(kFullMask, ssum, o);
  float inv_rms = rsqrtf(ssum / static_cast<float>(head_dim) + eps);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    float xv = v[e];
    v[e] = to_f32<T>(from_f32<T>(xv * inv_rms * wv[e]));
  }
}

// In place: v = T(v * rsqrt(mean(v^2) + eps) * w).
template <typename T, int D>
__device__ __forceinline__ void row_rmsnorm(float (&v)[D / 32], const T* __restrict__ w, int head_dim, float eps,
                                            int lane) {
  float wv[D / 32];
  row_load<T, D>(w, wv, lane);
  row_rmsnorm_w<T, D>(v, wv, head_dim, eps);
}

// In place rotate-half RoPE at `position`: pairs (i, i + D/2). Lanes 0..15 hold the
// first half of the row and lanes 16..31 the second half, so partners are 16 lanes apart.
template <typename T, int D>
__device__ __forceinline__ void row_rope(float (&v)[D / 32], int head_dim, int position, float rope_theta,
                                         int lane) {
  constexpr int E = D / 32;
  const bool first = lane < 16;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    float other = __shfl_xor_sync(kFullMask, v[e], 16);
    float x0 = first ? v[e] : other;
    float x1 = first ? other : v[e];
    int d = (lane & 15) * E + e;
    float inv_freq = powf(rope_theta, -2.0f * static_cast<float>(d) / static_cast<float>(head_dim));
    float angle = static_cast<float>(position) * inv_freq;
    float c = cosf(angle);
    float s = sinf(angle);
    float y0 = x0 * c - x1 * s;
    float y1 = x1 * c + x0 * s;
    v[e] = to_f32<T>(from_f32<T>(first ? y0 : y1));
  }
}

// row_rope in two halves: the rotation of this lane's elements at `position` (depends
// on neither row, so it can be computed before the row is loaded), then its application.
// The same expressions as row_rope, so the same bytes.
template <int D>
__device__ __forceinline__ void row_rope_coeffs(float (&c)[D / 32], float (&sn)[D / 32], int head_dim, int position,
                                                float rope_theta, int lane) {
  constexpr int E = D / 32;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    int d = (lane & 15) * E + e;
    float inv_freq = powf(rope_theta, -2.0f * static_cast<float>(d) / static_cast<float>(head_dim));
    float angle = static_cast<float>(position) * inv_freq;
    c[e] = cosf(angle);
    sn[e] = sinf(angle);
  }
}

template <typename T, int D>
__device__ __forceinline__ void row_rope_apply(float (&v)[D / 32], const float (&c)[D / 32], const float (&sn)[D / 32],
                                               int lane) {
  constexpr int E = D / 32;
  const bool first = lane < 16;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    float other = __shfl_xor_sync(kFullMask, v[e], 16);
    float x0 = first ? v[e] : other;
    float x1 = first ? other : v[e];
    float y0 = x0 * c[e] - x1 * sn[e];
    float y1 = x1 * c[e] + x0 * sn[e];
    v[e] = to_f32<T>(from_f32<T>(first ? y0 : y1));
  }
}

}  // namespace qic
