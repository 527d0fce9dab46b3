// Weight-streaming GEMV projections of one decode token for B200 (sm_100a).
//
// Replaces QwenMiniModel::gemv (src/model.cpp:603-617 of the QweninCuda project): a
// cuBLAS GEMM with one column over column-major fp16 weights, out[o] = sum_i
// W[i*out_dim + o] x[i] with fp32 accumulation and a 16-bit result, and, fused into
// the same launch, its neighbours in the decode loop: the RMSNorm of the input
// (launch_rmsnorm, src/kernels.cu:50-76), the SwiGLU of the gate/up pair
// (launch_swiglu, src/kernels.cu:186-198) and the residual add (launch_add_inplace,
// src/kernels.cu:129-136). Several projections of the same input (q, k and v) run as
// one launch over their separate weight buffers ("segments").
//
// At batch 1 every weight byte is read once per token and used for one multiply-add:
// the bound is HBM bandwidth, not the tensor cores.
//
// Design
//  * A CTA (8 warps) owns a 256-column tile of one segment (or, for SwiGLU, the same
//    256 columns of gate and up) and a contiguous range of input rows. Lane l of a
//    warp reads columns [8l, 8l+8) of a row: each row of the tile is one 512-byte
//    coalesced run, 16 bytes per lane (evict-first L2 policy: weights are streamed
//    once per token). A warp takes blocks of 8 consecutive rows and keeps the next
//    block's loads in flight while it multiplies the current one.
//  * The CTAs of one tile split its rows and form a thread-block cluster (up to 16
//    CTAs). Each CTA sums its warps' partials through shared memory in warp order,
//    then every CTA of the cluster sums one slice of the tile's columns over the
//    cluster's CTAs through distributed shared memory, in rank order: the result does
//    not depend on scheduling.
//  * The normalised input x_norm[i] = T(x[i] * rsqrt(mean(x^2) + eps) * w[i]) (the
//    reference rounds it to its 16-bit buffer) is computed by every CTA for its own
//    rows; the sum of squares over the whole input costs one 8-24 KB read from L2.
//  * Epilogue per column: T(sum); SwiGLU: T(silu(g) * u) from the rounded g and u, as
//    the reference's swiglu kernel; residual: T(T(sum) + r), as its add kernel.
//  * Programmatic dependent launch (QIC_PDL): the first block of weight rows is
//    loaded before griddepcontrol.wait (weights are constants), the input, norm
//    weights and residual after it.
//
// Compiled with --use_fast_math, like the reference build, so rsqrtf and expf in the
// fused norm and SwiGLU are the same approximations.
#include <algorithm>

#include "qic_internal.h"
#include "rowops.cuh"

namespace qic {

namespace {

constexpr int kWarps = kGemvThreads / 32;
constexpr int kTile = kGemvTile;  // columns per tile
constexpr int kU = 8;             // rows per block of a warp
constexpr int kRedRow = kTile + 4;

__device__ __forceinline__ uint4 ld_weights(const void* p, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}

template <typename T>
__device__ __forceinline__ void fma8(float (&acc)[8], const uint4& w, float x) {
  const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = fmaf(x, to_f32<T>(e[i]), acc[i]);
}

__device__ __forceinline__ void pdl_wait_gemv() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_gemv() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename X>
__device__ __forceinline__ X* map_rank(X* p, int rank) {
  uint64_t out;
  asm volatile("mapa.u64 %0, %1, %2;" : "=l"(out) : "l"(reinterpret_cast<uint64_t>(p)), "r"(rank));
  return reinterpret_cast<X*>(out);
}

}  // namespace

// PAIR: segments 0 and 1 are the gate and up projections of a SwiGLU (warps 0-3 read
// gate rows, warps 4-7 the same columns of up); out = silu(gate) * up into segment 0.
template <typename T, bool PAIR, bool NORM>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(16) float gsm[];
  float* xs = gsm;                                   // [rows of this CTA] normalised input
  float* red = gsm + p.xs_floats;                    // [kWarps][kRedRow] warp partials
  float* part = red + kWarps * kRedRow;              // [2][kTile] this CTA's partial (gate, up)
  __shared__ float wsum[kWarps];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = p.splits;
  const int crank = blockIdx.x;  // rank in the cluster = split of the rows
  const int tile = blockIdx.y;
  // the tile's segment and first column
  int s = 0;
#pragma unroll
  for (int k = 1; k < kGemvMaxSegments; ++k)
    if (k < p.nseg && tile >= p.seg[k].tile0) s = k;
  const int c0 = (tile - p.seg[s].tile0) * kTile;
  const int N = p.seg[s].N;
  const int r0 = crank * p.rows_per_split;
  const int r1 = min(p.K, r0 + p.rows_per_split);
  const int nrows = max(0, r1 - r0);

  // this warp's weights: its segment (gate or up for a pair), column block of the lane
  const int wseg = PAIR ? (warp >= kWarps / 2 ? 1 : 0) : s;
  const int wslot = PAIR ? (warp & (kWarps / 2 - 1)) : warp;   // warp index within its group
  const int wstride = PAIR ? kWarps / 2 : kWarps;              // warps sharing the rows
  const int col = c0 + lane * 8;
  const bool col_ok = col < N;
  const T* wbase = static_cast<const T*>(p.seg[wseg].w) + static_cast<size_t>(r0) * N + col;
  const uint64_t pol = l2_policy_evict_first();
  const int nblk = (nrows + kU - 1) / kU;  // blocks of kU rows in this CTA's range

  pdl_launch_gemv();

  auto load_block = [&](uint4 (&v)[kU], int blk) {
    const int rb = blk * kU;
#pragma unroll
    for (int j = 0; j < kU; ++j) {
      const int r = rb + j;
      if (col_ok && r < nrows)
        v[j] = ld_weights(wbase + static_cast<size_t>(r) * N, pol);
      else
        v[j] = make_uint4(0u, 0u, 0u, 0u);
    }
  };

  // first block of weights before the preceding kernel's outputs are waited for
  uint4 bufA[kU], bufB[kU];
  int blk = wslot;
  if (blk < nblk) load_block(bufA, blk);
  if (p.flags & QIC_PDL) pdl_wait_gemv();

  // ---- the input of this CTA's rows, normalised when NORM ----
  float inv = 1.0f;
  if (NORM) {
    // sum of squares of the whole input: thread t takes i = t, t + 256, ... (the
    // reference's loop), then warps and the block in fixed order
    const T* x = static_cast<const T*>(p.x);
    float ss = 0.0f;
    for (int i = threadIdx.x; i < p.K; i += kGemvThreads) {
      const float v = to_f32<T>(x[i]);
      ss += v * v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(kFullMask, ss, o);
    if (lane == 0) wsum[warp] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) tot += wsum[w];
    inv = rsqrtf(tot / static_cast<float>(p.K) + p.eps);
  }
  {
    const T* x = static_cast<const T*>(p.x) + r0;
    const T* nw = NORM ? static_cast<const T*>(p.norm_w) + r0 : nullptr;
    for (int i = threadIdx.x; i < nblk * kU; i += kGemvThreads) {
      float v = 0.0f;
      if (i < nrows) {
        v = to_f32<T>(x[i]);
        if (NORM) v = to_f32<T>(from_f32<T>(v * inv * to_f32<T>(nw[i])));
      }
      xs[i] = v;
    }
  }
  __syncthreads();

  // ---- stream the rows: block blk in one buffer while the next one loads ----
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
  auto fma_block = [&](const uint4 (&v)[kU], int b) {
    const float4 xa = *reinterpret_cast<const float4*>(xs + b * kU);
    const float4 xb = *reinterpret_cast<const float4*>(xs + b * kU + 4);
    fma8<T>(acc, v[0], xa.x);
    fma8<T>(acc, v[1], xa.y);
    fma8<T>(acc, v[2], xa.z);
    fma8<T>(acc, v[3], xa.w);
    fma8<T>(acc, v[4], xb.x);
    fma8<T>(acc, v[5], xb.y);
    fma8<T>(acc, v[6], xb.z);
    fma8<T>(acc, v[7], xb.w);
  };
#pragma unroll 1
  while (blk < nblk) {
    const int nb = blk + wstride;
    if (nb < nblk) load_block(bufB, nb);
    fma_block(bufA, blk);
    if (nb >= nblk) break;
    const int nb2 = nb + wstride;
    if (nb2 < nblk) load_block(bufA, nb2);
    fma_block(bufB, nb);
    blk = nb2;
  }

  // ---- the CTA's partial: warps summed in order ----
  {
    float4* dst = reinterpret_cast<float4*>(red + warp * kRedRow + lane * 8);
    dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
  __syncthreads();
  {
    const int t = threadIdx.x;  // column t of the tile
    if (PAIR) {
      float g = 0.0f, u = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps / 2; ++w) g += red[w * kRedRow + t];
#pragma unroll
      for (int w = kWarps / 2; w < kWarps; ++w) u += red[w * kRedRow + t];
      part[t] = g;
      part[kTile + t] = u;
    } else {
      float v = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) v += red[w * kRedRow + t];
      part[t] = v;
    }
  }

  // ---- the cluster's CTAs each finish one slice of the tile's columns ----
  const int slice = (kTile + C - 1) / C;
  const int lo = crank * slice, hi = min(kTile, lo + slice);
  if (C > 1) {
    __syncwarp();
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
  } else {
    __syncthreads();
  }
  const int t = lo + threadIdx.x;
  if (t < hi) {
    float g = 0.0f, u = 0.0f;
    if (C > 1) {
      float pg[kGemvMaxSplits], pu[kGemvMaxSplits];
#pragma unroll
      for (int c = 0; c < kGemvMaxSplits; ++c) {
        if (c < C) {
          const float* rp = map_rank(part, c);
          pg[c] = rp[t];
          pu[c] = PAIR ? rp[kTile + t] : 0.0f;
        }
      }
#pragma unroll
      for (int c = 0; c < kGemvMaxSplits; ++c) {
        if (c < C) {
          g += pg[c];
          u += pu[c];
        }
      }
    } else {
      g = part[t];
      u = PAIR ? part[kTile + t] : 0.0f;
    }
    const int oc = c0 + t;
    if (oc < N) {
      T* out = static_cast<T*>(p.seg[s].out);
      if (PAIR) {
        const float gv = to_f32<T>(from_f32<T>(g));
        const float uv = to_f32<T>(from_f32<T>(u));
        const float sig = 1.0f / (1.0f + expf(-gv));
        out[oc] = from_f32<T>((gv * sig) * uv);
      } else {
        T y = from_f32<T>(g);
        if (p.seg[s].res != nullptr) y = from_f32<T>(to_f32<T>(y) + to_f32<T>(static_cast<const T*>(p.seg[s].res)[oc]));
        out[oc] = y;
      }
    }
  }
  if (C > 1) {
    // the peers' reads of this CTA's partial are done once every CTA has arrived
    asm volatile("barrier.cluster.arrive.relaxed;\n\tbarrier.cluster.wait;" ::: "memory");
  }
}

namespace {

template <typename T, bool PAIR, bool NORM>
cudaError_t launch_gemv_typed(const GemvParams& p, size_t smem, cudaStream_t stream) {
  auto kern = gemv_kernel<T, PAIR, NORM>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.splits, p.n_tiles, 1);
  cfg.blockDim = dim3(kGemvThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (p.flags & QIC_PDL) ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = static_cast<unsigned>(p.splits);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_gemv_dtype(const GemvParams& p, size_t smem, bool pair, bool norm, cudaStream_t stream) {
  if (pair) return norm ? launch_gemv_typed<T, true, true>(p, smem, stream) : launch_gemv_typed<T, true, false>(p, smem, stream);
  return norm ? launch_gemv_typed<T, false, true>(p, smem, stream) : launch_gemv_typed<T, false, false>(p, smem, stream);
}

template <typename T>
int max_clusters_typed(int cluster, size_t smem) {
  auto kern = gemv_kernel<T, false, true>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess ||
      cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cluster, 1, 1);
  cfg.blockDim = dim3(kGemvThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cluster);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

}  // namespace

size_t gemv_smem_bytes(int rows_per_split) {
  const int xs = ((rows_per_split + kU - 1) / kU) * kU;
  return static_cast<size_t>(xs + kWarps * kRedRow + 2 * kTile) * sizeof(float);
}

int gemv_max_active_clusters(int dtype, int cluster, int rows_per_split) {
  // cached per device, cluster size and shared-memory size class (rows rounded up to 1024)
  static int cache[64][kGemvMaxSplits + 1][9] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || cluster < 1 || cluster > kGemvMaxSplits) return 0;
  const int cls = std::min(8, (rows_per_split + 1023) / 1024);
  int& c = cache[dev][cluster][cls];
  if (c == 0) {
    const size_t smem = gemv_smem_bytes(cls * 1024);
    c = dtype == QIC_DTYPE_BF16 ? max_clusters_typed<__nv_bfloat16>(cluster, smem)
                                : max_clusters_typed<__half>(cluster, smem);
    if (c == 0) c = -1;
  }
  return c;
}

cudaError_t launch_gemv(int dtype, const GemvParams& p, bool pair, bool norm, cudaStream_t stream) {
  const size_t smem = gemv_smem_bytes(p.rows_per_split);
  if (dtype == QIC_DTYPE_BF16) return launch_gemv_dtype<__nv_bfloat16>(p, smem, pair, norm, stream);
  return launch_gemv_dtype<__half>(p, smem, pair, norm, stream);
}

}  // namespace qic
