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
//    256 columns of gate and up) and a contiguous range of input rows. A warp takes
//    blocks of 8 consecutive rows of the tile (8 x 512 contiguous bytes per row) and
//    streams them through its own 3-slot shared-memory ring with 2D TMA copies that
//    its lane 0 issues (evict-first L2 policy: weights are streamed once per token);
//    each slot is refilled as soon as the warp has multiplied it, and no warp waits
//    for another. Lane l multiplies columns [8l, 8l+8) of every row (16-byte shared
//    loads, fp32 fused multiply-adds in row order). Measured against an earlier
//    version that kept two blocks of 16-byte global loads in registers per warp: the
//    registers capped the bytes in flight per SM and the stream at about 81% of the
//    copy bandwidth even in the longest launch.
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
//  * Programmatic dependent launch (QIC_PDL): the ring's first fill is issued before
//    griddepcontrol.wait (weights are constants), the input, norm weights and
//    residual are read after it.
//  * Every wait is bounded (ptx.cuh): on timeout the warp records QIC_DEV_TIMEOUT in
//    the caller's status word (if any), drains its copies (bounded) and the CTA
//    finishes without writing outputs.
//
// Compiled with --use_fast_math, like the reference build, so rsqrtf and expf in the
// fused norm and SwiGLU are the same approximations.
#include <algorithm>

#include "qic_internal.h"
#include "rowops.cuh"

namespace qic {

namespace {

constexpr int kWarps = kGemvThreads / 32;
constexpr int kTile = kGemvTile;                         // columns per tile
constexpr int kRowsSlot = kGemvRowsPerSlot;              // rows per TMA box (one ring slot)
constexpr int kSlotsW = kGemvSlotsPerWarp;               // ring slots per warp
constexpr int kSlotBytes = kRowsSlot * kTile * 2;        // 4 KB
constexpr int kRingBytes = kWarps * kSlotsW * kSlotBytes;  // 96 KB
constexpr int kRedRow = kTile + 4;
static_assert(kRingBytes >= (kWarps * kRedRow + 2 * kTile) * 4, "warp partials reuse the ring");

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
  extern __shared__ uint8_t gsm_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kRingBytes);  // [kWarps][kSlotsW]
  float* xs = reinterpret_cast<float*>(full + kWarps * kSlotsW);     // [rows of this CTA] input
  // after the stream the ring is free: warp partials and the CTA's partial live there
  float* red = reinterpret_cast<float*>(ring);                       // [kWarps][kRedRow]
  float* part = red + kWarps * kRedRow;                              // [2][kTile] (gate, up)
  __shared__ float wsum[kWarps];
  __shared__ int aborted;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = p.splits;
  const int crank = blockIdx.x;  // rank in the cluster = split of the rows
  // the tile columns this CTA finishes after the cluster's reduction (a division by
  // the runtime cluster size, done here rather than after the stream)
  const int slice = (kTile + C - 1) / C;
  const int lo = crank * slice, hi = min(kTile, lo + slice);
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
  const int nblk = (nrows + kRowsSlot - 1) / kRowsSlot;  // blocks of kRowsSlot rows in this CTA's range

  // this warp's weights (gate or up for a pair) and its blocks: wslot, wslot + wstride, ...
  const int wseg = PAIR ? (warp >= kWarps / 2 ? 1 : 0) : s;
  const int wslot = PAIR ? (warp & (kWarps / 2 - 1)) : warp;
  const int wstride = PAIR ? kWarps / 2 : kWarps;
  const int nmine = wslot < nblk ? (nblk - wslot + wstride - 1) / wstride : 0;
  const CUtensorMap* tm = &p.tm[wseg];
  uint8_t* wring = ring + warp * kSlotsW * kSlotBytes;
  uint64_t* wfull = full + warp * kSlotsW;
  const uint64_t pol = l2_policy_evict_first();
  const uint64_t deadline = globaltimer_ns() + p.timeout_ns;

  if (lane == 0) {
    if (warp == 0) aborted = 0;
#pragma unroll
    for (int k = 0; k < kSlotsW; ++k) mbar_init(&wfull[k], 1);
    fence_mbar_init();
    tma_prefetch_desc(tm);
  }
  __syncwarp();
  pdl_launch_gemv();

  // Block m of this warp: rows r0 + (wslot + m*wstride)*kRowsSlot .. +kRowsSlot, all
  // kTile columns of the tile, one 2D TMA box into ring slot m % kSlotsW. Rows past
  // the input's end are filled with zeros by the copy.
  auto issue = [&](int m) {
    if (lane == 0) {
      const int k = m % kSlotsW;
      mbar_arrive_expect_tx(&wfull[k], kSlotBytes);
      tma_load_2d(wring + k * kSlotBytes, tm, &wfull[k], c0, r0 + (wslot + m * wstride) * kRowsSlot, pol);
    }
  };
  // the ring's first fill before the preceding kernel's outputs are waited for
  // (weights are constants). Measured and not kept: also prefetching the warp's next
  // 4 / 16 / 64 blocks into L2 here (Qwen3-8B projection chain 19.6 -> 19.7 / 21.0 /
  // 22.0 us per launch).
#pragma unroll
  for (int m = 0; m < kSlotsW; ++m)
    if (m < nmine) issue(m);
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
    for (int i = threadIdx.x; i < nblk * kRowsSlot; i += kGemvThreads) {
      float v = 0.0f;
      if (i < nrows) {
        v = to_f32<T>(x[i]);
        if (NORM) v = to_f32<T>(from_f32<T>(v * inv * to_f32<T>(nw[i])));
      }
      xs[i] = v;
    }
  }
  __syncthreads();

  // ---- stream: wait for a slot, multiply its rows, refill it ----
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
  bool ok = true;
  int m = 0;
#pragma unroll 1
  for (; m < nmine; ++m) {
    const int k = m % kSlotsW;
    if (!__all_sync(kFullMask, mbar_wait(&wfull[k], (m / kSlotsW) & 1, deadline))) {
      ok = false;
      break;
    }
    const uint8_t* slot = wring + k * kSlotBytes + lane * 16;
    const float* xb = xs + (wslot + m * wstride) * kRowsSlot;
    const float4 xa = *reinterpret_cast<const float4*>(xb);
    const float4 xc = *reinterpret_cast<const float4*>(xb + 4);
    const float xr[8] = {xa.x, xa.y, xa.z, xa.w, xc.x, xc.y, xc.z, xc.w};
#pragma unroll
    for (int j = 0; j < kRowsSlot; ++j) {
      const uint4 w = *reinterpret_cast<const uint4*>(slot + j * (kTile * 2));
      fma8<T>(acc, w, xr[j]);
    }
    // the slot's values are consumed (the accumulators depend on every row) before
    // the copy that overwrites it is issued
    asm volatile("" ::"f"(acc[0]), "f"(acc[1]), "f"(acc[2]), "f"(acc[3]), "f"(acc[4]), "f"(acc[5]), "f"(acc[6]),
                 "f"(acc[7])
                 : "memory");
    __syncwarp();
    if (m + kSlotsW < nmine) issue(m + kSlotsW);
  }
  if (!ok) {
    if (lane == 0) {
      record_status(p.status, QIC_DEV_TIMEOUT);
      aborted = 1;
    }
    // wait (bounded) for this warp's copies still in flight before the ring is reused
    const uint64_t dl2 = globaltimer_ns() + p.timeout_ns;
    for (int mm = m; mm < nmine && mm < m + kSlotsW; ++mm)
      mbar_wait(&wfull[mm % kSlotsW], (mm / kSlotsW) & 1, dl2);
    __syncwarp();
  }
  __syncthreads();  // every warp is past its stream: the ring holds no copy in flight

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
  if (C > 1) {
    __syncwarp();
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
  } else {
    __syncthreads();
  }
  const int t = lo + threadIdx.x;
  if (t < hi) {
    float g = 0.0f, u = 0.0f;
    int bad = 0;  // a CTA of the cluster gave up on a copy: its partial is incomplete
    if (C > 1) {
      float pg[kGemvMaxSplits], pu[kGemvMaxSplits];
      int pb[kGemvMaxSplits];
#pragma unroll
      for (int c = 0; c < kGemvMaxSplits; ++c) {
        if (c < C) {
          const float* rp = map_rank(part, c);
          pg[c] = rp[t];
          pu[c] = PAIR ? rp[kTile + t] : 0.0f;
          pb[c] = *map_rank(&aborted, c);
        }
      }
#pragma unroll
      for (int c = 0; c < kGemvMaxSplits; ++c) {
        if (c < C) {
          g += pg[c];
          u += pu[c];
          bad |= pb[c];
        }
      }
    } else {
      g = part[t];
      u = PAIR ? part[kTile + t] : 0.0f;
      bad = aborted;
    }
    const int oc = c0 + t;
    if (oc < N && !bad) {
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

// Kernel attributes, set once per device: the largest dynamic shared memory any launch
// uses, and clusters above 8 CTAs.
template <typename T, bool PAIR, bool NORM>
cudaError_t configure_gemv() {
  static unsigned long long configured = 0;  // one bit per device ordinal
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 64 && (configured & (1ull << dev))) return cudaSuccess;
  auto kern = gemv_kernel<T, PAIR, NORM>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(gemv_smem_bytes(kGemvMaxRowsPerSplit)));
  if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e == cudaSuccess && dev < 64) configured |= 1ull << dev;
  return e;
}

template <typename T, bool PAIR, bool NORM>
cudaError_t launch_gemv_typed(const GemvParams& p, size_t smem, cudaStream_t stream) {
  auto kern = gemv_kernel<T, PAIR, NORM>;
  cudaError_t e = configure_gemv<T, PAIR, NORM>();
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
  if (configure_gemv<T, false, true>() != cudaSuccess) {
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
  const int xs = ((rows_per_split + kRowsSlot - 1) / kRowsSlot) * kRowsSlot;
  return 1024 + kRingBytes + kWarps * kSlotsW * sizeof(uint64_t) + static_cast<size_t>(xs) * sizeof(float);
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
