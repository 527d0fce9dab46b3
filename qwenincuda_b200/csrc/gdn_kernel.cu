// Qwen3.5 GatedDeltaNet decode step on the device (sm_100a).
//
// Restates the host loop of run_linear_attention_block (src/model.cpp:692-791 of
// the QweninCuda project) as one kernel with the conv state and the recurrent state
// resident in HBM:
//   conv:   window <- [window[1..K-1], x];  mixed = silu(sum_t w[c,t] window[t])
//   split:  q = mixed[0:Hk*dk], k = mixed[Hk*dk:2*Hk*dk], v = mixed[2*Hk*dk:]
//   norm:   q, k L2-normalised per key head; value head h uses key head h/(Hv/Hk);
//           q scaled by 1/sqrt(dk)
//   gates:  beta = sigmoid(b), g = exp(-exp(A_log) * softplus(a + dt_bias))
//   state:  S *= g; kv_mem = S^T k; S += k (beta (v - kv_mem))^T; o = S^T q
//   out:    o * rsqrt(mean(o^2) + eps) * norm_w * silu(z)
//
// Work split: one thread-block cluster per key head, holding the value heads that
// share it (REP = Hv/Hk) times CB column blocks of the 128x128 fp32 state. Every CTA
// of a cluster recomputes the 2x128 q/k conv channels from the old conv state; a
// cluster barrier orders all those reads before any CTA writes the new conv state.
// The gated RMSNorm needs the sum of squares over all 128 columns of a value head,
// which the CB CTAs of that head exchange through distributed shared memory.
//
// Compiled without --use_fast_math: exp/log1p/sqrt follow the reference's host
// arithmetic (std::exp, std::log1pf, std::sqrt), and the per-element multiply/add
// chains use explicit round-to-nearest intrinsics so no FMA contraction is added.
#include <cooperative_groups.h>

#include "qic_internal.h"
#include "ptx.cuh"

namespace cg = cooperative_groups;

namespace qic {

constexpr int kGdnThreads = 128;
constexpr int kGdnDk = 128;
constexpr int kGdnDv = 128;

template <typename T, int REP, int CB>
__global__ void __launch_bounds__(kGdnThreads, 1) gated_delta_kernel(const qic_gdn_args a) {
  constexpr int NC = kGdnDv / CB;            // state columns owned by this CTA
  constexpr int QUADS = NC / 4;              // float4 column groups
  constexpr int RG = kGdnThreads / QUADS;    // row groups
  constexpr int RPT = kGdnDk / RG;           // rows per thread
  static_assert(RPT * RG == kGdnDk, "row split");

  // the next kernel in the stream may start (its own griddepcontrol.wait keeps it
  // from reading this kernel's outputs early)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int vloc = rank / CB;
  const int cb = rank % CB;
  const int kh = blockIdx.x / (REP * CB);
  const int Hk = a.num_k_heads;
  const int vh = kh * REP + vloc;
  const int K = a.conv_kernel;
  const int tid = threadIdx.x;

  __shared__ float q_s[kGdnDk];
  __shared__ float k_s[kGdnDk];
  __shared__ float v_s[NC];
  __shared__ float red[kGdnThreads / 32][NC];
  __shared__ float col_s[NC];
  __shared__ float scal[4];
  __shared__ float ssq_all[CB];  // the value head's CB partial sums of squares, pushed by their CTAs

  const T* qkv = static_cast<const T*>(a.qkv);
  const T* conv_w = static_cast<const T*>(a.conv_w);
  float* conv_state = a.conv_state;

  // ---- 0. every global load that does not depend on another is issued first. The
  // weights (conv taps, dt_bias, a_log, norm_w) are never written by a kernel, so they
  // are loaded before griddepcontrol.wait, while the preceding kernel may still run.
  // The states may be written by an earlier kernel that is still running (with
  // programmatic dependent launch a kernel further back in the stream can be, e.g.
  // this layer's previous step): before the wait they are only prefetched into L2,
  // the point of coherence, and read after it together with the step's inputs ----
  const int quad = tid % QUADS;
  const int rg = tid / QUADS;
  float* state = a.recurrent_state + static_cast<size_t>(vh) * kGdnDk * kGdnDv + cb * NC + quad * 4;
  // thread t: q channel t and k channel t of key head kh; v channel t (t < NC)
  const int cq = kh * kGdnDk + tid;
  const int ck = Hk * kGdnDk + kh * kGdnDk + tid;
  const int cv = 2 * Hk * kGdnDk + vh * kGdnDv + cb * NC + tid;
  // row `tid` of this CTA's state block (NC columns: one or two lines) and the three
  // conv windows
  {
    const float* row = a.recurrent_state + static_cast<size_t>(vh) * kGdnDk * kGdnDv +
                       static_cast<size_t>(tid) * kGdnDv + cb * NC;
#pragma unroll
    for (int c = 0; c < NC; c += 32) prefetch_l2(row + c);
  }
  prefetch_l2(conv_state + static_cast<size_t>(cq) * K);
  prefetch_l2(conv_state + static_cast<size_t>(ck) * K);
  if (tid < NC) prefetch_l2(conv_state + static_cast<size_t>(cv) * K);
  const T dt_raw = static_cast<const T*>(a.dt_bias)[vh];
  const T al_raw = static_cast<const T*>(a.a_log)[vh];
  T nw_raw = T();
  if (tid < NC) nw_raw = static_cast<const T*>(a.norm_w)[cb * NC + tid];
  T wt_q[8], wt_k[8], wt_v[8];  // conv taps of the three channels
  auto taps = [&](int c, T (&wt)[8]) {
#pragma unroll
    for (int t = 0; t < 8; ++t) wt[t] = (t < K) ? conv_w[static_cast<size_t>(c) * K + t] : T();
  };
  taps(cq, wt_q);
  taps(ck, wt_k);
  if (tid < NC) taps(cv, wt_v);

  asm volatile("griddepcontrol.wait;" ::: "memory");
  float4 s[RPT];
#pragma unroll
  for (int r = 0; r < RPT; ++r) s[r] = *reinterpret_cast<const float4*>(state + static_cast<size_t>(rg + RG * r) * kGdnDv);
  const T bv_raw = static_cast<const T*>(a.b)[vh];
  const T av_raw = static_cast<const T*>(a.a)[vh];
  T z_raw = T();
  if (tid < NC) z_raw = static_cast<const T*>(a.z)[static_cast<size_t>(vh) * kGdnDv + cb * NC + tid];

  // ---- 1. causal conv + SiLU from the old conv state ----
  // win: the channel's new window [old[1..K-1], x]
  float win_q[8], win_k[8], win_v[8];
  auto conv_channel = [&](int c, float (&win)[8], const T (&wt)[8]) -> float {
    const float x = to_f32<T>(qkv[c]);
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      win[t] = (t < K - 1) ? conv_state[static_cast<size_t>(c) * K + t + 1] : ((t == K - 1) ? x : 0.0f);
    }
    float acc = 0.0f;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      if (t < K) acc = __fadd_rn(acc, __fmul_rn(to_f32<T>(wt[t]), win[t]));
    }
    return acc / (1.0f + expf(-acc));
  };
  q_s[tid] = conv_channel(cq, win_q, wt_q);
  k_s[tid] = conv_channel(ck, win_k, wt_k);
  if (tid < NC) v_s[tid] = conv_channel(cv, win_v, wt_v);

  // every CTA of the cluster has read the old conv state past this point (first
  // phase of the cluster barrier; the conv-state writes wait for it further down)
  asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
  __syncthreads();

  // ---- 3. L2 norms of q and k, q scale (src/model.cpp:721-735) ----
  {
    const int w = tid >> 5, lane = tid & 31;
    float sq = 0.0f, sk = 0.0f;
    if (w == 0) {
#pragma unroll
      for (int i = lane; i < kGdnDk; i += 32) sq = __fadd_rn(sq, __fmul_rn(q_s[i], q_s[i]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
      if (lane == 0) scal[0] = 1.0f / sqrtf(sq + 1e-6f);
    } else if (w == 1) {
#pragma unroll
      for (int i = lane; i < kGdnDk; i += 32) sk = __fadd_rn(sk, __fmul_rn(k_s[i], k_s[i]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sk += __shfl_xor_sync(0xffffffffu, sk, o);
      if (lane == 0) scal[1] = 1.0f / sqrtf(sk + 1e-6f);
    }
  }
  __syncthreads();
  {
    const float qscale = 1.0f / sqrtf(static_cast<float>(kGdnDk));
    q_s[tid] = __fmul_rn(__fmul_rn(q_s[tid], scal[0]), qscale);
    k_s[tid] = __fmul_rn(k_s[tid], scal[1]);
  }
  __syncthreads();

  // ---- 4. gates (src/model.cpp:739-742) ----
  const float bval = to_f32<T>(bv_raw);
  const float beta = 1.0f / (1.0f + expf(-bval));
  const float av = to_f32<T>(av_raw) + to_f32<T>(dt_raw);
  const float softp = log1pf(expf(av));
  const float g = expf(-expf(to_f32<T>(al_raw)) * softp);

  // ---- 5. state block (loaded at the start): rows i = rg + RG*r, columns cb*NC + 4*quad .. +3 ----

  auto block_colsum = [&](float4 part) {
    // sum `part` over all threads with the same quad, result in col_s[4*quad + 0..3]
#pragma unroll
    for (int o = QUADS; o < 32; o <<= 1) {
      part.x += __shfl_xor_sync(0xffffffffu, part.x, o);
      part.y += __shfl_xor_sync(0xffffffffu, part.y, o);
      part.z += __shfl_xor_sync(0xffffffffu, part.z, o);
      part.w += __shfl_xor_sync(0xffffffffu, part.w, o);
    }
    const int w = tid >> 5, lane = tid & 31;
    if (lane < QUADS) {
      red[w][4 * quad + 0] = part.x;
      red[w][4 * quad + 1] = part.y;
      red[w][4 * quad + 2] = part.z;
      red[w][4 * quad + 3] = part.w;
    }
    __syncthreads();
    if (tid < NC) {
      float acc = 0.0f;
#pragma unroll
      for (int ww = 0; ww < kGdnThreads / 32; ++ww) acc += red[ww][tid];
      col_s[tid] = acc;
    }
    __syncthreads();
  };

  // decay, then kv_mem = S^T k
  float4 part = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int r = 0; r < RPT; ++r) {
    const float kr = k_s[rg + RG * r];
    s[r].x = __fmul_rn(s[r].x, g);
    s[r].y = __fmul_rn(s[r].y, g);
    s[r].z = __fmul_rn(s[r].z, g);
    s[r].w = __fmul_rn(s[r].w, g);
    part.x = __fadd_rn(part.x, __fmul_rn(s[r].x, kr));
    part.y = __fadd_rn(part.y, __fmul_rn(s[r].y, kr));
    part.z = __fadd_rn(part.z, __fmul_rn(s[r].z, kr));
    part.w = __fadd_rn(part.w, __fmul_rn(s[r].w, kr));
  }
  block_colsum(part);
  // delta = beta (v - kv_mem); S += k delta^T; o = S^T q
  float4 delta;
  delta.x = __fmul_rn(v_s[4 * quad + 0] - col_s[4 * quad + 0], beta);
  delta.y = __fmul_rn(v_s[4 * quad + 1] - col_s[4 * quad + 1], beta);
  delta.z = __fmul_rn(v_s[4 * quad + 2] - col_s[4 * quad + 2], beta);
  delta.w = __fmul_rn(v_s[4 * quad + 3] - col_s[4 * quad + 3], beta);
  __syncthreads();  // col_s is reused below
  part = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int r = 0; r < RPT; ++r) {
    const float kr = k_s[rg + RG * r];
    const float qr = q_s[rg + RG * r];
    s[r].x = __fadd_rn(s[r].x, __fmul_rn(kr, delta.x));
    s[r].y = __fadd_rn(s[r].y, __fmul_rn(kr, delta.y));
    s[r].z = __fadd_rn(s[r].z, __fmul_rn(kr, delta.z));
    s[r].w = __fadd_rn(s[r].w, __fmul_rn(kr, delta.w));
    part.x = __fadd_rn(part.x, __fmul_rn(s[r].x, qr));
    part.y = __fadd_rn(part.y, __fmul_rn(s[r].y, qr));
    part.z = __fadd_rn(part.z, __fmul_rn(s[r].z, qr));
    part.w = __fadd_rn(part.w, __fmul_rn(s[r].w, qr));
    *reinterpret_cast<float4*>(state + static_cast<size_t>(rg + RG * r) * kGdnDv) = s[r];
  }
  block_colsum(part);  // col_s = o for this CTA's columns

  // ---- 6. gated RMSNorm over the value head's 128 columns (src/model.cpp:777-791) ----
  float ss_mine = 0.0f;  // this CTA's sum of squares (warp 0)
  if (tid < 32) {
    float ss = 0.0f;
    for (int j = tid; j < NC; j += 32) ss = __fadd_rn(ss, __fmul_rn(col_s[j], col_s[j]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    ss_mine = ss;
  }
  // every CTA of the cluster is running and has read the old conv state
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
  // this CTA's partial goes into slot cb of every CTA of its value head (DSMEM stores
  // before the cluster barrier below), so after that barrier every CTA reads only its
  // own shared memory and may exit without waiting for its peers
  if (tid < CB) *cluster.map_shared_rank(&ssq_all[cb], vloc * CB + tid) = ss_mine;
  // the new conv state (q/k channels by the first value head's CTAs, v channels by
  // their owner)
  if (vloc == 0) {
    constexpr int QK_PER = kGdnDk / CB;
    if (tid >= cb * QK_PER && tid < (cb + 1) * QK_PER) {
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        if (t < K) {
          conv_state[static_cast<size_t>(cq) * K + t] = win_q[t];
          conv_state[static_cast<size_t>(ck) * K + t] = win_k[t];
        }
      }
    }
  }
  if (tid < NC) {
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      if (t < K) conv_state[static_cast<size_t>(cv) * K + t] = win_v[t];
    }
  }
  cluster.sync();  // every partial of this value head is in ssq_all
  float ss = 0.0f;
#pragma unroll
  for (int c = 0; c < CB; ++c) ss += ssq_all[c];
  const float inv = 1.0f / sqrtf(ss / static_cast<float>(kGdnDv) + a.eps);
  if (tid < NC) {
    const int j = cb * NC + tid;
    const float normed = __fmul_rn(col_s[tid], inv);
    const float zv = to_f32<T>(z_raw);
    const float gate = zv / (1.0f + expf(-zv));
    const float ww = to_f32<T>(nw_raw);
    static_cast<T*>(a.out)[static_cast<size_t>(vh) * kGdnDv + j] = from_f32<T>(__fmul_rn(__fmul_rn(normed, ww), gate));
  }
}

template <typename T, int REP, int CB>
static cudaError_t launch_gdn_typed(const qic_gdn_args& a, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.num_k_heads * REP * CB, 1, 1);
  cfg.blockDim = dim3(kGdnThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = REP * CB;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = (a.flags & QIC_PDL) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gated_delta_kernel<T, REP, CB>, a);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_gdn_rep(const qic_gdn_args& a, cudaStream_t stream) {
  switch (a.num_v_heads / a.num_k_heads) {
    case 1: return launch_gdn_typed<T, 1, 4>(a, stream);
    case 2: return launch_gdn_typed<T, 2, 4>(a, stream);
    case 4: return launch_gdn_typed<T, 4, 2>(a, stream);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_gated_delta(const qic_gdn_args& a, cudaStream_t stream) {
  if (a.dtype == QIC_DTYPE_BF16) return launch_gdn_rep<__nv_bfloat16>(a, stream);
  return launch_gdn_rep<__half>(a, stream);
}

}  // namespace qic
