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
// The read-out uses o = (g S)^T q + (k . q) delta, equal to S'^T q, so the two column
// sums over the state come from one pass and one reduction (with the q/k norms),
// before the state update.
//
// Work split: one thread-block cluster per key head, holding the value heads that
// share it (REP = Hv/Hk) times CB column blocks of the 128x128 fp32 state. Every CTA
// of a cluster recomputes the 2x128 q/k conv channels from the old conv state; a
// cluster barrier orders all those reads before any CTA writes the new conv state.
// The gated RMSNorm needs the sum of squares over all 128 columns of a value head:
// each of the CB CTAs of that head stores its partial into every peer's shared memory
// with st.async, and each CTA waits on its own mbarrier for the CB partials (no
// cluster-wide barrier at the end, whose release would wait for this CTA's state
// stores to drain).
//
// Compiled with --use_fast_math: exp, log1p, sqrt and the divisions of the gates, the
// norms and SiLU are the hardware approximations (the step's outputs and state stay
// within the tolerances of the reference's host arithmetic, std::exp / std::log1pf /
// std::sqrt; the IEEE forms cost 0.4 us of a 3.85 us step), while the state's
// per-element multiply/add chains keep explicit round-to-nearest intrinsics, so no FMA
// contraction changes their order.
#include <cooperative_groups.h>

#include "qic_internal.h"
#include "ptx.cuh"

namespace cg = cooperative_groups;

namespace qic {

constexpr int kGdnThreads = 128;
constexpr int kGdnDk = 128;
constexpr int kGdnDv = 128;
constexpr uint64_t kGdnWaitNs = 2000000000ull;  // bound on the wait for the value head's peers

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
  __shared__ float red[kGdnThreads / 32][NC];   // warp partials of S_g^T q
  __shared__ float redk[kGdnThreads / 32][NC];  // warp partials of S_g^T k
  __shared__ float redn[kGdnThreads / 32][4];   // warp partials of |q|^2, |k|^2, k . q
  __shared__ __align__(16) float delta_s[NC];
  __shared__ float col_s[NC];
  __shared__ float ssq_all[CB];  // the value head's CB partial sums of squares, pushed by their CTAs
  __shared__ __align__(8) uint64_t ssq_bar;  // completes when all CB partials have landed in ssq_all
  if (tid == 0) {
    mbar_init(&ssq_bar, 1);
    mbar_arrive_expect_tx(&ssq_bar, CB * 4);
    fence_mbar_init();  // visible to the peers' st.async after the cluster barrier's first phase
  }

  const T* qkv = static_cast<const T*>(a.qkv);
  const T* conv_w = static_cast<const T*>(a.conv_w);
  float* conv_state = a.conv_state;

  // ---- 0. every global load that does not depend on another is issued first. The
  // weights (conv taps, dt_bias, a_log, norm_w) are never written by a kernel, so they
  // are loaded before griddepcontrol.wait, while the preceding kernel may still run.
  // The states may be written by an earlier kernel that is still running (with
  // programmatic dependent launch a kernel further back in the stream can be, e.g.
  // this layer's previous step): before the wait they are only prefetched into L2,
  // the point of coherence, and read after it together with the step's inputs, unless
  // the caller guarantees their writer has completed (QIC_GDN_STATES_READY) ----
  const int quad = tid % QUADS;
  const int rg = tid / QUADS;
  float* state = a.recurrent_state + static_cast<size_t>(vh) * kGdnDk * kGdnDv + cb * NC + quad * 4;
  // thread t: q channel t and k channel t of key head kh; v channel t (t < NC)
  const int cq = kh * kGdnDk + tid;
  const int ck = Hk * kGdnDk + kh * kGdnDk + tid;
  const int cv = 2 * Hk * kGdnDk + vh * kGdnDv + cb * NC + tid;
  // With QIC_GDN_STATES_READY the caller guarantees that the states' last writer has
  // completed, so they are read here; otherwise row `tid` of this CTA's state block (NC
  // columns: one or two lines) and the three conv windows are prefetched.
  const bool states_ready = (a.flags & QIC_GDN_STATES_READY) != 0;
  float4 s[RPT];
  // win: the channel's new window [old[1..K-1], x] (x is filled in after the wait)
  float win_q[8], win_k[8], win_v[8];
  auto load_state = [&]() {
#pragma unroll
    for (int r = 0; r < RPT; ++r)
      s[r] = *reinterpret_cast<const float4*>(state + static_cast<size_t>(rg + RG * r) * kGdnDv);
  };
  auto load_window = [&](int c, float (&win)[8]) {
#pragma unroll
    for (int t = 0; t < 8; ++t) win[t] = (t < K - 1) ? conv_state[static_cast<size_t>(c) * K + t + 1] : 0.0f;
  };
  auto load_windows = [&]() {
    load_window(cq, win_q);
    load_window(ck, win_k);
    if (tid < NC) load_window(cv, win_v);
  };
  if (states_ready) {
    load_state();
    load_windows();
  } else {
    const float* row = a.recurrent_state + static_cast<size_t>(vh) * kGdnDk * kGdnDv +
                       static_cast<size_t>(tid) * kGdnDv + cb * NC;
#pragma unroll
    for (int c = 0; c < NC; c += 32) prefetch_l2(row + c);
    prefetch_l2(conv_state + static_cast<size_t>(cq) * K);
    prefetch_l2(conv_state + static_cast<size_t>(ck) * K);
    if (tid < NC) prefetch_l2(conv_state + static_cast<size_t>(cv) * K);
  }
  // The step's inputs may still be written by the preceding kernel: they are only
  // brought into L2 here (no value is read; L2 is the point of coherence, so a later
  // write lands there) and read after the wait. One prefetch per 64-byte run of a warp.
  if ((tid & 31) == 0) {
    prefetch_l2(qkv + cq);
    prefetch_l2(qkv + ck);
    if (tid < NC) {
      prefetch_l2(qkv + cv);
      prefetch_l2(static_cast<const T*>(a.z) + static_cast<size_t>(vh) * kGdnDv + cb * NC + tid);
    }
    if (tid == 0) {
      prefetch_l2(static_cast<const T*>(a.b) + vh);
      prefetch_l2(static_cast<const T*>(a.a) + vh);
    }
  }
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
  if (!states_ready) {
    load_state();
    load_windows();
  }
  const T bv_raw = static_cast<const T*>(a.b)[vh];
  const T av_raw = static_cast<const T*>(a.a)[vh];
  T z_raw = T();
  if (tid < NC) z_raw = static_cast<const T*>(a.z)[static_cast<size_t>(vh) * kGdnDv + cb * NC + tid];

  // ---- 1. causal conv + SiLU from the old conv state ----
  auto conv_channel = [&](int c, float (&win)[8], const T (&wt)[8]) -> float {
    const float x = to_f32<T>(qkv[c]);
#pragma unroll
    for (int t = 0; t < 8; ++t)
      if (t == K - 1) win[t] = x;
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

  // ---- 3-4. gates (src/model.cpp:739-742) ----
  const float bval = to_f32<T>(bv_raw);
  const float beta = 1.0f / (1.0f + expf(-bval));
  const float av = to_f32<T>(av_raw) + to_f32<T>(dt_raw);
  const float softp = log1pf(expf(av));
  const float g = expf(-expf(to_f32<T>(al_raw)) * softp);

  // ---- 5. one pass over the decayed state (src/model.cpp:721-775) ----
  // With q^ = q / |q| / sqrt(dk), k^ = k / |k| and S_g = g S (the decayed state):
  //   kv_mem = S_g^T k^,  delta = beta (v - kv_mem),  S' = S_g + k^ delta^T,
  //   o = S'^T q^ = S_g^T q^ + (k^ . q^) delta.
  // So the column sums S_g^T q and S_g^T k (raw conv outputs, scaled afterwards) and
  // the sums |q|^2, |k|^2 and k . q come out of one reduction, and the state update
  // is off the output's path. The state rows of this CTA were loaded at the start:
  // rows i = rg + RG*r, columns cb*NC + 4*quad .. +3.
  float4 pq = make_float4(0.f, 0.f, 0.f, 0.f), pk = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int r = 0; r < RPT; ++r) {
    const float qr = q_s[rg + RG * r];
    const float kr = k_s[rg + RG * r];
    s[r].x = __fmul_rn(s[r].x, g);
    s[r].y = __fmul_rn(s[r].y, g);
    s[r].z = __fmul_rn(s[r].z, g);
    s[r].w = __fmul_rn(s[r].w, g);
    pq.x = __fadd_rn(pq.x, __fmul_rn(s[r].x, qr));
    pq.y = __fadd_rn(pq.y, __fmul_rn(s[r].y, qr));
    pq.z = __fadd_rn(pq.z, __fmul_rn(s[r].z, qr));
    pq.w = __fadd_rn(pq.w, __fmul_rn(s[r].w, qr));
    pk.x = __fadd_rn(pk.x, __fmul_rn(s[r].x, kr));
    pk.y = __fadd_rn(pk.y, __fmul_rn(s[r].y, kr));
    pk.z = __fadd_rn(pk.z, __fmul_rn(s[r].z, kr));
    pk.w = __fadd_rn(pk.w, __fmul_rn(s[r].w, kr));
  }
  // channel tid's contributions to |q|^2, |k|^2 and k . q
  float nq = __fmul_rn(q_s[tid], q_s[tid]), nk = __fmul_rn(k_s[tid], k_s[tid]), nqk = __fmul_rn(q_s[tid], k_s[tid]);
  const int w = tid >> 5, lane = tid & 31;
#pragma unroll
  for (int o = QUADS; o < 32; o <<= 1) {
    pq.x += __shfl_xor_sync(0xffffffffu, pq.x, o);
    pq.y += __shfl_xor_sync(0xffffffffu, pq.y, o);
    pq.z += __shfl_xor_sync(0xffffffffu, pq.z, o);
    pq.w += __shfl_xor_sync(0xffffffffu, pq.w, o);
    pk.x += __shfl_xor_sync(0xffffffffu, pk.x, o);
    pk.y += __shfl_xor_sync(0xffffffffu, pk.y, o);
    pk.z += __shfl_xor_sync(0xffffffffu, pk.z, o);
    pk.w += __shfl_xor_sync(0xffffffffu, pk.w, o);
  }
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    nq += __shfl_xor_sync(0xffffffffu, nq, o);
    nk += __shfl_xor_sync(0xffffffffu, nk, o);
    nqk += __shfl_xor_sync(0xffffffffu, nqk, o);
  }
  if (lane < QUADS) {
    red[w][4 * quad + 0] = pq.x;
    red[w][4 * quad + 1] = pq.y;
    red[w][4 * quad + 2] = pq.z;
    red[w][4 * quad + 3] = pq.w;
    redk[w][4 * quad + 0] = pk.x;
    redk[w][4 * quad + 1] = pk.y;
    redk[w][4 * quad + 2] = pk.z;
    redk[w][4 * quad + 3] = pk.w;
  }
  if (lane == 0) {
    redn[w][0] = nq;
    redn[w][1] = nk;
    redn[w][2] = nqk;
  }
  __syncthreads();
  // the norms (every thread, warps summed in order)
  float sq = 0.0f, sk = 0.0f, sqk = 0.0f;
#pragma unroll
  for (int ww = 0; ww < kGdnThreads / 32; ++ww) {
    sq += redn[ww][0];
    sk += redn[ww][1];
    sqk += redn[ww][2];
  }
  const float inv_q = 1.0f / sqrtf(sq + 1e-6f);
  const float inv_k = 1.0f / sqrtf(sk + 1e-6f);
  const float qscale = __fmul_rn(inv_q, 1.0f / sqrtf(static_cast<float>(kGdnDk)));
  const float kq = __fmul_rn(__fmul_rn(sqk, inv_k), qscale);  // k^ . q^
  // Warp 0 sends this CTA's sum of squares into slot cb of every CTA of its value head
  // (after the cluster barrier's first phase: every CTA runs, has initialised its
  // mbarrier and has read the old conv state); each CTA then reads only its own shared
  // memory once its mbarrier shows all CB slots written, so no CTA waits at exit for
  // its peers.
  auto push_ssq = [&](float ss) {
    asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
    if (tid < CB) st_async_cluster_f32(&ssq_all[cb], &ssq_bar, vloc * CB + tid, ss);
  };
  if (tid < NC) {
    float cq_sum = 0.0f, ck_sum = 0.0f;
#pragma unroll
    for (int ww = 0; ww < kGdnThreads / 32; ++ww) {
      cq_sum += red[ww][tid];
      ck_sum += redk[ww][tid];
    }
    const float kv_mem = __fmul_rn(ck_sum, inv_k);
    const float delta = __fmul_rn(v_s[tid] - kv_mem, beta);
    delta_s[tid] = delta;
    const float o = __fadd_rn(__fmul_rn(cq_sum, qscale), __fmul_rn(kq, delta));
    col_s[tid] = o;
    if constexpr (NC == 32) {
      // warp 0 holds all of this CTA's columns: its sum of squares goes to the value
      // head's CTAs now, ahead of the state update
      float ss = __fmul_rn(o, o);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      push_ssq(ss);
    }
  }
  __syncthreads();
  // the new state: S' = S_g + k^ delta^T
  {
    const float4 delta = *reinterpret_cast<const float4*>(&delta_s[4 * quad]);
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
      const float kr = __fmul_rn(k_s[rg + RG * r], inv_k);
      s[r].x = __fadd_rn(s[r].x, __fmul_rn(kr, delta.x));
      s[r].y = __fadd_rn(s[r].y, __fmul_rn(kr, delta.y));
      s[r].z = __fadd_rn(s[r].z, __fmul_rn(kr, delta.z));
      s[r].w = __fadd_rn(s[r].w, __fmul_rn(kr, delta.w));
      *reinterpret_cast<float4*>(state + static_cast<size_t>(rg + RG * r) * kGdnDv) = s[r];
    }
  }

  // ---- 6. gated RMSNorm over the value head's 128 columns (src/model.cpp:777-791) ----
  if constexpr (NC != 32) {
    float ss = 0.0f;  // this CTA's sum of squares (warp 0)
    if (tid < 32) {
      for (int j = tid; j < NC; j += 32) ss = __fadd_rn(ss, __fmul_rn(col_s[j], col_s[j]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      push_ssq(ss);
    }
  }
  // the threads that did not send a partial: every CTA of the cluster has read the old
  // conv state before any conv-state write below
  if (tid >= 32) asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
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
  if (tid >= NC) return;
  // every partial of this value head is in ssq_all (bounded wait: the peers of a
  // cluster run together, so only a broken launch gives up)
  if (!mbar_wait(&ssq_bar, 0, globaltimer_ns() + kGdnWaitNs)) {
    if (a.status != nullptr) record_status(a.status, QIC_DEV_TIMEOUT);
    return;
  }
  float ss = 0.0f;
#pragma unroll
  for (int c = 0; c < CB; ++c) ss += ssq_all[c];
  const float inv = 1.0f / sqrtf(ss / static_cast<float>(kGdnDv) + a.eps);
  const int j = cb * NC + tid;
  const float normed = __fmul_rn(col_s[tid], inv);
  const float zv = to_f32<T>(z_raw);
  const float gate = zv / (1.0f + expf(-zv));
  const float ww = to_f32<T>(nw_raw);
  static_cast<T*>(a.out)[static_cast<size_t>(vh) * kGdnDv + j] = from_f32<T>(__fmul_rn(__fmul_rn(normed, ww), gate));
}

template <typename T, int REP, int CB>
static cudaError_t launch_gdn_typed(const qic_gdn_args& a, cudaStream_t stream) {
  if constexpr (REP * CB > 8) {
    // clusters of more than 8 CTAs are non-portable: allowed once per device
    static unsigned long long allowed = 0;  // one bit per device ordinal
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 64 || !(allowed & (1ull << dev))) {
      e = cudaFuncSetAttribute(gated_delta_kernel<T, REP, CB>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess) return e;
      if (dev < 64) allowed |= 1ull << dev;
    }
  }
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
    // two value heads per key head (Qwen3.5): 8 column blocks each, clusters of 16
    // (32-layer chain, A/B on one box: 4 blocks 3.97 us per layer, 8 blocks 3.86)
    case 2: return launch_gdn_typed<T, 2, 8>(a, stream);
    case 4: return launch_gdn_typed<T, 4, 2>(a, stream);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_gated_delta(const qic_gdn_args& a, cudaStream_t stream) {
  if (a.dtype == QIC_DTYPE_BF16) return launch_gdn_rep<__nv_bfloat16>(a, stream);
  return launch_gdn_rep<__half>(a, stream);
}

}  // namespace qic
