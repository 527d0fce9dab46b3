// Split-KV decode attention for B200 (sm_100a), contiguous or paged K/V.
//
// Replaces flash_attention_kernel / paged_attention_kernel (src/kernels.cu:200-374
// of the QweninCuda project): ctx[h] = softmax_t(q_h . K[t, h/g] / sqrt(d)) V[t, h/g].
//
// Design
//  * grid = (splits, kv heads). A CTA owns one kv head and a contiguous range of
//    32-token stages, and serves every query head of the GQA group, so each K/V
//    byte is read from HBM once.
//  * One producer warp streams K and V stages into a shared-memory ring with 2D
//    TMA tile loads (box = 64 elements x box_h tokens, 128-byte swizzle,
//    evict-first L2 policy). Paged layouts are gathered by issuing one box per
//    page segment at the physical row page_table[t/P]*P + t%P; the page-table
//    window is prefetched one window ahead.
//  * Four consumer warps take whole stages round-robin. Scores are computed as
//    S^T = K Q^T with mma.sync m16n8k16 (16 tokens x 8 query-head columns), the
//    online softmax runs in the exp2 domain on the accumulator fragments, P^T is
//    turned into the B operand with movmatrix, and O^T += V^T P accumulates in
//    registers.
//  * Optionally fused: the q prologue (head RMSNorm + RoPE of q) and the K/V append
//    of the new token (head RMSNorm + RoPE of k, written straight into its page
//    slot before the producer loads that stage), and the sigmoid output gate.
//  * Splits write (lse, o) partials to the caller's workspace; the last CTA of a kv
//    head (atomic counter) merges them by log-sum-exp and writes the output.
//  * Every wait is bounded (see ptx.cuh); on timeout the CTA records
//    QIC_DEV_TIMEOUT, waits (bounded) for its own copies in flight and exits.
//
// This translation unit is compiled with --use_fast_math so that the fused norm /
// RoPE / gate arithmetic matches the reference build bit for bit.
#include "qic_internal.h"
#include "rowops.cuh"

namespace qic {

template <int D>
struct AttnShape {
  static constexpr int kChunks = D / 64;                       // 128-byte rows per token row
  static constexpr int kKBytes = kStageTokens * D * 2;         // K bytes of one stage
  static constexpr int kStageBytes = 2 * kKBytes;              // K + V
  static constexpr int kRing = (D == 256) ? 6 : ((D == 128) ? 12 : 24);
  static constexpr int kRingBytes = kRing * kStageBytes;       // 192 KiB
  static constexpr int kCtrlBytes = 8 * (2 * kRing + 2);       // full[], empty[], append barrier, pad
  static constexpr int kQBytes = kMaxGroup * D * 2;
  static constexpr int kFlagBytes = 64;
  static constexpr int kSmemBytes = 1024 + kRingBytes + kCtrlBytes + kQBytes + kFlagBytes;
};

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

template <typename T, int D>
__global__ void __launch_bounds__(kAttnThreads, 1) decode_attn_kernel(const __grid_constant__ AttnParams p) {
  using Sh = AttnShape<D>;
  constexpr int kRing = Sh::kRing;
  constexpr int KS = D / 16;  // k-steps of 16 dims / m-tiles of 16 dims

  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + Sh::kRingBytes);
  uint64_t* empty = full + kRing;
  uint64_t* append_bar = empty + kRing;
  T* q_s = reinterpret_cast<T*>(ring + Sh::kRingBytes + Sh::kCtrlBytes);
  volatile int* flags_s = reinterpret_cast<volatile int*>(ring + Sh::kRingBytes + Sh::kCtrlBytes + Sh::kQBytes);
  // flags_s[0]: abort, flags_s[1]: this CTA merges, flags_s[2]: stages issued (producer)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = blockIdx.x;
  const int kvh = blockIdx.y;
  const int nsplit = p.n_splits;
  const int st_lo = static_cast<int>(static_cast<long long>(split) * p.n_stages / nsplit);
  const int st_hi = static_cast<int>(static_cast<long long>(split + 1) * p.n_stages / nsplit);
  const int nst = st_hi - st_lo;
  const int S = p.seq_len;
  const int G = p.G;
  const bool do_append = (p.flags & QIC_FUSE_APPEND) && st_hi == p.n_stages;
  const uint64_t deadline = globaltimer_ns() + p.timeout_ns;

  if (threadIdx.x == 0) {
#pragma unroll 1
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(append_bar, 1);
    flags_s[0] = 0;
    flags_s[1] = 0;
    flags_s[2] = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ======================= producer warp =======================
    const uint64_t pol = l2_policy_evict_first();
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_k);
      tma_prefetch_desc(&p.tm_v);
    }
    const bool paged = p.page_table != nullptr;
    const int bh = p.box_h;
    const int box_row_bytes = bh * 128;   // one 64-element chunk of bh token rows
    const int box_bytes = bh * D * 2;     // all chunks of bh token rows
    const int P = p.page_size;
    const int npages = paged ? (S + P - 1) / P : 0;
    // page-table window: lane l holds entry wbase + l; `nxt` holds the next window
    int wbase = 0, cur = 0, nxt = 0;
    if (paged) {
      wbase = (st_lo * kStageTokens) / P;
      int e0 = wbase + lane, e1 = wbase + 32 + lane;
      cur = e0 < npages ? __ldg(p.page_table + e0) : 0;
      nxt = e1 < npages ? __ldg(p.page_table + e1) : 0;
    }
    int issued = 0;
    bool ok = true;
#pragma unroll 1
    for (int i = 0; i < nst; ++i) {
      const int slot = i % kRing;
      if (i >= kRing) {
        if (!__all_sync(kFullMask, mbar_wait(&empty[slot], ((i / kRing) - 1) & 1, deadline))) {
          ok = false;
          break;
        }
      }
      if (__shfl_sync(kFullMask, flags_s[0], 0)) {
        ok = false;
        break;
      }
      const int t0 = (st_lo + i) * kStageTokens;
      const int nvalid = min(kStageTokens, S - t0);
      if (do_append && i == nst - 1) {
        // the stage holding the new token is loaded after the append has landed
        if (!__all_sync(kFullMask, mbar_wait(append_bar, 0, deadline))) {
          ok = false;
          break;
        }
      }
      const int nbox = (nvalid + bh - 1) / bh;
      uint8_t* sk = ring + slot * Sh::kStageBytes;
      if (lane == 0) mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(nbox * box_bytes * 2));
#pragma unroll 1
      for (int j = 0; j < nbox; ++j) {
        const int tb = t0 + j * bh;
        int row = tb;
        if (paged) {
          const int e = tb / P;
          while (e >= wbase + 32) {  // uniform across the warp
            cur = nxt;
            wbase += 32;
            const int en = wbase + 32 + lane;
            nxt = en < npages ? __ldg(p.page_table + en) : 0;
          }
          const int page = __shfl_sync(kFullMask, cur, e - wbase);
          long long r = static_cast<long long>(page) * P + (tb - e * P);
          if (page < 0 || (p.cache_tokens > 0 && r + bh > p.cache_tokens)) {
            if (lane == 0) record_status(p.status, QIC_DEV_BAD_PAGE);
            r = tb - e * P;  // clamp to page 0
          }
          row = static_cast<int>(r);
        }
        if (lane == 0) {
#pragma unroll
          for (int c = 0; c < Sh::kChunks; ++c) {
            uint8_t* dst = sk + j * box_bytes + c * box_row_bytes;
            const int x = kvh * D + c * 64;
            tma_load_2d(dst, &p.tm_k, &full[slot], x, row, pol);
            tma_load_2d(dst + Sh::kKBytes, &p.tm_v, &full[slot], x, row, pol);
          }
        }
      }
      issued = i + 1;
      __syncwarp();
    }
    if (!ok) {
      if (lane == 0) {
        record_status(p.status, QIC_DEV_TIMEOUT);
        flags_s[0] = 1;
        // wait (bounded) for the copies this CTA still has in flight
        const uint64_t dl2 = globaltimer_ns() + p.timeout_ns;
        for (int i = max(0, issued - kRing); i < issued; ++i) mbar_wait(&full[i % kRing], (i / kRing) & 1, dl2);
      }
    }
    return;
  }

  // ======================= consumer warps =======================
  const int ctid = threadIdx.x;  // 0..127
  const int hd = p.head_dim;
  // ---- prologue: q rows into shared memory, and the fused append ----
  {
    const int nrows = G + (do_append ? 1 : 0);
#pragma unroll 1
    for (int r = warp; r < nrows; r += kConsumerWarps) {
      float v[D / 32];
      if (r < G) {
        const int h = kvh * G + r;
        row_load<T, D>(static_cast<const T*>(p.q) + static_cast<size_t>(h) * D, v, lane);
        if (p.flags & QIC_FUSE_Q_PROLOGUE) {
          row_rmsnorm<T, D>(v, static_cast<const T*>(p.q_norm_w), hd, p.eps, lane);
          row_rope<T, D>(v, hd, S - 1, p.theta, lane);
        }
        row_store<T, D>(q_s + r * D, v, lane);
      } else {
        // K/V append at position S-1 (src/model.cpp:634,637,639-641)
        const int pos = S - 1;
        long long slot = pos;
        if (p.page_table != nullptr) {
          const int e = pos / p.page_size;
          slot = static_cast<long long>(__ldg(p.page_table + e)) * p.page_size + (pos - e * p.page_size);
        }
        const size_t kv_dim = static_cast<size_t>(p.Hkv) * D;
        if (slot >= 0 && slot < p.cache_tokens) {
          row_load<T, D>(static_cast<const T*>(p.k_new) + static_cast<size_t>(kvh) * D, v, lane);
          row_rmsnorm<T, D>(v, static_cast<const T*>(p.k_norm_w), hd, p.eps, lane);
          row_rope<T, D>(v, hd, pos, p.theta, lane);
          T* kdst = static_cast<T*>(p.k_cache) + static_cast<size_t>(slot) * kv_dim + static_cast<size_t>(kvh) * D;
          row_store<T, D>(kdst, v, lane);
          float vv[D / 32];
          row_load<T, D>(static_cast<const T*>(p.v_new) + static_cast<size_t>(kvh) * D, vv, lane);
          T* vdst = static_cast<T*>(p.v_cache) + static_cast<size_t>(slot) * kv_dim + static_cast<size_t>(kvh) * D;
          row_store<T, D>(vdst, vv, lane);
        } else if (lane == 0) {
          record_status(p.status, QIC_DEV_BAD_PAGE);
        }
        fence_proxy_async_global();
        __syncwarp();
        if (lane == 0) mbar_arrive(append_bar);
      }
    }
  }
  consumer_sync();

  // ---- B fragments of Q^T (k = dims, n = query heads of the group) ----
  const int hq = lane >> 2;         // n index held by this lane in B fragments
  const int kq = (lane & 3) * 2;    // k pair held by this lane
  uint32_t qf[KS][2];
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
    if (hq < G) {
      qf[ks][0] = *reinterpret_cast<const uint32_t*>(q_s + hq * D + ks * 16 + kq);
      qf[ks][1] = *reinterpret_cast<const uint32_t*>(q_s + hq * D + ks * 16 + kq + 8);
    } else {
      qf[ks][0] = 0u;
      qf[ks][1] = 0u;
    }
  }

  // ---- per-lane shared-memory address pieces (swizzled, chunk-major boxes) ----
  const int bh = p.box_h;
  const int lbh = p.log2_box_h;
  const int box_bytes = bh * D * 2;
  const int box_row_bytes = bh * 128;
  const int q8 = lane >> 3;   // ldmatrix matrix index supplied by this lane
  const int rr = lane & 7;    // row within that 8x8 matrix
  uint32_t rowK[2], rowV[2];
#pragma unroll
  for (int g2 = 0; g2 < 2; ++g2) {
    const int tk = g2 * 16 + (q8 & 1) * 8 + rr;
    const int tv = g2 * 16 + (q8 >> 1) * 8 + rr;
    rowK[g2] = static_cast<uint32_t>((tk >> lbh) * box_bytes + (tk & (bh - 1)) * 128);
    rowV[g2] = static_cast<uint32_t>((tv >> lbh) * box_bytes + (tv & (bh - 1)) * 128);
  }
  const uint32_t xk = static_cast<uint32_t>(((q8 >> 1) ^ rr) << 4);
  const uint32_t xv = static_cast<uint32_t>(((q8 & 1) ^ rr) << 4);

  float acc[KS][4];
#pragma unroll
  for (int j = 0; j < KS; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  const float sl2 = p.scale_log2;
  bool ok = true;

#pragma unroll 1
  for (int i = warp; i < nst; i += kConsumerWarps) {
    const int slot = i % kRing;
    if (!__all_sync(kFullMask, mbar_wait(&full[slot], (i / kRing) & 1, deadline))) {
      ok = false;
      break;
    }
    const int t0 = (st_lo + i) * kStageTokens;
    const int nvalid = min(kStageTokens, S - t0);
    uint8_t* sk = ring + slot * Sh::kStageBytes;
    const uint32_t bk = smem_u32(sk);
    const uint32_t bv = bk + Sh::kKBytes;
    if (nvalid < kStageTokens) {
      // rows past the sequence end hold stale or unloaded data: zero V there so
      // P = 0 rows cannot turn into NaN in the PV product
      uint8_t* sv = sk + Sh::kKBytes;
      const int nz = (kStageTokens - nvalid) * Sh::kChunks * 8;  // 16-byte units
      for (int u = lane; u < nz; u += 32) {
        const int t = nvalid + u / (Sh::kChunks * 8);
        const int rem = u % (Sh::kChunks * 8);
        const int c = rem >> 3, w16 = rem & 7;
        uint8_t* dst = sv + (t >> lbh) * box_bytes + c * box_row_bytes + (t & (bh - 1)) * 128 + w16 * 16;
        *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
      }
      // these generic writes precede a later TMA write into the same slot
      fence_proxy_async_smem();
      __syncwarp();
    }

    // S^T = K Q^T for the two 16-token groups of the stage
    float sc[2][4];
#pragma unroll
    for (int g2 = 0; g2 < 2; ++g2) {
      sc[g2][0] = sc[g2][1] = sc[g2][2] = sc[g2][3] = 0.0f;
      if (g2 * 16 < nvalid) {
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          uint32_t a0, a1, a2, a3;
          const uint32_t addr =
              bk + rowK[g2] + (ks >> 2) * box_row_bytes + (xk ^ static_cast<uint32_t>(((2 * ks) & 7) << 4));
          ldsm_x4(addr, a0, a1, a2, a3);
          MmaOp<T>::run(sc[g2], a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
        }
      }
    }
    // scale, mask, online softmax (per head column)
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int g2 = 0; g2 < 2; ++g2) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int t = g2 * 16 + hq + r * 8;
        const bool valid = t < nvalid;
        sc[g2][2 * r + 0] = valid ? sc[g2][2 * r + 0] * sl2 : -INFINITY;
        sc[g2][2 * r + 1] = valid ? sc[g2][2 * r + 1] * sl2 : -INFINITY;
        mx0 = fmaxf(mx0, sc[g2][2 * r + 0]);
        mx1 = fmaxf(mx1, sc[g2][2 * r + 1]);
      }
    }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(kFullMask, mx0, o));
      mx1 = fmaxf(mx1, __shfl_xor_sync(kFullMask, mx1, o));
    }
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float mu0 = (mn0 == -INFINITY) ? 0.0f : mn0;
    const float mu1 = (mn1 == -INFINITY) ? 0.0f : mn1;
    const float al0 = exp2f(m0 - mu0), al1 = exp2f(m1 - mu1);
    m0 = mn0;
    m1 = mn1;
    float ps0 = 0.0f, ps1 = 0.0f;
#pragma unroll
    for (int g2 = 0; g2 < 2; ++g2) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        sc[g2][2 * r + 0] = exp2f(sc[g2][2 * r + 0] - mu0);
        sc[g2][2 * r + 1] = exp2f(sc[g2][2 * r + 1] - mu1);
        ps0 += sc[g2][2 * r + 0];
        ps1 += sc[g2][2 * r + 1];
      }
    }
    l0 = l0 * al0 + ps0;
    l1 = l1 * al1 + ps1;
#pragma unroll
    for (int j = 0; j < KS; ++j) {
      acc[j][0] *= al0;
      acc[j][1] *= al1;
      acc[j][2] *= al0;
      acc[j][3] *= al1;
    }
    // O^T += V^T P
#pragma unroll
    for (int g2 = 0; g2 < 2; ++g2) {
      if (g2 * 16 < nvalid) {
        const uint32_t b0 = movmatrix_trans(pack2<T>(sc[g2][0], sc[g2][1]));
        const uint32_t b1 = movmatrix_trans(pack2<T>(sc[g2][2], sc[g2][3]));
#pragma unroll
        for (int j = 0; j < KS; ++j) {
          uint32_t a0, a1, a2, a3;
          const uint32_t addr =
              bv + rowV[g2] + (j >> 2) * box_row_bytes + (xv ^ static_cast<uint32_t>(((2 * j) & 7) << 4));
          ldsm_x4_trans(addr, a0, a1, a2, a3);
          MmaOp<T>::run(acc[j], a0, a1, a2, a3, b0, b1);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  if (!ok) {
    if (lane == 0) {
      record_status(p.status, QIC_DEV_TIMEOUT);
      flags_s[0] = 1;
    }
  }
  // full row sums per head column
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    l0 += __shfl_xor_sync(kFullMask, l0, o);
    l1 += __shfl_xor_sync(kFullMask, l1, o);
  }
  consumer_sync();
  if (flags_s[0]) return;  // aborted: the producer drains its copies

  // ---- combine the four consumer warps (ring memory is free now) ----
  float* cm = reinterpret_cast<float*>(ring);         // [4][8] m
  float* cl = cm + kConsumerWarps * 8;                // [4][8] l
  float* co = cl + kConsumerWarps * 8;                // [4][8][D] o
  {
    const int hA = (lane & 3) * 2, hB = hA + 1;
    if (lane < 4) {
      cm[warp * 8 + hA] = m0;
      cm[warp * 8 + hB] = m1;
      cl[warp * 8 + hA] = l0;
      cl[warp * 8 + hB] = l1;
    }
#pragma unroll
    for (int j = 0; j < KS; ++j) {
      const int d0 = j * 16 + hq;
      co[(warp * 8 + hA) * D + d0] = acc[j][0];
      co[(warp * 8 + hB) * D + d0] = acc[j][1];
      co[(warp * 8 + hA) * D + d0 + 8] = acc[j][2];
      co[(warp * 8 + hB) * D + d0 + 8] = acc[j][3];
    }
  }
  consumer_sync();

  const size_t qoff = static_cast<size_t>(kvh) * G * D;  // first output row of this group
  const int pf = partial_floats(G, D);
  float* mypart = p.part + (static_cast<size_t>(kvh) * nsplit + split) * pf;
#pragma unroll 1
  for (int idx = ctid; idx < G * D; idx += kConsumerWarps * 32) {
    const int h = idx / D, d = idx - (idx / D) * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, cm[w * 8 + h]);
    const float Mu = (M == -INFINITY) ? 0.0f : M;
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float wt = exp2f(cm[w * 8 + h] - Mu);
      L += cl[w * 8 + h] * wt;
      O += co[(w * 8 + h) * D + d] * wt;
    }
    if (nsplit == 1) {
      const float inv_l = 1.0f / fmaxf(L, 1e-12f);
      T ot = from_f32<T>(O * inv_l);
      if (p.gate != nullptr) {
        const float g = to_f32<T>(static_cast<const T*>(p.gate)[qoff + idx]);
        const float sig = 1.0f / (1.0f + expf(-g));
        ot = from_f32<T>(to_f32<T>(ot) * sig);
      }
      static_cast<T*>(p.out)[qoff + idx] = ot;
    } else {
      mypart[G + idx] = (L > 0.0f) ? O / L : 0.0f;
      if (d == 0) mypart[h] = (L > 0.0f) ? Mu + log2f(L) : -INFINITY;
    }
  }
  if (nsplit == 1) return;

  // ---- cross-split merge by the last CTA of this kv head ----
  __threadfence();
  consumer_sync();
  if (ctid == 0) {
    const int prev = atomicAdd(p.counters + kvh, 1);
    flags_s[1] = (prev == nsplit - 1) ? 1 : 0;
  }
  consumer_sync();
  if (!flags_s[1]) return;
  __threadfence();
  float* lse_s = reinterpret_cast<float*>(ring);  // [G] merged lse
  const float* gpart = p.part + static_cast<size_t>(kvh) * nsplit * pf;
  {
#pragma unroll 1
    for (int h = warp; h < G; h += kConsumerWarps) {
      float mx = -INFINITY;
      for (int s = lane; s < nsplit; s += 32) mx = fmaxf(mx, __ldcg(gpart + static_cast<size_t>(s) * pf + h));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, o));
      const float mxu = (mx == -INFINITY) ? 0.0f : mx;
      float sum = 0.0f;
      for (int s = lane; s < nsplit; s += 32) sum += exp2f(__ldcg(gpart + static_cast<size_t>(s) * pf + h) - mxu);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(kFullMask, sum, o);
      if (lane == 0) lse_s[h] = (sum > 0.0f) ? mxu + log2f(sum) : 0.0f;
    }
  }
  consumer_sync();
#pragma unroll 1
  for (int idx = ctid; idx < G * D; idx += kConsumerWarps * 32) {
    const int h = idx / D;
    const float lse = lse_s[h];
    float o = 0.0f;
#pragma unroll 4
    for (int s = 0; s < nsplit; ++s) {
      const float* ps = gpart + static_cast<size_t>(s) * pf;
      o += __ldcg(ps + G + idx) * exp2f(__ldcg(ps + h) - lse);
    }
    T ot = from_f32<T>(o);
    if (p.gate != nullptr) {
      const float g = to_f32<T>(static_cast<const T*>(p.gate)[qoff + idx]);
      const float sig = 1.0f / (1.0f + expf(-g));
      ot = from_f32<T>(to_f32<T>(ot) * sig);
    }
    static_cast<T*>(p.out)[qoff + idx] = ot;
  }
  if (ctid == 0) p.counters[kvh] = 0;  // ready for the next call
}

// ----------------------------------------------------------------------------
// host launcher
// ----------------------------------------------------------------------------
size_t decode_attention_smem_bytes(int head_dim) {
  switch (head_dim) {
    case 64: return AttnShape<64>::kSmemBytes;
    case 128: return AttnShape<128>::kSmemBytes;
    case 256: return AttnShape<256>::kSmemBytes;
    default: return 0;
  }
}

template <typename T, int D>
static cudaError_t launch_typed(const AttnParams& p, cudaStream_t stream) {
  static unsigned long long configured = 0;  // one bit per device ordinal
  const int smem = AttnShape<D>::kSmemBytes;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 64 && !(configured & (1ull << dev))) {
    e = cudaFuncSetAttribute(decode_attn_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured |= 1ull << dev;
  }
  dim3 grid(p.n_splits, p.Hkv);
  decode_attn_kernel<T, D><<<grid, kAttnThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_decode_attention(int dtype, int head_dim, const AttnParams& p, cudaStream_t stream) {
  if (dtype == QIC_DTYPE_BF16) {
    switch (head_dim) {
      case 64: return launch_typed<__nv_bfloat16, 64>(p, stream);
      case 128: return launch_typed<__nv_bfloat16, 128>(p, stream);
      case 256: return launch_typed<__nv_bfloat16, 256>(p, stream);
    }
  } else {
    switch (head_dim) {
      case 64: return launch_typed<__half, 64>(p, stream);
      case 128: return launch_typed<__half, 128>(p, stream);
      case 256: return launch_typed<__half, 256>(p, stream);
    }
  }
  return cudaErrorInvalidValue;
}

}  // namespace qic
