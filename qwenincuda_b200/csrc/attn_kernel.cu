// Split-KV decode attention for B200 (sm_100a), contiguous or paged K/V.
//
// Replaces flash_attention_kernel / paged_attention_kernel (src/kernels.cu:200-374
// of the QweninCuda project): ctx[h] = softmax_t(q_h . K[t, h/g] / sqrt(d)) V[t, h/g].
//
// Design
//  * A CTA owns one kv head of one sequence and a contiguous range of pipeline
//    stages (32 tokens, 16 at head_dim 256), and serves every query head of the GQA
//    group, so each K/V byte is read from HBM once. Single-sequence launches use a
//    (splits, kv heads) grid; batched launches read one WorkItem per CTA.
//  * Four warps; warp w consumes stages w, w+4, ... of a 4-stage (64 KB) shared-memory
//    ring (8 stages at head_dim 64) and issues each slot's next copy itself as soon as
//    it has finished with the slot: 3D TMA tile loads, one box = every 64-element
//    chunk of bh token rows (128-byte swizzle, evict-first L2 policy), K boxes from
//    lanes 0-15 and V boxes from lanes 16-31. A stage-level %globaltimer trace showed
//    separate producer warps to be the limit: a producer's wake-up, page lookup and
//    issue cost 0.5-0.8 us per stage, so each slot sat idle 2-2.5 us per lap. Three
//    CTAs fit per SM (registers and shared memory), 12 issuing warps per SM. Paged
//    layouts are gathered with one box per page segment at row
//    page_table[t/P]*P + t%P; each warp loads the table entries of its next stage
//    one stage ahead.
//  * Slots are owned by one warp (ring depth is a multiple of four), so mbarrier
//    parities cannot alias. Scores are S^T = K Q^T with mma.sync m16n8k16 (16 tokens
//    x 8 query-head columns); the online softmax runs in the exp2 domain on the
//    fragments; P^T is turned into the B operand with movmatrix; O^T += V^T P
//    accumulates in registers.
//  * Fused options: the q prologue (head RMSNorm + RoPE of q, read from q or from
//    the interleaved q/gate projection), the K/V append of the new token (head
//    RMSNorm + RoPE of k written into its page slot; a stage holding it that was
//    copied before the append gets the row written into shared memory, and a token
//    alone in the last stage is taken from registers without copying that stage),
//    and the sigmoid output gate.
//  * The splits of a kv head form thread-block clusters. CTA c of a cluster owns
//    output slice c: every CTA sends slice c of its (o, lse) partial into CTA c's
//    shared memory with st.async (distributed shared memory, bytes counted by CTA c's
//    mbarrier), and each CTA merges its slice once all contributions have landed: no
//    cluster-wide barrier after the stage loops. When a kv head spans several
//    clusters, each cluster slice is written to the caller's workspace and the last
//    arriving CTA of that slice (release/acquire counter) merges the cluster partials
//    by log-sum-exp.
//  * Long sequences hand out their first eighth of stages one at a time (a per-kv-head
//    ticket counter in the workspace) to the warps that finish their own range first.
//  * Programmatic dependent launch (QIC_PDL): the CTA signals its dependents at
//    start; the norm weights, page-table entries, cached K/V rows and a device-resident
//    length (QIC_DEVICE_SEQ_LEN) are read before griddepcontrol.wait, q, k_new,
//    v_new, the gate and the workspace's counters and partials after it (a bad page
//    or length may be OR-ed into the status word before it), so the next call's K/V
//    prefetch overlaps this call's tail.
//  * Every wait is bounded (ptx.cuh); on timeout the CTA records QIC_DEV_TIMEOUT,
//    drains its own copies (bounded) and exits.
//
// Compiled with --use_fast_math so the fused norm / RoPE / gate arithmetic matches
// the reference build bit for bit where bytes are stored and compared: the appended k
// row (head norm with the reference's ascending sum order, RoPE) and the gate. The q
// rows' head norm sums its squares with a shuffle tree: q feeds only the attention
// output, which is checked within tolerance.
#include "qic_internal.h"
#include "rowops.cuh"

namespace qic {

template <int D>
struct AttnShape {
  static constexpr int kTok = stage_tokens(D);                 // tokens per stage
  static constexpr int kGroups = kTok / 16;                     // 16-token mma groups per stage
  static constexpr int kChunks = D / 64;                        // 128-byte rows per token row
  static constexpr int kKBytes = kTok * D * 2;                  // K bytes of one stage
  static constexpr int kStageBytes = 2 * kKBytes;               // K + V
  static constexpr int kRing = (D == 64) ? 8 : 4;
  static_assert(kRing % kConsumerWarps == 0, "a ring slot must always be consumed by the same warp");
  static constexpr int kRingBytes = kRing * kStageBytes;        // 64 KB
  static constexpr int kCombineBytes = kConsumerWarps * (kMaxGroup * (D + 4) + 2 * kMaxGroup) * 4;
  static_assert(kCombineBytes + (kMaxGroup * (D + 1) + 4) * 4 <= kRingBytes, "combine buffer + partial");
  static constexpr int kCtrlBytes = 128;                         // full[] barriers
  static constexpr int kQBytes = kMaxGroup * D * 2;
  static constexpr int kFlagBytes = 64;
  static constexpr int kMlBytes = 2 * kConsumerWarps * 8 * 4;       // every warp's (m, l) per head column
  static constexpr int kAppBytes = 2 * D * 2;                         // the appended k and v rows
  static constexpr int kSmemBytes = 1024 + kRingBytes + kCtrlBytes + kQBytes + kFlagBytes + kMlBytes + kAppBytes;
  // the cluster merge's receive buffer follows (attn_rx_bytes, sized per launch)
  static constexpr int kMaxRxBytes = (kMaxGroup * D + kMaxCluster * (kMaxGroup + 1)) * 4;
};

// Receive buffer of the cluster merge: one contribution per CTA of the cluster, each
// a slice of ceil(G*D/C) outputs and the G per-head log-sum-exps padded to a multiple
// of four (none for C = 1).
__host__ __device__ constexpr int attn_rx_bytes(int G, int D, int C) {
  return C > 1 ? C * ((G * D + C - 1) / C + ((G + 3) & ~3)) * 4 : 0;
}

__device__ __forceinline__ void consumer_sync() {
  __syncwarp();
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

__device__ __forceinline__ int atomic_add_acq_rel_gpu(int* addr, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
  return old;
}

// out[i] = T(o), then the optional sigmoid gate gate[gi] as the reference applies it.
template <typename T>
__device__ __forceinline__ void write_out(T* ob, const T* gb, size_t i, size_t gi, float o) {
  T ot = from_f32<T>(o);
  if (gb != nullptr) {
    const float g = to_f32<T>(gb[gi]);
    const float sig = 1.0f / (1.0f + expf(-g));
    ot = from_f32<T>(to_f32<T>(ot) * sig);
  }
  ob[i] = ot;
}

// Contribution (parity, source rank, kv head, slice c) in the exchange buffer at
// `base`: cp_slice_words 8-byte words.
__device__ __forceinline__ uint2* cp_slot(void* base, int par, int src, int world, int Hkv, int kvh, int c,
                                          int words) {
  const size_t i = ((static_cast<size_t>(par) * world + src) * Hkv + kvh) * kCpSlices + c;
  return static_cast<uint2*>(base) + i * words;
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// CP: context-parallel launch (the in-kernel exchange); a separate instantiation so
// that single-GPU launches carry none of its code.
template <typename T, int D, bool CP>
__global__ void __launch_bounds__(kAttnThreads, 3) decode_attn_kernel(const __grid_constant__ AttnParams p) {
  using Sh = AttnShape<D>;
  constexpr int kRing = Sh::kRing;
  constexpr int TOK = Sh::kTok;
  constexpr int NG = Sh::kGroups;
  constexpr int KS = D / 16;  // k-steps of 16 dims / m-tiles of 16 dims

  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + Sh::kRingBytes);
  T* q_s = reinterpret_cast<T*>(ring + Sh::kRingBytes + Sh::kCtrlBytes);
  volatile int* flags_s = reinterpret_cast<volatile int*>(ring + Sh::kRingBytes + Sh::kCtrlBytes + Sh::kQBytes);
  // [4][8] m then [4][8] l of the warps, written as each warp leaves its stage loop
  float* ml_s = reinterpret_cast<float*>(ring + Sh::kRingBytes + Sh::kCtrlBytes + Sh::kQBytes + Sh::kFlagBytes);
  // the cluster merge: contributions of the cluster's CTAs to this CTA's output slice,
  // and the mbarrier that counts their bytes (control slot 15; ring slots use 0-7)
  // the appended k row then v row, as stored into the cache
  T* app_s = reinterpret_cast<T*>(ring + Sh::kRingBytes + Sh::kCtrlBytes + Sh::kQBytes + Sh::kFlagBytes + Sh::kMlBytes);
  float* rx = reinterpret_cast<float*>(ring + Sh::kRingBytes + Sh::kCtrlBytes + Sh::kQBytes + Sh::kFlagBytes +
                                       Sh::kMlBytes + Sh::kAppBytes);
  uint64_t* rx_bar = full + 15;
  // flags_s[0]: abort, flags_s[1]: this CTA merges, flags_s[2]: app_s holds the append

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- this CTA's unit of work ----
  int b, kvh, split, nsplit, st_lo, st_hi, S, part_base;
  // Single-sequence launches whose appended token is alone in the sequence's last stage
  // (S - 1 a multiple of the stage size: positions 2^k, for instance) take that token's
  // contribution from the appending warp's registers and never copy the stage.
  bool tail_regs = false;
  if (p.plan != nullptr) {
    const WorkItem w = p.plan[blockIdx.x];
    b = w.b;
    kvh = w.kvh;
    split = w.split;
    nsplit = w.nsplit;
    st_lo = w.st_lo;
    st_hi = w.st_hi;
    S = w.seq_len;
    part_base = w.part_base;
  } else {
    b = 0;
    kvh = blockIdx.y;
    split = blockIdx.x;
    nsplit = p.n_splits;
    S = p.seq_len;
    if (p.seq_len_dev != nullptr) {
      // the current length, written before this launch like the page table; the launch
      // is sized for p.seq_len, so a length outside [1, p.seq_len] is clamped into it
      int sd = *p.seq_len_dev;
      if (sd < 1 || sd > p.seq_len) {
        if (threadIdx.x == 0) record_status(p.status, QIC_DEV_BAD_LENGTH);
        sd = sd < 1 ? 1 : p.seq_len;
      }
      S = sd;
    }
    tail_regs = (p.flags & QIC_FUSE_APPEND) && S > 1 && (S - 1) % TOK == 0;
    const int nst = (S + TOK - 1) / TOK - (tail_regs ? 1 : 0);  // stages copied
    st_lo = static_cast<int>(static_cast<long long>(split) * nst / nsplit);
    st_hi = static_cast<int>(static_cast<long long>(split + 1) * nst / nsplit);
    part_base = kvh * (nsplit / p.cluster);  // one global slot per cluster
  }
  if (p.cluster == 1 && nsplit > 1 &&
      (part_base + split >= p.part_slots || b * p.Hkv + kvh >= p.num_counters || nsplit > kMaxSplits)) {
    // a planned work item that does not fit the workspace is reported, not executed
    // (cluster launches are shaped on the host and never take this exit)
    if (threadIdx.x == 0) record_status(p.status, QIC_DEV_BAD_PLAN);
    return;
  }
  const int n_stages_seq = (S + TOK - 1) / TOK;
  const int n_copy = n_stages_seq - (tail_regs ? 1 : 0);  // stages that go through the ring
  // Stages of this CTA (absolute indices in the sequence): its own contiguous range
  // [a0, a1), and, in single-sequence launches with a workspace and at least 8
  // stages per split, a share of the first eighth of the sequence, [0, pool_n),
  // handed out one stage at a time by the kv head's ticket counter once a warp's own
  // stages are all issued: CTAs that start late or stream slowly take fewer of them.
  // The own ranges split the rest evenly; the last one holds the appended token.
  // Batched work items keep their planned range.
  int a0 = st_lo, a1 = st_hi, pool_n = 0;
  int* stage_ctr = nullptr;
  if (p.plan == nullptr && p.stage_ctr != nullptr && n_copy >= 8 * nsplit) {
    pool_n = n_copy / 8;
    const int rest = n_copy - pool_n;
    a0 = pool_n + static_cast<int>(static_cast<long long>(split) * rest / nsplit);
    a1 = pool_n + static_cast<int>(static_cast<long long>(split + 1) * rest / nsplit);
    stage_ctr = p.stage_ctr + kvh;
  }
  const int G = p.G;
  // The cluster merge's geometry (divisions by the runtime cluster size, done here,
  // off the merge's path): CTA `rank` of cluster `cid` owns outputs [lo, hi).
  const int C = p.cluster;
  const int GD = G * D;
  const int rank = split % C, cid = split / C, nclust = nsplit / C;
  const int slice = (GD + C - 1) / C;
  const int lo = rank * slice, hi = min(GD, lo + slice);
  const bool do_append = (p.flags & QIC_FUSE_APPEND) && a1 == n_copy && a1 > a0;
  const int32_t* table = p.page_table != nullptr ? p.page_table + static_cast<size_t>(b) * p.table_bstride : nullptr;
  const uint64_t deadline = globaltimer_ns() + p.timeout_ns;

  if (threadIdx.x == 0) {
#pragma unroll 1
    for (int i = 0; i < kRing; ++i) mbar_init(&full[i], 1);
    if (p.cluster > 1) {
      // bytes this CTA receives in the cluster merge: from each of the C CTAs, its
      // share of this CTA's output slice and its G log-sum-exps
      const int cnt = max(0, hi - lo);
      const int nl = (slice % 4 == 0) ? ((G + 3) & ~3) : G;  // log-sum-exps sent (padded with 16-byte stores)
      mbar_init(rx_bar, 1);
      mbar_arrive_expect_tx(rx_bar, static_cast<uint32_t>(C * (cnt + nl) * 4));
    }
    flags_s[0] = 0;
    flags_s[1] = 0;
    flags_s[2] = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // first cluster barrier phase: this CTA runs and its receive mbarrier is initialised
  // (waited for just before the merge's first remote store)
  if (p.cluster > 1) asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
  pdl_launch_dependents();

  // ---- stage copies: every warp streams its own ring slots ----
  // Warp w owns slots w, w+4, ... and consumes them in turn; as soon as it has
  // finished with a slot it issues the slot's next stage itself, so a slot never
  // waits on another warp. Lane l < 16 copies K box l of a stage and lane 16 + l the
  // V box l; a box is every 64-element chunk of bh token rows, at row
  // page_table[t/P]*P + t%P when paged.
  constexpr int kSlots = kRing / kConsumerWarps;  // slots per warp
  const uint64_t pol = l2_policy_evict_first();
  if (lane == 0) {
    tma_prefetch_desc(&p.tm_k);
    tma_prefetch_desc(&p.tm_v);
  }
  const int bh = p.box_h;
  const int lbh = p.log2_box_h;
  const int box_bytes = bh * D * 2;  // all chunks of bh token rows
  const int P = p.page_size;
  const int bx = lane & 15;
  const CUtensorMap* tmap = lane < 16 ? &p.tm_k : &p.tm_v;
  const int kv_off = lane < 16 ? 0 : Sh::kKBytes;
  const int append_stage = (do_append && !tail_regs) ? n_stages_seq - 1 : -1;  // copied stage holding it
  // token index / page size: a shift for power-of-two pages (the common case), so a
  // refill does not wait on an integer division
  const int lP = (P > 0 && (P & (P - 1)) == 0) ? __ffs(P) - 1 : -1;
  auto page_of = [&](int t) -> int { return lP >= 0 ? (t >> lP) : t / P; };
  // page-table entry holding box bx of stage j, or -1
  auto box_entry = [&](int j) -> int {
    const int tb = j * TOK + bx * bh;
    return (j >= 0 && bx * bh < TOK && tb < S) ? page_of(tb) : -1;
  };
  auto load_entry = [&](int e) -> int { return e >= 0 ? __ldg(table + e) : 0; };
  auto issue = [&](int j, int page, int slot) {
    const int t0 = j * TOK;
    const int nbox = (min(TOK, S - t0) + bh - 1) >> lbh;
    const int tb = t0 + bx * bh;
    long long row = tb;
    if (table != nullptr && bx < nbox) {
      const int e = page_of(tb);
      row = static_cast<long long>(page) * P + (tb - e * P);
      if (page < 0 || (p.cache_tokens > 0 && row + bh > p.cache_tokens)) {
        record_status(p.status, QIC_DEV_BAD_PAGE);
        row = tb - e * P;  // clamp to page 0
      }
    }
    if (lane == 0) mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(2 * nbox * box_bytes));
    __syncwarp();
    if (bx < nbox) {
      // the warp's ldmatrix reads of this slot have completed: their results fed the
      // mma instructions issued before this copy
      tma_load_3d(ring + slot * Sh::kStageBytes + kv_off + bx * box_bytes, tmap, &full[slot], 0,
                  static_cast<int>(row), kvh * Sh::kChunks, pol);
    }
  };
  // cur[k]: stage in this warp's k-th slot (issued, not yet consumed) or -1
  int cur[kSlots], lap[kSlots];
  int live = 0;  // slots holding a stage
#pragma unroll
  for (int k = 0; k < kSlots; ++k) {
    const int j = a0 + warp + k * kConsumerWarps;
    cur[k] = j < a1 ? j : -1;
    lap[k] = 0;
    live += cur[k] >= 0 ? 1 : 0;
  }
  // initial fill, before the inputs of the preceding kernel are waited for. The stage
  // holding the appended token is copied too, with the row's old bytes: its consumer
  // overwrites that row in shared memory with the appended k and v rows (app_s) before
  // using it, so the append's global write is not waited for by a copy. pg_st[k]:
  // page-table entry of the slot's next own stage (cur[k] + kRing), loaded one stage
  // ahead.
  int pg_st[kSlots];
  bool app_patch = false;  // this warp copied the stage holding the appended row before the append
#pragma unroll
  for (int k = 0; k < kSlots; ++k) {
    pg_st[k] = 0;
    if (cur[k] < 0) continue;
    const int pg0 = table != nullptr ? load_entry(box_entry(cur[k])) : 0;
    if (table != nullptr && cur[k] + kRing < a1) pg_st[k] = load_entry(box_entry(cur[k] + kRing));
    if (cur[k] == append_stage) app_patch = true;
    issue(cur[k], pg0, warp + k * kConsumerWarps);
  }
  // Measured and not kept: also prefetching each slot's next 1 / 2 / 4 own stages
  // into L2 here, so that a chained layer's K/V stream while the previous layer
  // merges (S=8192 chain 12.5 -> 13.3 us per layer, 32K 30.0 -> 30.6-32.7, S=1025
  // 7.63 -> 7.74).

  const int ctid = threadIdx.x;  // 0..127
  const int hd = p.head_dim;
  const T* qb = static_cast<const T*>(p.q) + static_cast<size_t>(b) * p.q_bstride;
  const T* gb = p.gate != nullptr ? static_cast<const T*>(p.gate) + static_cast<size_t>(b) * p.q_bstride : nullptr;
  T* ob = static_cast<T*>(p.out) + static_cast<size_t>(b) * p.out_bstride;
  const int qhs = p.q_hstride;  // D, or 2D for the interleaved q/gate projection
  // RoPE position of q and of the appended k: the last attended token, or the
  // caller's global position when this launch holds one shard of a longer sequence
  const int rpos = (p.plan == nullptr && p.rope_pos >= 0) ? static_cast<int>(p.rope_pos) : S - 1;
  // Before the preceding kernel has completed: the norm weights (constants) and the
  // page-table entry of the appended row. The q rows go to warp w (rows w and w+4),
  // the append to a warp with the fewest q rows; each warp issues all its row loads
  // before it computes, so its prologue costs one load round trip.
  const bool fuse_q = (p.flags & QIC_FUSE_Q_PROLOGUE) != 0;
  const bool my_append = do_append && warp == G % kConsumerWarps;
  float qw[D / 32], kw[D / 32];
  if (fuse_q) row_load<T, D>(static_cast<const T*>(p.q_norm_w), qw, lane);
  long long app_slot = S - 1;  // K/V append at position S-1 (src/model.cpp:634,637,639-641)
  if (my_append) {
    row_load<T, D>(static_cast<const T*>(p.k_norm_w), kw, lane);
    if (table != nullptr) {
      const int pos = S - 1, e = pos / p.page_size;
      app_slot = static_cast<long long>(__ldg(table + e)) * p.page_size + (pos - e * p.page_size);
    }
  }
  const bool app_ok = app_slot >= 0 && app_slot < p.cache_tokens;
  // the rotation at rpos (the same for q and the appended k), before the wait
  float rc[D / 32], rs[D / 32];
  if (fuse_q || my_append) row_rope_coeffs<D>(rc, rs, hd, rpos, p.theta, lane);
  // inputs written by the preceding kernel are read only after it has completed
  pdl_wait();
  // ---- prologue: q rows into shared memory, and the fused append ----
  {
    const int r0 = warp, r1 = warp + kConsumerWarps;  // G <= 8
    float v0[D / 32], v1[D / 32], kr[D / 32], vr[D / 32];
    const size_t nb = static_cast<size_t>(b) * p.kv_new_bstride + static_cast<size_t>(kvh) * D;
    if (r0 < G) row_load<T, D>(qb + static_cast<size_t>(kvh * G + r0) * qhs, v0, lane);
    if (r1 < G) row_load<T, D>(qb + static_cast<size_t>(kvh * G + r1) * qhs, v1, lane);
    if (my_append && app_ok) {
      row_load<T, D>(static_cast<const T*>(p.k_new) + nb, kr, lane);
      row_load<T, D>(static_cast<const T*>(p.v_new) + nb, vr, lane);
    }
    if (r0 < G) {
      if (fuse_q) {
        row_rmsnorm_w_tree<T, D>(v0, qw, hd, p.eps);
        row_rope_apply<T, D>(v0, rc, rs, lane);
      }
      row_store<T, D>(q_s + r0 * D, v0, lane);
    }
    if (r1 < G) {
      if (fuse_q) {
        row_rmsnorm_w_tree<T, D>(v1, qw, hd, p.eps);
        row_rope_apply<T, D>(v1, rc, rs, lane);
      }
      row_store<T, D>(q_s + r1 * D, v1, lane);
    }
    if (my_append) {
      if (app_ok) {
        // the reference's ascending-order sum of squares (app_s is free until the row
        // is staged there below)
        row_rmsnorm_w_staged<T, D>(kr, kw, hd, p.eps, reinterpret_cast<float*>(app_s), lane);
        row_rope_apply<T, D>(kr, rc, rs, lane);
        const size_t at = static_cast<size_t>(app_slot) * static_cast<size_t>(p.Hkv) * D + static_cast<size_t>(kvh) * D;
        row_store<T, D>(static_cast<T*>(p.k_cache) + at, kr, lane);
        row_store<T, D>(static_cast<T*>(p.v_cache) + at, vr, lane);
        // the same bytes for the consumer of the stage holding this row
        row_store<T, D>(app_s, kr, lane);
        row_store<T, D>(app_s + D, vr, lane);
        if (lane == 0) flags_s[2] = 1;
      } else if (lane == 0) {
        record_status(p.status, QIC_DEV_BAD_PAGE);
      }
      // a later copy of this row (a stage issued after the barrier below) goes through
      // TMA, the async proxy
      fence_proxy_async_global();
      __syncwarp();
    }
  }
  consumer_sync();
  // Tickets of the pool: a warp asks for its next stage when it issues one, and
  // reads the answer (and starts loading that stage's page-table entries) when it
  // begins the following stage, so the atomic and the table load overlap compute.
  // Tickets are taken only after griddepcontrol.wait: the counter is reset by the
  // previous call's last merger.
  unsigned tk_raw = 0;      // lane 0: the pending ticket
  bool tk_pending = false;  // a ticket has been asked for and not read yet
  int tk_next = -1;         // next pool stage of this warp (read), or -1
  int pg_tk = 0;            // its page-table entry (lane's box)
  // The first ticket is asked for when the warp issues its last own stage (here, if
  // the initial copies already were); a warp with no stage of its own never reads a
  // ticket, so it takes none.
  auto ask_ticket = [&]() {
    if (lane == 0) tk_raw = atomicAdd(reinterpret_cast<unsigned*>(stage_ctr), 1u);
    tk_pending = true;
  };
  if (pool_n > 0 && live > 0 && a0 + warp + kSlots * kConsumerWarps >= a1) ask_ticket();

  // ---- B fragments of Q^T (k = dims, n = query heads of the group) ----
  const int hq = lane >> 2;       // n index held by this lane in B fragments
  const int kq = (lane & 3) * 2;  // k pair held by this lane
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
  const int box_row_bytes = bh * 128;
  const int q8 = lane >> 3;  // ldmatrix matrix index supplied by this lane
  const int rr = lane & 7;   // row within that 8x8 matrix
  uint32_t rowK[NG], rowV[NG];
#pragma unroll
  for (int g2 = 0; g2 < NG; ++g2) {
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
  if (tail_regs && do_append && warp == G % kConsumerWarps && flags_s[2] != 0) {
    // the appended token, alone in the uncopied last stage: this warp's softmax state
    // starts from it (score against each q row, l = 1, o = its v row), with its k and
    // v rows as stored into the cache (app_s)
    float kk[D / 32];
    row_load<T, D>(app_s, kk, lane);
    const int ha = (lane & 3) * 2;  // this lane's head columns ha, ha + 1
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) {
      float part = 0.0f;
      if (h < G) {
        float qv[D / 32];
        row_load<T, D>(q_s + h * D, qv, lane);
#pragma unroll
        for (int e = 0; e < D / 32; ++e) part += qv[e] * kk[e];
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(kFullMask, part, off);
      if (h == ha) m0 = part * sl2;
      if (h == ha + 1) m1 = part * sl2;
    }
    // l is kept as per-lane partial sums over the lanes of a head column (summed after
    // the stage loop): the token counts once, in the lane with hq == 0
    l0 = hq == 0 ? 1.0f : 0.0f;
    l1 = hq == 0 ? 1.0f : 0.0f;
#pragma unroll
    for (int j = 0; j < KS; ++j) {
      const float va = to_f32<T>(app_s[D + j * 16 + hq]), vb = to_f32<T>(app_s[D + j * 16 + hq + 8]);
      acc[j][0] = va;
      acc[j][1] = va;
      acc[j][2] = vb;
      acc[j][3] = vb;
    }
  }

#pragma unroll 1
  for (int k = 0; live > 0; k = (k + 1 == kSlots) ? 0 : k + 1) {
    if (cur[k] < 0) continue;
    const int i = cur[k];
    const int slot = warp + k * kConsumerWarps;
    if (!__all_sync(kFullMask, mbar_wait(&full[slot], lap[k] & 1, deadline))) {
      ok = false;
      break;
    }
    if (tk_pending) {
      const int v = static_cast<int>(__shfl_sync(kFullMask, tk_raw, 0));
      tk_next = v < pool_n ? v : -1;
      if (tk_next >= 0 && table != nullptr) pg_tk = load_entry(box_entry(tk_next));
      tk_pending = false;
    }
    const int t0 = i * TOK;
    const int nvalid = min(TOK, S - t0);
    uint8_t* sk = ring + slot * Sh::kStageBytes;
    const uint32_t bk = smem_u32(sk);
    const uint32_t bv = bk + Sh::kKBytes;
    if (app_patch && i == append_stage && flags_s[2] != 0) {
      // the appended token's k and v rows: 16-byte units u of row tl in chunk c at the
      // 128-byte-swizzled position u ^ (tl % 8), as TMA lays them out
      const int tl = (S - 1) - t0;
      constexpr int UR = D / 8;  // 16-byte units per row
      for (int u = lane; u < 2 * UR; u += 32) {
        const int kind = u / UR, g = u - kind * UR;
        const int c = g >> 3, w16 = g & 7;
        uint8_t* dst = sk + kind * Sh::kKBytes + (tl >> lbh) * box_bytes + c * (bh * 128) + (tl & (bh - 1)) * 128 +
                       ((w16 ^ (tl & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(app_s + kind * D + g * 8);
      }
      // these generic writes precede a later TMA write into the same slot
      fence_proxy_async_smem();
      __syncwarp();
    }
    if (nvalid < TOK) {
      // rows past the sequence end hold stale or unloaded data: zero V there so
      // P = 0 rows cannot turn into NaN in the PV product
      uint8_t* sv = sk + Sh::kKBytes;
      const int nz = (TOK - nvalid) * Sh::kChunks * 8;  // 16-byte units
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

    // S^T = K Q^T for each 16-token group of the stage
    float sc[NG][4];
#pragma unroll
    for (int g2 = 0; g2 < NG; ++g2) {
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
    for (int g2 = 0; g2 < NG; ++g2) {
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
    for (int g2 = 0; g2 < NG; ++g2) {
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
    for (int g2 = 0; g2 < NG; ++g2) {
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
    ++lap[k];
    // refill this slot right away: the slot's next own stage, else the warp's next
    // pool stage, if any
    if (i >= a0 && i + kRing < a1) {  // (a pool stage has no own continuation)
      const int j = i + kRing;
      issue(j, pg_st[k], slot);
      cur[k] = j;
      if (table != nullptr && j + kRing < a1) pg_st[k] = load_entry(box_entry(j + kRing));
      // the warp's last own stage is issued: ask for a pool stage for the next refill
      if (pool_n > 0 && j + kConsumerWarps >= a1) ask_ticket();
    } else if (tk_next >= 0) {
      issue(tk_next, pg_tk, slot);
      cur[k] = tk_next;
      tk_next = -1;
      ask_ticket();
    } else {
      cur[k] = -1;
      --live;
    }
  }
  if (!ok) {
    if (lane == 0) {
      record_status(p.status, QIC_DEV_TIMEOUT);
      flags_s[0] = 1;
    }
    // wait (bounded) for this warp's copies still in flight before the CTA exits
    const uint64_t dl2 = globaltimer_ns() + p.timeout_ns;
#pragma unroll
    for (int k = 0; k < kSlots; ++k)
      if (cur[k] >= 0) mbar_wait(&full[warp + k * kConsumerWarps], lap[k] & 1, dl2);
    __syncwarp();
  }
  // full row sums per head column
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    l0 += __shfl_xor_sync(kFullMask, l0, o);
    l1 += __shfl_xor_sync(kFullMask, l1, o);
  }
  const int hA = (lane & 3) * 2, hB = hA + 1;
  // this warp's (m, l) go outside the ring (other warps may still read their slots),
  // so one barrier both ends the stage loops and publishes them
  float* cm = ml_s;                    // [4][8] m
  float* cl = ml_s + kConsumerWarps * 8;  // [4][8] l
  if (lane < 4) {
    cm[warp * 8 + hA] = m0;
    cm[warp * 8 + hB] = m1;
    cl[warp * 8 + hA] = l0;
    cl[warp * 8 + hB] = l1;
  }
  consumer_sync();
  const bool aborted = flags_s[0] != 0;

  // ---- combine the four warps (ring memory is free now) ----
  // Each warp's share of head h is weighted by exp2(m_w - M) / L with M, L the
  // head's maximum and normaliser over the four warps; the weights are applied to
  // the accumulators in registers, so the cross-warp step is a plain sum.
  float* co = reinterpret_cast<float*>(ring);  // [4][8][D + 4] weighted o (padded rows: no bank conflicts)
  float* mine = reinterpret_cast<float*>(ring + Sh::kCombineBytes);  // this split: [o: G*D][lse: G]
  constexpr int kCoRow = D + 4;
  if (!aborted) {
    float MA = -INFINITY, MB = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      MA = fmaxf(MA, cm[w * 8 + hA]);
      MB = fmaxf(MB, cm[w * 8 + hB]);
    }
    const float MAu = (MA == -INFINITY) ? 0.0f : MA, MBu = (MB == -INFINITY) ? 0.0f : MB;
    float LA = 0.0f, LB = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      LA += cl[w * 8 + hA] * exp2f(cm[w * 8 + hA] - MAu);
      LB += cl[w * 8 + hB] * exp2f(cm[w * 8 + hB] - MBu);
    }
    const float wA = LA > 0.0f ? exp2f(m0 - MAu) / LA : 0.0f;
    const float wB = LB > 0.0f ? exp2f(m1 - MBu) / LB : 0.0f;
    float* coA = co + (warp * 8 + hA) * kCoRow + hq;
    float* coB = co + (warp * 8 + hB) * kCoRow + hq;
#pragma unroll
    for (int j = 0; j < KS; ++j) {
      coA[j * 16] = acc[j][0] * wA;
      coB[j * 16] = acc[j][1] * wB;
      coA[j * 16 + 8] = acc[j][2] * wA;
      coB[j * 16 + 8] = acc[j][3] * wB;
    }
    // this split's log-sum-exp per head (log2 domain)
    if (warp == 0 && lane < 4 && (nsplit > 1 || p.part_out != nullptr)) {
      if (hA < G) mine[G * D + hA] = LA > 0.0f ? MAu + log2f(LA) : -INFINITY;
      if (hB < G) mine[G * D + hB] = LB > 0.0f ? MBu + log2f(LB) : -INFINITY;
    }
  }
  consumer_sync();
  const size_t qoff = static_cast<size_t>(kvh) * G * D;  // first output row of this group
  // gate element of output idx of this group (head idx / D, dim idx % D)
  auto gidx = [&](int idx) -> size_t {
    return static_cast<size_t>(kvh * G + idx / D) * qhs + (idx % D);
  };
  const int pf = partial_floats(G, D);
  constexpr bool cp = CP;
  unsigned cp_e = 0;  // exchange epoch of this call (slice mergers, context parallel)
  // Destination of the final value o of output idx (head h, log-sum-exp lse): the
  // output or the caller's fp32 partial (QIC_PARTIAL_OUT).
  auto emit = [&](int idx, int h, float o, float lse, bool head_first) {
    if (p.part_out != nullptr) {
      float* po = p.part_out + static_cast<size_t>(kvh) * pf;
      po[idx] = o;
      if (head_first) po[GD + h] = lse;
    } else {
      write_out<T>(ob, gb, qoff + idx, gidx(idx), o);
    }
  };
  // the sum over the four warps: into the output (one split), into `mine` (a cluster
  // of one CTA), or, in a cluster, on the way into the st.async stores below
  if (!aborted && (nsplit == 1 || C == 1)) {
#pragma unroll 2
    for (int idx = ctid; idx < GD; idx += kConsumerWarps * 32) {
      const int h = idx / D, d = idx - h * D;
      float o = 0.0f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) o += co[(w * 8 + h) * kCoRow + d];
      if (nsplit == 1) {
        emit(idx, h, o, mine[GD + h], d == 0);
      } else {
        mine[idx] = o;
      }
    }
  }
  if (nsplit == 1) {
    // every warp of the kv head's only CTA is past its stage loop: ready for the next call
    if (stage_ctr != nullptr && ctid == 0) *stage_ctr = 0;
    return;
  }

  // ---- merge the partials of this cluster: CTA c owns output slice c. Every CTA
  // sends slice c of its partial, and its per-head log-sum-exps, into CTA c's receive
  // buffer with st.async, then merges its own slice from its own shared memory once
  // its mbarrier has counted all C contributions: no cluster-wide barrier, and no CTA
  // waits at exit for its peers (its shared memory is only written, never read, by
  // them, and every write to it has landed before it merges) ----
  const int Gp = (G + 3) & ~3;
  const int rxs = slice + Gp;  // floats of one contribution in the receive buffer
  if (C == 1) consumer_sync();  // `mine` is complete (the merge below reads it across threads)
  if (C > 1) {
    // every CTA of the cluster runs and has initialised its receive mbarrier (the
    // phase completed long ago; this orders nothing inside the CTA)
    asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
    if (slice % 4 == 0) {
      // 16-byte stores (the combine rows, the slices and the receive rows are 16-byte
      // aligned), each the four warps' sum of four outputs of one head; the
      // log-sum-exp quads are padded with -inf
      const int q4 = rxs / 4;
      // item i = (destination c, quad e4): one division per thread, then steps of a
      // CTA's thread count
      constexpr int kStep = kConsumerWarps * 32;
      const int step_c = kStep / q4, step_e = kStep - step_c * q4;
      int c = ctid / q4, e4 = ctid - (ctid / q4) * q4;
#pragma unroll 1
      for (int i = ctid; i < C * q4; i += kStep) {
        const int e = e4 * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        bool send = true;
        if (e < slice) {
          const int idx = c * slice + e;
          send = idx < GD;
          if (send && !aborted) {
            const int h = idx / D, d = idx - h * D;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) {
              const float4 x = *reinterpret_cast<const float4*>(co + (w * 8 + h) * kCoRow + d);
              v.x += x.x;
              v.y += x.y;
              v.z += x.z;
              v.w += x.w;
            }
          }
        } else {
          const int h = e - slice;
          v.x = (!aborted && h < G) ? mine[GD + h] : -INFINITY;
          v.y = (!aborted && h + 1 < G) ? mine[GD + h + 1] : -INFINITY;
          v.z = (!aborted && h + 2 < G) ? mine[GD + h + 2] : -INFINITY;
          v.w = (!aborted && h + 3 < G) ? mine[GD + h + 3] : -INFINITY;
        }
        if (send) st_async_cluster_f32x4(rx + rank * rxs + e, rx_bar, c, v);
        e4 += step_e;
        c += step_c;
        if (e4 >= q4) {
          e4 -= q4;
          ++c;
        }
      }
    } else {
#pragma unroll 1
      for (int i = ctid; i < C * (slice + G); i += kConsumerWarps * 32) {
        const int c = i / (slice + G), e = i - c * (slice + G);
        float v;
        if (e < slice) {
          const int idx = c * slice + e;
          if (idx >= GD) continue;
          v = 0.0f;
          if (!aborted) {
            const int h = idx / D, d = idx - h * D;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) v += co[(w * 8 + h) * kCoRow + d];
          }
        } else {
          v = aborted ? -INFINITY : mine[GD + e - slice];  // an aborted CTA contributes nothing
        }
        st_async_cluster_f32(rx + rank * rxs + e, rx_bar, c, v);
      }
    }
    // Bounded: a peer whose stage loop gave up at the deadline still sends, after
    // draining its copies for at most one more timeout.
    if (!mbar_wait(rx_bar, 0, deadline + 2 * p.timeout_ns)) {
      if (ctid == 0) record_status(p.status, QIC_DEV_TIMEOUT);
      return;
    }
  }
  // a kv head that is one cluster is past every stage loop (each contribution is sent
  // after its CTA's loop): reset its ticket counter
  if (nclust == 1 && rank == 0 && stage_ctr != nullptr && ctid == 0) *stage_ctr = 0;
  // contribution c: rx_o[c * rxs + idx - o_off] for output idx, rx_l[c * rxs + h] for
  // head h (with one CTA per cluster, its own partial)
  const float* rx_o = C > 1 ? rx : mine;
  const float* rx_l = C > 1 ? rx + slice : mine + GD;
  const int o_off = C > 1 ? lo : 0;
  // context parallel: this rank's merged slice (after the cross-cluster merge when the
  // kv head spans several clusters) goes to every rank as one contribution
  const int cpw = cp_slice_words(G, D);
  unsigned cp_tag = 0;
  if (cp) {
    cp_e = ld_relaxed_gpu_u32(p.cp_epoch) + 1;
    cp_tag = ((cp_e & 0xffffffu) << 8) | 1u;
  }
  auto cp_push = [&](int idx, float o, float lse) {
    for (int r = 0; r < p.cp_world; ++r) {
      uint2* slot = cp_slot(p.cp_peer[r], cp_e & 1, p.cp_rank, p.cp_world, p.Hkv, kvh, rank, cpw);
      st_word_sys(slot + (idx - lo), o, cp_tag);
      if (idx == lo) st_word_sys(slot + cpw - 2, lse, cp_tag);
      if (idx == hi - 1) st_word_sys(slot + cpw - 1, lse, cp_tag);
    }
  };
  float* gslot = p.part + static_cast<size_t>(part_base + cid) * pf;  // [o: G*D][lse: G]
  // one lane per output: the max over the C contributions, then their weights
  // (measured against spreading an output's contributions over up to C lanes with a
  // shuffle combine: the runtime lane count's division and the shuffles cost more
  // than the shorter chain saved, S=8192 11.64 vs 11.96 us per layer)
#pragma unroll 1
  for (int idx = lo + ctid; idx < hi; idx += kConsumerWarps * 32) {
    const int h = idx / D;
    float mx = -INFINITY, sum = 0.0f, o = 0.0f;
#pragma unroll 4
    for (int c = 0; c < C; ++c) mx = fmaxf(mx, rx_l[c * rxs + h]);
    if (mx != -INFINITY) {
#pragma unroll 4
      for (int c = 0; c < C; ++c) {
        const float w = exp2f(rx_l[c * rxs + h] - mx);
        sum += w;
        o += w * rx_o[c * rxs + idx - o_off];
      }
    }
    const float lse = sum > 0.0f ? mx + log2f(sum) : -INFINITY;
    o = sum > 0.0f ? o / sum : 0.0f;
    if (cp && nclust == 1) {
      cp_push(idx, o, lse);
    } else if (nclust == 1) {
      emit(idx, h, o, lse, idx == lo || idx - h * D == 0);
    } else {
      gslot[idx] = o;
      if (idx == lo || idx - h * D == 0) gslot[GD + h] = lse;
    }
  }
  if (nclust > 1) {
    // ---- merge the cluster partials of this slice: last arriving cluster ----
    consumer_sync();
    const int counter = (b * p.Hkv + kvh) * C + rank;
    if (ctid == 0) {
      const int prev = atomic_add_acq_rel_gpu(p.counters + counter, 1);
      flags_s[1] = (prev == nclust - 1) ? 1 : 0;
    }
    consumer_sync();
    if (flags_s[1]) {
      const float* g0 = p.part + static_cast<size_t>(part_base) * pf;
#pragma unroll 1
      for (int idx = lo + ctid; idx < hi; idx += kConsumerWarps * 32) {
        const int h = idx / D;
        // online log-sum-exp over the cluster partials, eight loads in flight at a time
        float mx = -INFINITY, sum = 0.0f, o = 0.0f;
#pragma unroll 1
        for (int k0 = 0; k0 < nclust; k0 += 8) {
          float lk[8], ok[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int k = k0 + u;
            lk[u] = k < nclust ? __ldcg(g0 + static_cast<size_t>(k) * pf + GD + h) : -INFINITY;
            ok[u] = k < nclust ? __ldcg(g0 + static_cast<size_t>(k) * pf + idx) : 0.0f;
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const float mn = fmaxf(mx, lk[u]);
            if (mn == -INFINITY) continue;
            const float sc = exp2f(mx - mn), w = exp2f(lk[u] - mn);
            sum = sum * sc + w;
            o = o * sc + w * ok[u];
            mx = mn;
          }
        }
        if (cp) {
          cp_push(idx, sum > 0.0f ? o / sum : 0.0f, sum > 0.0f ? mx + log2f(sum) : -INFINITY);
        } else {
          emit(idx, h, sum > 0.0f ? o / sum : 0.0f, sum > 0.0f ? mx + log2f(sum) : -INFINITY,
               idx == lo || idx - h * D == 0);
        }
      }
      if (ctid == 0) {
        p.counters[counter] = 0;  // ready for the next call
        // every cluster of this kv head has arrived: past every stage loop
        if (rank == 0 && stage_ctr != nullptr) *stage_ctr = 0;
      }
    }
  }
  if (cp && (nclust == 1 || flags_s[1] != 0)) {
    // ---- context parallel: the CTA that produced this rank's slice `rank` of the kv
    // head merges that slice from every rank's contribution, polling the tagged
    // words (one contribution per rank: its clusters are merged already) ----
    const int W = p.cp_world, par = cp_e & 1;
    const unsigned want = cp_e & 0xffffffu;
    const uint64_t dl = globaltimer_ns() + p.timeout_ns;
    bool late = false;
#pragma unroll 1
    for (int idx = lo + ctid; idx < hi; idx += kConsumerWarps * 32) {
      const int h = idx / D;
      const int lw = (h == lo / D) ? cpw - 2 : cpw - 1;  // log-sum-exp word of this output's head
      float mx = -INFINITY, sum = 0.0f, o = 0.0f;
      auto fold = [&](uint2 wo, uint2 wl) {
        const float lk = __uint_as_float(wl.x), ov = __uint_as_float(wo.x);
        const float mn = fmaxf(mx, lk);
        if (mn == -INFINITY) return;
        const float sc = exp2f(mx - mn), w = exp2f(lk - mn);
        sum = sum * sc + w;
        o = o * sc + w * ov;
        mx = mn;
      };
      // one contribution per rank; all of them are read together and re-read until
      // every tag is this call's
      uint2 wo[kMaxRanks], wl[kMaxRanks];
      unsigned have = 0;  // bit r: rank r's words are this call's
      const unsigned all = (1u << W) - 1u;
      bool ok = true;
#pragma unroll 1
      for (uint32_t it = 0;; ++it) {
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r) {
          if (r < W && !(have & (1u << r))) {
            const uint2* slot = cp_slot(p.cp_peer[p.cp_rank], par, r, W, p.Hkv, kvh, rank, cpw);
            wo[r] = ld_word_sys(slot + (idx - lo));
            wl[r] = ld_word_sys(slot + lw);
          }
        }
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r)
          if (r < W && (wo[r].y >> 8) == want && (wl[r].y >> 8) == want) have |= 1u << r;
        if (have == all) break;
        if ((it & 15u) == 15u && globaltimer_ns() > dl) {
          ok = false;
          break;
        }
        __nanosleep(32);
      }
      if (ok) {
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r)
          if (r < W) fold(wo[r], wl[r]);
      }
      if (ok && !aborted) {
        write_out<T>(ob, gb, qoff + idx, gidx(idx), sum > 0.0f ? o / sum : 0.0f);
      } else if (!ok) {
        late = true;
      }
    }
    if (late) record_status(p.status, QIC_DEV_PEER_TIMEOUT);
    // the last slice merger of this call advances the epoch for the next call
    consumer_sync();
    if (ctid == 0) {
      const unsigned prev = atomicAdd(p.cp_done, 1u);
      if (prev == static_cast<unsigned>(p.cp_mergers) - 1u) {
        *p.cp_done = 0u;
        *p.cp_epoch = cp_e;
      }
    }
  }
}

// ----------------------------------------------------------------------------
// log-sum-exp merge of QIC_PARTIAL_OUT partials (one thread per output element)
// ----------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(256) merge_partials_kernel(const float* __restrict__ partials, int n, int H,
                                                             int Hkv, const T* __restrict__ gate, T* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= H * D) return;
  const int G = H / Hkv, pf = partial_floats(G, D);
  const int h = i / D, d = i - h * D, kvh = h / G, hh = h - kvh * G;
  float mx = -INFINITY;
  for (int k = 0; k < n; ++k) mx = fmaxf(mx, partials[(static_cast<size_t>(k) * Hkv + kvh) * pf + G * D + hh]);
  const float mxu = (mx == -INFINITY) ? 0.0f : mx;
  float sum = 0.0f, o = 0.0f;
  for (int k = 0; k < n; ++k) {
    const float* pk = partials + (static_cast<size_t>(k) * Hkv + kvh) * pf;
    const float w = exp2f(pk[G * D + hh] - mxu);
    sum += w;
    o += w * pk[hh * D + d];
  }
  write_out<T>(out, gate, static_cast<size_t>(i), static_cast<size_t>(i), sum > 0.0f ? o / sum : 0.0f);
}

template <typename T, int D>
static cudaError_t launch_merge_typed(const float* partials, int n, int H, int Hkv, const void* gate, void* out,
                                      cudaStream_t stream) {
  const int total = H * D;
  merge_partials_kernel<T, D><<<(total + 255) / 256, 256, 0, stream>>>(partials, n, H, Hkv,
                                                                     static_cast<const T*>(gate), static_cast<T*>(out));
  return cudaGetLastError();
}

cudaError_t launch_attention_merge(int dtype, int head_dim, const float* partials, int n, int H, int Hkv,
                                   const void* gate, void* out, cudaStream_t stream) {
  if (dtype == QIC_DTYPE_BF16) {
    switch (head_dim) {
      case 64: return launch_merge_typed<__nv_bfloat16, 64>(partials, n, H, Hkv, gate, out, stream);
      case 128: return launch_merge_typed<__nv_bfloat16, 128>(partials, n, H, Hkv, gate, out, stream);
      case 256: return launch_merge_typed<__nv_bfloat16, 256>(partials, n, H, Hkv, gate, out, stream);
    }
  } else {
    switch (head_dim) {
      case 64: return launch_merge_typed<__half, 64>(partials, n, H, Hkv, gate, out, stream);
      case 128: return launch_merge_typed<__half, 128>(partials, n, H, Hkv, gate, out, stream);
      case 256: return launch_merge_typed<__half, 256>(partials, n, H, Hkv, gate, out, stream);
    }
  }
  return cudaErrorInvalidValue;
}

// ----------------------------------------------------------------------------
// host launcher
// ----------------------------------------------------------------------------
template <typename T, int D>
static cudaError_t configure_typed() {
  static unsigned long long configured = 0;  // one bit per device ordinal
  const int smem = AttnShape<D>::kSmemBytes + AttnShape<D>::kMaxRxBytes;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 64 && (configured & (1ull << dev))) return cudaSuccess;
  e = cudaFuncSetAttribute(decode_attn_kernel<T, D, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(decode_attn_kernel<T, D, false>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(decode_attn_kernel<T, D, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(decode_attn_kernel<T, D, true>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e == cudaSuccess && dev < 64) configured |= 1ull << dev;
  return e;
}

template <typename T, int D>
static cudaError_t launch_typed(const AttnParams& p, dim3 grid, cudaStream_t stream) {
  const int smem = AttnShape<D>::kSmemBytes + attn_rx_bytes(p.G, D, p.cluster);
  cudaError_t e = configure_typed<T, D>();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kAttnThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (p.flags & QIC_PDL) ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = static_cast<unsigned>(p.cluster);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = p.cp_world > 0 ? cudaLaunchKernelEx(&cfg, decode_attn_kernel<T, D, true>, p)
                     : cudaLaunchKernelEx(&cfg, decode_attn_kernel<T, D, false>, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <typename T, int D>
static int max_active_clusters_typed(int cluster, int group) {
  // cached per device, cluster size and query heads per kv head: clusters of `cluster`
  // CTAs that fit on the GPU at once
  static int cache[64][kMaxCluster + 1][kMaxGroup + 1] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || cluster < 1 || cluster > kMaxCluster ||
      group < 1 || group > kMaxGroup)
    return 0;
  if (cache[dev][cluster][group] != 0) return cache[dev][cluster][group];
  const int smem = AttnShape<D>::kSmemBytes + attn_rx_bytes(group, D, cluster);
  if (configure_typed<T, D>() != cudaSuccess) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cluster, 1, 1);
  cfg.blockDim = dim3(kAttnThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cluster);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, decode_attn_kernel<T, D, false>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  cache[dev][cluster][group] = n;
  return n;
}

int decode_attention_max_active_clusters(int dtype, int head_dim, int cluster, int group) {
  if (dtype == QIC_DTYPE_BF16) {
    switch (head_dim) {
      case 64: return max_active_clusters_typed<__nv_bfloat16, 64>(cluster, group);
      case 128: return max_active_clusters_typed<__nv_bfloat16, 128>(cluster, group);
      case 256: return max_active_clusters_typed<__nv_bfloat16, 256>(cluster, group);
    }
  } else {
    switch (head_dim) {
      case 64: return max_active_clusters_typed<__half, 64>(cluster, group);
      case 128: return max_active_clusters_typed<__half, 128>(cluster, group);
      case 256: return max_active_clusters_typed<__half, 256>(cluster, group);
    }
  }
  return 0;
}

cudaError_t launch_decode_attention(int dtype, int head_dim, const AttnParams& p, cudaStream_t stream) {
  const dim3 grid = p.plan != nullptr ? dim3(p.n_splits, 1, 1) : dim3(p.n_splits, p.Hkv, 1);
  if (dtype == QIC_DTYPE_BF16) {
    switch (head_dim) {
      case 64: return launch_typed<__nv_bfloat16, 64>(p, grid, stream);
      case 128: return launch_typed<__nv_bfloat16, 128>(p, grid, stream);
      case 256: return launch_typed<__nv_bfloat16, 256>(p, grid, stream);
    }
  } else {
    switch (head_dim) {
      case 64: return launch_typed<__half, 64>(p, grid, stream);
      case 128: return launch_typed<__half, 128>(p, grid, stream);
      case 256: return launch_typed<__half, 256>(p, grid, stream);
    }
  }
  return cudaErrorInvalidValue;
}

}  // namespace qic
