// Host/device shared declarations of the qic library (not part of the public ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/qic.h"

namespace qic {

constexpr int kConsumerWarps = 4;    // warps of an attention CTA; each streams and consumes its own ring slots
constexpr int kAttnThreads = kConsumerWarps * 32;
constexpr int kMaxCluster = 16;      // CTAs of one (sequence, kv head) merged through DSMEM
constexpr int kMaxGroup = 8;         // query heads per kv head handled by one n8 mma tile
constexpr int kMaxSplits = 256;      // KV splits per kv head
constexpr uint64_t kDefaultTimeoutNs = 2000000000ull;  // 2 s bound on every device wait

// Workspace layout, the same for every shape so one workspace can serve calls of any
// shape: [status word | pad to 256 B][kMaxCounters merge counters][partial slots].
// Counters are only ever used as counters and are left at zero by every call.
constexpr size_t kWsHeader = 256;
constexpr int kMaxCounters = 8192;
constexpr size_t kWsPartialOffset = kWsHeader + static_cast<size_t>(kMaxCounters) * sizeof(int);
// The last kMaxStageCounters counters of that region are the stage-pool ticket
// counters of single-sequence launches (one per kv head), never merge counters.
constexpr int kMaxStageCounters = 64;

// Tokens per TMA pipeline stage: one stage is 16 KB of K+V for head_dim 128/256
// (32 / 16 tokens) and 8 KB for head_dim 64 (32 tokens).
__host__ __device__ constexpr int stage_tokens(int head_dim) { return head_dim > 128 ? 16 : 32; }

// One partial of a (kv head, split): o[G][D] (normalised) then lse[G] (log2 domain),
// fp32, padded to a multiple of 4 floats.
__host__ __device__ constexpr int partial_floats(int G, int D) { return ((G * (D + 1)) + 3) & ~3; }

// Context parallelism. Workspace header words: calls completed (the exchange epoch)
// at byte 64, slice mergers finished in the current call at byte 128.
constexpr size_t kWsCpEpoch = 64;
constexpr size_t kWsCpDone = 128;
constexpr int kMaxRanks = QIC_MAX_RANKS;
constexpr int kCpSlices = 8;  // exchange slices per kv head: one per CTA of an 8-CTA cluster
// Exchange words: 8 bytes, {fp32 value, tag}, written with one 8-byte store so a
// reader that sees the tag sees the value (no fence, no separate flag). tag =
// (epoch & 0xffffff) << 8 | contributions of the writing rank (1).
// Exchange buffer of one rank: [2 parities][world sources][Hkv][kCpSlices]
// contributions of cp_slice_words words each: the slice's outputs, then the
// log-sum-exp of the head of its first and of its last output.
__host__ __device__ constexpr int cp_slice_words(int G, int D) { return (G * D + kCpSlices - 1) / kCpSlices + 2; }
__host__ __device__ constexpr size_t cp_exchange_bytes(int G, int D, int Hkv, int world) {
  return static_cast<size_t>(2) * world * Hkv * kCpSlices * cp_slice_words(G, D) * 8;
}

// Work of one CTA in a planned (batched) launch: stages [st_lo, st_hi) of sequence b
// for kv head kvh, being split `split` of `nsplit` for that (b, kvh); its partial goes
// to slot part_base + split. 32 bytes.
struct WorkItem {
  int b, kvh, split, nsplit;
  int st_lo, st_hi, seq_len, part_base;
};

struct AttnParams {
  CUtensorMap tm_k;                  // 2D map over [tokens, kv_dim], box {64, box_h}, 128B swizzle
  CUtensorMap tm_v;
  const void* q;                     // [H, q_hstride]
  const void* gate;                  // [H, q_hstride] or null
  void* out;                         // [H, D]
  void* k_cache;                     // generic pointers for the fused append
  void* v_cache;
  const int32_t* page_table;         // null = contiguous
  const void* q_norm_w;
  const void* k_norm_w;
  const void* k_new;
  const void* v_new;
  float* part;                       // partial slots, partial_floats each
  int* counters;                     // one merge counter per (sequence, kv head)
  int* status;                       // device status word
  const WorkItem* plan;              // null: one sequence, grid (n_splits, Hkv)
  long long q_bstride;               // elements between sequences in q / gate
  long long out_bstride;             // elements between sequences in out
  int q_hstride;                     // elements between heads in q / gate: D, or 2D when interleaved
  long long kv_new_bstride;          // elements between sequences in k_new / v_new
  int table_bstride;                 // entries between sequences' block-table rows
  int part_slots;                    // partial slots available in the workspace
  int num_counters;                  // merge counters available in the workspace
  int64_t cache_tokens;
  int H, Hkv, G;
  int head_dim;                      // runtime copy of D (mirrors the reference's runtime arithmetic)
  int seq_len;
  int page_size;
  int box_h, log2_box_h;
  int n_splits;                      // cluster * n_clusters CTAs per kv head (stages: from seq_len)
  int cluster;                       // CTAs per thread-block cluster along the splits
  int flags;
  float eps, theta, scale_log2;
  uint64_t timeout_ns;
  long long rope_pos;                // RoPE position of q and the appended k (single-sequence launches)
  float* part_out;                   // QIC_PARTIAL_OUT: [Hkv][partial_floats] instead of out
  int* stage_ctr;                    // per kv head ticket counters of the stage pool, or null
  const int32_t* seq_len_dev;        // QIC_DEVICE_SEQ_LEN: the current length (seq_len is its bound), or null
  // context parallelism (cp_world == 0: off)
  int cp_rank, cp_world;
  int cp_mergers;                    // slice mergers per call on this rank: Hkv * kCpSlices
  unsigned* cp_epoch;                // workspace words kWsCpEpoch / kWsCpDone
  unsigned* cp_done;
  void* cp_peer[kMaxRanks];          // every rank's exchange buffer, addressable here
};

// Weight-streaming GEMV (gemv_kernel.cu): 256 threads per CTA, 256-column tiles, up to
// kGemvMaxSegments projections of one input per launch, the rows of a tile split over
// a thread-block cluster of up to kGemvMaxSplits CTAs.
constexpr int kGemvThreads = 256;
constexpr int kGemvTile = 256;
constexpr int kGemvMaxSegments = QIC_GEMV_MAX_SEGMENTS;
constexpr int kGemvMaxSplits = 16;
constexpr int kGemvMaxRowsPerSplit = 8192;  // normalised input rows kept in shared memory
constexpr int kGemvRowsPerSlot = 8;         // rows per TMA box / ring slot (8 x 512 B)
constexpr int kGemvSlotsPerWarp = 3;        // ring slots per warp

struct GemvSeg {
  const void* w;    // [K, N], N contiguous
  void* out;        // [N]
  const void* res;  // [N] residual or null
  int N;
  int tile0;        // first tile of this segment in the grid
};

struct GemvParams {
  CUtensorMap tm[kGemvMaxSegments];  // 2D map of each segment's weights {N, K}, box {kGemvTile, kGemvRowsPerSlot}
  const void* x;       // [K]
  const void* norm_w;  // [K] or null
  float eps;
  int K;
  int flags;           // QIC_PDL
  int nseg;
  int n_tiles;
  int splits;          // CTAs per cluster along the rows
  int rows_per_split;
  int xs_floats;       // floats of the input slice in shared memory (rows_per_split rounded up to 8)
  int* status;         // device status word (QIC_DEV_TIMEOUT) or null
  uint64_t timeout_ns;
  GemvSeg seg[kGemvMaxSegments];
};

cudaError_t launch_gemv(int dtype, const GemvParams& p, bool pair, bool norm, cudaStream_t stream);
size_t gemv_smem_bytes(int rows_per_split);
// Clusters of `cluster` GEMV CTAs resident at once (-1 or 0 if unknown).
int gemv_max_active_clusters(int dtype, int cluster, int rows_per_split);

// Launchers (attn_kernel.cu)
cudaError_t launch_decode_attention(int dtype, int head_dim, const AttnParams& p, cudaStream_t stream);
// out = log-sum-exp merge of n partials [n][Hkv][partial_floats] (+ gate)
cudaError_t launch_attention_merge(int dtype, int head_dim, const float* partials, int n, int H, int Hkv,
                                   const void* gate, void* out, cudaStream_t stream);
// Clusters of `cluster` CTAs of the decode kernel that can be resident at once (0 if unknown).
int decode_attention_max_active_clusters(int dtype, int head_dim, int cluster, int group);

// Standalone ops (rowops.cu)
cudaError_t launch_head_rmsnorm(int dtype, const void* x, const void* w, int num_heads, int head_dim, float eps,
                                void* out, cudaStream_t stream);
cudaError_t launch_rope_inplace(int dtype, void* x, int num_heads, int head_dim, int position, float theta,
                                cudaStream_t stream);
cudaError_t launch_sigmoid_mul_inplace(int dtype, void* x, const void* gate, int n, cudaStream_t stream);
cudaError_t launch_kv_append(int dtype, const void* k_new, const void* v_new, const void* k_norm_w, float eps,
                             float theta, int position, const int32_t* page_table, int page_size, int64_t cache_tokens,
                             void* k_cache, void* v_cache, int num_kv_heads, int head_dim, cudaStream_t stream);

// GatedDeltaNet (gdn_kernel.cu)
cudaError_t launch_gated_delta(const qic_gdn_args& a, cudaStream_t stream);

}  // namespace qic
