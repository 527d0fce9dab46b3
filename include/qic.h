/*
 * qic.h — C-ABI of the QweninCuda decode-time KV-cache hot path for B200 (sm_100a).
 *
 * Plain C types only: device pointers as void*, sizes as int32/int64, CUDA streams
 * as an opaque pointer (binary-compatible with cudaStream_t / CUstream). Every entry
 * point returns a qic_status (0 = success) and, except qic_device_alloc, never
 * allocates device memory; scratch space is passed in by the caller (see
 * qic_decode_workspace_bytes).
 *
 * Element types: QIC_DTYPE_F16 (the reference's `half`) or QIC_DTYPE_BF16.
 *
 * Reference interfaces replaced (paths inside the QweninCuda project):
 *   launch_head_rmsnorm        include/kernels.cuh:7-8,   src/kernels.cu:78-112,392-396
 *   launch_rope_inplace        include/kernels.cuh:13,    src/kernels.cu:150-183,418-424
 *   launch_sigmoid_mul_inplace include/kernels.cuh:12,    src/kernels.cu:138-148,412-416
 *   launch_flash_attention     include/kernels.cuh:15-16, src/kernels.cu:200-290,432-438
 *   launch_paged_attention     include/kernels.cuh:17-19, src/kernels.cu:292-374,440-447
 *   K/V append (cudaMemcpy D2D at position*kv_dim)        src/model.cpp:31-33,639-641
 *   full-attention block body (norm, RoPE, append, attn)  src/model.cpp:633-652
 *   GatedDeltaNet host loop (conv, delta rule, gated norm) src/model.cpp:692-793
 * The exact C++ signatures of include/kernels.cuh are provided as well, by
 * include/qic_kernels_compat.h, on top of these entry points.
 */
#ifndef QIC_H_
#define QIC_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* qic_stream_t; /* same type as cudaStream_t */

typedef enum qic_status {
  QIC_SUCCESS = 0,
  QIC_ERROR_INVALID_VALUE = 1,   /* null pointer, non-positive size, H % Hkv != 0, position outside cache */
  QIC_ERROR_NOT_SUPPORTED = 2,   /* head_dim / group size / page size outside the compiled set */
  QIC_ERROR_MISALIGNED = 3,      /* a pointer or row stride breaks the 16-byte TMA rule */
  QIC_ERROR_WORKSPACE = 4,       /* workspace missing or smaller than required */
  QIC_ERROR_CUDA = 5,            /* CUDA runtime or launch error (qic_last_cuda_error) */
  QIC_ERROR_DEVICE_TIMEOUT = 6,  /* a bounded device-side wait gave up (device status word) */
  QIC_ERROR_BAD_PAGE = 7,        /* a page-table entry points outside the cache (device status word) */
  QIC_ERROR_PEER = 8             /* peer-exchange set-up failed */
} qic_status;

enum { QIC_DTYPE_F16 = 0, QIC_DTYPE_BF16 = 1 };

/* Bits of the device status word kept in the workspace (qic_workspace_status). */
enum {
  QIC_DEV_TIMEOUT = 1,           /* a bounded wait timed out */
  QIC_DEV_BAD_PAGE = 2,          /* an out-of-range page-table entry was clamped to page 0 */
  QIC_DEV_PEER_TIMEOUT = 4,      /* a peer never published its partial */
  QIC_DEV_BAD_PLAN = 8,          /* a batched work item does not fit the workspace; it was skipped */
  QIC_DEV_BAD_LENGTH = 16        /* a device-resident sequence length was outside [1, seq_len]; clamped */
};

/* Flags of qic_decode_args.flags */
enum {
  QIC_FUSE_Q_PROLOGUE = 1,       /* q := RoPE(head_rmsnorm(q, q_norm_w)) inside the attention kernel */
  QIC_FUSE_APPEND = 2,           /* k_new/v_new appended at position seq_len-1 inside the kernel */
  QIC_PDL = 4,                   /* programmatic dependent launch: the kernel may start while the previous
                                    kernel in the stream runs and prefetch cached K/V rows (all but the
                                    appended one) and page-table entries; q, k_new, v_new, gate and the
                                    workspace are touched only after that kernel has completed. No
                                    kernel that can still be running may write the page table or those
                                    cached rows: when every kernel in between lets its dependents start
                                    early (this one does), that includes kernels several launches back.
                                    In a layer stack their writers (this layer's previous step, the
                                    caller's page-table update) are a whole stack of layers back. */
  QIC_PARTIAL_OUT = 8,           /* out is float [Hkv][qic_partial_floats()]: per kv head, the G*d
                                    outputs normalised by their own softmax sum, then G log-sum-exp
                                    values (log2 of the sum of 2^(score*log2(e)/sqrt(d))), padded to a
                                    multiple of 4 floats; no gate. Partials of disjoint token ranges
                                    of one sequence combine with qic_attention_merge. */
  QIC_EXPLICIT_POSITION = 16,    /* args->position is the token position used for RoPE of q and of the
                                    appended k (default seq_len-1). The append still writes the last
                                    attended row (index seq_len-1 of this call's cache or page table):
                                    a rank that holds the final shard of a longer sequence. */
  QIC_DETERMINISTIC = 32,        /* bitwise-reproducible outputs. Without it, single-sequence calls with
                                    a workspace and at least 8 stages per split hand the first eighth
                                    of the sequence's stages to whichever CTA asks first (load
                                    balance), so the order in which split partials are summed, and the
                                    last bits of the output, can change from call to call. */
  QIC_Q_GATE_INTERLEAVED = 64,   /* q is the interleaved q/gate projection [H, 2d] (per head d q values,
                                    then d gate values) and out *= sigmoid(gate) with that gate; `gate`
                                    must be NULL. Folds launch_split_q_gate_interleaved
                                    (src/kernels.cu:113-127, src/model.cpp:628) into the kernel. Batched
                                    calls: q is [B, H, 2d]. Partial outputs carry no gate. */
  QIC_DEVICE_SEQ_LEN = 128       /* the number of tokens attended is read from device memory
                                    (args->seq_len_dev, an int32 in [1, args->seq_len]) when the kernel
                                    starts; args->seq_len is the largest it may be and sizes the launch.
                                    A decode loop captured once in a CUDA graph then replays for every
                                    token: the caller advances the length (and any new page-table
                                    entry) in device memory before each replay. The length is read
                                    early like the page table (QIC_PDL). Needs a workspace (an
                                    out-of-range length is clamped and reported as QIC_DEV_BAD_LENGTH);
                                    not with context parallelism. */
};

/* Longest sequence (tokens attended, and token positions) any entry point accepts:
 * 2^30, beyond any cache that fits a GPU. Longer lengths return QIC_ERROR_INVALID_VALUE. */
#define QIC_MAX_SEQ_LEN 1073741824

const char* qic_status_string(int status);
int qic_last_cuda_error(void);    /* cudaError_t of the last QIC_ERROR_CUDA on this thread */
int qic_version(void);

/* ------------------------------------------------------------------------- */
/* Standalone ops, numerically identical to the reference kernels.           */
/* ------------------------------------------------------------------------- */

/* out[h,:] = x[h,:] * rsqrt(mean(x[h,:]^2) + eps) * weight, rounded to dtype.
 * Replaces launch_head_rmsnorm (include/kernels.cuh:7-8). x == out allowed. */
int qic_head_rmsnorm(int dtype, const void* x, const void* weight, int num_heads, int head_dim, float eps,
                     void* out, qic_stream_t stream);

/* Rotate-half RoPE over all head_dim dims, in place.
 * Replaces launch_rope_inplace (include/kernels.cuh:13). */
int qic_rope_inplace(int dtype, void* x, int num_heads, int head_dim, int position, float rope_theta,
                     qic_stream_t stream);

/* x[i] *= sigmoid(gate[i]). Replaces launch_sigmoid_mul_inplace (include/kernels.cuh:12). */
int qic_sigmoid_mul_inplace(int dtype, void* x, const void* gate, int n, qic_stream_t stream);

/* ------------------------------------------------------------------------- */
/* K/V append fused with k head-RMSNorm and RoPE.                            */
/* ------------------------------------------------------------------------- */

/* k_cache[slot] = RoPE(head_rmsnorm(k_new, k_norm_w)), v_cache[slot] = v_new, for all
 * num_kv_heads heads, where slot = page_table[position/page_size]*page_size +
 * position%page_size (paged) or slot = position (page_table == NULL). Byte-identical
 * to the reference chain launch_head_rmsnorm -> launch_rope_inplace -> cudaMemcpy
 * (src/model.cpp:634,637,639-641), written straight into the page that
 * launch_paged_attention reads for token `position` (src/kernels.cu:320-323).
 * Caches are [cache_tokens, num_kv_heads, head_dim]. */
int qic_kv_append(int dtype, const void* k_new, const void* v_new, const void* k_norm_w, float eps,
                  float rope_theta, int position, void* k_cache, void* v_cache, const int32_t* page_table,
                  int page_size, int64_t cache_tokens, int num_kv_heads, int head_dim, qic_stream_t stream);

/* ------------------------------------------------------------------------- */
/* Split-KV decode attention (contiguous = flash layout, or paged).          */
/* ------------------------------------------------------------------------- */

typedef struct qic_decode_args {
  int32_t dtype;            /* QIC_DTYPE_* */
  int32_t num_heads;        /* H query heads */
  int32_t num_kv_heads;     /* Hkv, H % Hkv == 0, group H/Hkv <= 8 */
  int32_t head_dim;         /* d in {64, 128, 256} */
  int32_t seq_len;          /* S tokens attended (position+1 when appending); 0 writes zeros */
  int32_t page_size;        /* tokens per page when page_table != NULL (multiple of 8) */
  int64_t cache_tokens;     /* token rows in k_cache / v_cache (bounds for loads and table entries) */
  const void* q;            /* [H, d] (raw projection when QIC_FUSE_Q_PROLOGUE) */
  void* k_cache;            /* [cache_tokens, Hkv, d], 16-byte aligned */
  void* v_cache;            /* [cache_tokens, Hkv, d], 16-byte aligned */
  const int32_t* page_table;/* [ceil(S/page_size)] physical page of each logical page; NULL = contiguous */
  const void* gate;         /* [H, d] output gate (out *= sigmoid(gate)) or NULL */
  void* out;                /* [H, d] */
  uint32_t flags;           /* QIC_FUSE_* */
  float eps;                /* head-RMSNorm epsilon (fused prologue / append) */
  float rope_theta;         /* RoPE base (fused prologue / append) */
  const void* q_norm_w;     /* [d] (QIC_FUSE_Q_PROLOGUE) */
  const void* k_norm_w;     /* [d] (QIC_FUSE_APPEND) */
  const void* k_new;        /* [Hkv, d] raw k projection (QIC_FUSE_APPEND) */
  const void* v_new;        /* [Hkv, d] v projection (QIC_FUSE_APPEND) */
  void* workspace;          /* scratch from the caller, zeroed once by qic_workspace_init */
  size_t workspace_bytes;
  int32_t num_splits;       /* KV splits per kv head; 0 = chosen from the SM count */
  int32_t cluster_size;     /* splits merged on chip per thread-block cluster (1..16, divides
                               num_splits); 0 = chosen with num_splits */
  int64_t position;         /* QIC_EXPLICIT_POSITION: RoPE position of q and the appended k */
  const int32_t* seq_len_dev; /* QIC_DEVICE_SEQ_LEN: device int32, the current seq_len */
} qic_decode_args;

/* Scratch bytes qic_decode_attention needs for this shape (any seq_len up to max_seq_len).
 * A workspace holds the status word, merge and stage-ticket counters, split partials
 * and (context parallel) the call epoch: calls that may run at the same time on the
 * GPU (different streams) need different workspaces; calls in stream order may share
 * one, whatever their shapes. Every call leaves the counters at zero. */
size_t qic_decode_workspace_bytes(int num_heads, int num_kv_heads, int head_dim, int max_seq_len);

/* Zeroes a workspace (counters and the device status word). Call once after allocating it. */
int qic_workspace_init(void* workspace, size_t bytes, qic_stream_t stream);

/* Reads and clears the device status word (QIC_DEV_* bits); synchronises `stream`. */
int qic_workspace_status(void* workspace, qic_stream_t stream, int* dev_status);

/* context[h,:] = sum_t softmax_t(q_h . K[t,h/g] / sqrt(d)) V[t,h/g] over t < seq_len,
 * optionally preceded by the fused q prologue and append and followed by the gate.
 * Replaces launch_flash_attention / launch_paged_attention (include/kernels.cuh:15-19)
 * and, with flags, the block src/model.cpp:633-652. */
int qic_decode_attention(const qic_decode_args* args, qic_stream_t stream);

/* The launch shape qic_decode_attention uses for these arguments: splits per kv head
 * and CTAs per thread-block cluster (its own choice when num_splits / cluster_size
 * are 0), or 0 and 0 when seq_len is 0 (nothing is launched). With QIC_DEVICE_SEQ_LEN
 * the shape follows seq_len, the bound. Reads the device's occupancy for the kernel;
 * touches no argument pointer and allocates nothing. */
int qic_decode_launch_shape(const qic_decode_args* args, int* num_splits, int* cluster_size);

/* Same computation as qic_decode_attention, for callers that cannot allocate device
 * memory: code written against the reference's kernels.cuh interface has no workspace
 * to pass, and a per-token decode loop (or a host that reserves all HBM for its own
 * page pool) must not call cudaMalloc, which synchronises the device. The split-KV
 * scratch is a 2 MiB array inside this library (qic_noalloc_scratch_bytes), held by
 * every GPU that loads it until the process exits; args->workspace and
 * args->workspace_bytes are ignored. The first call on a device (and again after a
 * cudaDeviceReset) looks up the array's address: make it before any stream capture.
 * Each call clears the array's merge counters; calls that overlap on the GPU share
 * the array and race. The array's device status word (QIC_DEV_* bits: bad page, bad
 * device length, timeout) accumulates over calls until qic_noalloc_status reads it.
 * Shapes whose partials do not fit return QIC_ERROR_WORKSPACE. No counterpart in the
 * reference: its kernels keep no scratch. Allocates nothing. */
int qic_decode_attention_noalloc(const qic_decode_args* args, qic_stream_t stream);

/* Size in bytes of the array qic_decode_attention_noalloc uses. */
size_t qic_noalloc_scratch_bytes(void);

/* Reads and clears the device status word of the current device's
 * qic_decode_attention_noalloc array (QIC_DEV_* bits of every call since the last
 * read); synchronises `stream`. No counterpart in the reference. */
int qic_noalloc_status(qic_stream_t stream, int* dev_status);

/* Floats per kv head of a QIC_PARTIAL_OUT partial: ((H/Hkv)*(d+1)+3) & ~3. */
size_t qic_partial_floats(int num_heads, int num_kv_heads, int head_dim);

/* out[h,:] = log-sum-exp merge of num_partials QIC_PARTIAL_OUT partials of one
 * sequence (stacked [num_partials][Hkv][qic_partial_floats]), each over a disjoint set
 * of tokens, then the optional gate (out *= sigmoid(gate)); out is [H, d] of dtype.
 * The partial/merge pair gives the all-gather form of context parallelism (partials
 * exchanged by a collective library); qic_cp_decode_attention fuses the exchange. */
int qic_attention_merge(int dtype, const float* partials, int num_partials, int num_heads, int num_kv_heads,
                        int head_dim, const void* gate, void* out, qic_stream_t stream);

/* ------------------------------------------------------------------------- */
/* Context parallelism: one sequence's K/V split across GPUs.                 */
/* No counterpart in the reference (single GPU); the shards' partials are      */
/* exchanged over NVLink inside the attention kernel and merged by log-sum-exp. */
/* ------------------------------------------------------------------------- */

#define QIC_MAX_RANKS 8
#define QIC_IPC_HANDLE_BYTES 64

typedef struct qic_cp_args {
  int32_t rank;             /* this GPU's shard, 0 <= rank < world */
  int32_t world;            /* shards of the sequence, 1..QIC_MAX_RANKS */
  void* exchange;           /* this rank's exchange buffer, qic_cp_exchange_bytes, zeroed before first use */
  size_t exchange_bytes;
  void* peer_exchange[QIC_MAX_RANKS]; /* every rank's exchange buffer as addressable from this process
                                         (peer memory opened with qic_ipc_open_handle);
                                         peer_exchange[rank] == exchange */
  int32_t timeout_ms;       /* bound of the device-side wait for the other ranks (0 = 2000 ms) */
  int32_t reserved;
} qic_cp_args;

/* Bytes of one rank's exchange buffer. */
size_t qic_cp_exchange_bytes(int num_heads, int num_kv_heads, int head_dim, int world);

/* Decode attention of one shard of a sequence, fused with the exchange: the rank's
 * (o, lse) partial of every (kv head, slice), merged over the rank's 8-CTA
 * clusters, is stored into every rank's exchange buffer over NVLink as 8-byte words
 * {value, call tag} (one store each: no fence or flag); the CTA that produced the
 * slice polls the words of every rank's contribution (bounded wait), merges them by
 * log-sum-exp and writes out (with the gate). Every rank calls it once per step
 * with the same shapes, cluster size (8) and number of calls; args->workspace is
 * required (it keeps the call epoch).
 * Shard layout: each rank's args describe its own tokens (seq_len, page_table or
 * contiguous rows); q is the same on every rank; QIC_EXPLICIT_POSITION gives the
 * global position for RoPE; the rank holding the last token sets QIC_FUSE_APPEND.
 * A peer that does not publish within timeout_ms sets QIC_DEV_PEER_TIMEOUT in the
 * device status word; the kernel then returns without writing out. */
int qic_cp_decode_attention(const qic_decode_args* args, const qic_cp_args* cp, qic_stream_t stream);

/* Device memory for exchange buffers: cudaMalloc'd and zeroed (an IPC handle must
 * name the start of an allocation). */
int qic_device_alloc(size_t bytes, void** ptr);
int qic_device_free(void* ptr);
/* CUDA IPC: handle (QIC_IPC_HANDLE_BYTES) of a qic_device_alloc buffer, and the
 * mapping of another process's buffer into this one (peer access enabled). */
int qic_ipc_get_handle(const void* ptr, void* handle);
int qic_ipc_open_handle(const void* handle, void** ptr);
int qic_ipc_close_handle(void* ptr);

/* ------------------------------------------------------------------------- */
/* Batched paged decode over one shared page pool.                            */
/* ------------------------------------------------------------------------- */

typedef struct qic_batch_decode_args {
  int32_t dtype;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t batch;              /* B sequences */
  int32_t page_size;          /* P, multiple of 8 */
  int64_t cache_tokens;       /* token rows in the shared pool */
  int32_t max_pages_per_seq;  /* row length of block_tables */
  uint32_t flags;             /* QIC_FUSE_*, QIC_PDL; the append goes to position seq_len-1 of each sequence */
  const void* q;              /* [B, H, d] */
  void* k_cache;              /* pool [cache_tokens, Hkv, d] */
  void* v_cache;
  const int32_t* block_tables;/* [B, max_pages_per_seq] */
  const void* gate;           /* [B, H, d] or NULL */
  void* out;                  /* [B, H, d] */
  float eps;
  float rope_theta;
  const void* q_norm_w;       /* [d] */
  const void* k_norm_w;       /* [d] */
  const void* k_new;          /* [B, Hkv, d] */
  const void* v_new;          /* [B, Hkv, d] */
  const void* plan;           /* device copy of the work items written by qic_batch_plan */
  int32_t plan_items;
  int32_t reserved;
  void* workspace;            /* >= the bytes qic_batch_plan reported, zeroed once by qic_workspace_init */
  size_t workspace_bytes;
} qic_batch_decode_args;

/* Bytes of one plan work item. */
#define QIC_PLAN_ITEM_BYTES 32

/* Host-side planner. seq_lens[b] (host memory) is the number of tokens sequence b
 * attends (position+1 when appending). Cuts every (sequence, kv head) into work items of
 * at most ~total/(target_ctas) pipeline stages, ordered longest first, and writes them to
 * `plan` (host memory, max_items * QIC_PLAN_ITEM_BYTES bytes). target_ctas 0 picks whole
 * waves of the CTAs the GPU holds at once, with about 1 MiB or more of K/V per item and
 * at most 16 items per SM. Returns the item count and the workspace size the plan needs. */
int qic_batch_plan(const int32_t* seq_lens, int batch, int num_heads, int num_kv_heads, int head_dim,
                   int target_ctas, void* plan, int max_items, int* items, size_t* workspace_bytes);

/* out[b] = decode attention of sequence b over its block-table row, for all b, in one
 * launch (with the fused prologue/append/gate options of qic_decode_attention).
 * Replaces one launch_paged_attention per sequence (include/kernels.cuh:17-19). */
int qic_batch_decode_attention(const qic_batch_decode_args* args, qic_stream_t stream);

/* ------------------------------------------------------------------------- */
/* Weight-streaming GEMV projections of one token, fused with the neighbouring */
/* RMSNorm, SwiGLU and residual add.                                           */
/* ------------------------------------------------------------------------- */

#define QIC_GEMV_MAX_SEGMENTS 4

/* Flags of qic_gemv_args.flags (QIC_PDL = 4 is accepted too: the kernel may start
 * while the previous kernel in the stream runs and load its first weight rows; x,
 * norm_w and the residuals are read after that kernel has completed). */
enum {
  QIC_GEMV_RMSNORM = 1,   /* x := T(x * rsqrt(mean(x^2) + eps) * norm_w) first (launch_rmsnorm) */
  QIC_GEMV_SWIGLU = 2,    /* two segments of equal out_dim, gate then up: seg[0].out = T(silu(gate) * up)
                             from the 16-bit gate and up (launch_swiglu); seg[1].out is not written */
  QIC_GEMV_RESIDUAL = 8   /* seg[k].out = T(T(product) + seg[k].residual) (launch_add_inplace);
                             residual may be the same buffer as out */
};

typedef struct qic_gemv_segment {
  const void* w;          /* [in_dim, out_dim], out_dim contiguous: element (i, o) at w[i*out_dim + o],
                             the reference's column-major weights (lda = out_dim); 16-byte aligned */
  void* out;              /* [out_dim] */
  const void* residual;   /* [out_dim] (QIC_GEMV_RESIDUAL) */
  int32_t out_dim;        /* multiple of 8 */
  int32_t reserved;
} qic_gemv_segment;

typedef struct qic_gemv_args {
  int32_t dtype;          /* QIC_DTYPE_*: x, weights, outputs */
  int32_t in_dim;         /* K, 1..131072 */
  int32_t num_segments;   /* projections of the same x in this launch, 1..QIC_GEMV_MAX_SEGMENTS */
  uint32_t flags;         /* QIC_GEMV_*, QIC_PDL */
  const void* x;          /* [in_dim]; must not overlap any out */
  const void* norm_w;     /* [in_dim] (QIC_GEMV_RMSNORM) */
  float eps;              /* RMSNorm epsilon */
  int32_t splits;         /* CTAs splitting the rows of a column tile (one cluster), 1..16; 0 = chosen */
  qic_gemv_segment seg[QIC_GEMV_MAX_SEGMENTS];
  void* status;           /* device int32 status word (QIC_DEV_TIMEOUT is OR-ed in when a bounded wait
                             for a weight copy gives up; the outputs are then not written), or NULL */
} qic_gemv_args;

/* seg[k].out[o] = T(sum_i x[i] * seg[k].w[i*out_dim + o]) with fp32 accumulation, for every
 * segment, in one launch, optionally with the input RMSNorm, the SwiGLU of a gate/up pair and
 * the residual add fused. Replaces QwenMiniModel::gemv (src/model.cpp:603-617: cublasGemmEx, one
 * column, fp32 compute) and, with the flags, launch_rmsnorm -> gemv of q, k and v (or of the
 * linear layer's qkv, z, b, a) (src/model.cpp:832, 627-631, 667-670), launch_rmsnorm -> gemv(w_gate),
 * gemv(w_up) -> launch_swiglu (src/model.cpp:800-804), gemv(w_down) -> launch_add_inplace
 * (src/model.cpp:805-806) and gemv(wo / out_proj) -> launch_add_inplace (src/model.cpp:653 or 794,
 * then 840), with the residual copies (src/model.cpp:799, 831) dropped. Deterministic: the same
 * inputs give the same bits on every call. Allocates nothing. */
int qic_gemv(const qic_gemv_args* args, qic_stream_t stream);

/* The split count qic_gemv uses for these arguments (its own choice when args->splits is 0). */
int qic_gemv_launch_shape(const qic_gemv_args* args, int* splits, int* tiles);

/* ------------------------------------------------------------------------- */
/* Qwen3.5 GatedDeltaNet decode step (state resident on the device).          */
/* ------------------------------------------------------------------------- */

typedef struct qic_gdn_args {
  int32_t dtype;            /* element type of the 16-bit inputs and of out */
  int32_t num_k_heads;      /* Hk */
  int32_t num_v_heads;      /* Hv, Hv % Hk == 0, Hv/Hk in {1, 2, 4} */
  int32_t k_head_dim;       /* dk == 128 */
  int32_t v_head_dim;       /* dv == 128 */
  int32_t conv_kernel;      /* K in [1, 8] */
  float eps;                /* gated RMSNorm epsilon */
  uint32_t flags;           /* QIC_PDL: may start while the previous kernel in the stream runs,
                               loading the weights (conv_w, dt_bias, a_log, norm_w, which no kernel
                               may write meanwhile) and prefetching the states into L2; the states
                               and qkv, z, b, a are read after that kernel has completed. The
                               kernel always lets the next kernel in the stream start early.
                               QIC_GDN_STATES_READY (with QIC_PDL): the states are read, not only
                               prefetched, before that point (see below). */
  const void* qkv;          /* [2*Hk*dk + Hv*dv] in_proj_qkv output (conv input) */
  const void* z;            /* [Hv*dv] */
  const void* b;            /* [Hv] */
  const void* a;            /* [Hv] */
  const void* conv_w;       /* [conv_dim, K] */
  const void* dt_bias;      /* [Hv] */
  const void* a_log;        /* [Hv] */
  const void* norm_w;       /* [dv] */
  float* conv_state;        /* [conv_dim, K] fp32, updated in place */
  float* recurrent_state;   /* [Hv, dk, dv] fp32, updated in place */
  void* out;                /* [Hv*dv] gated-norm output (input of out_proj) */
  int32_t* status;          /* optional device word (NULL: none): QIC_DEV_TIMEOUT is OR-ed in if a
                               CTA gives up waiting for its value head's peers (the output of that
                               head is then not written) */
} qic_gdn_args;

/* Flag of qic_gdn_args.flags. The caller guarantees that every kernel which wrote
 * conv_state or recurrent_state has completed before this launch starts, so with QIC_PDL
 * the kernel reads them before waiting for the previous kernel (only the step's inputs
 * qkv, z, b, a are read after it). This holds when a stream operation without
 * programmatic dependent launch lies between the states' last writer and this launch: a
 * copy, a kernel launched without QIC_PDL, or the boundary between two CUDA graph
 * launches (a layer stack captured as one graph per decode step, each layer's states
 * written once per step). It does not hold for two PDL launches of the same layer
 * back to back. */
#define QIC_GDN_STATES_READY 256u

/* One decode step of src/model.cpp:692-791 on the device: conv-state shift and causal
 * conv + SiLU, L2-norm of q/k, head repeat, beta/g gates, delta-rule state update and
 * read-out, gated RMSNorm. */
int qic_gated_delta_decode(const qic_gdn_args* args, qic_stream_t stream);

/* ------------------------------------------------------------------------- */
/* Decode-step runner: decode_next as one captured CUDA graph.                 */
/* ------------------------------------------------------------------------- */

/* The model's shape: the fields of QwenMiniConfig (include/model.hpp:10-28), in the
 * order of the qmini v4 header (src/model.cpp:345-366). layer_types[i]: 0 full
 * attention, 1 linear attention (GatedDeltaNet). */
typedef struct qic_model_config {
  int32_t vocab_size, hidden_size, intermediate_size, num_layers;
  int32_t num_heads, num_kv_heads, head_dim;
  int32_t linear_num_key_heads, linear_num_value_heads, linear_key_head_dim, linear_value_head_dim;
  int32_t linear_conv_kernel_dim;
  int32_t max_seq_len;
  float rms_norm_eps, rope_theta;
  const int32_t* layer_types;  /* [num_layers] */
} qic_model_config;

/* Device weights of one layer: QwenMiniModel::LayerWeights (include/model.hpp:55-79),
 * the same shapes and column-major [in][out] projection layout. */
typedef struct qic_layer_weights {
  int32_t is_linear;
  const void* attn_norm;
  const void *wq, *wk, *wv, *q_norm, *k_norm, *wo;  /* full attention (wq: [hidden, 2*H*d], q and gate) */
  const void *linear_in_qkv, *linear_in_z, *linear_in_b, *linear_in_a, *linear_conv1d_w, *linear_dt_bias,
      *linear_a_log, *linear_norm_w, *linear_out_proj;  /* linear attention */
  const void *ffn_norm, *w_gate, *w_up, *w_down;
} qic_layer_weights;

typedef struct qic_model_weights {
  const void* tok_embeddings;        /* [vocab, hidden] */
  const void* final_norm;            /* [hidden] */
  const void* lm_head;               /* [hidden, vocab] */
  const qic_layer_weights* layers;   /* [num_layers] */
} qic_model_weights;

typedef struct qic_model qic_model;

/* A runner over the caller's device weights (they must outlive it). Allocates the
 * K/V caches ([max_seq_len, kv_dim] per full-attention layer), the fp32 conv and
 * recurrent states, the runtime buffers and the attention workspace, runs one step,
 * captures the step as a CUDA graph and clears the caches and states. No counterpart
 * function in the reference: its QwenMiniModel is set up by load() (src/model.cpp:
 * 319-428) and alloc_runtime() (src/model.cpp:430-502). */
int qic_model_create(const qic_model_config* cfg, int dtype, const qic_model_weights* weights, qic_model** model);

/* A runner over the weights of a qmini v4 file (QwenMiniModel::load, src/model.cpp:
 * 319-428: the same header checks and tensor order), kept as 16-bit values on the
 * device (QIC_DTYPE_F16). max_seq_len 0 keeps the file's. */
int qic_model_load(const char* path, int max_seq_len, qic_model** model);

/* The runner's shape (layer_types not returned) and its file weight bytes (0 for qic_model_create). */
int qic_model_info(const qic_model* model, qic_model_config* cfg, size_t* weight_bytes);

/* Clears the K/V caches, the linear-attention states and the device status words (a new sequence). */
int qic_model_reset(qic_model* model);

/* One decode step at `position` (0-based; the caches hold positions 0..position-1):
 * QwenMiniModel::decode_next (src/model.cpp:823-845). Copies the token and length to
 * the device, replays the step's graph on `stream`, and returns the greedy token
 * (argmax_host, src/model.cpp:78-89: first index of the largest logit) in
 * *next_token and, when logits is not NULL, the vocab_size 16-bit logits (host
 * memory). Synchronises `stream`. QIC_ERROR_DEVICE_TIMEOUT / QIC_ERROR_BAD_PAGE report
 * a device-side status bit of this step. */
int qic_model_decode(qic_model* model, int token, int position, void* logits, int* next_token, qic_stream_t stream);

/* The two halves of qic_model_decode without the synchronisation, for callers that
 * time or chain steps: write the token and position (stream-ordered), then replay the
 * step's graph. The greedy token stays on the device. */
int qic_model_set_position(qic_model* model, int token, int position, qic_stream_t stream);
int qic_model_step_graph(qic_model* model, qic_stream_t stream);

/* Frees the runner (and the weights qic_model_load read); synchronises the device. */
int qic_model_free(qic_model* model);

#ifdef __cplusplus
}
#endif

#endif /* QIC_H_ */
