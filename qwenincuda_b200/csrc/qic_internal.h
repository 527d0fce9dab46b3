// Host/device shared declarations of the qic library (not part of the public ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/qic.h"

namespace qic {

constexpr int kStageTokens = 32;     // tokens per TMA pipeline stage
constexpr int kConsumerWarps = 4;    // warps that run the mma pipeline
constexpr int kAttnThreads = (kConsumerWarps + 1) * 32;  // + one producer warp
constexpr int kMaxGroup = 8;         // query heads per kv head handled by one n8 mma tile
constexpr int kMaxSplits = 256;      // KV splits per kv head
constexpr uint64_t kDefaultTimeoutNs = 2000000000ull;  // 2 s bound on every device wait

// Workspace layout: [status int | pad to 256][counters int[Hkv*batch] | pad to 256][partials]
constexpr size_t kWsHeader = 256;

// One partial of a (kv head, split): lse[G] (log2 domain) then o[G][D] (normalised), fp32.
__host__ __device__ constexpr int partial_floats(int G, int D) { return ((G * (D + 1)) + 3) & ~3; }

struct AttnParams {
  CUtensorMap tm_k;                  // 2D map over [tokens, kv_dim], box {64, box_h}, 128B swizzle
  CUtensorMap tm_v;
  const void* q;                     // [H, D]
  const void* gate;                  // [H, D] or null
  void* out;                         // [H, D]
  void* k_cache;                     // generic pointers for the fused append
  void* v_cache;
  const int32_t* page_table;         // null = contiguous
  const void* q_norm_w;
  const void* k_norm_w;
  const void* k_new;
  const void* v_new;
  float* part;                       // [Hkv][n_splits][partial_floats]
  int* counters;                     // [Hkv]
  int* status;                       // device status word
  int64_t cache_tokens;
  int H, Hkv, G;
  int head_dim;                      // runtime copy of D (mirrors the reference's runtime arithmetic)
  int seq_len;
  int page_size;
  int box_h, log2_box_h;
  int n_stages, n_splits;
  int flags;
  float eps, theta, scale_log2;
  uint64_t timeout_ns;
};

// Launchers (attn_kernel.cu)
cudaError_t launch_decode_attention(int dtype, int head_dim, const AttnParams& p, cudaStream_t stream);
size_t decode_attention_smem_bytes(int head_dim);

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
