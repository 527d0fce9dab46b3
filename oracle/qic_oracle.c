/*
 * qic_oracle.c — TEST INFRASTRUCTURE ONLY. CPU restatement of the QweninCuda
 * decode-time KV-cache hot path, used as the checker by tests/, by
 * __graft_entry__.smoke() and by bench.py's CPU-baseline legs. Nothing in the
 * product library links or calls this file.
 *
 * Each function follows the reference's algorithm and operation order with fp32
 * arithmetic and 16-bit storage rounding (round-to-nearest-even), citing the file
 * and lines it restates (paths inside the QweninCuda project). The reference GPU
 * build uses --use_fast_math (CMakeLists.txt:9-14), whose hardware approximations
 * (rsqrt, pow, sin, cos, exp) this CPU code cannot reproduce, so CPU-vs-GPU
 * comparisons are tolerance checks; byte-exact checks are GPU-vs-GPU against the
 * reference kernels compiled by oracle/Makefile into oracle/_ref/.
 *
 * Parity pin: the reference ships no golden vectors or unit tests. This oracle is
 * pinned against outputs of the reference kernels themselves (tests/golden/, made
 * by tests/golden/make_golden.py from oracle/_ref on a B200).
 *
 * Storage: 16-bit tensors are passed as uint16_t bit patterns; dtype 0 = IEEE
 * binary16 (the reference's `half`), 1 = bfloat16.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------------------
 * 16-bit conversions (round to nearest, ties to even), written from the IEEE
 * 754 binary16 / bfloat16 definitions.
 * ------------------------------------------------------------------------- */
static float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

static float f16_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu;
  uint32_t m = h & 0x3ffu;
  uint32_t x;
  if (e == 0) {
    float v = ldexpf((float)m, -24);
    memcpy(&x, &v, 4);
    x |= sign;
  } else if (e == 31) {
    x = sign | 0x7f800000u | (m << 13);
  } else {
    x = sign | ((e - 15 + 127) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &x, 4);
  return f;
}

static uint16_t f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to inf */
  if (ax < 0x38800000u) {                                   /* below 2^-14: subnormal range */
    float av;
    memcpy(&av, &ax, 4);
    float q = nearbyintf(av * 16777216.0f); /* multiples of 2^-24, ties to even */
    return (uint16_t)(sign | (uint32_t)q);
  }
  uint32_t e = (ax >> 23) - 127 + 15;
  uint32_t mant = ax & 0x7fffffu;
  uint32_t h = (e << 10) | (mant >> 13);
  uint32_t rem = mant & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

static inline float ld(int dtype, uint16_t v) { return dtype ? bf16_to_f32(v) : f16_to_f32(v); }
static inline uint16_t st(int dtype, float v) { return dtype ? f32_to_bf16(v) : f32_to_f16(v); }

void qico_to_f32(int dtype, const uint16_t* src, float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = ld(dtype, src[i]);
}

void qico_from_f32(int dtype, const float* src, uint16_t* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = st(dtype, src[i]);
}

/* ---------------------------------------------------------------------------
 * head RMSNorm — src/kernels.cu:78-112 (head_rmsnorm_kernel). The reference sums
 * the squares with a shared-memory atomicAdd per thread; the oracle sums them in
 * ascending index order.
 * ------------------------------------------------------------------------- */
void qico_head_rmsnorm(int dtype, const uint16_t* x, const uint16_t* w, int num_heads, int head_dim, float eps,
                       uint16_t* out) {
  for (int h = 0; h < num_heads; ++h) {
    const uint16_t* xh = x + (int64_t)h * head_dim;
    uint16_t* oh = out + (int64_t)h * head_dim;
    float ssum = 0.0f;
    for (int i = 0; i < head_dim; ++i) {
      float v = ld(dtype, xh[i]);
      float sq = v * v;
      ssum = ssum + sq;
    }
    float inv_rms = 1.0f / sqrtf(ssum / (float)head_dim + eps);
    for (int i = 0; i < head_dim; ++i) {
      float xv = ld(dtype, xh[i]);
      float wv = ld(dtype, w[i]);
      oh[i] = st(dtype, xv * inv_rms * wv);
    }
  }
}

/* ---------------------------------------------------------------------------
 * rotate-half RoPE, in place — src/kernels.cu:150-183 (rope_inplace_kernel):
 * pairs (i, i + d/2), inv_freq = theta^(-2i/d), angle = position * inv_freq.
 * ------------------------------------------------------------------------- */
void qico_rope_inplace(int dtype, uint16_t* x, int num_heads, int head_dim, int position, float theta) {
  int half_dim = head_dim / 2;
  for (int h = 0; h < num_heads; ++h) {
    uint16_t* xh = x + (int64_t)h * head_dim;
    for (int d = 0; d < half_dim; ++d) {
      float x0 = ld(dtype, xh[d]);
      float x1 = ld(dtype, xh[d + half_dim]);
      float inv_freq = powf(theta, -2.0f * (float)d / (float)head_dim);
      float angle = (float)position * inv_freq;
      float c = cosf(angle);
      float s = sinf(angle);
      float y0 = x0 * c - x1 * s;
      float y1 = x1 * c + x0 * s;
      xh[d] = st(dtype, y0);
      xh[d + half_dim] = st(dtype, y1);
    }
  }
}

/* x *= sigmoid(gate) — src/kernels.cu:138-148 (sigmoid_mul_inplace_kernel). */
void qico_sigmoid_mul_inplace(int dtype, uint16_t* x, const uint16_t* gate, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    float g = ld(dtype, gate[i]);
    float sig = 1.0f / (1.0f + expf(-g));
    x[i] = st(dtype, ld(dtype, x[i]) * sig);
  }
}

/* Physical token row of logical token t — src/kernels.cu:320-323. */
static inline int64_t phys_token(const int32_t* page_table, int page_size, int64_t t) {
  if (!page_table) return t;
  return (int64_t)page_table[t / page_size] * page_size + (t % page_size);
}

/* ---------------------------------------------------------------------------
 * K/V append — src/model.cpp:634 (head_rmsnorm k), :637 (RoPE k), :639-641 (copy
 * into the cache). The slot is the one paged_attention reads for token
 * `position` (src/kernels.cu:320-323); with page_table == NULL it is the
 * reference's logical offset position*kv_dim (src/model.cpp:31-33).
 * ------------------------------------------------------------------------- */
void qico_kv_append(int dtype, const uint16_t* k_new, const uint16_t* v_new, const uint16_t* k_norm_w, float eps,
                    float theta, int position, uint16_t* k_cache, uint16_t* v_cache, const int32_t* page_table,
                    int page_size, int num_kv_heads, int head_dim) {
  int kv_dim = num_kv_heads * head_dim;
  uint16_t* k = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)kv_dim);
  qico_head_rmsnorm(dtype, k_new, k_norm_w, num_kv_heads, head_dim, eps, k);
  qico_rope_inplace(dtype, k, num_kv_heads, head_dim, position, theta);
  int64_t slot = phys_token(page_table, page_size, position);
  memcpy(k_cache + slot * kv_dim, k, sizeof(uint16_t) * (size_t)kv_dim);
  memcpy(v_cache + slot * kv_dim, v_new, sizeof(uint16_t) * (size_t)kv_dim);
  free(k);
}

/* ---------------------------------------------------------------------------
 * Decode attention — src/kernels.cu:200-290 (flash_attention_kernel) and
 * :292-374 (paged_attention_kernel): per query head h, kv head h/(H/Hkv), a
 * sequential online softmax over t in [0, seq_len): s = (q.k) * rsqrt(d),
 * new_m = max(m, s), alpha = exp(m-new_m), beta = exp(s-new_m), l = l*alpha+beta,
 * acc = acc*alpha + beta*v; out = acc * (1/max(l, 1e-12)). Parallel over heads.
 * ------------------------------------------------------------------------- */
static void attention_head(int dtype, const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                           const int32_t* page_table, int page_size, int num_heads, int num_kv_heads, int head_dim,
                           int seq_len, int h, uint16_t* context, float* acc, float* qf) {
  int group = num_heads / num_kv_heads;
  int kv_h = h / group;
  int64_t kv_dim = (int64_t)num_kv_heads * head_dim;
  for (int d = 0; d < head_dim; ++d) qf[d] = ld(dtype, q[(int64_t)h * head_dim + d]);
  for (int d = 0; d < head_dim; ++d) acc[d] = 0.0f;
  float m = -INFINITY, l = 0.0f;
  float inv_scale = 1.0f / sqrtf((float)head_dim);
  for (int64_t t = 0; t < seq_len; ++t) {
    int64_t pt = phys_token(page_table, page_size, t);
    const uint16_t* kh = k_cache + pt * kv_dim + (int64_t)kv_h * head_dim;
    const uint16_t* vh = v_cache + pt * kv_dim + (int64_t)kv_h * head_dim;
    float dot = 0.0f;
    for (int d = 0; d < head_dim; ++d) dot += qf[d] * ld(dtype, kh[d]);
    float s = dot * inv_scale;
    float new_m = fmaxf(m, s);
    float alpha = expf(m - new_m);
    float beta = expf(s - new_m);
    m = new_m;
    l = l * alpha + beta;
    for (int d = 0; d < head_dim; ++d) acc[d] = acc[d] * alpha + beta * ld(dtype, vh[d]);
  }
  float inv_l = 1.0f / fmaxf(l, 1e-12f);
  for (int d = 0; d < head_dim; ++d) context[(int64_t)h * head_dim + d] = st(dtype, acc[d] * inv_l);
}

void qico_attention(int dtype, const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                    const int32_t* page_table, int page_size, int num_heads, int num_kv_heads, int head_dim,
                    int seq_len, uint16_t* context) {
#pragma omp parallel for schedule(dynamic, 1)
  for (int h = 0; h < num_heads; ++h) {
    float* acc = (float*)malloc(sizeof(float) * (size_t)head_dim * 2);
    attention_head(dtype, q, k_cache, v_cache, page_table, page_size, num_heads, num_kv_heads, head_dim, seq_len,
                   h, context, acc, acc + head_dim);
    free(acc);
  }
}

/* Batched paged decode: one launch_paged_attention per sequence, each with its own
 * block-table row (the per-sequence check of the batched workload). */
void qico_batched_attention(int dtype, const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                            const int32_t* block_tables, int max_pages_per_seq, const int32_t* seq_lens, int batch,
                            int page_size, int num_heads, int num_kv_heads, int head_dim, uint16_t* out) {
  int64_t qstride = (int64_t)num_heads * head_dim;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int b = 0; b < batch; ++b) {
    for (int h = 0; h < num_heads; ++h) {
      float* acc = (float*)malloc(sizeof(float) * (size_t)head_dim * 2);
      attention_head(dtype, q + b * qstride, k_cache, v_cache, block_tables + (int64_t)b * max_pages_per_seq,
                     page_size, num_heads, num_kv_heads, head_dim, seq_lens[b], h, out + b * qstride, acc,
                     acc + head_dim);
      free(acc);
    }
  }
}

/* ---------------------------------------------------------------------------
 * GatedDeltaNet decode step — src/model.cpp:692-791 (host loop of
 * run_linear_attention_block), same loop order, fp32 state and std::exp /
 * std::log1p / std::sqrt arithmetic. Inputs are read as the reference reads its
 * 16-bit device buffers. Parallel over value heads for the state update.
 * ------------------------------------------------------------------------- */
static inline float silu(float x) { return x / (1.0f + expf(-x)); }

static void l2norm_inplace(float* x, int n) {
  float ss = 0.0f;
  for (int i = 0; i < n; ++i) ss += x[i] * x[i];
  float inv = 1.0f / sqrtf(ss + 1e-6f);
  for (int i = 0; i < n; ++i) x[i] *= inv;
}

void qico_gated_delta_decode(int dtype, int num_k_heads, int num_v_heads, int dk, int dv, int conv_kernel, float eps,
                             const uint16_t* qkv, const uint16_t* z, const uint16_t* b, const uint16_t* a,
                             const uint16_t* conv_w, const uint16_t* dt_bias, const uint16_t* a_log,
                             const uint16_t* norm_w, float* conv_state, float* recurrent_state, uint16_t* out) {
  const int key_dim = num_k_heads * dk;
  const int val_dim = num_v_heads * dv;
  const int conv_dim = key_dim * 2 + val_dim;
  const int K = conv_kernel;
  float* mixed = (float*)malloc(sizeof(float) * (size_t)conv_dim);
  /* model.cpp:692-708: shift the conv window, append the new input, conv + SiLU */
  for (int c = 0; c < conv_dim; ++c) {
    for (int t = 0; t < K - 1; ++t) conv_state[c * K + t] = conv_state[c * K + t + 1];
    conv_state[c * K + (K - 1)] = ld(dtype, qkv[c]);
    float acc = 0.0f;
    for (int t = 0; t < K; ++t) acc += ld(dtype, conv_w[c * K + t]) * conv_state[c * K + t];
    mixed[c] = silu(acc);
  }
  /* model.cpp:710-724: split q/k/v and L2-normalise each key head */
  float* q = mixed;
  float* k = mixed + key_dim;
  float* v = mixed + 2 * key_dim;
  for (int h = 0; h < num_k_heads; ++h) {
    l2norm_inplace(q + h * dk, dk);
    l2norm_inplace(k + h * dk, dk);
  }
  int repeat = num_v_heads / num_k_heads;
  float* o = (float*)malloc(sizeof(float) * (size_t)val_dim);
  /* model.cpp:726-775: repeat to value heads, gates, decay, delta rule, read-out */
#pragma omp parallel for schedule(static)
  for (int h = 0; h < num_v_heads; ++h) {
    int src_h = h / repeat;
    float* q_rep = (float*)malloc(sizeof(float) * (size_t)dk * 2);
    float* k_rep = q_rep + dk;
    float* kv_mem = (float*)malloc(sizeof(float) * (size_t)dv);
    for (int d = 0; d < dk; ++d) {
      q_rep[d] = q[src_h * dk + d] * (1.0f / sqrtf((float)dk));
      k_rep[d] = k[src_h * dk + d];
    }
    float beta = 1.0f / (1.0f + expf(-ld(dtype, b[h])));
    float av = ld(dtype, a[h]) + ld(dtype, dt_bias[h]);
    float softp = log1pf(expf(av));
    float g = expf(-expf(ld(dtype, a_log[h])) * softp);
    float* state = recurrent_state + (int64_t)h * dk * dv;
    for (int i = 0; i < dk; ++i)
      for (int j = 0; j < dv; ++j) state[i * dv + j] *= g;
    for (int j = 0; j < dv; ++j) {
      float m = 0.0f;
      for (int i = 0; i < dk; ++i) m += state[i * dv + j] * k_rep[i];
      kv_mem[j] = m;
    }
    for (int j = 0; j < dv; ++j) {
      float delta = (v[h * dv + j] - kv_mem[j]) * beta;
      for (int i = 0; i < dk; ++i) state[i * dv + j] += k_rep[i] * delta;
    }
    for (int j = 0; j < dv; ++j) {
      float y = 0.0f;
      for (int i = 0; i < dk; ++i) y += state[i * dv + j] * q_rep[i];
      o[h * dv + j] = y;
    }
    free(kv_mem);
    free(q_rep);
  }
  /* model.cpp:777-791: gated RMSNorm per value head */
  for (int h = 0; h < num_v_heads; ++h) {
    float ss = 0.0f;
    for (int j = 0; j < dv; ++j) ss += o[h * dv + j] * o[h * dv + j];
    float inv = 1.0f / sqrtf(ss / (float)dv + eps);
    for (int j = 0; j < dv; ++j) {
      float normed = o[h * dv + j] * inv;
      float gate = silu(ld(dtype, z[h * dv + j]));
      float ww = ld(dtype, norm_w[j]);
      out[h * dv + j] = st(dtype, normed * ww * gate);
    }
  }
  free(o);
  free(mixed);
}

int qico_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void qico_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
