// Decode-step runner: the reference's QwenMiniModel::decode_next (src/model.cpp:823-845
// of the QweninCuda project) as one CUDA graph of this library's kernels, replayed for
// every token.
//
// Per token the graph runs the embedding row of the token, then per layer
//   full attention: RMSNorm + q/gate, k, v projections (one qic_gemv launch), the fused
//     attention (q head-norm + RoPE, k head-norm + RoPE + append, attention over the
//     cache, sigmoid gate; qic_decode_attention), o projection + residual (qic_gemv);
//   linear attention: RMSNorm + qkv, z, b, a projections (one qic_gemv), the
//     GatedDeltaNet step with device-resident states (qic_gated_delta_decode), out
//     projection + residual (qic_gemv);
//   FFN: RMSNorm + gate/up + SwiGLU (qic_gemv), down projection + residual (qic_gemv);
// then the final RMSNorm + lm_head (qic_gemv) and the greedy token (argmax). Every
// launch lets the next one start early (programmatic dependent launch). The token and
// the sequence length are read from device memory, so the graph captured once serves
// every position: compared with decode_next, the 2 residual copies per layer, the 8
// device-to-host and 1 host-to-device copies of every linear-attention layer
// (src/model.cpp:672-693, 793) and the per-call host work are gone.
//
// Weights: either the caller's device buffers (qic_model_create, the layout of the
// reference's LayerWeights, include/model.hpp:55-79) or read from a qmini v4 file
// (qic_model_load, the format of QwenMiniModel::load, src/model.cpp:319-428).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <memory>
#include <string>
#include <vector>

#include "qic_internal.h"

namespace qic {
cudaError_t launch_embed(int dtype, const void* table, int vocab, int hidden, const int32_t* token, void* out,
                         cudaStream_t stream);
cudaError_t launch_argmax(int dtype, const void* x, int n, int32_t* out, cudaStream_t stream);
}  // namespace qic

struct qic_model {
  qic_model_config cfg = {};
  int dtype = QIC_DTYPE_F16;
  std::vector<qic_layer_weights> layers;
  const void* tok_embeddings = nullptr;
  const void* final_norm = nullptr;
  const void* lm_head = nullptr;
  std::vector<void*> owned;  // device buffers this model frees (weights read from a file, runtime buffers)
  // runtime buffers
  void* x = nullptr;        // [hidden] residual stream
  void* qg = nullptr;       // [2 * q_dim] packed q / gate projection
  void* k = nullptr;        // [kv_dim]
  void* v = nullptr;
  void* ctx = nullptr;      // [q_dim] attention output (gated)
  void* lqkv = nullptr;     // [conv_dim]
  void* lz = nullptr;       // [val_dim]
  void* lb = nullptr;       // [Hv]
  void* la = nullptr;
  void* lout = nullptr;     // [val_dim]
  void* hidden_ffn = nullptr;  // [inter]
  void* logits = nullptr;   // [vocab]
  void* ws = nullptr;       // attention workspace
  size_t ws_bytes = 0;
  int32_t* dev_scalars = nullptr;  // [0] token, [1] sequence length, [2] greedy token, [3] GEMV / GatedDeltaNet status
  int32_t* host_scalars = nullptr; // pinned: dev_scalars[0..3], then the attention workspace's status word
  std::vector<void*> k_cache, v_cache;               // per layer ([max_seq_len, kv_dim]) or null
  std::vector<float*> conv_state, recurrent_state;   // per layer or null
  cudaStream_t capture_stream = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  size_t weight_bytes = 0;
};

namespace {

int cuda_fail(cudaError_t e) { return e == cudaSuccess ? QIC_SUCCESS : QIC_ERROR_CUDA; }

size_t elem(int dtype) { return 2; }

struct Dims {
  size_t hidden, inter, vocab, q_dim, kv_dim, key_dim, val_dim, conv_dim;
};

Dims dims_of(const qic_model_config& c) {
  Dims d;
  d.hidden = static_cast<size_t>(c.hidden_size);
  d.inter = static_cast<size_t>(c.intermediate_size);
  d.vocab = static_cast<size_t>(c.vocab_size);
  d.q_dim = static_cast<size_t>(c.num_heads) * c.head_dim;
  d.kv_dim = static_cast<size_t>(c.num_kv_heads) * c.head_dim;
  d.key_dim = static_cast<size_t>(c.linear_num_key_heads) * c.linear_key_head_dim;
  d.val_dim = static_cast<size_t>(c.linear_num_value_heads) * c.linear_value_head_dim;
  d.conv_dim = 2 * d.key_dim + d.val_dim;
  return d;
}

// The shapes this library's kernels take; mirrors validate_qwen35_config
// (src/model.cpp:58-76) plus the kernels' own limits.
int check_config(const qic_model_config& c) {
  if (c.vocab_size <= 0 || c.hidden_size <= 0 || c.intermediate_size <= 0 || c.num_layers <= 0 ||
      c.max_seq_len <= 0 || c.max_seq_len > QIC_MAX_SEQ_LEN || c.layer_types == nullptr)
    return QIC_ERROR_INVALID_VALUE;
  bool any_full = false, any_linear = false;
  for (int i = 0; i < c.num_layers; ++i) {
    if (c.layer_types[i] != 0 && c.layer_types[i] != 1) return QIC_ERROR_INVALID_VALUE;
    (c.layer_types[i] == 0 ? any_full : any_linear) = true;
  }
  const Dims d = dims_of(c);
  if (d.hidden % 8 || d.inter % 8 || d.vocab % 8) return QIC_ERROR_NOT_SUPPORTED;
  if (any_full) {
    if (c.num_heads <= 0 || c.num_kv_heads <= 0 || c.num_heads % c.num_kv_heads) return QIC_ERROR_INVALID_VALUE;
    if ((c.head_dim != 64 && c.head_dim != 128 && c.head_dim != 256) || c.num_heads / c.num_kv_heads > 8)
      return QIC_ERROR_NOT_SUPPORTED;
  }
  if (any_linear) {
    if (c.linear_num_key_heads <= 0 || c.linear_num_value_heads <= 0 ||
        c.linear_num_value_heads % c.linear_num_key_heads || c.linear_conv_kernel_dim <= 0)
      return QIC_ERROR_INVALID_VALUE;
    const int rep = c.linear_num_value_heads / c.linear_num_key_heads;
    if (c.linear_key_head_dim != 128 || c.linear_value_head_dim != 128 || (rep != 1 && rep != 2 && rep != 4) ||
        c.linear_conv_kernel_dim > 8 || c.linear_num_value_heads % 8)
      return QIC_ERROR_NOT_SUPPORTED;
  }
  return QIC_SUCCESS;
}

int alloc(qic_model* m, size_t bytes, void** p) {
  *p = nullptr;
  if (cudaMalloc(p, std::max<size_t>(bytes, 16)) != cudaSuccess) return QIC_ERROR_CUDA;
  m->owned.push_back(*p);
  if (cudaMemset(*p, 0, std::max<size_t>(bytes, 16)) != cudaSuccess) return QIC_ERROR_CUDA;
  return QIC_SUCCESS;
}

int check(int rc, bool& ok) {
  if (rc != QIC_SUCCESS) ok = false;
  return rc;
}

// The decode step's launches on `s` (captured into the graph).
int record_step(qic_model* m, cudaStream_t s) {
  const qic_model_config& c = m->cfg;
  const Dims d = dims_of(c);
  const qic_stream_t st = reinterpret_cast<qic_stream_t>(s);
  int rc = qic::launch_embed(m->dtype, m->tok_embeddings, c.vocab_size, c.hidden_size, m->dev_scalars, m->x, s) ==
                   cudaSuccess
               ? QIC_SUCCESS
               : QIC_ERROR_CUDA;
  if (rc != QIC_SUCCESS) return rc;
  int32_t* gemv_status = m->dev_scalars + 3;
  auto gemv = [&](const void* x, int in_dim, uint32_t flags, const void* norm_w,
                  std::initializer_list<qic_gemv_segment> segs) {
    qic_gemv_args g = {};
    g.dtype = m->dtype;
    g.in_dim = in_dim;
    g.x = x;
    g.flags = flags | QIC_PDL;
    g.norm_w = norm_w;
    g.eps = c.rms_norm_eps;
    g.num_segments = static_cast<int32_t>(segs.size());
    int k = 0;
    for (const qic_gemv_segment& sg : segs) g.seg[k++] = sg;
    g.status = gemv_status;
    return qic_gemv(&g, st);
  };
  for (int i = 0; i < c.num_layers && rc == QIC_SUCCESS; ++i) {
    const qic_layer_weights& w = m->layers[i];
    if (c.layer_types[i] == 0) {
      rc = gemv(m->x, c.hidden_size, QIC_GEMV_RMSNORM, w.attn_norm,
                {{w.wq, m->qg, nullptr, static_cast<int32_t>(2 * d.q_dim), 0},
                 {w.wk, m->k, nullptr, static_cast<int32_t>(d.kv_dim), 0},
                 {w.wv, m->v, nullptr, static_cast<int32_t>(d.kv_dim), 0}});
      if (rc != QIC_SUCCESS) break;
      qic_decode_args a = {};
      a.dtype = m->dtype;
      a.num_heads = c.num_heads;
      a.num_kv_heads = c.num_kv_heads;
      a.head_dim = c.head_dim;
      a.seq_len = c.max_seq_len;  // the bound; the current length is read from device memory
      a.seq_len_dev = m->dev_scalars + 1;
      a.cache_tokens = c.max_seq_len;
      a.q = m->qg;
      a.k_cache = m->k_cache[i];
      a.v_cache = m->v_cache[i];
      a.out = m->ctx;
      a.flags = QIC_FUSE_Q_PROLOGUE | QIC_FUSE_APPEND | QIC_Q_GATE_INTERLEAVED | QIC_PDL | QIC_DEVICE_SEQ_LEN;
      a.eps = c.rms_norm_eps;
      a.rope_theta = c.rope_theta;
      a.q_norm_w = w.q_norm;
      a.k_norm_w = w.k_norm;
      a.k_new = m->k;
      a.v_new = m->v;
      a.workspace = m->ws;
      a.workspace_bytes = m->ws_bytes;
      rc = qic_decode_attention(&a, st);
      if (rc != QIC_SUCCESS) break;
      rc = gemv(m->ctx, static_cast<int>(d.q_dim), QIC_GEMV_RESIDUAL, nullptr,
                {{w.wo, m->x, m->x, c.hidden_size, 0}});
    } else {
      const int Hv = c.linear_num_value_heads;
      rc = gemv(m->x, c.hidden_size, QIC_GEMV_RMSNORM, w.attn_norm,
                {{w.linear_in_qkv, m->lqkv, nullptr, static_cast<int32_t>(d.conv_dim), 0},
                 {w.linear_in_z, m->lz, nullptr, static_cast<int32_t>(d.val_dim), 0},
                 {w.linear_in_b, m->lb, nullptr, Hv, 0},
                 {w.linear_in_a, m->la, nullptr, Hv, 0}});
      if (rc != QIC_SUCCESS) break;
      qic_gdn_args g = {};
      g.dtype = m->dtype;
      g.num_k_heads = c.linear_num_key_heads;
      g.num_v_heads = Hv;
      g.k_head_dim = c.linear_key_head_dim;
      g.v_head_dim = c.linear_value_head_dim;
      g.conv_kernel = c.linear_conv_kernel_dim;
      g.eps = c.rms_norm_eps;
      // each layer's states are written once per step and every step is its own graph
      // launch (or the eager first step after the states were cleared), so their writer
      // has completed before this launch starts
      g.flags = QIC_PDL | QIC_GDN_STATES_READY;
      g.qkv = m->lqkv;
      g.z = m->lz;
      g.b = m->lb;
      g.a = m->la;
      g.conv_w = w.linear_conv1d_w;
      g.dt_bias = w.linear_dt_bias;
      g.a_log = w.linear_a_log;
      g.norm_w = w.linear_norm_w;
      g.conv_state = m->conv_state[i];
      g.recurrent_state = m->recurrent_state[i];
      g.out = m->lout;
      g.status = gemv_status;  // a bounded wait's timeout, reported like the GEMV's
      rc = qic_gated_delta_decode(&g, st);
      if (rc != QIC_SUCCESS) break;
      rc = gemv(m->lout, static_cast<int>(d.val_dim), QIC_GEMV_RESIDUAL, nullptr,
                {{w.linear_out_proj, m->x, m->x, c.hidden_size, 0}});
    }
    if (rc != QIC_SUCCESS) break;
    rc = gemv(m->x, c.hidden_size, QIC_GEMV_RMSNORM | QIC_GEMV_SWIGLU, w.ffn_norm,
              {{w.w_gate, m->hidden_ffn, nullptr, c.intermediate_size, 0},
               {w.w_up, nullptr, nullptr, c.intermediate_size, 0}});
    if (rc != QIC_SUCCESS) break;
    rc = gemv(m->hidden_ffn, c.intermediate_size, QIC_GEMV_RESIDUAL, nullptr,
              {{w.w_down, m->x, m->x, c.hidden_size, 0}});
  }
  if (rc != QIC_SUCCESS) return rc;
  rc = gemv(m->x, c.hidden_size, QIC_GEMV_RMSNORM, m->final_norm, {{m->lm_head, m->logits, nullptr, c.vocab_size, 0}});
  if (rc != QIC_SUCCESS) return rc;
  return qic::launch_argmax(m->dtype, m->logits, c.vocab_size, m->dev_scalars + 2, s) == cudaSuccess ? QIC_SUCCESS
                                                                                                       : QIC_ERROR_CUDA;
}

// Runtime buffers, caches and states; the graph.
int finish(qic_model* m) {
  const qic_model_config& c = m->cfg;
  const Dims d = dims_of(c);
  const size_t e = elem(m->dtype);
  int rc = QIC_SUCCESS;
  bool ok = true;
  check(alloc(m, d.hidden * e, &m->x), ok);
  check(alloc(m, std::max<size_t>(2 * d.q_dim, 8) * e, &m->qg), ok);
  check(alloc(m, std::max<size_t>(d.kv_dim, 8) * e, &m->k), ok);
  check(alloc(m, std::max<size_t>(d.kv_dim, 8) * e, &m->v), ok);
  check(alloc(m, std::max<size_t>(d.q_dim, 8) * e, &m->ctx), ok);
  check(alloc(m, std::max<size_t>(d.conv_dim, 8) * e, &m->lqkv), ok);
  check(alloc(m, std::max<size_t>(d.val_dim, 8) * e, &m->lz), ok);
  check(alloc(m, std::max<int>(c.linear_num_value_heads, 8) * e, &m->lb), ok);
  check(alloc(m, std::max<int>(c.linear_num_value_heads, 8) * e, &m->la), ok);
  check(alloc(m, std::max<size_t>(d.val_dim, 8) * e, &m->lout), ok);
  check(alloc(m, d.inter * e, &m->hidden_ffn), ok);
  check(alloc(m, d.vocab * e, &m->logits), ok);
  void* sc = nullptr;
  check(alloc(m, 4 * sizeof(int32_t), &sc), ok);
  m->dev_scalars = static_cast<int32_t*>(sc);
  if (!ok) return QIC_ERROR_CUDA;
  if (cudaMallocHost(reinterpret_cast<void**>(&m->host_scalars), 5 * sizeof(int32_t)) != cudaSuccess)
    return QIC_ERROR_CUDA;
  m->k_cache.assign(c.num_layers, nullptr);
  m->v_cache.assign(c.num_layers, nullptr);
  m->conv_state.assign(c.num_layers, nullptr);
  m->recurrent_state.assign(c.num_layers, nullptr);
  bool any_full = false;
  for (int i = 0; i < c.num_layers; ++i) {
    if (c.layer_types[i] == 0) {
      any_full = true;
      check(alloc(m, static_cast<size_t>(c.max_seq_len) * d.kv_dim * e, &m->k_cache[i]), ok);
      check(alloc(m, static_cast<size_t>(c.max_seq_len) * d.kv_dim * e, &m->v_cache[i]), ok);
    } else {
      void* cs = nullptr;
      void* rs = nullptr;
      check(alloc(m, d.conv_dim * c.linear_conv_kernel_dim * sizeof(float), &cs), ok);
      check(alloc(m, static_cast<size_t>(c.linear_num_value_heads) * c.linear_key_head_dim * c.linear_value_head_dim *
                         sizeof(float),
                  &rs),
            ok);
      m->conv_state[i] = static_cast<float*>(cs);
      m->recurrent_state[i] = static_cast<float*>(rs);
    }
  }
  if (any_full) {
    m->ws_bytes = qic_decode_workspace_bytes(c.num_heads, c.num_kv_heads, c.head_dim, c.max_seq_len);
    check(alloc(m, m->ws_bytes, &m->ws), ok);
  }
  if (!ok) return QIC_ERROR_CUDA;
  if (cudaStreamCreateWithFlags(&m->capture_stream, cudaStreamNonBlocking) != cudaSuccess) return QIC_ERROR_CUDA;
  // one eager step first (per-device kernel set-up happens outside the capture), then
  // the capture; the caches and states the eager step touched are cleared after
  m->host_scalars[0] = 0;
  m->host_scalars[1] = 1;
  if (cudaMemcpyAsync(m->dev_scalars, m->host_scalars, 2 * sizeof(int32_t), cudaMemcpyHostToDevice,
                      m->capture_stream) != cudaSuccess)
    return QIC_ERROR_CUDA;
  rc = record_step(m, m->capture_stream);
  if (rc != QIC_SUCCESS) return rc;
  if (cudaStreamSynchronize(m->capture_stream) != cudaSuccess) return QIC_ERROR_CUDA;
  if (cudaStreamBeginCapture(m->capture_stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
    return QIC_ERROR_CUDA;
  rc = record_step(m, m->capture_stream);
  cudaGraph_t g = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(m->capture_stream, &g);
  if (rc != QIC_SUCCESS) {
    if (g != nullptr) cudaGraphDestroy(g);
    return rc;
  }
  if (ce != cudaSuccess) return QIC_ERROR_CUDA;
  m->graph = g;
  if (cudaGraphInstantiate(&m->exec, g, 0) != cudaSuccess) return QIC_ERROR_CUDA;
  return qic_model_reset(m);
}

template <typename X>
bool read_raw(std::ifstream& in, X* v, size_t n = 1) {
  in.read(reinterpret_cast<char*>(v), static_cast<std::streamsize>(n * sizeof(X)));
  return static_cast<bool>(in);
}

// One tensor of the file: uint64 element count, then that many 16-bit values.
int read_tensor(std::ifstream& in, qic_model* m, size_t expected, const void** out) {
  uint64_t n = 0;
  if (!read_raw(in, &n) || n != expected) return QIC_ERROR_INVALID_VALUE;
  std::vector<uint16_t> host(n);
  if (!read_raw(in, host.data(), n)) return QIC_ERROR_INVALID_VALUE;
  void* dev = nullptr;
  if (cudaMalloc(&dev, std::max<size_t>(n * 2, 16)) != cudaSuccess) return QIC_ERROR_CUDA;
  m->owned.push_back(dev);
  if (cudaMemcpy(dev, host.data(), n * 2, cudaMemcpyHostToDevice) != cudaSuccess) return QIC_ERROR_CUDA;
  m->weight_bytes += n * 2;
  *out = dev;
  return QIC_SUCCESS;
}

}  // namespace

extern "C" {

int qic_model_create(const qic_model_config* cfg, int dtype, const qic_model_weights* w, qic_model** out) {
  if (cfg == nullptr || w == nullptr || out == nullptr || (dtype != QIC_DTYPE_F16 && dtype != QIC_DTYPE_BF16) ||
      w->layers == nullptr || w->tok_embeddings == nullptr || w->final_norm == nullptr || w->lm_head == nullptr)
    return QIC_ERROR_INVALID_VALUE;
  *out = nullptr;
  int rc = check_config(*cfg);
  if (rc != QIC_SUCCESS) return rc;
  std::unique_ptr<qic_model> m(new qic_model());
  m->cfg = *cfg;
  // the layer kinds are kept by the model (the caller's array may go away)
  auto* types = new int32_t[cfg->num_layers];
  std::memcpy(types, cfg->layer_types, sizeof(int32_t) * cfg->num_layers);
  m->cfg.layer_types = types;
  m->dtype = dtype;
  m->tok_embeddings = w->tok_embeddings;
  m->final_norm = w->final_norm;
  m->lm_head = w->lm_head;
  m->layers.assign(w->layers, w->layers + cfg->num_layers);
  rc = finish(m.get());
  if (rc != QIC_SUCCESS) {
    qic_model_free(m.release());
    return rc;
  }
  *out = m.release();
  return QIC_SUCCESS;
}

int qic_model_load(const char* path, int max_seq_len, qic_model** out) {
  if (path == nullptr || out == nullptr || max_seq_len < 0 || max_seq_len > QIC_MAX_SEQ_LEN)
    return QIC_ERROR_INVALID_VALUE;
  *out = nullptr;
  std::ifstream in(path, std::ios::binary);
  if (!in) return QIC_ERROR_INVALID_VALUE;
  char magic[8] = {};
  int32_t version = 0;
  if (!read_raw(in, magic, 8) || std::memcmp(magic, "QWENMINI", 8) != 0 || !read_raw(in, &version) ||
      version != 4)
    return QIC_ERROR_INVALID_VALUE;
  // header: src/model.cpp:345-366 (int32 fields in this order, then eps and theta as
  // float, then one int32 layer kind per layer)
  qic_model_config c = {};
  int32_t f[13];
  if (!read_raw(in, f, 13) || !read_raw(in, &c.rms_norm_eps) || !read_raw(in, &c.rope_theta))
    return QIC_ERROR_INVALID_VALUE;
  c.vocab_size = f[0];
  c.hidden_size = f[1];
  c.intermediate_size = f[2];
  c.num_layers = f[3];
  c.num_heads = f[4];
  c.num_kv_heads = f[5];
  c.head_dim = f[6];
  c.linear_num_key_heads = f[7];
  c.linear_num_value_heads = f[8];
  c.linear_key_head_dim = f[9];
  c.linear_value_head_dim = f[10];
  c.linear_conv_kernel_dim = f[11];
  c.max_seq_len = max_seq_len > 0 ? max_seq_len : f[12];
  if (c.num_layers <= 0 || c.num_layers > 4096) return QIC_ERROR_INVALID_VALUE;
  std::vector<int32_t> types(c.num_layers);
  if (!read_raw(in, types.data(), types.size())) return QIC_ERROR_INVALID_VALUE;
  c.layer_types = types.data();
  int rc = check_config(c);
  if (rc != QIC_SUCCESS) return rc;
  std::unique_ptr<qic_model> m(new qic_model());
  m->cfg = c;
  auto* kinds = new int32_t[c.num_layers];  // the model's own copy, freed with it
  std::memcpy(kinds, types.data(), sizeof(int32_t) * c.num_layers);
  m->cfg.layer_types = kinds;
  m->dtype = QIC_DTYPE_F16;  // the format's element type (the reference's half)
  const Dims d = dims_of(c);
  auto fail = [&](int code) {
    qic_model_free(m.release());
    return code;
  };
  // tensors: src/model.cpp:383-421
  if ((rc = read_tensor(in, m.get(), d.vocab * d.hidden, &m->tok_embeddings)) != QIC_SUCCESS) return fail(rc);
  m->layers.assign(c.num_layers, qic_layer_weights{});
  for (int i = 0; i < c.num_layers && rc == QIC_SUCCESS; ++i) {
    qic_layer_weights& l = m->layers[i];
    l.is_linear = types[i] == 1;
    rc = read_tensor(in, m.get(), d.hidden, &l.attn_norm);
    if (rc == QIC_SUCCESS && l.is_linear) {
      const size_t Hv = static_cast<size_t>(c.linear_num_value_heads);
      if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), d.hidden * d.conv_dim, &l.linear_in_qkv);
      if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), d.hidden * d.val_dim, &l.linear_in_z);
      if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), d.hidden * Hv, &l.linear_in_b);
      if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), d.hidden * Hv, &l.linear_in_a);
      if (rc == QIC_SUCCESS)
        rc = read_tensor(in, m.get(), d.conv_dim * c.linear_conv_kernel_dim, &l.linear_conv1d_w);
      if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), Hv, &l.linear_dt_bias);
      if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), Hv, &l.linear_a_log);
      if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), c.linear_value_head_dim, &l.linear_norm_w);
      if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), d.val_dim * d.hidden, &l.linear_out_proj);
    } else if (rc == QIC_SUCCESS) {
      if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), d.hidden * 2 * d.q_dim, &l.wq);
      if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), d.hidden * d.kv_dim, &l.wk);
      if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), d.hidden * d.kv_dim, &l.wv);
      if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), c.head_dim, &l.q_norm);
      if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), c.head_dim, &l.k_norm);
      if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), d.q_dim * d.hidden, &l.wo);
    }
    if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), d.hidden, &l.ffn_norm);
    if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), d.hidden * d.inter, &l.w_gate);
    if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), d.hidden * d.inter, &l.w_up);
    if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), d.inter * d.hidden, &l.w_down);
  }
  if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), d.hidden, &m->final_norm);
  if (rc == QIC_SUCCESS) rc = read_tensor(in, m.get(), d.hidden * d.vocab, &m->lm_head);
  if (rc != QIC_SUCCESS) return fail(rc);
  rc = finish(m.get());
  if (rc != QIC_SUCCESS) return fail(rc);
  *out = m.release();
  return QIC_SUCCESS;
}

int qic_model_info(const qic_model* m, qic_model_config* cfg, size_t* weight_bytes) {
  if (m == nullptr) return QIC_ERROR_INVALID_VALUE;
  if (cfg != nullptr) {
    *cfg = m->cfg;
    cfg->layer_types = nullptr;  // the model's own array stays private
  }
  if (weight_bytes != nullptr) *weight_bytes = m->weight_bytes;
  return QIC_SUCCESS;
}

int qic_model_reset(qic_model* m) {
  if (m == nullptr) return QIC_ERROR_INVALID_VALUE;
  const Dims d = dims_of(m->cfg);
  cudaStream_t s = m->capture_stream;
  for (int i = 0; i < m->cfg.num_layers; ++i) {
    if (m->k_cache[i] != nullptr) {
      const size_t bytes = static_cast<size_t>(m->cfg.max_seq_len) * d.kv_dim * 2;
      if (cudaMemsetAsync(m->k_cache[i], 0, bytes, s) != cudaSuccess ||
          cudaMemsetAsync(m->v_cache[i], 0, bytes, s) != cudaSuccess)
        return QIC_ERROR_CUDA;
    }
    if (m->conv_state[i] != nullptr) {
      if (cudaMemsetAsync(m->conv_state[i], 0, d.conv_dim * m->cfg.linear_conv_kernel_dim * sizeof(float), s) !=
              cudaSuccess ||
          cudaMemsetAsync(m->recurrent_state[i], 0,
                          static_cast<size_t>(m->cfg.linear_num_value_heads) * m->cfg.linear_key_head_dim *
                              m->cfg.linear_value_head_dim * sizeof(float),
                          s) != cudaSuccess)
        return QIC_ERROR_CUDA;
    }
  }
  if (m->ws != nullptr && cudaMemsetAsync(m->ws, 0, m->ws_bytes, s) != cudaSuccess) return QIC_ERROR_CUDA;
  if (cudaMemsetAsync(m->dev_scalars, 0, 4 * sizeof(int32_t), s) != cudaSuccess) return QIC_ERROR_CUDA;
  return cuda_fail(cudaStreamSynchronize(s));
}

int qic_model_decode(qic_model* m, int token, int position, void* logits, int* next_token, qic_stream_t stream) {
  if (m == nullptr || m->exec == nullptr || position < 0 || position >= m->cfg.max_seq_len)
    return QIC_ERROR_INVALID_VALUE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  m->host_scalars[0] = token;
  m->host_scalars[1] = position + 1;
  cudaError_t e = cudaMemcpyAsync(m->dev_scalars, m->host_scalars, 2 * sizeof(int32_t), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaGraphLaunch(m->exec, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(m->host_scalars + 2, m->dev_scalars + 2, 2 * sizeof(int32_t), cudaMemcpyDeviceToHost, s);
  m->host_scalars[4] = 0;
  if (e == cudaSuccess && m->ws != nullptr)
    e = cudaMemcpyAsync(m->host_scalars + 4, m->ws, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess && logits != nullptr)
    e = cudaMemcpyAsync(logits, m->logits, static_cast<size_t>(m->cfg.vocab_size) * 2, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return QIC_ERROR_CUDA;
  const int gemv_status = m->host_scalars[3], attn_status = m->host_scalars[4];
  if (gemv_status != 0 || attn_status != 0) {
    // report once: the words are cleared for the next step
    if (cudaMemsetAsync(m->dev_scalars + 3, 0, sizeof(int32_t), s) != cudaSuccess ||
        (m->ws != nullptr && cudaMemsetAsync(m->ws, 0, sizeof(int32_t), s) != cudaSuccess) ||
        cudaStreamSynchronize(s) != cudaSuccess)
      return QIC_ERROR_CUDA;
    if (gemv_status != 0 || (attn_status & (QIC_DEV_TIMEOUT | QIC_DEV_PEER_TIMEOUT)))
      return QIC_ERROR_DEVICE_TIMEOUT;
    return QIC_ERROR_BAD_PAGE;  // a bad page entry or device length, clamped by the kernel
  }
  if (next_token != nullptr) *next_token = m->host_scalars[2];
  return QIC_SUCCESS;
}

int qic_model_step_graph(qic_model* m, qic_stream_t stream) {
  if (m == nullptr || m->exec == nullptr) return QIC_ERROR_INVALID_VALUE;
  return cuda_fail(cudaGraphLaunch(m->exec, reinterpret_cast<cudaStream_t>(stream)));
}

int qic_model_set_position(qic_model* m, int token, int position, qic_stream_t stream) {
  if (m == nullptr || position < 0 || position >= m->cfg.max_seq_len) return QIC_ERROR_INVALID_VALUE;
  m->host_scalars[0] = token;
  m->host_scalars[1] = position + 1;
  return cuda_fail(cudaMemcpyAsync(m->dev_scalars, m->host_scalars, 2 * sizeof(int32_t), cudaMemcpyHostToDevice,
                                   reinterpret_cast<cudaStream_t>(stream)));
}

int qic_model_free(qic_model* m) {
  if (m == nullptr) return QIC_SUCCESS;
  if (m->capture_stream != nullptr) cudaStreamSynchronize(m->capture_stream);
  cudaDeviceSynchronize();
  if (m->exec != nullptr) cudaGraphExecDestroy(m->exec);
  if (m->graph != nullptr) cudaGraphDestroy(m->graph);
  if (m->capture_stream != nullptr) cudaStreamDestroy(m->capture_stream);
  for (void* p : m->owned) cudaFree(p);
  if (m->host_scalars != nullptr) cudaFreeHost(m->host_scalars);
  delete[] m->cfg.layer_types;
  delete m;
  return QIC_SUCCESS;
}

}  // extern "C"
