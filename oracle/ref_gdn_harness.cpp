// TEST INFRASTRUCTURE ONLY: runs the reference's own GatedDeltaNet decode step (fp16
// as it ships, or a bfloat16 instance built with QICREF_GDN_BF16).
//
// The reference keeps this step in a private member, QwenMiniModel::
// run_linear_attention_block (src/model.cpp:656-795 of the QweninCuda project): four
// cuBLAS projections of x_norm_, eight device-to-host copies, the conv / delta-rule /
// gated-norm loop on the host, one host-to-device copy of the result and the out
// projection. This file compiles that source unmodified, in place (oracle/Makefile
// passes the reference's src/ and include/ directories), opening the class's members
// to this translation unit only, and drives the member function on caller-given
// inputs: with hidden_size 1 and x_norm_ = [1.0], each in-projection returns its one
// weight column exactly (fp16 x 1.0 in fp32), so those "weights" are the step's qkv,
// z, b and a. The 16-bit result is read from linear_out_; the conv and recurrent
// states are the LayerCache host vectors the loop updates in place.
//
// Every standard and CUDA header the reference includes is included first, so the
// access-specifier redefinition below reaches only the reference's own declarations.
#include <cublas_v2.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iomanip>
#include <iostream>
#include <numeric>
#include <random>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#ifdef QICREF_GDN_BF16
// bfloat16 instance: the reference's `half`, its two conversion calls and the cuBLAS
// element type of its GEMV renamed to their bfloat16 counterparts, after every header
// that defines them (the same renaming oracle/ref_bf16_shim.h applies to kernels.cu)
#include <cuda_bf16.h>
#define half __nv_bfloat16
#define __half2float __bfloat162float
#define __float2half __float2bfloat16
#define CUDA_R_16F CUDA_R_16BF
#endif

#define private public
#include "model.cpp"
#undef private

namespace {

half* to_device(const void* src, size_t bytes) {
  half* d = nullptr;
  CUDA_CHECK(cudaMalloc(&d, bytes));
  if (src != nullptr) {
    CUDA_CHECK(cudaMemcpy(d, src, bytes, cudaMemcpyHostToDevice));
  } else {
    CUDA_CHECK(cudaMemset(d, 0, bytes));
  }
  return d;
}

}  // namespace

// The reference model set up for one linear-attention layer: weights and runtime
// buffers on the device, the LayerCache states on the host, the cuBLAS handle
// created once, as the reference's load() does.
struct RefGdn {
  QwenMiniModel m;  // its destructor frees the runtime buffers and the cuBLAS handle
  QwenMiniModel::LayerWeights w;
  QwenMiniModel::LayerCache cache;
  size_t key_dim = 0, val_dim = 0, conv_dim = 0;
  int Hv = 0, K = 0, dk = 0, dv = 0;
  ~RefGdn() {
    for (half* p : {w.linear_in_qkv, w.linear_in_z, w.linear_in_b, w.linear_in_a, w.linear_conv1d_w,
                    w.linear_dt_bias, w.linear_a_log, w.linear_norm_w, w.linear_out_proj})
      if (p != nullptr) cudaFree(p);
  }
};

// Host fp16 weights (conv_w [conv_dim*K], dt_bias/a_log [Hv], norm_w [dv]) and fp32
// initial states (conv_state [conv_dim*K], recurrent_state [Hv*dk*dv]). Returns a
// handle, or null after printing the reference's CUDA/cuBLAS error.
extern "C" void* qicref_gdn_create(int Hk, int Hv, int dk, int dv, int K, float eps, const void* conv_w,
                                   const void* dt_bias, const void* a_log, const void* norm_w,
                                   const float* conv_state, const float* recurrent_state) {
  RefGdn* r = new RefGdn();
  try {
    r->key_dim = static_cast<size_t>(Hk) * dk;
    r->val_dim = static_cast<size_t>(Hv) * dv;
    r->conv_dim = 2 * r->key_dim + r->val_dim;
    r->Hv = Hv;
    r->K = K;
    r->dk = dk;
    r->dv = dv;
    QwenMiniModel& m = r->m;
    m.cfg_.hidden_size = 1;
    m.cfg_.linear_num_key_heads = Hk;
    m.cfg_.linear_num_value_heads = Hv;
    m.cfg_.linear_key_head_dim = dk;
    m.cfg_.linear_value_head_dim = dv;
    m.cfg_.linear_conv_kernel_dim = K;
    m.cfg_.rms_norm_eps = eps;
    CUBLAS_CHECK(cublasCreate(&m.cublas_));
    const half one = __float2half(1.0f);
    m.x_norm_ = to_device(&one, sizeof(half));
    m.x_ = to_device(nullptr, sizeof(half));
    m.linear_mixed_qkv_ = to_device(nullptr, r->conv_dim * sizeof(half));
    m.linear_z_ = to_device(nullptr, r->val_dim * sizeof(half));
    m.linear_b_ = to_device(nullptr, Hv * sizeof(half));
    m.linear_a_ = to_device(nullptr, Hv * sizeof(half));
    m.linear_out_ = to_device(nullptr, r->val_dim * sizeof(half));
    QwenMiniModel::LayerWeights& w = r->w;
    w.is_linear = true;
    w.linear_in_qkv = to_device(nullptr, r->conv_dim * sizeof(half));
    w.linear_in_z = to_device(nullptr, r->val_dim * sizeof(half));
    w.linear_in_b = to_device(nullptr, Hv * sizeof(half));
    w.linear_in_a = to_device(nullptr, Hv * sizeof(half));
    w.linear_conv1d_w = to_device(conv_w, r->conv_dim * K * sizeof(half));
    w.linear_dt_bias = to_device(dt_bias, Hv * sizeof(half));
    w.linear_a_log = to_device(a_log, Hv * sizeof(half));
    w.linear_norm_w = to_device(norm_w, dv * sizeof(half));
    w.linear_out_proj = to_device(nullptr, r->val_dim * sizeof(half));
    r->cache.linear_conv_state.assign(conv_state, conv_state + r->conv_dim * K);
    r->cache.linear_recurrent_state.assign(recurrent_state, recurrent_state + Hv * static_cast<size_t>(dk) * dv);
  } catch (const std::exception& e) {
    std::fprintf(stderr, "reference GatedDeltaNet set-up failed: %s\n", e.what());
    delete r;
    return nullptr;
  }
  return r;
}

// One decode step of the reference's linear-attention block. qkv [conv_dim], z
// [Hv*dv], b and a [Hv] (host fp16) become the step's projections (null: the previous
// step's again); out [Hv*dv] (host fp16) receives the gated-norm output, or null.
extern "C" int qicref_gdn_run(void* handle, const void* qkv, const void* z, const void* b, const void* a, void* out) {
  RefGdn* r = static_cast<RefGdn*>(handle);
  try {
    if (qkv != nullptr) {
      CUDA_CHECK(cudaMemcpy(r->w.linear_in_qkv, qkv, r->conv_dim * sizeof(half), cudaMemcpyHostToDevice));
      CUDA_CHECK(cudaMemcpy(r->w.linear_in_z, z, r->val_dim * sizeof(half), cudaMemcpyHostToDevice));
      CUDA_CHECK(cudaMemcpy(r->w.linear_in_b, b, r->Hv * sizeof(half), cudaMemcpyHostToDevice));
      CUDA_CHECK(cudaMemcpy(r->w.linear_in_a, a, r->Hv * sizeof(half), cudaMemcpyHostToDevice));
    }
    r->m.run_linear_attention_block(r->w, r->cache);
    if (out != nullptr)
      CUDA_CHECK(cudaMemcpy(out, r->m.linear_out_, r->val_dim * sizeof(half), cudaMemcpyDeviceToHost));
  } catch (const std::exception& e) {
    std::fprintf(stderr, "reference GatedDeltaNet step failed: %s\n", e.what());
    return 1;
  }
  return 0;
}

// Copies the current states out (host fp32).
extern "C" void qicref_gdn_states(void* handle, float* conv_state, float* recurrent_state) {
  const RefGdn* r = static_cast<const RefGdn*>(handle);
  std::memcpy(conv_state, r->cache.linear_conv_state.data(), r->conv_dim * r->K * sizeof(float));
  std::memcpy(recurrent_state, r->cache.linear_recurrent_state.data(),
              r->Hv * static_cast<size_t>(r->dk) * r->dv * sizeof(float));
}

extern "C" void qicref_gdn_destroy(void* handle) { delete static_cast<RefGdn*>(handle); }

// One step on fresh state: conv_state and recurrent_state (host fp32) are updated in
// place; out receives the step's output. Returns 0, or 1 after printing the error.
extern "C" int qicref_gdn_step(int Hk, int Hv, int dk, int dv, int K, float eps, const void* qkv, const void* z,
                               const void* b, const void* a, const void* conv_w, const void* dt_bias,
                               const void* a_log, const void* norm_w, float* conv_state, float* recurrent_state,
                               void* out) {
  void* h = qicref_gdn_create(Hk, Hv, dk, dv, K, eps, conv_w, dt_bias, a_log, norm_w, conv_state, recurrent_state);
  if (h == nullptr) return 1;
  const int rc = qicref_gdn_run(h, qkv, z, b, a, out);
  if (rc == 0) qicref_gdn_states(h, conv_state, recurrent_state);
  qicref_gdn_destroy(h);
  return rc;
}

// ---------------------------------------------------------------------------
// The reference's projections: QwenMiniModel::gemv (src/model.cpp:603-617, cuBLAS
// with the reference's own arguments) and run_ffn_block (src/model.cpp:797-807), run
// on caller device buffers through one model object whose cuBLAS handle is created
// once, as the reference's load() does. The model's runtime buffers that these
// members use are set to caller or scratch memory; free_all() never sees them.
// ---------------------------------------------------------------------------
namespace {

struct RefProj {
  QwenMiniModel m;
  std::vector<void*> scratch;
  RefProj() { CUBLAS_CHECK(cublasCreate(&m.cublas_)); }
  ~RefProj() {
    m.x_ = m.x_resid_ = m.x_norm_ = m.ffn_gate_ = m.ffn_up_ = m.ffn_hidden_ = nullptr;
    for (void* p : scratch) cudaFree(p);
  }
  half* buf(size_t elems) {
    void* p = nullptr;
    CUDA_CHECK(cudaMalloc(&p, elems * sizeof(half)));
    scratch.push_back(p);
    return static_cast<half*>(p);
  }
};

RefProj* ref_proj() {
  static RefProj* r = new RefProj();  // kept until exit, like the reference's model
  return r;
}

}  // namespace

// out[out_dim] = the reference's gemv of x[in_dim] with w[in_dim, out_dim] (device buffers).
extern "C" int qicref_gemv(const void* x, const void* w, int in_dim, int out_dim, void* out) {
  try {
    ref_proj()->m.gemv(static_cast<const half*>(x), static_cast<const half*>(w), in_dim, out_dim,
                       static_cast<half*>(out));
    CUDA_CHECK(cudaDeviceSynchronize());
  } catch (const std::exception& e) {
    std::fprintf(stderr, "reference gemv failed: %s\n", e.what());
    return 1;
  }
  return 0;
}

// x[hidden] (device, in place) = the reference's FFN block: x + down(swiglu(gate(norm(x)), up(norm(x)))).
extern "C" int qicref_ffn_block(void* x, const void* ffn_norm, const void* w_gate, const void* w_up, const void* w_down,
                                int hidden, int inter, float eps) {
  try {
    RefProj* r = ref_proj();
    QwenMiniModel& m = r->m;
    m.cfg_.hidden_size = hidden;
    m.cfg_.intermediate_size = inter;
    m.cfg_.rms_norm_eps = eps;
    m.x_ = static_cast<half*>(x);
    m.x_resid_ = r->buf(hidden);
    m.x_norm_ = r->buf(hidden);
    m.ffn_gate_ = r->buf(inter);
    m.ffn_up_ = r->buf(inter);
    m.ffn_hidden_ = r->buf(inter);
    QwenMiniModel::LayerWeights lw;
    lw.ffn_norm = const_cast<half*>(static_cast<const half*>(ffn_norm));
    lw.w_gate = const_cast<half*>(static_cast<const half*>(w_gate));
    lw.w_up = const_cast<half*>(static_cast<const half*>(w_up));
    lw.w_down = const_cast<half*>(static_cast<const half*>(w_down));
    m.run_ffn_block(lw);
    CUDA_CHECK(cudaDeviceSynchronize());
    m.x_ = m.x_resid_ = m.x_norm_ = m.ffn_gate_ = m.ffn_up_ = m.ffn_hidden_ = nullptr;
    for (void* p : r->scratch) cudaFree(p);
    r->scratch.clear();
  } catch (const std::exception& e) {
    std::fprintf(stderr, "reference FFN block failed: %s\n", e.what());
    return 1;
  }
  return 0;
}

// ---------------------------------------------------------------------------
// The reference model end to end: QwenMiniModel::load of a qmini v4 file
// (src/model.cpp:319-428) and decode_next (src/model.cpp:823-845), unmodified.
// ---------------------------------------------------------------------------
extern "C" void* qicref_model_load(const char* path) {
  QwenMiniModel* m = new QwenMiniModel();
  try {
    if (!m->load(path)) {
      delete m;
      return nullptr;
    }
  } catch (const std::exception& e) {
    std::fprintf(stderr, "reference load failed: %s\n", e.what());
    delete m;
    return nullptr;
  }
  return m;
}

// One decode_next step; logits (host, vocab 16-bit values) may be null. Returns the
// greedy token, or -1 after printing the reference's error.
extern "C" int qicref_model_decode(void* handle, int token, int position, void* logits) {
  QwenMiniModel* m = static_cast<QwenMiniModel*>(handle);
  try {
    std::vector<half> host;
    const int next = m->decode_next(token, position, &host);
    if (logits != nullptr) std::memcpy(logits, host.data(), host.size() * sizeof(half));
    return next;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "reference decode_next failed: %s\n", e.what());
    return -1;
  }
}

extern "C" void qicref_model_free(void* handle) { delete static_cast<QwenMiniModel*>(handle); }
