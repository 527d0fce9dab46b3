// TEST INFRASTRUCTURE ONLY: runs the reference's own GatedDeltaNet decode step.
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

// One decode step of the reference's linear-attention block on host fp16 inputs
// (qkv [2*Hk*dk + Hv*dv], z [Hv*dv], b/a/dt_bias/a_log [Hv], conv_w [conv_dim*K],
// norm_w [dv]); conv_state [conv_dim*K] and recurrent_state [Hv*dk*dv] (fp32, host)
// are updated in place; out [Hv*dv] receives the fp16 gated-norm output. Returns 0,
// or 1 after printing the reference's CUDA/cuBLAS error.
extern "C" int qicref_gdn_step(int Hk, int Hv, int dk, int dv, int K, float eps, const void* qkv, const void* z,
                               const void* b, const void* a, const void* conv_w, const void* dt_bias,
                               const void* a_log, const void* norm_w, float* conv_state, float* recurrent_state,
                               void* out) {
  QwenMiniModel::LayerWeights w;
  int rc = 0;
  try {
    const size_t key_dim = static_cast<size_t>(Hk) * dk;
    const size_t val_dim = static_cast<size_t>(Hv) * dv;
    const size_t conv_dim = 2 * key_dim + val_dim;
    QwenMiniModel m;  // its destructor frees the runtime buffers and the cuBLAS handle set below
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
    m.linear_mixed_qkv_ = to_device(nullptr, conv_dim * sizeof(half));
    m.linear_z_ = to_device(nullptr, val_dim * sizeof(half));
    m.linear_b_ = to_device(nullptr, Hv * sizeof(half));
    m.linear_a_ = to_device(nullptr, Hv * sizeof(half));
    m.linear_out_ = to_device(nullptr, val_dim * sizeof(half));
    w.is_linear = true;
    w.linear_in_qkv = to_device(qkv, conv_dim * sizeof(half));
    w.linear_in_z = to_device(z, val_dim * sizeof(half));
    w.linear_in_b = to_device(b, Hv * sizeof(half));
    w.linear_in_a = to_device(a, Hv * sizeof(half));
    w.linear_conv1d_w = to_device(conv_w, conv_dim * K * sizeof(half));
    w.linear_dt_bias = to_device(dt_bias, Hv * sizeof(half));
    w.linear_a_log = to_device(a_log, Hv * sizeof(half));
    w.linear_norm_w = to_device(norm_w, dv * sizeof(half));
    w.linear_out_proj = to_device(nullptr, val_dim * sizeof(half));
    QwenMiniModel::LayerCache cache;
    cache.linear_conv_state.assign(conv_state, conv_state + conv_dim * K);
    cache.linear_recurrent_state.assign(recurrent_state, recurrent_state + Hv * static_cast<size_t>(dk) * dv);
    m.run_linear_attention_block(w, cache);
    CUDA_CHECK(cudaMemcpy(out, m.linear_out_, val_dim * sizeof(half), cudaMemcpyDeviceToHost));
    std::memcpy(conv_state, cache.linear_conv_state.data(), conv_dim * K * sizeof(float));
    std::memcpy(recurrent_state, cache.linear_recurrent_state.data(), Hv * static_cast<size_t>(dk) * dv * sizeof(float));
  } catch (const std::exception& e) {
    std::fprintf(stderr, "reference GatedDeltaNet step failed: %s\n", e.what());
    rc = 1;
  }
  for (half* p : {w.linear_in_qkv, w.linear_in_z, w.linear_in_b, w.linear_in_a, w.linear_conv1d_w, w.linear_dt_bias,
                  w.linear_a_log, w.linear_norm_w, w.linear_out_proj})
    if (p != nullptr) cudaFree(p);
  return rc;
}
