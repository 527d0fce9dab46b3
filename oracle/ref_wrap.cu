// ref_wrap.cu — TEST INFRASTRUCTURE ONLY. extern "C" entry points over the
// reference's own launch_* functions (include/kernels.cuh:5-19 of the QweninCuda
// project), so tests can drive the unmodified reference kernels through ctypes.
// Linked with the reference's src/kernels.cu into oracle/_ref/libqicref_{f16,bf16}.so
// by oracle/Makefile. With -include ref_bf16_shim.h, `half` below is bfloat16.
#include "kernels.cuh"

#include <cuda_runtime.h>

extern "C" {

int qicref_head_rmsnorm(const void* x, const void* w, int num_heads, int head_dim, float eps, void* out) {
  launch_head_rmsnorm(static_cast<const half*>(x), static_cast<const half*>(w), num_heads, head_dim, eps,
                      static_cast<half*>(out));
  return static_cast<int>(cudaGetLastError());
}

int qicref_rope_inplace(void* x, int num_heads, int head_dim, int position, float theta) {
  launch_rope_inplace(static_cast<half*>(x), num_heads, head_dim, position, theta);
  return static_cast<int>(cudaGetLastError());
}

int qicref_sigmoid_mul_inplace(void* x, const void* gate, int n) {
  launch_sigmoid_mul_inplace(static_cast<half*>(x), static_cast<const half*>(gate), n);
  return static_cast<int>(cudaGetLastError());
}

int qicref_split_q_gate(const void* packed, int num_heads, int head_dim, void* q, void* gate) {
  launch_split_q_gate_interleaved(static_cast<const half*>(packed), num_heads, head_dim, static_cast<half*>(q),
                                  static_cast<half*>(gate));
  return static_cast<int>(cudaGetLastError());
}

int qicref_flash_attention(const void* q, const void* k, const void* v, int num_heads, int num_kv_heads,
                           int head_dim, int seq_len, void* ctx) {
  launch_flash_attention(static_cast<const half*>(q), static_cast<const half*>(k), static_cast<const half*>(v),
                         num_heads, num_kv_heads, head_dim, seq_len, static_cast<half*>(ctx));
  return static_cast<int>(cudaGetLastError());
}

int qicref_paged_attention(const void* q, const void* k, const void* v, const int* page_table, int page_size,
                           int num_heads, int num_kv_heads, int head_dim, int seq_len, void* ctx) {
  launch_paged_attention(static_cast<const half*>(q), static_cast<const half*>(k), static_cast<const half*>(v),
                         page_table, page_size, num_heads, num_kv_heads, head_dim, seq_len,
                         static_cast<half*>(ctx));
  return static_cast<int>(cudaGetLastError());
}

// The reference appends with two device-to-device cudaMemcpy calls on the legacy
// default stream (src/model.cpp:639-641); this replays them at a given row.
int qicref_copy_row(void* cache, const void* row, long long row_index, int kv_dim) {
  size_t bytes = static_cast<size_t>(kv_dim) * sizeof(half);
  char* dst = static_cast<char*>(cache) + static_cast<size_t>(row_index) * bytes;
  return static_cast<int>(cudaMemcpy(dst, row, bytes, cudaMemcpyDeviceToDevice));
}

int qicref_rmsnorm(const void* x, const void* w, int n, float eps, void* out) {
  launch_rmsnorm(static_cast<const half*>(x), static_cast<const half*>(w), n, eps, static_cast<half*>(out));
  return static_cast<int>(cudaGetLastError());
}

int qicref_add_inplace(void* x, const void* y, int n) {
  launch_add_inplace(static_cast<half*>(x), static_cast<const half*>(y), n);
  return static_cast<int>(cudaGetLastError());
}

int qicref_swiglu(const void* gate, const void* up, int n, void* out) {
  launch_swiglu(static_cast<const half*>(gate), static_cast<const half*>(up), n, static_cast<half*>(out));
  return static_cast<int>(cudaGetLastError());
}

int qicref_synchronize(void) { return static_cast<int>(cudaDeviceSynchronize()); }

}  // extern "C"
