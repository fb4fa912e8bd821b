// The library's C ABI (include/cozy_ulysses.h): thin extern "C" wrappers that turn the
// stream handle into a cudaStream_t and forward to the kernels' launchers. Nothing here throws;
// every entry point returns a cudaError_t value as an int.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/cozy_ulysses.h"

namespace cozy {
int attention_forward(const void* q, const void* k, const void* v, void* out, int batch,
                      int seq_q, int seq_k, int heads_q, int heads_kv, int head_dim,
                      const long long* q_strides, const long long* k_strides,
                      const long long* v_strides, const long long* o_strides,
                      const CozyHeadMap* head_map, const CozyScatter* scatter, int causal,
                      float scale, int* status, cudaStream_t stream);
int attention_split_plan(int batch, int seq_q, int seq_k, int heads_q, int head_dim, int causal,
                         long long* whole, int* parts);
int attention_split_plan_for(int batch, int seq_q, int seq_k, int heads_q, int head_dim,
                             int causal, int sms, long long* whole, int* parts);
int key_sum(const void* key, const long long* strides, int rows, int batch, int heads,
            int head_dim, float* sum, cudaStream_t stream);
int narrow_shift(const float* sum, long long count, int batch, int heads, int head_dim,
                 float* shift, cudaStream_t stream);
int narrow_pack(const CozyNarrowTensor* tensors, int count, int world, int rows, int batch,
                int head_dim, cudaStream_t stream);
int narrow_widen(const CozyWidenSource* sources, int count, int batch, int head_dim, void* out,
                 const long long* out_strides, cudaStream_t stream);
int ulysses_pack(const CozyPackTensor* tensors, int count, int world, int rows, int batch,
                 int head_dim, const CozyRope* rope, cudaStream_t stream);
int head_norm_rope(const void* x, void* out, int batch, int seq, int heads, int head_dim,
                   const long long* x_strides, const long long* out_strides,
                   const CozyRope* rope, int normalize, const float* weight, float offset,
                   float eps, cudaStream_t stream);
int ulysses_land(const void* returned, int world, int rows, int batch, int head_dim,
                 const int* head_lo, const int* head_n, void* out, const long long* out_strides,
                 cudaStream_t stream);
}  // namespace cozy

static inline cudaStream_t as_stream(uintptr_t s) { return reinterpret_cast<cudaStream_t>(s); }

extern "C" {

int cozy_attention_fwd(const void* q, const void* k, const void* v, void* out, int batch,
                       int seq_q, int seq_k, int heads_q, int heads_kv, int head_dim,
                       const long long* q_strides, const long long* k_strides,
                       const long long* v_strides, const long long* o_strides,
                       const CozyHeadMap* head_map, const CozyScatter* scatter, int causal,
                       float scale, int* status, uintptr_t stream) {
  if (!q_strides || !k_strides || !v_strides || (!o_strides && !scatter))
    return cudaErrorInvalidValue;
  return cozy::attention_forward(q, k, v, out, batch, seq_q, seq_k, heads_q, heads_kv, head_dim,
                                 q_strides, k_strides, v_strides, o_strides, head_map, scatter, causal, scale,
                                 status, as_stream(stream));
}

int cozy_attention_split_plan(int batch, int seq_q, int seq_k, int heads_q, int head_dim,
                              int causal, long long* whole_tiles, int* parts) {
  return cozy::attention_split_plan(batch, seq_q, seq_k, heads_q, head_dim, causal, whole_tiles,
                                    parts);
}

int cozy_key_sum(const void* key, const long long* strides, int rows, int batch, int heads,
                 int head_dim, float* sum, uintptr_t stream) {
  return cozy::key_sum(key, strides, rows, batch, heads, head_dim, sum, as_stream(stream));
}

int cozy_narrow_shift(const float* sum, long long count, int batch, int heads, int head_dim,
                      float* shift, uintptr_t stream) {
  return cozy::narrow_shift(sum, count, batch, heads, head_dim, shift, as_stream(stream));
}

int cozy_narrow_pack(const CozyNarrowTensor* tensors, int count, int world, int rows, int batch,
                     int head_dim, uintptr_t stream) {
  return cozy::narrow_pack(tensors, count, world, rows, batch, head_dim, as_stream(stream));
}

int cozy_narrow_widen(const CozyWidenSource* sources, int count, int batch, int head_dim,
                      void* out, const long long* out_strides, uintptr_t stream) {
  return cozy::narrow_widen(sources, count, batch, head_dim, out, out_strides, as_stream(stream));
}

int cozy_attention_split_plan_for(int batch, int seq_q, int seq_k, int heads_q, int head_dim,
                                  int causal, int sms, long long* whole_tiles, int* parts) {
  return cozy::attention_split_plan_for(batch, seq_q, seq_k, heads_q, head_dim, causal, sms,
                                        whole_tiles, parts);
}

int cozy_ulysses_pack(const CozyPackTensor* tensors, int count, int world, int rows, int batch,
                      int head_dim, const CozyRope* rope, uintptr_t stream) {
  if (!tensors) return cudaErrorInvalidValue;
  return cozy::ulysses_pack(tensors, count, world, rows, batch, head_dim, rope,
                            as_stream(stream));
}

int cozy_ulysses_land(const void* returned, int world, int rows, int batch, int head_dim,
                      const int* head_lo, const int* head_n, void* out,
                      const long long* out_strides, uintptr_t stream) {
  if (!head_lo || !head_n || !out_strides) return cudaErrorInvalidValue;
  return cozy::ulysses_land(returned, world, rows, batch, head_dim, head_lo, head_n, out,
                            out_strides, as_stream(stream));
}

int cozy_head_norm_rope(const void* x, void* out, int batch, int seq, int heads, int head_dim,
                        const long long* x_strides, const long long* out_strides,
                        const CozyRope* rope, int normalize, const float* weight, float offset,
                        float eps, uintptr_t stream) {
  if (!x_strides || !out_strides) return cudaErrorInvalidValue;
  return cozy::head_norm_rope(x, out, batch, seq, heads, head_dim, x_strides, out_strides, rope,
                              normalize, weight, offset, eps, as_stream(stream));
}

const char* cozy_error_name(int code) {
  return cudaGetErrorName(static_cast<cudaError_t>(code));
}

int cozy_abi_version(void) { return 104; }

}  // extern "C"

namespace cozy {
int attention_forward_fp8(const void* q, const void* k, const void* v, const float* q_scale,
                          const float* k_scale, const float* v_scale, long long scale_seq,
                          const int* cuts, int n_cuts, void* out, int batch, int seq_q, int seq_k, int heads_q, int heads_kv,
                          int head_dim, const long long* q_strides, const long long* k_strides,
                          const long long* v_strides, const long long* o_strides,
                          const CozyHeadMap* head_map, const CozyScatter* scatter, int causal,
                          float scale, int* status, cudaStream_t stream);
int fp8_stats(const CozyFp8Stats* a, cudaStream_t stream);
int fp8_pack(const CozyFp8Pack* a, cudaStream_t stream);
int fp8_head_amax(const CozyFp8Pack* a, cudaStream_t stream);
}  // namespace cozy

extern "C" {

int cozy_fp8_stats(const CozyFp8Stats* stats, uintptr_t stream) {
  if (!stats || !stats->key || !stats->value || !stats->k_sum || !stats->v_amax)
    return cudaErrorInvalidValue;
  return cozy::fp8_stats(stats, as_stream(stream));
}

int cozy_fp8_pack(const CozyFp8Pack* pack, uintptr_t stream) {
  if (!pack) return cudaErrorInvalidValue;
  return cozy::fp8_pack(pack, as_stream(stream));
}

int cozy_fp8_head_amax(const CozyFp8Pack* pack, uintptr_t stream) {
  if (!pack) return cudaErrorInvalidValue;
  return cozy::fp8_head_amax(pack, as_stream(stream));
}

int cozy_attention_fwd_fp8(const void* q, const void* k, const void* v, const float* q_scale,
                           const float* k_scale, const float* v_scale, long long scale_seq,
                           const int* cuts, int n_cuts, void* out, int batch, int seq_q, int seq_k, int heads_q, int heads_kv,
                           int head_dim, const long long* q_strides, const long long* k_strides,
                           const long long* v_strides, const long long* o_strides,
                           const CozyHeadMap* head_map, const CozyScatter* scatter, int causal,
                           float scale, int* status, uintptr_t stream) {
  if (!q_strides || !k_strides || !v_strides || (!o_strides && !scatter))
    return cudaErrorInvalidValue;
  return cozy::attention_forward_fp8(q, k, v, q_scale, k_scale, v_scale, scale_seq, cuts, n_cuts,
                                     out, batch,
                                     seq_q, seq_k, heads_q, heads_kv, head_dim, q_strides,
                                     k_strides, v_strides, o_strides, head_map, scatter, causal,
                                     scale, status, as_stream(stream));
}

}  // extern "C"
