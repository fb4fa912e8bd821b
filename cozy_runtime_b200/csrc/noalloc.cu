// Degree-1 attention with RoPE on Q and K that allocates nothing: the rotated Q and K go to a
// file-scope device array instead of a buffer the caller (or this library) allocates.
//
// Who needs this: code that may not call cudaMalloc while it runs — a stream being captured into
// a CUDA graph (allocation calls are not capturable), a serving loop that owns all device memory
// up front through a fixed arena and forbids further driver allocations, or a host thread with
// hard latency limits (cudaMalloc can synchronize the device). They pass inputs and the output;
// the intermediate rotated copies live in `g_noalloc_scratch`.
//
// Limits and sharing: the array holds COZY_NOALLOC_SCRATCH_BYTES (64 MiB) on every GPU that loads
// this library, until the process exits. Every call on a device uses the same array, so calls
// whose kernels overlap on the GPU (two streams, or two host threads) race and corrupt each
// other's results; serialize them. Nothing in the array has to start at zero: each call writes
// every byte it reads before reading it. The first call on a device looks up the array's device
// address (cudaGetSymbolAddress, with that device current); make that first call before any
// stream capture begins.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "../../include/cozy_ulysses.h"

namespace cozy {
int attention_forward_unsplit(const void* q, const void* k, const void* v, void* out, int batch,
                      int seq_q, int seq_k, int heads_q, int heads_kv, int head_dim,
                      const long long* q_strides, const long long* k_strides,
                      const long long* v_strides, const long long* o_strides,
                      const CozyHeadMap* head_map, const CozyScatter* scatter, int causal,
                      float scale, int* status, cudaStream_t stream);
int ulysses_pack(const CozyPackTensor* tensors, int count, int world, int rows, int batch,
                 int head_dim, const CozyRope* rope, cudaStream_t stream);
}  // namespace cozy

// The scratch array. In host code this name is a host-side stand-in, not a device address:
// kernels are given the address cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) uint8_t g_noalloc_scratch[COZY_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_address[kMaxDevices] = {};

// The array's device address on the current device, looked up once per device.
cudaError_t scratch_address(void** out) {
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_address[device] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_address[device] = ptr;
  }
  *out = g_scratch_address[device];
  return cudaSuccess;
}
}  // namespace

extern "C" int cozy_rope_attention_fwd_noalloc(
    const void* q, const void* k, const void* v, void* out, int batch, int seq, int heads_q,
    int heads_kv, int head_dim, const long long* q_strides, const long long* k_strides,
    const long long* v_strides, const long long* o_strides, const CozyRope* rope, int normalize,
    float norm_eps, int causal, float scale, int* status, uintptr_t stream) {
  if (!q || !k || !v || !out || !q_strides || !k_strides || !v_strides || !o_strides || !rope)
    return cudaErrorInvalidValue;
  if (batch <= 0 || seq <= 0 || heads_q <= 0 || heads_kv <= 0 || head_dim <= 0)
    return cudaErrorInvalidValue;
  if (head_dim != 64 && head_dim != 128) return cudaErrorNotSupported;
  // Everything the attention checks is checked here first, so a refused call launches nothing
  // and leaves the shared array as the last call left it.
  if (heads_q % heads_kv != 0 || batch > 65535 || heads_q > 65535) return cudaErrorInvalidValue;
  const void* aligned[4] = {q, k, v, out};
  for (const void* ptr : aligned)
    if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0) return cudaErrorInvalidValue;
  const long long* given[4] = {q_strides, k_strides, v_strides, o_strides};
  for (const long long* st : given)
    for (int i = 0; i < 3; ++i)
      if (st[i] <= 0 || st[i] % 8 != 0) return cudaErrorInvalidValue;
  if (rope->cos == nullptr || rope->sin == nullptr || rope->rotary < 0 ||
      rope->rotary > head_dim || rope->rotary % 2 != 0)
    return cudaErrorInvalidValue;
  if (!rope->interleaved && rope->rotary % 16 != 0) return cudaErrorNotSupported;
  // Rotated Q and K, [seq][batch][heads][head_dim] bf16 each, must fit the array.
  const unsigned long long q_bytes = 2ull * seq * batch * heads_q * head_dim;
  const unsigned long long k_bytes = 2ull * seq * batch * heads_kv * head_dim;
  if (q_bytes + k_bytes > COZY_NOALLOC_SCRATCH_BYTES) return cudaErrorInvalidValue;
  void* base = nullptr;
  cudaError_t e = scratch_address(&base);
  if (e != cudaSuccess) return e;
  uint8_t* q_rot = static_cast<uint8_t*>(base);
  uint8_t* k_rot = q_rot + q_bytes;

  CozyPackTensor t[2] = {};
  const void* srcs[2] = {q, k};
  const long long* strides[2] = {q_strides, k_strides};
  const int heads[2] = {heads_q, heads_kv};
  void* dsts[2] = {q_rot, k_rot};
  for (int i = 0; i < 2; ++i) {
    t[i].src = srcs[i];
    for (int j = 0; j < 3; ++j) t[i].src_strides[j] = strides[i][j];
    t[i].heads = heads[i];
    t[i].normalize = normalize ? 1 : 0;
    t[i].norm_weight = nullptr;
    t[i].norm_offset = 0.f;
    t[i].norm_eps = norm_eps;
    t[i].rotate = 1;
    t[i].dst[0] = dsts[i];
    t[i].head_lo[0] = 0;
    t[i].head_n[0] = heads[i];
  }
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int code = cozy::ulysses_pack(t, 2, 1, seq, batch, head_dim, rope, s);
  if (code != cudaSuccess) return code;
  const long long qs[3] = {1LL * batch * heads_q * head_dim, head_dim, 1LL * heads_q * head_dim};
  const long long ks[3] = {1LL * batch * heads_kv * head_dim, head_dim,
                           1LL * heads_kv * head_dim};
  return cozy::attention_forward_unsplit(q_rot, k_rot, v, out, batch, seq, seq, heads_q, heads_kv,
                                 head_dim, qs, ks, v_strides, o_strides, nullptr, nullptr, causal,
                                 scale, status, s);
}
