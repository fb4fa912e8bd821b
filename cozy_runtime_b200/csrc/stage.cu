// The memory-bound stages around the attention: the fused first stage of the seq->head exchange
// (per-head RMSNorm + RoPE + transpose into per-peer blocks, one pass over Q/K/V) and the landing
// of returned output rows into [batch, rows, heads, head_dim].
//
// Both move 16-byte vectors: a row of head_dim bf16 is head_dim/8 consecutive threads, so a
// warp reads and writes whole 128-byte lines. These kernels are bounded by HBM (or, when the
// destination is a peer's buffer, by NVLink).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/cozy_ulysses.h"
#include "norm_rope.cuh"

namespace cozy {

struct PackArgs {
  CozyPackTensor t[3];
  CozyRope rope;
  int count, world, rows, batch;
  int max_rows_per_peer;  // rows × batch × max(head_n): the grid's x extent
};

// A CTA's destination rows are contiguous at their destination (blocks are [rows][batch][n][D]).
// With more than one destination most of them are other GPUs' memory: there the rows go out as
// one bulk copy of the CTA's rows, staged in shared memory, instead of one 16-byte store a
// thread (small writes cross NVLink at about half its rate).
__device__ __forceinline__ void bulk_store(void* dst, const void* src_smem, uint32_t bytes) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(src_smem));
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
               :: "l"(dst), "r"(s), "r"(bytes) : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  // complete, writes included, before the CTA leaves: the kernel's end then orders them before
  // the arrival flag the next kernel publishes
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 x = __bfloat1622float2(h[i]);
    f[2 * i] = x.x;
    f[2 * i + 1] = x.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 v;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

// Destination rows a thread carries: their loads are issued before the first row's math. Two
// rows at 8 CTAs an SM (32 registers) measured best on B200 (C2 first stage: 291 µs at one row,
// 268 µs at two, 301 µs at two without the register cap, 335 µs at four); the limit is the
// 16-byte reads an SM keeps in flight.
constexpr int kPackRows = 2;

// grid: x covers rows × batch × head_n[p] destination rows (CHUNKS threads each, kPackRows
// passes of 256 / CHUNKS rows per CTA), y = peer, z = tensor. One thread = 8 channels of one
// destination row per pass.
template <int HD, bool BULK>
__global__ void __launch_bounds__(256, 8) pack_kernel(const PackArgs a) {
  constexpr int CHUNKS = HD / 8;
  constexpr int ROWS_PER_PASS = 256 / CHUNKS;
  constexpr int kCtaRows = kPackRows * ROWS_PER_PASS;
  __shared__ __align__(128) __nv_bfloat16 staged[BULK ? kCtaRows * HD : 8];
  const CozyPackTensor& t = a.t[blockIdx.z];
  const int peer = blockIdx.y;
  const unsigned n = static_cast<unsigned>(t.head_n[peer]);
  const int chunk = threadIdx.x % CHUNKS;
  // destination rows number below 2^31 (checked on the host): 32-bit index arithmetic
  const unsigned total = static_cast<unsigned>(a.rows) * a.batch * n;
  const unsigned cta_first = blockIdx.x * kCtaRows;
  const unsigned first = cta_first + threadIdx.x / CHUNKS;
  // The CTA leaves as a whole when it has no row (the bulk path's barrier needs every thread).
  if (n == 0 || cta_first >= total) return;
  if (!BULK && first >= total) return;  // whole row groups leave together
  const int d0 = chunk * 8;
  float x[kPackRows][8];
  unsigned token[kPackRows];
#pragma unroll
  for (int k = 0; k < kPackRows; ++k) {
    const unsigned row = first + k * ROWS_PER_PASS;
    token[k] = 0;
    if (row < total) {
      // destination order [rows][batch][n]
      const unsigned hh = row % n;
      const unsigned sb = row / n;
      const unsigned b = sb % static_cast<unsigned>(a.batch);
      const unsigned s = sb / static_cast<unsigned>(a.batch);
      token[k] = s;
      const int head = t.head_lo[peer] + static_cast<int>(hh);
      const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(t.src) +
                                 s * t.src_strides[0] + head * t.src_strides[1] +
                                 b * t.src_strides[2];
      unpack8(*reinterpret_cast<const uint4*>(src + d0), x[k]);
    }
  }
#pragma unroll
  for (int k = 0; k < kPackRows; ++k) {
    const unsigned row = first + k * ROWS_PER_PASS;
    if (row >= total) break;
    norm_rope_row<HD>(x[k], d0, chunk, row_group_mask<CHUNKS>(), a.rope.token0 + token[k], t,
                      a.rope);
    if constexpr (BULK) {
      *reinterpret_cast<uint4*>(staged + (row - cta_first) * HD + d0) = pack8(x[k]);
    } else {
      __nv_bfloat16* dst =
          static_cast<__nv_bfloat16*>(t.dst[peer]) + static_cast<long long>(row) * HD + d0;
      *reinterpret_cast<uint4*>(dst) = pack8(x[k]);
    }
  }
  if constexpr (BULK) {
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned rows_here = min(static_cast<unsigned>(kCtaRows), total - cta_first);
      bulk_store(static_cast<__nv_bfloat16*>(t.dst[peer]) + static_cast<long long>(cta_first) * HD,
                 staged, rows_here * HD * 2u);
    }
  }
}

// The standalone form: [batch, seq, heads, HD] in, the same shape out, any strides.
struct NormRopeArgs {
  CozyPackTensor t;  // src, src_strides, heads, norm fields, rotate; dst[0] = out
  long long out_strides[3];
  CozyRope rope;
  int seq, batch;
};

template <int HD>
__global__ void __launch_bounds__(256, 8) head_norm_rope_kernel(const NormRopeArgs a) {
  constexpr int CHUNKS = HD / 8;
  constexpr int ROWS_PER_PASS = 256 / CHUNKS;
  const int chunk = threadIdx.x % CHUNKS;
  const unsigned heads = static_cast<unsigned>(a.t.heads);
  const unsigned total = static_cast<unsigned>(a.batch) * a.seq * heads;
  // rows in [b][s][h] order; kPackRows of them a thread, loads first (as pack_kernel)
  const unsigned first = blockIdx.x * (kPackRows * ROWS_PER_PASS) + threadIdx.x / CHUNKS;
  if (first >= total) return;
  const int d0 = chunk * 8;
  float x[kPackRows][8];
  unsigned token[kPackRows];
  __nv_bfloat16* dst[kPackRows];
#pragma unroll
  for (int k = 0; k < kPackRows; ++k) {
    const unsigned row = first + k * ROWS_PER_PASS;
    token[k] = 0;
    dst[k] = nullptr;
    if (row < total) {
      const unsigned h = row % heads;
      const unsigned bs = row / heads;
      const unsigned s = bs % static_cast<unsigned>(a.seq);
      const unsigned b = bs / static_cast<unsigned>(a.seq);
      token[k] = s;
      const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(a.t.src) +
                                 s * a.t.src_strides[0] + h * a.t.src_strides[1] +
                                 b * a.t.src_strides[2];
      unpack8(*reinterpret_cast<const uint4*>(src + d0), x[k]);
      dst[k] = static_cast<__nv_bfloat16*>(a.t.dst[0]) + s * a.out_strides[0] +
               h * a.out_strides[1] + b * a.out_strides[2] + d0;
    }
  }
#pragma unroll
  for (int k = 0; k < kPackRows; ++k) {
    if (first + k * ROWS_PER_PASS >= total) break;
    norm_rope_row<HD>(x[k], d0, chunk, row_group_mask<CHUNKS>(), a.rope.token0 + token[k], a.t,
                      a.rope);
    *reinterpret_cast<uint4*>(dst[k]) = pack8(x[k]);
  }
}

int head_norm_rope(const void* x, void* out, int batch, int seq, int heads, int head_dim,
                   const long long* x_strides, const long long* out_strides,
                   const CozyRope* rope, int normalize, const float* weight, float offset,
                   float eps, cudaStream_t stream) {
  if (head_dim != 64 && head_dim != 128) return cudaErrorNotSupported;
  if (x == nullptr || out == nullptr || batch < 1 || seq < 0 || heads < 1)
    return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
    return cudaErrorInvalidValue;
  for (int k = 0; k < 3; ++k)
    if (x_strides[k] % 8 || out_strides[k] % 8) return cudaErrorInvalidValue;
  if (rope != nullptr) {
    if (rope->cos == nullptr || rope->sin == nullptr) return cudaErrorInvalidValue;
    if (rope->rotary < 0 || rope->rotary > head_dim || rope->rotary % 2) return cudaErrorInvalidValue;
    if (!rope->interleaved && rope->rotary % 16) return cudaErrorNotSupported;
  }
  const long long rows = static_cast<long long>(batch) * seq * heads;
  if (rows == 0) return cudaSuccess;
  if (rows >= (1LL << 31)) return cudaErrorInvalidValue;
  NormRopeArgs a = {};
  a.t.src = x;
  for (int k = 0; k < 3; ++k) {
    a.t.src_strides[k] = x_strides[k];
    a.out_strides[k] = out_strides[k];
  }
  a.t.heads = heads;
  a.t.normalize = normalize ? 1 : 0;
  a.t.norm_weight = weight;
  a.t.norm_offset = offset;
  a.t.norm_eps = eps;
  a.t.rotate = rope != nullptr;
  a.t.dst[0] = out;
  if (rope != nullptr) a.rope = *rope;
  a.seq = seq;
  a.batch = batch;
  const int rows_per_block = kPackRows * 256 / (head_dim / 8);
  const unsigned blocks = static_cast<unsigned>((rows + rows_per_block - 1) / rows_per_block);
  if (head_dim == 128)
    head_norm_rope_kernel<128><<<blocks, 256, 0, stream>>>(a);
  else
    head_norm_rope_kernel<64><<<blocks, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

// remote: the destinations are mostly other GPUs' memory (bulk copies out of shared memory);
// otherwise every destination is this GPU's own memory (16-byte stores a thread).
int ulysses_pack_to(const CozyPackTensor* tensors, int count, int world, int rows, int batch,
                    int head_dim, const CozyRope* rope, bool remote, cudaStream_t stream);

int ulysses_pack(const CozyPackTensor* tensors, int count, int world, int rows, int batch,
                 int head_dim, const CozyRope* rope, cudaStream_t stream) {
  return ulysses_pack_to(tensors, count, world, rows, batch, head_dim, rope, world > 1, stream);
}

int ulysses_pack_to(const CozyPackTensor* tensors, int count, int world, int rows, int batch,
                    int head_dim, const CozyRope* rope, bool remote, cudaStream_t stream) {
  if (count < 1 || count > 3 || world < 1 || world > COZY_MAX_PEERS || rows < 0 || batch < 1)
    return cudaErrorInvalidValue;
  if (head_dim != 64 && head_dim != 128) return cudaErrorNotSupported;
  PackArgs a = {};
  int max_n = 0;
  bool any_rotate = false;
  for (int i = 0; i < count; ++i) {
    a.t[i] = tensors[i];
    const CozyPackTensor& t = tensors[i];
    if (t.src == nullptr || reinterpret_cast<uintptr_t>(t.src) % 16) return cudaErrorInvalidValue;
    for (int k = 0; k < 3; ++k)
      if (t.src_strides[k] % 8) return cudaErrorInvalidValue;
    for (int p = 0; p < world; ++p) {
      if (t.head_n[p] < 0 || t.head_lo[p] < 0 || t.head_lo[p] + t.head_n[p] > t.heads)
        return cudaErrorInvalidValue;
      if (t.head_n[p] > 0 && (t.dst[p] == nullptr || reinterpret_cast<uintptr_t>(t.dst[p]) % 16))
        return cudaErrorInvalidValue;
      max_n = t.head_n[p] > max_n ? t.head_n[p] : max_n;
    }
    any_rotate = any_rotate || t.rotate;
  }
  if (any_rotate) {
    if (rope == nullptr || rope->cos == nullptr || rope->sin == nullptr) return cudaErrorInvalidValue;
    if (rope->rotary < 0 || rope->rotary > head_dim || rope->rotary % 2) return cudaErrorInvalidValue;
    if (!rope->interleaved && rope->rotary % 16) return cudaErrorNotSupported;
    a.rope = *rope;
  }
  a.count = count;
  a.world = world;
  a.rows = rows;
  a.batch = batch;
  const long long dest_rows = static_cast<long long>(rows) * batch * max_n;
  if (dest_rows == 0) return cudaSuccess;
  if (dest_rows >= (1LL << 31)) return cudaErrorInvalidValue;  // the kernel indexes in 32 bits
  const int rows_per_block = kPackRows * 256 / (head_dim / 8);
  const long long blocks = (dest_rows + rows_per_block - 1) / rows_per_block;
  dim3 grid(static_cast<unsigned>(blocks), world, count);
  if (remote) {
    if (head_dim == 128) pack_kernel<128, true><<<grid, 256, 0, stream>>>(a);
    else pack_kernel<64, true><<<grid, 256, 0, stream>>>(a);
  } else {
    if (head_dim == 128) pack_kernel<128, false><<<grid, 256, 0, stream>>>(a);
    else pack_kernel<64, false><<<grid, 256, 0, stream>>>(a);
  }
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------- landing
struct LandArgs {
  const __nv_bfloat16* returned;
  __nv_bfloat16* out;
  long long out_s, out_h, out_b;
  long long offset[COZY_MAX_PEERS];  // element offset of source p's block in `returned`
  int head_lo[COZY_MAX_PEERS], head_n[COZY_MAX_PEERS];
  int rows, batch;
};

template <int HD>
__global__ void __launch_bounds__(256) land_kernel(const LandArgs a) {
  constexpr int CHUNKS = HD / 8;
  constexpr int ROWS_PER_BLOCK = 256 / CHUNKS;
  const int p = blockIdx.y;
  const int n = a.head_n[p];
  const long long row = static_cast<long long>(blockIdx.x) * ROWS_PER_BLOCK + threadIdx.x / CHUNKS;
  if (n == 0 || row >= static_cast<long long>(a.rows) * a.batch * n) return;
  const int chunk = threadIdx.x % CHUNKS;
  const int hh = static_cast<int>(row % n);
  const long long sb = row / n;
  const int b = static_cast<int>(sb % a.batch);
  const int s = static_cast<int>(sb / a.batch);
  const uint4 v = *reinterpret_cast<const uint4*>(a.returned + a.offset[p] + row * HD + chunk * 8);
  __nv_bfloat16* dst =
      a.out + s * a.out_s + (a.head_lo[p] + hh) * a.out_h + b * a.out_b + chunk * 8;
  *reinterpret_cast<uint4*>(dst) = v;
}

int ulysses_land(const void* returned, int world, int rows, int batch, int head_dim,
                 const int* head_lo, const int* head_n, void* out, const long long* out_strides,
                 cudaStream_t stream) {
  if (world < 1 || world > COZY_MAX_PEERS || rows < 0 || batch < 1) return cudaErrorInvalidValue;
  if (head_dim != 64 && head_dim != 128) return cudaErrorNotSupported;
  if (returned == nullptr || out == nullptr || reinterpret_cast<uintptr_t>(returned) % 16 ||
      reinterpret_cast<uintptr_t>(out) % 16)
    return cudaErrorInvalidValue;
  for (int k = 0; k < 3; ++k)
    if (out_strides[k] % 8) return cudaErrorInvalidValue;
  LandArgs a = {};
  a.returned = static_cast<const __nv_bfloat16*>(returned);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_s = out_strides[0];
  a.out_h = out_strides[1];
  a.out_b = out_strides[2];
  a.rows = rows;
  a.batch = batch;
  long long offset = 0;
  int max_n = 0;
  for (int p = 0; p < world; ++p) {
    if (head_n[p] < 0 || head_lo[p] < 0) return cudaErrorInvalidValue;
    a.offset[p] = offset;
    a.head_lo[p] = head_lo[p];
    a.head_n[p] = head_n[p];
    offset += static_cast<long long>(rows) * batch * head_n[p] * head_dim;
    max_n = head_n[p] > max_n ? head_n[p] : max_n;
  }
  const long long dest_rows = static_cast<long long>(rows) * batch * max_n;
  if (dest_rows == 0) return cudaSuccess;
  const int rows_per_block = 256 / (head_dim / 8);
  dim3 grid(static_cast<unsigned>((dest_rows + rows_per_block - 1) / rows_per_block), world, 1);
  if (head_dim == 128)
    land_kernel<128><<<grid, 256, 0, stream>>>(a);
  else
    land_kernel<64><<<grid, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace cozy
