// The int8 wire of the exchange ("narrow"): rows of Q, K and V (K less a shift every GPU
// shares) and of the attention's output cross as int8 with one bf16 scale per row, after a turn
// by the orthonormal Hadamard matrix of the head dimension; the receiver turns them back.
//
// Law (src/cozy_runtime/internal/parallel/turn.py:60-82, `law` and `law_back`), per row x of
// D = 64 or 128 bf16 values:
//   t     = (x · H) · D^-½ − shift                  H: Sylvester ±1 matrix of order D
//   scale = bf16(max(max|t| · (1/127), 2^-126))     round to nearest even
//   code  = sign(q) · ⌊|q| + ½⌋,  q = clamp(t / scale, −127, 127)   (IEEE division)
//   back  = bf16((code · H) · (scale · D^-½))
// The turn is a fast Walsh-Hadamard transform across the warp that holds the row (the same
// matrix: H of order 2n is [[H, H], [H, −H]], one butterfly per index bit). Back, the codes'
// transform is exact in fp32 (|sum| ≤ 127·128), so `back` equals law_back bit for bit; forward,
// the fp32 sums of the turn may round in another order than the reference's matrix product.
//
// key_sum_kernel:     this rank's fp32 column sums of K in a fixed order, one 8-CTA cluster per
//                     (batch, head) (the all-reduced sum /
//                     total is the shift's source, as src/cozy_runtime/internal/parallel/
//                     ulysses.py:588-604).
// narrow_shift_kernel: shift = turned(sum / total), per (batch, head).
// narrow_pack_kernel: one warp per row (token, head, batch) of a tensor, its codes and scale
//                     written to every destination whose rows and heads contain it: by head for
//                     the first stage (every peer takes its heads of all this rank's rows), by
//                     row for the output's return (every owner takes its rows of all heads).
// narrow_widen_kernel: one warp per received row, back to bf16 at any strides.
#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/cozy_ulysses.h"

namespace cozy {

namespace cg = cooperative_groups;

constexpr float kTiny = 1.17549435e-38f;  // 2^-126, bf16's smallest normal

template <int D>
struct Turn {
  static constexpr int kPer = D / 32;  // values a lane holds: lane L has [L·kPer, L·kPer + kPer)
  static constexpr float kNorm = D == 128 ? 0.08838834764831845f : 0.125f;  // D^-1/2
};

// x·H for a row spread over the warp (unnormalised).
template <int D>
__device__ __forceinline__ void fwht(float (&x)[D / 32], int lane) {
  constexpr int kPer = D / 32;
#pragma unroll
  for (int bit = 1; bit < kPer; bit <<= 1)
#pragma unroll
    for (int i = 0; i < kPer; ++i)
      if (!(i & bit)) {
        const float u = x[i], w = x[i | bit];
        x[i] = u + w;
        x[i | bit] = u - w;
      }
#pragma unroll
  for (int lanes = 1; lanes < 32; lanes <<= 1) {
    // the lane holding the butterfly's upper half keeps (other - x), the lower (x + other):
    // other + sign·x, one FMA (exact: sign is ±1)
    const float sign = (lane & lanes) ? -1.f : 1.f;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const float other = __shfl_xor_sync(0xffffffffu, x[i], lanes);
      x[i] = __fmaf_rn(sign, x[i], other);
    }
  }
}

// One 8-CTA cluster per (batch, head): CTA c of the cluster sums rows [c·rows/8, (c+1)·rows/8),
// its warp w rows w, w + 32, ... of that share (lane L: channels [L·kPer, +kPer)); the warps'
// sums are added in warp order, then CTA 0 adds the eight CTAs' sums in rank order through
// distributed shared memory. The same order every call, so the shift, and every code narrowed
// against it, repeat bit for bit.
constexpr int kSumCluster = 8;

constexpr int kSumWarps = 32;

template <int D>
__global__ void __cluster_dims__(kSumCluster, 1, 1) __launch_bounds__(kSumWarps * 32)
    key_sum_kernel(const __nv_bfloat16* key, long long s_seq, long long s_head, long long s_batch,
                   int rows, int heads, float* sum) {
  constexpr int kPer = D / 32;
  __shared__ float part[kSumWarps][D];
  __shared__ float cta_total[D];
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int head = blockIdx.x / kSumCluster, b = blockIdx.y;
  const int r0 = static_cast<int>(static_cast<long long>(rows) * rank / kSumCluster);
  const int r1 = static_cast<int>(static_cast<long long>(rows) * (rank + 1) / kSumCluster);
  const __nv_bfloat16* k = key + b * s_batch + head * s_head + lane * kPer;
  // four rows in flight a warp, four accumulators (rows r + 32u of each pass), added in that
  // order at the end
  float acc[4][kPer];
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int i = 0; i < kPer; ++i) acc[u][i] = 0.f;
  for (int r = r0 + warp; r < r1; r += 4 * kSumWarps) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (r + kSumWarps * u >= r1) break;
      const __nv_bfloat16* row = k + static_cast<long long>(r + kSumWarps * u) * s_seq;
      if constexpr (kPer == 4) {
        const uint2 v = *reinterpret_cast<const uint2*>(row);
        const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.x));
        const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.y));
        acc[u][0] += lo.x, acc[u][1] += lo.y, acc[u][2] += hi.x, acc[u][3] += hi.y;
      } else {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(row));
        acc[u][0] += f.x, acc[u][1] += f.y;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    part[warp][lane * kPer + i] = ((acc[0][i] + acc[1][i]) + acc[2][i]) + acc[3][i];
  __syncthreads();
  if (threadIdx.x < D) {
    float total = 0.f;
#pragma unroll
    for (int w = 0; w < kSumWarps; ++w) total += part[w][threadIdx.x];
    cta_total[threadIdx.x] = total;
  }
  cluster.sync();  // every CTA's share is in its shared memory
  if (rank == 0 && threadIdx.x < D) {
    float total = 0.f;
#pragma unroll
    for (int c = 0; c < kSumCluster; ++c) total += cluster.map_shared_rank(cta_total, c)[threadIdx.x];
    sum[(static_cast<long long>(b) * heads + head) * D + threadIdx.x] += total;
  }
  cluster.sync();  // no CTA leaves while CTA 0 still reads its shared memory
}

// One warp per (batch, head): shift = ((sum / count) · H) · D^-½.
template <int D>
__global__ void narrow_shift_kernel(const float* sum, float count, int rows_total, float* shift) {
  constexpr int kPer = D / 32;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows_total) return;
  float x[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    x[i] = __fdiv_rn(sum[static_cast<long long>(row) * D + lane * kPer + i], count);
  fwht<D>(x, lane);
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    shift[static_cast<long long>(row) * D + lane * kPer + i] = __fmul_rn(x[i], Turn<D>::kNorm);
}

struct NarrowArgs {
  CozyNarrowTensor t[3];
  int count, world, rows, batch;
};

#ifndef COZY_NARROW_PACK_GROUP
#define COZY_NARROW_PACK_GROUP 1
#endif
#ifndef COZY_NARROW_WIDEN_GROUP
#define COZY_NARROW_WIDEN_GROUP 1
#endif
// Heads a warp loads before it turns the first. Measured on B200 at C2 (24 heads × 33272 rows):
// pack of Q/K/V 555 µs at 1, 588 at 2, 626 at 4; widen 104 µs at 1, 111 at 4, 139 at 8 — the
// kernels issue ~160 instructions a row (the turn's five shuffle rounds, the quantisation), so
// extra loads in flight cost occupancy for no gain.
constexpr int kPackGroup = COZY_NARROW_PACK_GROUP;
constexpr int kWidenGroup = COZY_NARROW_WIDEN_GROUP;
// Scales from here up divide by one reciprocal and a correction (below): the residual of the
// quotient cannot underflow.
constexpr float kFastDivide = 7.88860905e-31f;  // 2^-100

// One row (token r, batch b, head h) held by the warp: turned, shifted, scaled and quantised,
// then written to every destination that holds it.
template <int D>
__device__ __forceinline__ void narrow_row(float (&x)[D / 32], int lane, const float* shift,
                                           const NarrowArgs& a, const CozyNarrowTensor& t, int r,
                                           int b, int h) {
  constexpr int kPer = D / 32;
  fwht<D>(x, lane);
  uint32_t amax_bits = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    x[i] = __fmul_rn(x[i], Turn<D>::kNorm);
    if (shift) x[i] = __fsub_rn(x[i], shift[i]);
    amax_bits = max(amax_bits, __float_as_uint(fabsf(x[i])));
  }
  // non-negative floats order like their bit patterns: one warp reduction instruction
  const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, amax_bits));
  const __nv_bfloat16 scale = __float2bfloat16_rn(fmaxf(__fmul_rn(amax, 1.0f / 127.0f), kTiny));
  const float sf = __bfloat162float(scale);
  // q = t / scale rounded to nearest, as IEEE division: q0 = t·(1/scale), then one correction
  // by the exact residual t − q0·scale (Markstein's step; checked equal to division on 4M
  // fp32 samples with ties and their neighbours, scales 2^-100 ... 2^100). Smaller scales
  // (rows of tiny values) divide outright. `sf` is the same in the whole warp.
  const bool fast = sf >= kFastDivide;
  const float inv = __frcp_rn(sf);
  uint32_t word = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    float q;
    if (fast) {
      const float q0 = __fmul_rn(x[i], inv);
      q = __fmaf_rn(__fmaf_rn(-q0, sf, x[i]), inv, q0);
    } else {
      q = __fdiv_rn(x[i], sf);
    }
    q = fminf(fmaxf(q, -127.f), 127.f);
    // half away from zero: |q| + 1/2 is exact below 2^23, so truncation rounds it
    const int code = __float2int_rz(__fadd_rn(q, copysignf(0.5f, q)));
    word |= (static_cast<uint32_t>(code) & 0xffu) << (8 * i);
  }
  for (int p = 0; p < a.world; ++p) {
    if (r < t.row_lo[p] || r >= t.row_lo[p] + t.row_n[p]) continue;
    if (h < t.head_lo[p] || h >= t.head_lo[p] + t.head_n[p]) continue;
    const long long at =
        (static_cast<long long>(r - t.row_lo[p]) * a.batch + b) * t.head_n[p] + (h - t.head_lo[p]);
    int8_t* dst = static_cast<int8_t*>(t.dst[p]) + at * D + lane * kPer;
    if constexpr (kPer == 4) *reinterpret_cast<uint32_t*>(dst) = word;
    else *reinterpret_cast<uint16_t*>(dst) = static_cast<uint16_t>(word);
    if (lane == 0) static_cast<__nv_bfloat16*>(t.scale_dst[p])[at] = scale;
  }
}

// One warp per (row, batch) pair of a tensor, its heads in turn: the pair's index math runs once
// (32-bit: rows × batch < 2^31, checked on the host), each head's row is one 8- or 4-byte load a
// lane.
template <int D>
__global__ void __launch_bounds__(256) narrow_pack_kernel(const NarrowArgs a) {
  constexpr int kPer = D / 32;
  const CozyNarrowTensor& t = a.t[blockIdx.y];
  const int lane = threadIdx.x & 31;
  const unsigned pairs = static_cast<unsigned>(a.rows) * static_cast<unsigned>(a.batch);
  const unsigned warps = gridDim.x * (blockDim.x >> 5);
  for (unsigned rb = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); rb < pairs;
       rb += warps) {
    const int b = static_cast<int>(rb % static_cast<unsigned>(a.batch));
    const int r = static_cast<int>(rb / static_cast<unsigned>(a.batch));
    const __nv_bfloat16* base = static_cast<const __nv_bfloat16*>(t.src) + b * t.src_strides[2] +
                                static_cast<long long>(r) * t.src_strides[0] + lane * kPer;
    const float* shift_base =
        t.shift ? t.shift + static_cast<long long>(b) * t.heads * D + lane * kPer : nullptr;
    for (int h0 = 0; h0 < t.heads; h0 += kPackGroup) {
      // the group's rows are loaded before any is turned: kPackGroup reads in flight a lane
      float x[kPackGroup][kPer];
#pragma unroll
      for (int g = 0; g < kPackGroup; ++g) {
        const int h = h0 + g;
        if (h >= t.heads) break;
        const __nv_bfloat16* src = base + h * t.src_strides[1];
        if constexpr (kPer == 4) {
          const uint2 v = *reinterpret_cast<const uint2*>(src);
          const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.x));
          const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.y));
          x[g][0] = lo.x, x[g][1] = lo.y, x[g][2] = hi.x, x[g][3] = hi.y;
        } else {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src));
          x[g][0] = f.x, x[g][1] = f.y;
        }
      }
#pragma unroll
      for (int g = 0; g < kPackGroup; ++g) {
        const int h = h0 + g;
        if (h >= t.heads) break;
        narrow_row<D>(x[g], lane, shift_base ? shift_base + h * D : nullptr, a, t, r, b, h);
      }
    }
  }
}

struct WidenArgs {
  CozyWidenSource s[COZY_MAX_PEERS];
  int count, batch;
  __nv_bfloat16* out;
  long long s_seq, s_head, s_batch;
};

// One warp per (row, batch) pair of a source, its heads in turn (codes are [rows][batch][n]).
template <int D>
__global__ void __launch_bounds__(256) narrow_widen_kernel(const WidenArgs a) {
  constexpr int kPer = D / 32;
  const CozyWidenSource& s = a.s[blockIdx.y];
  const int lane = threadIdx.x & 31;
  const unsigned pairs = static_cast<unsigned>(s.rows) * static_cast<unsigned>(a.batch);
  const unsigned warps = gridDim.x * (blockDim.x >> 5);
  for (unsigned rb = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); rb < pairs;
       rb += warps) {
    const int b = static_cast<int>(rb % static_cast<unsigned>(a.batch));
    const int r = static_cast<int>(rb / static_cast<unsigned>(a.batch));
    const long long first = static_cast<long long>(rb) * s.head_n;  // item of head 0
    __nv_bfloat16* out = a.out + b * a.s_batch + static_cast<long long>(s.row_lo + r) * a.s_seq +
                         static_cast<long long>(s.head_lo) * a.s_head + lane * kPer;
    for (int h0 = 0; h0 < s.head_n; h0 += kWidenGroup) {
      // the group's codes and scales are loaded before any row is turned back
      float x[kWidenGroup][kPer];
      float scale[kWidenGroup];
#pragma unroll
      for (int g = 0; g < kWidenGroup; ++g) {
        const long long it = first + h0 + g;
        if (h0 + g >= s.head_n) break;
        const int8_t* codes = static_cast<const int8_t*>(s.codes) + it * D + lane * kPer;
        if constexpr (kPer == 4) {
          const char4 c = *reinterpret_cast<const char4*>(codes);
          x[g][0] = c.x, x[g][1] = c.y, x[g][2] = c.z, x[g][3] = c.w;
        } else {
          const char2 c = *reinterpret_cast<const char2*>(codes);
          x[g][0] = c.x, x[g][1] = c.y;
        }
        scale[g] = __bfloat162float(static_cast<const __nv_bfloat16*>(s.scales)[it]);
      }
#pragma unroll
      for (int g = 0; g < kWidenGroup; ++g) {
        if (h0 + g >= s.head_n) break;
        fwht<D>(x[g], lane);  // integers: exact
        const float factor = __fmul_rn(scale[g], Turn<D>::kNorm);
        __nv_bfloat16* dst = out + (h0 + g) * a.s_head;
        if constexpr (kPer == 4) {
          __nv_bfloat162 lo =
              __floats2bfloat162_rn(__fmul_rn(x[g][0], factor), __fmul_rn(x[g][1], factor));
          __nv_bfloat162 hi =
              __floats2bfloat162_rn(__fmul_rn(x[g][2], factor), __fmul_rn(x[g][3], factor));
          uint2 v;
          v.x = *reinterpret_cast<uint32_t*>(&lo);
          v.y = *reinterpret_cast<uint32_t*>(&hi);
          *reinterpret_cast<uint2*>(dst) = v;
        } else {
          *reinterpret_cast<__nv_bfloat162*>(dst) =
              __floats2bfloat162_rn(__fmul_rn(x[g][0], factor), __fmul_rn(x[g][1], factor));
        }
      }
    }
  }
}

static int grid_for(long long items) {
  const long long blocks = (items + 7) / 8;  // 8 warps a block, one (row, batch) pair each at first
  return static_cast<int>(blocks < 148 * 16 ? (blocks > 0 ? blocks : 1) : 148 * 16);
}

int key_sum(const void* key, const long long* strides, int rows, int batch, int heads,
            int head_dim, float* sum, cudaStream_t stream) {
  if (head_dim != 64 && head_dim != 128) return cudaErrorNotSupported;
  if (key == nullptr || strides == nullptr || sum == nullptr || rows < 0 || batch < 1 || heads < 1)
    return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  const int vec = head_dim / 32;
  if (reinterpret_cast<uintptr_t>(key) % (2 * vec)) return cudaErrorInvalidValue;
  for (int i = 0; i < 3; ++i)
    if (strides[i] <= 0 || strides[i] % vec) return cudaErrorInvalidValue;
  if (batch > 65535 || heads > (1 << 24)) return cudaErrorInvalidValue;
  dim3 grid(heads * kSumCluster, batch);
  const __nv_bfloat16* k = static_cast<const __nv_bfloat16*>(key);
  if (head_dim == 128)
    key_sum_kernel<128><<<grid, kSumWarps * 32, 0, stream>>>(k, strides[0], strides[1], strides[2],
                                                             rows, heads, sum);
  else
    key_sum_kernel<64><<<grid, kSumWarps * 32, 0, stream>>>(k, strides[0], strides[1], strides[2],
                                                            rows, heads, sum);
  return cudaGetLastError();
}

int narrow_shift(const float* sum, long long count, int batch, int heads, int head_dim,
                 float* shift, cudaStream_t stream) {
  if (head_dim != 64 && head_dim != 128) return cudaErrorNotSupported;
  if (sum == nullptr || shift == nullptr || count <= 0 || count > (1LL << 24) || batch < 1 ||
      heads < 1)
    return cudaErrorInvalidValue;
  const int rows = batch * heads;
  const int blocks = (rows + 7) / 8;
  const float c = static_cast<float>(count);  // exact: count ≤ 2^24
  if (head_dim == 128) narrow_shift_kernel<128><<<blocks, 256, 0, stream>>>(sum, c, rows, shift);
  else narrow_shift_kernel<64><<<blocks, 256, 0, stream>>>(sum, c, rows, shift);
  return cudaGetLastError();
}

int narrow_pack(const CozyNarrowTensor* tensors, int count, int world, int rows, int batch,
                int head_dim, cudaStream_t stream) {
  if (head_dim != 64 && head_dim != 128) return cudaErrorNotSupported;
  if (tensors == nullptr || count < 1 || count > 3 || world < 1 || world > COZY_MAX_PEERS ||
      rows < 0 || batch < 1)
    return cudaErrorInvalidValue;
  NarrowArgs a;
  a.count = count;
  a.world = world;
  a.rows = rows;
  a.batch = batch;
  const int vec = head_dim / 32;  // elements a lane loads: 4 (8 bytes) or 2 (4 bytes)
  for (int i = 0; i < count; ++i) {
    const CozyNarrowTensor& t = tensors[i];
    if (t.src == nullptr || t.heads < 1 || reinterpret_cast<uintptr_t>(t.src) % (2 * vec))
      return cudaErrorInvalidValue;
    for (int k = 0; k < 3; ++k)
      if (t.src_strides[k] <= 0 || t.src_strides[k] % vec) return cudaErrorInvalidValue;
    if (t.shift != nullptr && reinterpret_cast<uintptr_t>(t.shift) % 4) return cudaErrorInvalidValue;
    for (int p = 0; p < world; ++p) {
      if (t.head_n[p] < 0 || t.row_n[p] < 0 || t.head_lo[p] < 0 || t.row_lo[p] < 0 ||
          t.head_lo[p] + t.head_n[p] > t.heads || t.row_lo[p] + t.row_n[p] > rows)
        return cudaErrorInvalidValue;
      if (t.head_n[p] > 0 && t.row_n[p] > 0 &&
          (t.dst[p] == nullptr || t.scale_dst[p] == nullptr ||
           reinterpret_cast<uintptr_t>(t.dst[p]) % vec ||
           reinterpret_cast<uintptr_t>(t.scale_dst[p]) % 2))
        return cudaErrorInvalidValue;
    }
    a.t[i] = t;
  }
  const long long pairs = static_cast<long long>(rows) * batch;
  if (pairs == 0) return cudaSuccess;
  if (pairs >= (1LL << 31)) return cudaErrorInvalidValue;  // 32-bit pair index
  dim3 grid(grid_for(pairs), count);
  if (head_dim == 128) narrow_pack_kernel<128><<<grid, 256, 0, stream>>>(a);
  else narrow_pack_kernel<64><<<grid, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

int narrow_widen(const CozyWidenSource* sources, int count, int batch, int head_dim, void* out,
                 const long long* out_strides, cudaStream_t stream) {
  if (head_dim != 64 && head_dim != 128) return cudaErrorNotSupported;
  if (sources == nullptr || count < 1 || count > COZY_MAX_PEERS || batch < 1 || out == nullptr ||
      out_strides == nullptr)
    return cudaErrorInvalidValue;
  const int vec = head_dim / 32;
  if (reinterpret_cast<uintptr_t>(out) % (2 * vec)) return cudaErrorInvalidValue;
  for (int k = 0; k < 3; ++k)
    if (out_strides[k] <= 0 || out_strides[k] % vec) return cudaErrorInvalidValue;
  WidenArgs a;
  a.count = count;
  a.batch = batch;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.s_seq = out_strides[0];
  a.s_head = out_strides[1];
  a.s_batch = out_strides[2];
  long long most = 0;
  for (int i = 0; i < count; ++i) {
    const CozyWidenSource& s = sources[i];
    if (s.rows < 0 || s.head_n < 0 || s.row_lo < 0 || s.head_lo < 0) return cudaErrorInvalidValue;
    if (s.rows > 0 && s.head_n > 0 &&
        (s.codes == nullptr || s.scales == nullptr ||
         reinterpret_cast<uintptr_t>(s.codes) % vec || reinterpret_cast<uintptr_t>(s.scales) % 2))
      return cudaErrorInvalidValue;
    a.s[i] = s;
    const long long pairs = static_cast<long long>(s.rows) * batch;
    if (pairs >= (1LL << 31)) return cudaErrorInvalidValue;  // 32-bit pair index
    most = pairs > most ? pairs : most;
  }
  if (most == 0) return cudaSuccess;
  dim3 grid(grid_for(most), count);
  if (head_dim == 128) narrow_widen_kernel<128><<<grid, 256, 0, stream>>>(a);
  else narrow_widen_kernel<64><<<grid, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace cozy
