// The FP8 first stage of the exchange: e4m3 Q, K and V crossing the wire with their scales.
//
// Recipe (the FP8 video configuration): K less its per-(batch, head) mean over the WHOLE
// sequence (attention is unchanged by a shift of every key; the reference's narrow wire does the
// same with one all-reduce, src/cozy_runtime/internal/parallel/ulysses.py:588-604); Q and K
// quantised with one fp32 scale per 64-token × head block, scale = max(absmax / 448, 1e-12)
// (the reference's per-head law, src/cozy_runtime/internal/attention_fp8.py:162-169, at block
// granularity; a block is 64 rows of the whole sequence starting at a multiple of 64, clipped to
// this rank's rows); V quantised with one fp32 scale per
// (batch, head, channel) over the whole sequence. Codes are round-to-nearest-even, saturating.
//
// With RoPE / RMSNorm (the first stage's law, norm_rope.cuh) the recipe applies to the rotated
// Q and K, rounded to bf16 as the bf16 first stage leaves them: one pass over HBM does all of it.
//
// fp8_stats_kernel: this rank's partial K sums and V channel absmax (the host all-reduces them).
// fp8_pack_kernel:  one CTA per (block, head, batch) of one tensor: rows loaded once,
//                   mean subtracted, block absmax reduced in the CTA, codes written to every
//                   peer that owns the head, one scale per row to its per-token scale array.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "../../include/cozy_ulysses.h"
#include "norm_rope.cuh"

namespace cozy {

constexpr float kE4M3Max = 448.0f;
constexpr float kScaleFloor = 1e-12f;

// bf16 rounding of the first stage's fp32 result (the bf16 first stage stores exactly this)
__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

template <typename T>
__device__ __host__ __forceinline__ bool first_stage_law(const T& t) {
  return t.normalize || t.rotate;
}

__device__ __forceinline__ void unpack8(const uint4& v, float (&x)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

// blockIdx: x = slab of kStatsRows rows, y = head, z = batch. 256 threads: 16 a row (8 channels
// each, 16-byte loads), 16 rows a pass; UNROLL rows a thread are loaded (raw, 16 bytes each of K
// and V) before their math.
constexpr int kStatsRows = 256;

template <bool LAW>
__global__ void __launch_bounds__(256, 3) fp8_stats_kernel(const CozyFp8Stats a) {
  constexpr int UNROLL = LAW ? 2 : 4;
  const int chunk = threadIdx.x & 15;
  const int row_in = threadIdx.x >> 4;
  const int d0 = chunk * 8;
  const int head = blockIdx.y, b = blockIdx.z;
  const int r0 = blockIdx.x * kStatsRows;
  const __nv_bfloat16* key = static_cast<const __nv_bfloat16*>(a.key) + b * a.k_strides[2] +
                             head * a.k_strides[1] + d0;
  const __nv_bfloat16* value = static_cast<const __nv_bfloat16*>(a.value) + b * a.v_strides[2] +
                               head * a.v_strides[1] + d0;
  float sum[8], amax[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) sum[i] = amax[i] = 0.f;
  for (int base = 0; base < kStatsRows; base += 16 * UNROLL) {
    uint4 kr[UNROLL], vr[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int r = r0 + base + u * 16 + row_in;
      kr[u] = vr[u] = make_uint4(0u, 0u, 0u, 0u);
      if (r < a.rows) {
        kr[u] = *reinterpret_cast<const uint4*>(key + r * a.k_strides[0]);
        vr[u] = *reinterpret_cast<const uint4*>(value + r * a.v_strides[0]);
      }
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int r = r0 + base + u * 16 + row_in;
      float x[8], y[8];
      unpack8(kr[u], x);
      unpack8(vr[u], y);
      if constexpr (LAW) {  // a row past the end is zeros: its table row is clamped, unused
        norm_rope_row<128>(x, d0, chunk, row_group_mask<16>(),
                           a.rope.token0 + min(r, a.rows - 1), a, a.rope);
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = r < a.rows ? bf16_round(x[i]) : 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        sum[i] += x[i];
        amax[i] = fmaxf(amax[i], fabsf(y[i]));
      }
    }
  }
  // the CTA's 16 row groups into one partial per channel, then one atomic per channel
  __shared__ float part_sum[16][128], part_max[16][128];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    part_sum[row_in][d0 + i] = sum[i];
    part_max[row_in][d0 + i] = amax[i];
  }
  __syncthreads();
  if (threadIdx.x < 128) {
    const int d = threadIdx.x;
    float s = 0.f, m = 0.f;
#pragma unroll
    for (int g = 0; g < 16; ++g) {
      s += part_sum[g][d];
      m = fmaxf(m, part_max[g][d]);
    }
    const int o = (b * a.heads + head) * 128 + d;
    atomicAdd(a.k_sum + o, s);
    // non-negative floats order like their bit patterns
    atomicMax(reinterpret_cast<unsigned int*>(a.v_amax) + o, __float_as_uint(m));
  }
}

__device__ __forceinline__ uint32_t e4m3x4(float a, float b, float c, float d) {
  uint16_t lo, hi;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;" : "=h"(lo) : "f"(a), "f"(b));
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;" : "=h"(hi) : "f"(c), "f"(d));
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// ------------------------------------------------------------------------ first stage
// One CTA per work item: (64-row block of the whole sequence clipped to this rank) x head x
// (batch, tensor); 512 threads, 16 a row (8 channels each), 2 rows a thread, both loaded before
// any math; three CTAs an SM. (A persistent form that kept loads in flight through the math with
// a cp.async ring measured slower on B200 — 316 against 200 us at C4's degree-8 share — since
// the stage is bound by its instructions, the Hadamard's shuffles above all, not by HBM.)
constexpr int kPackThreads = 512;
constexpr int kPackPasses = 64 * 16 / kPackThreads;
constexpr float kHadamardBf16 = 0.08837890625f;  // 1/sqrt(128) rounded to bf16

// The first stage's transform of an item's rows held in `x`: RMSNorm + RoPE (rounded to bf16),
// K less its mean (block law), the Hadamard rotation (Q and K); rows outside the rank stay 0.
template <bool LAW>
__device__ __forceinline__ void transform_rows(const CozyFp8Pack& a, const CozyFp8Tensor& t,
                                               int b, int head, int block0, int lo_row, int hi_row,
                                               float (&x)[kPackPasses][8]) {
  const int chunk = threadIdx.x & 15, row_in = threadIdx.x >> 4, d0 = chunk * 8;
  if constexpr (LAW) {
    if (first_stage_law(t)) {
#pragma unroll
      for (int pass = 0; pass < kPackPasses; ++pass) {
        const int r = block0 + pass * 32 + row_in;
        const bool in = r >= lo_row && r < hi_row;
        norm_rope_row<128>(x[pass], d0, chunk, row_group_mask<16>(),
                           a.rope.token0 + (in ? r : lo_row), t, a.rope);
#pragma unroll
        for (int i = 0; i < 8; ++i) x[pass][i] = in ? bf16_round(x[pass][i]) : 0.f;
      }
    }
  }
  if (t.mean_sum != nullptr) {
    const float* ms = t.mean_sum + (b * t.heads + head) * 128 + d0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float mean = ms[i] * t.mean_inv_count;
#pragma unroll
      for (int pass = 0; pass < kPackPasses; ++pass) {
        const int r = block0 + pass * 32 + row_in;
        if (r >= lo_row && r < hi_row) x[pass][i] -= mean;
      }
    }
  }
  if (t.hadamard) {
    // Fast Walsh-Hadamard transform of each row (128 channels, index bits 0-6): bits 0-2 are
    // this thread's 8 channels, bits 3-6 its chunk, i.e. lanes 1, 2, 4, 8 apart in the row's
    // group of 16. Butterfly (a, b) -> (a + b, a - b); then the orthonormal 1/sqrt(128). The
    // per-head law rotates as a bf16 matrix product does: the multiplier rounded to bf16, the
    // result rounded to bf16.
#pragma unroll
    for (int pass = 0; pass < kPackPasses; ++pass) {
#pragma unroll
      for (int bit = 1; bit < 8; bit <<= 1)
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (!(i & bit)) {
            const float u = x[pass][i], w = x[pass][i | bit];
            x[pass][i] = u + w;
            x[pass][i | bit] = u - w;
          }
#pragma unroll
      for (int lanes = 1; lanes < 16; lanes <<= 1) {
        const float sign = (chunk & lanes) ? -1.f : 1.f;  // the high lane keeps other - x
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float other = __shfl_xor_sync(0xffffffffu, x[pass][i], lanes);
          x[pass][i] = fmaf(sign, x[pass][i], other);
        }
      }
      if (a.per_head) {
#pragma unroll
        for (int i = 0; i < 8; ++i) x[pass][i] = bf16_round(x[pass][i] * kHadamardBf16);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) x[pass][i] *= 0.08838834764831845f;  // 1/sqrt(128)
      }
    }
  }
}

__device__ __forceinline__ float warp_amax(const float (&x)[kPackPasses][8]) {
  float amax = 0.f;
#pragma unroll
  for (int pass = 0; pass < kPackPasses; ++pass)
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(x[pass][i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  return amax;
}

// AMAX = false: the first stage (codes to every owner of the head, per-token scales).
// AMAX = true:  the per-head law's statistics: the absmax of every (batch, head) of every tensor
//               with `head_amax`, after the same transform (atomic max; the caller zero-fills).
// blockIdx: x = 64-row block of this rank, y = head, z = batch * 3 + tensor (0 Q, 1 K, 2 V).
template <bool LAW, bool AMAX>
__global__ void __launch_bounds__(kPackThreads, LAW ? 2 : 3) fp8_pack_kernel(const CozyFp8Pack a) {
  const int tensor = blockIdx.z % 3;
  const int b = blockIdx.z / 3;
  const CozyFp8Tensor& t = a.t[tensor];
  if (static_cast<int>(blockIdx.y) >= t.heads) return;
  if (AMAX && t.head_amax == nullptr) return;
  // heads from the launch's first head round (the grid's y extent is Q's head count; K/V
  // start at the same fraction of theirs)
  const int turn = static_cast<int>(static_cast<long long>(a.head_turn) * t.heads / a.t[0].heads);
  const int head = (static_cast<int>(blockIdx.y) + turn) % t.heads;
  const int chunk = threadIdx.x & 15;
  const int row_in = threadIdx.x >> 4;
  const int d0 = chunk * 8;
  // global block of this CTA, clipped to this rank's rows [row0, row0 + rows)
  const int gblock = a.row0 / 64 + static_cast<int>(blockIdx.x);
  const int lo_row = max(gblock * 64, a.row0) - a.row0;
  const int hi_row = min(gblock * 64 + 64, a.row0 + a.rows) - a.row0;
  const int block0 = gblock * 64 - a.row0;  // may be negative: rows below lo_row are skipped
  const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(t.src) + b * t.src_strides[2] +
                             head * t.src_strides[1] + d0;
  float x[kPackPasses][8];
  {
    uint4 raw[kPackPasses];
#pragma unroll
    for (int pass = 0; pass < kPackPasses; ++pass) {
      const int r = block0 + pass * 32 + row_in;
      raw[pass] = make_uint4(0u, 0u, 0u, 0u);
      if (r >= lo_row && r < hi_row) raw[pass] = *reinterpret_cast<const uint4*>(src + r * t.src_strides[0]);
    }
#pragma unroll
    for (int pass = 0; pass < kPackPasses; ++pass) unpack8(raw[pass], x[pass]);
  }
  transform_rows<LAW>(a, t, b, head, block0, lo_row, hi_row, x);
  if constexpr (AMAX) {
    const float m = warp_amax(x);
    // non-negative floats order like their bit patterns
    if ((threadIdx.x & 31) == 0)
      atomicMax(reinterpret_cast<unsigned int*>(t.head_amax) + b * t.heads + head, __float_as_uint(m));
    return;
  } else {
    float inv[8];
    float scale = 0.f;
    bool divide = a.per_head;
    if (t.channel_scale != nullptr) {  // per-channel (V): scale from the global channel absmax
      const float* cs = t.channel_scale + (b * t.heads + head) * 128 + d0;
#pragma unroll
      for (int i = 0; i < 8; ++i) inv[i] = divide ? cs[i] : 1.f / cs[i];
    } else if (t.head_scale != nullptr) {  // per (batch, head): the reference's law
      scale = t.head_scale[b * t.heads + head];
#pragma unroll
      for (int i = 0; i < 8; ++i) inv[i] = scale;
      divide = true;
    } else {  // per 64-token block: reduce the absmax over the CTA
      __shared__ float warp_max[kPackThreads / 32];
      const float m0 = warp_amax(x);
      if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m0;
      __syncthreads();
      float m = warp_max[0];
#pragma unroll
      for (int w = 1; w < kPackThreads / 32; ++w) m = fmaxf(m, warp_max[w]);
      scale = fmaxf(m / kE4M3Max, kScaleFloor);
      const float is = 1.f / scale;
#pragma unroll
      for (int i = 0; i < 8; ++i) inv[i] = is;
    }
    // codes: x·(1/scale) for the block and channel recipes; x / scale correctly rounded, as
    // the reference's per-head law divides, where the per-head law is asked for
    auto code = [&](int pass, int i) {
      return divide ? __fdiv_rn(x[pass][i], inv[i]) : x[pass][i] * inv[i];
    };
    for (int p = 0; p < a.world; ++p) {
      const int lo = t.head_lo[p], n = t.head_n[p];
      if (head < lo || head >= lo + n) continue;
      const int hh = head - lo;
      uint8_t* dst = static_cast<uint8_t*>(t.dst[p]);
      float* sdst = t.scale_dst[p];
#pragma unroll
      for (int pass = 0; pass < kPackPasses; ++pass) {
        const int r = block0 + pass * 32 + row_in;
        if (r < lo_row || r >= hi_row) continue;
        const uint2 codes = make_uint2(
            e4m3x4(code(pass, 0), code(pass, 1), code(pass, 2), code(pass, 3)),
            e4m3x4(code(pass, 4), code(pass, 5), code(pass, 6), code(pass, 7)));
        // destination [rows][batch][n][128] bytes
        *reinterpret_cast<uint2*>(dst + ((static_cast<long long>(r) * a.batch + b) * n + hh) * 128 + d0) =
            codes;
        if (sdst != nullptr && chunk == 0)  // per-token scales [batch][n][scale_seq] at this rank's row
          sdst[(static_cast<long long>(b) * n + hh) * t.scale_seq + r] = scale;
      }
    }
  }
}

// The RoPE table a rotating tensor reads (the bf16 first stage's checks).
static int check_rope(const CozyRope& r) {
  if (r.cos == nullptr || r.sin == nullptr) return cudaErrorInvalidValue;
  if (r.rotary < 0 || r.rotary > 128 || r.rotary % 2 || r.token0 < 0) return cudaErrorInvalidValue;
  if (!r.interleaved && r.rotary % 16) return cudaErrorNotSupported;
  return cudaSuccess;
}

int fp8_stats(const CozyFp8Stats* a, cudaStream_t stream) {
  if (a->head_dim != 128 || a->rows < 0 || a->batch < 1 || a->heads < 1) return cudaErrorNotSupported;
  if (a->key == nullptr || a->value == nullptr || a->k_sum == nullptr || a->v_amax == nullptr ||
      reinterpret_cast<uintptr_t>(a->key) % 16 || reinterpret_cast<uintptr_t>(a->value) % 16)
    return cudaErrorInvalidValue;
  for (int k = 0; k < 3; ++k)
    if (a->k_strides[k] % 8 || a->v_strides[k] % 8) return cudaErrorInvalidValue;
  if (a->rotate) {
    const int e = check_rope(a->rope);
    if (e != cudaSuccess) return e;
  }
  if (a->rows == 0) return cudaSuccess;
  dim3 grid((a->rows + kStatsRows - 1) / kStatsRows, a->heads, a->batch);
  if (first_stage_law(*a))
    fp8_stats_kernel<true><<<grid, 256, 0, stream>>>(*a);
  else
    fp8_stats_kernel<false><<<grid, 256, 0, stream>>>(*a);
  return cudaGetLastError();
}

// The checks both launches of the first-stage kernel make; `heads` gets the grid's head extent.
static int check_pack(const CozyFp8Pack* a, bool amax, int* heads) {
  if (a->head_dim != 128) return cudaErrorNotSupported;
  if (a->world < 1 || a->world > COZY_MAX_PEERS || a->rows < 0 || a->batch < 1)
    return cudaErrorInvalidValue;
  *heads = 0;
  for (int i = 0; i < 3; ++i) {
    const CozyFp8Tensor& t = a->t[i];
    if (t.src == nullptr || reinterpret_cast<uintptr_t>(t.src) % 16) return cudaErrorInvalidValue;
    for (int k = 0; k < 3; ++k)
      if (t.src_strides[k] % 8) return cudaErrorInvalidValue;
    if (!amax)
      for (int p = 0; p < a->world; ++p)
        if (t.head_n[p] > 0 && (t.dst[p] == nullptr || reinterpret_cast<uintptr_t>(t.dst[p]) % 8))
          return cudaErrorInvalidValue;
    *heads = t.heads > *heads ? t.heads : *heads;
    if (t.rotate) {
      const int e = check_rope(a->rope);
      if (e != cudaSuccess) return e;
    }
  }
  if (a->row0 < 0) return cudaErrorInvalidValue;
  if (a->head_turn < 0 || (a->t[0].heads > 0 && a->head_turn >= a->t[0].heads) ||
      a->t[0].heads != *heads)  // the grid walks Q's heads; K/V have as many or fewer
    return cudaErrorInvalidValue;
  return cudaSuccess;
}

template <bool AMAX>
static int launch_pack(const CozyFp8Pack* a, cudaStream_t stream) {
  int heads = 0;
  const int e = check_pack(a, AMAX, &heads);
  if (e != cudaSuccess) return e;
  if (a->rows == 0) return cudaSuccess;
  const int blocks = (a->row0 + a->rows + 63) / 64 - a->row0 / 64;
  dim3 grid(blocks, heads, a->batch * 3);
  if (first_stage_law(a->t[0]) || first_stage_law(a->t[1]) || first_stage_law(a->t[2]))
    fp8_pack_kernel<true, AMAX><<<grid, kPackThreads, 0, stream>>>(*a);
  else
    fp8_pack_kernel<false, AMAX><<<grid, kPackThreads, 0, stream>>>(*a);
  return cudaGetLastError();
}

int fp8_pack(const CozyFp8Pack* a, cudaStream_t stream) { return launch_pack<false>(a, stream); }

int fp8_head_amax(const CozyFp8Pack* a, cudaStream_t stream) {
  bool any = false;
  for (int i = 0; i < 3; ++i) any |= a->t[i].head_amax != nullptr;
  if (!any) return cudaErrorInvalidValue;
  return launch_pack<true>(a, stream);
}

}  // namespace cozy
