// Per-head RMSNorm then RoPE of one row held 8 channels a thread: the first stage's law
// (src/cozy_runtime/accel/fusion/_kernels.py:177-240 `head_norm_rope_kernel`), shared by the
// bf16 first stage (stage.cu) and the FP8 one (fp8.cu). `T` is any tensor descriptor with the
// fields normalize, norm_weight, norm_offset, norm_eps and rotate.
#pragma once

#include <cuda_runtime.h>

#include "../../include/cozy_ulysses.h"

namespace cozy {

// Per-head RMSNorm (when `t.normalize`) then RoPE (when `t.rotate`) of one row's 8 channels
// [d0, d0 + 8) held by this thread; the row's CHUNKS threads are consecutive lanes of one warp
// (`group_mask`). `token` is the row's RoPE table row. fp32 arithmetic, rounded once by the caller.
template <int HD, typename T>
__device__ __forceinline__ void norm_rope_row(float (&x)[8], int d0, int chunk,
                                              unsigned group_mask, long long token, const T& t,
                                              const CozyRope& r) {
  constexpr int CHUNKS = HD / 8;
  if (t.normalize) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(x[i], x[i], ss);
#pragma unroll
    for (int o = CHUNKS / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(group_mask, ss, o);
    const float inv = rsqrtf(ss / HD + t.norm_eps);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float w = t.norm_weight ? t.norm_weight[d0 + i] + t.norm_offset : 1.f;
      x[i] = t.norm_weight ? x[i] * inv * w : x[i] * inv;
    }
  }
  if (t.rotate && r.rotary > 0) {
    const float* cs = r.cos + token * r.stride_token;
    const float* sn = r.sin + token * r.stride_token;
    if (r.interleaved) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int d = d0 + 2 * i;
        if (d < r.rotary) {
          const int col = (d >> 1) * r.stride_channel;
          const float c = cs[col], sv = sn[col];
          const float lo = x[2 * i], hi = x[2 * i + 1];
          x[2 * i] = lo * c - hi * sv;
          x[2 * i + 1] = hi * c + lo * sv;
        }
      }
    } else {
      // split-half: channel j pairs with j ± rotary/2, a whole chunk (rotary/16) lanes away
      const int half_chunks = r.rotary / 16;
      const int lane = threadIdx.x & 31;
      const int base = lane - chunk;
      int partner = chunk;
      if (chunk < half_chunks) partner = chunk + half_chunks;
      else if (chunk < 2 * half_chunks) partner = chunk - half_chunks;
      float y[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = __shfl_sync(group_mask, x[i], base + partner);
      if (chunk < 2 * half_chunks) {
        const bool low = chunk < half_chunks;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int col = (d0 + i) * r.stride_channel;
          const float c = cs[col], sv = sn[col];
          x[i] = low ? x[i] * c - y[i] * sv : x[i] * c + y[i] * sv;
        }
      }
    }
  }
}

template <int CHUNKS>
__device__ __forceinline__ unsigned row_group_mask() {
  return (CHUNKS == 32) ? 0xffffffffu
                        : (((1u << CHUNKS) - 1u) << ((threadIdx.x & 31) / CHUNKS * CHUNKS));
}

}  // namespace cozy
