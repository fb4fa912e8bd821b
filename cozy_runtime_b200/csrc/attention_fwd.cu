// Flash-attention forward for sm_100a: softmax(Q Kᵀ · scale) V per head, bf16 in and out, fp32
// softmax statistics and accumulation, on the 5th-generation tensor cores.
//
// One CTA owns 256 query rows of one (batch, head): two 128-row query tiles that take turns on
// the tensor core, so one tile's softmax runs while the other's matrix products do.
//
//   warps 0-3   softmax for query tile 0 (thread = one query row = one TMEM lane)
//   warps 4-7   softmax for query tile 1
//   warp  8     TMA producer: Q and K_0 once, then V_j with K_{j+1} into a ring of shared-memory
//               slots; the pair completes one barrier, so the MMA warp waits once per key block
//               for both (each wait of that warp costs ~150 clocks while its MMAs are in flight)
//   warp  9     MMA issuer (one elected lane): S = Q·Kᵀ into TMEM, O += P·V, P read from TMEM
//   warps 10-11 idle (they complete the third warpgroup the register split needs)
//
// Tensor memory (512 columns × 128 lanes of 32 bits):
//   [0,128)   S/P of tile 0   (S fp32; P bf16 pairs overwrite its first HD/2... columns)
//   [128,256) S/P of tile 1
//   [256, 256+HD) O of tile 0, then O of tile 1
//
// The running max is rescaled lazily: a warp rescales its rows of O only when some row's max
// grew by more than 2^8 since the max its probabilities were taken against; otherwise P is
// formed against the stale max (values ≤ 256, exact in fp32 and safe in bf16).
//
// Memory layout of Q, K, V and O: any strides over (sequence, head, batch) with the head
// dimension contiguous, described to TMA by 4-D tensor maps (dims: head_dim, seq, head, batch).
// This reads both a rank's own [B, S, H, D] rows and the [S, B, h, D] receive buffers of the
// Ulysses exchange without a transpose.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <utility>

#include "../../include/cozy_ulysses.h"
#include "attention.h"
#include "sm100.cuh"

namespace cozy {

constexpr int kBlockM = 128;   // query rows per tile (TMEM lanes)
constexpr int kBlockN = 128;   // key rows per tile
constexpr int kQTiles = 2;     // query tiles per CTA
constexpr int kStages = 4;     // K/V ring slots
constexpr int kThreads = 384;  // 8 softmax warps + producer + MMA + 2 idle (a full warpgroup)
// Register split (setmaxnreg): the launch gives every thread 168 (384 × 168 = 64512 of 65536);
// the producer warpgroup drops to 80 so the two softmax warpgroups can hold 208 each:
// 256 × 208 + 128 × 80 = 63488 ≤ 64512, and per SM sub-partition 208 + 208 + 80 = 496 ≤ 512
// per lane.
constexpr int kSoftmaxRegs = 208;
constexpr int kProducerRegs = 80;
constexpr float kRescaleLog2 = 8.0f;

struct AttentionParams {
  int batch, seq_q, seq_k, heads_q, heads_kv;
  int group, q_base, kv_base;  // query head h reads key/value head (h + q_base) / group - kv_base
  int causal;
  int causal_offset;  // seq_k - seq_q: causal aligned bottom-right
  int q_blocks;       // ceil(seq_q / 256)
  float scale_log2;   // softmax scale × log2(e)
  __nv_bfloat16* out;
  long long out_s, out_h, out_b;  // element strides of O
  int* status;
  // scatter: rows go to their owners' outputs (possibly other GPUs' memory) instead of `out`
  int scatter, world, head_offset;
  int row_start[COZY_MAX_PEERS + 1];
  __nv_bfloat16* outs[COZY_MAX_PEERS];
  long long outs_strides[COZY_MAX_PEERS][3];
  // FP8 operands: per-token scales of Q rows and K columns ([batch][heads][scale_seq]) and the
  // per-channel scale of V ([batch][heads_kv][head_dim]); unused by the bf16 kernel
  const float* q_scale;
  const float* k_scale;
  const float* v_scale;
  long long scale_seq;
  // rows where one rank's rows end and the next one's begin: the only places a 64-key block of
  // K scales can change inside a 64-key half of a tile
  int n_cuts;
  int cuts[COZY_MAX_PEERS];
  // Split key ranges (the last partial wave of tiles): tiles [0, n_full) run whole, one CTA
  // each; every later tile runs as `parts` CTAs over consecutive key-block ranges. A part leaves
  // its unnormalised O rows and (max, sum) in `ws_o`/`ws_ml`; the part that arrives last at the
  // tile's counter (an atomic, no waiting) merges them and writes the output.
  int n_full, parts;
  float* ws_o;     // [split tile][part][query tile][HD / 4][128 rows] float4
  float2* ws_ml;   // [split tile][part][query tile][128 rows]
  int* counters;   // [split tile][query tile], zero at launch
  // Walk orders. Query blocks run from q_turn downwards, cyclically (q_turn = q_blocks - 1: the
  // last block first, which for causal calls is the heaviest); each tile's key blocks run from
  // kv_turn downwards, cyclically (kv_turn < 0: upwards from block 0).
  int q_turn, kv_turn, q_seg;
  // Rows still crossing from other GPUs: rows [src_start[s], src_start[s + 1]) come from source
  // s, resident once arrive[s] (a flag in this GPU's memory the source writes) reaches
  // arrive_seq; the producer waits for a source's flag before its first load of that source's
  // rows (bounded by arrive_limit_ns, then kStatusPeerTimeout). arrive == nullptr: all rows are
  // resident. Source arrive_self is resident from the start.
  const long long* arrive;
  long long arrive_seq, arrive_limit_ns;
  int n_src, arrive_self;
  int src_start[COZY_MAX_PEERS + 1];
};

// Tile index t -> (query block, head, batch). The query blocks are taken in walk order (from
// q_turn downwards, cyclically) in segments of q_seg blocks: every (head, batch) takes the
// first segment's blocks, then every (head, batch) the next segment's, and so on, consecutive
// tiles sharing a (head, batch) and with it their keys and values in L2. q_seg = q_blocks keeps
// each (head, batch)'s blocks together; a smaller segment (the query blocks of one GPU's rows)
// runs every head's resident rows before any rows still crossing.
struct TileAt {
  int qb, head, b;
};

__device__ __forceinline__ TileAt tile_at(const AttentionParams& p, int t) {
  const int hb = p.heads_q * p.batch;
  const int seg = t / (p.q_seg * hb);
  const int first = seg * p.q_seg;
  const int len = min(p.q_seg, p.q_blocks - first);
  const int within = t - seg * p.q_seg * hb;
  const int pair = within / len;
  int qb = p.q_turn - (first + within % len);
  if (qb < 0) qb += p.q_blocks;
  return {qb, pair % p.heads_q, pair / p.heads_q};
}

// The key block of walk step i for a tile with n_blocks key blocks.
__device__ __forceinline__ int walk_block(const AttentionParams& p, int i, int n_blocks) {
  if (p.kv_turn < 0) return i;
  const int first = min(p.kv_turn, n_blocks - 1);
  const int b = first - i;
  return b < 0 ? b + n_blocks : b;
}

// Waits (lane 0 of the calling warp, bounded) until *flag reaches seq with acquire semantics at
// system scope. Returns false when the time limit passes (status: peer timeout) or the CTA or
// launch already gave up.
__device__ __forceinline__ bool wait_flag(const long long* flag, long long seq, long long limit_ns,
                                          volatile int* abort, int* status) {
  const uint64_t start = global_timer_ns();
  for (uint32_t spin = 0;; ++spin) {
    long long v;
    asm volatile("ld.acquire.sys.global.s64 %0, [%1];" : "=l"(v) : "l"(flag) : "memory");
    if (v >= seq) return true;
    if ((spin & 63u) == 63u) {
      if (*abort) return false;
      if (status != nullptr && *reinterpret_cast<volatile int*>(status) != kStatusOk) {
        *abort = 1;
        return false;
      }
      if (global_timer_ns() - start > static_cast<uint64_t>(limit_ns)) {
        *abort = 1;
        if (status != nullptr) atomicCAS(status, kStatusOk, kStatusPeerTimeout);
        return false;
      }
    }
    __nanosleep(32);
  }
}

template <int HD, bool FP8>
struct AttentionSmem {
  static constexpr int kElem = FP8 ? 1 : 2;            // bytes per element
  static constexpr int kBoxes = HD * kElem / 128;     // 128-byte swizzle atoms per row
  static constexpr int kBoxBytes = 128 * 128;         // one box: 128 rows × 128 bytes
  static constexpr int kTileBytes = kBoxes * kBoxBytes;
  static constexpr int kQOffset = 0;
  static constexpr int kKVOffset = kQTiles * kTileBytes;
  static constexpr int kBarOffset = kKVOffset + kStages * kTileBytes;
  // barriers: q_full (Q and K_0), kv_full[2] (the pair V_j, K_{j+1} of block j, alternating),
  // kv_empty[S], s_full[2], p_ready[2][2 halves], o_final[2], drain
  static constexpr int kBars = 1 + 2 + kStages + 2 + 4 + 2 + 1;
  static constexpr int kMiscOffset = kBarOffset + kBars * 8;
  static constexpr int kBytes = kMiscOffset + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack to align the base to 1024 bytes
};

// Empty asm that ties 32 registers to a point in the program, so no use of a TMEM load's
// outputs moves above the tcgen05.wait::ld that makes them valid.
__device__ __forceinline__ void reg_fence(uint32_t (&r)[32]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                 "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31]));
}

// One lane of a converged warp (the same lane every time).
__device__ __forceinline__ bool elect_one() {
  uint32_t pred;
  asm volatile(
      "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// Named barrier `kId` over `kCount` threads (a multiple of 32) that also returns whether
// `pred` held in every one of them.
template <int kId, int kCount>
__device__ __forceinline__ bool named_bar_and(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "n"(kId), "n"(kCount)
      : "memory");
  return r != 0;
}

template <int kId, int kCount>
__device__ __forceinline__ void named_bar_sync() {
  asm volatile("bar.sync %0, %1;" ::"n"(kId), "n"(kCount) : "memory");
}

// This CTA's tile, and for a split tile its part and its index among the split tiles (part -1
// for a whole tile). Cheap enough to recompute where it is needed, rather than hold in registers.
__device__ __forceinline__ int unit_tile(const AttentionParams& p, int u, int* part,
                                         int* split_tile) {
  if (u < p.n_full) {
    *part = -1;
    *split_tile = 0;
    return u;
  }
  const int v = u - p.n_full;
  *split_tile = v / p.parts;
  *part = v - *split_tile * p.parts;
  return p.n_full + *split_tile;
}

// Thread and block index read anew (volatile: never merged with an earlier read), so values
// derived from them after a long loop are recomputed there instead of held through it.
__device__ __forceinline__ int fresh_tid() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%tid.x;" : "=r"(r));
  return static_cast<int>(r);
}

__device__ __forceinline__ int fresh_ctaid() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%ctaid.x;" : "=r"(r));
  return static_cast<int>(r);
}

// mbar_wait by every lane of a warp, with one answer for the whole warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          int* status) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, status));
}

// A wait that ignores the CTA's abort flag but still ends at the time limit: used to drain the
// asynchronous copies and MMAs a CTA issued before it unwinds.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity, int* status) {
  (void)status;  // a drain never gives up early on another CTA's report
  int never = 0;
  mbar_wait(bar, parity, reinterpret_cast<volatile int*>(&never), nullptr);
}

// -------------------------------------------------------------------------- softmax helpers
// 2^f on [0, 1) by a degree-3 polynomial, coefficients fitted for this kernel (relative-error
// weighted least squares on 20001 points, Lawson reweighting toward minimax): max relative
// error 7.6e-5, far below the bf16 rounding P is stored with.
constexpr float kExp2C0 = 0.99992478f;
constexpr float kExp2C1 = 0.69583595f;
constexpr float kExp2C2 = 0.22606595f;
constexpr float kExp2C3 = 0.07802287f;
// Pairs of every 8 whose exponentials run on the FMA pipe instead of the MUFU unit (16 results
// per clock per SM). Measured on B200 at the C2 shape (24 heads × 33272 tokens, elected MMA
// warp): 0/8 1201-1219 TFLOP/s, 1/8 1232, 2/8 1253, 3/8 1234, 4/8 1137.
#ifndef COZY_POLY_PER_EIGHT
#define COZY_POLY_PER_EIGHT 2
#endif
constexpr int kPolyPerEight = COZY_POLY_PER_EIGHT;

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float chunk_max(const uint32_t (&r)[32]) {
  float m0 = fmaxf(__uint_as_float(r[0]), __uint_as_float(r[1]));
  float m1 = fmaxf(__uint_as_float(r[2]), __uint_as_float(r[3]));
#pragma unroll
  for (int i = 4; i < 32; i += 4) {
    m0 = fmax3(m0, __uint_as_float(r[i]), __uint_as_float(r[i + 1]));
    m1 = fmax3(m1, __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
  }
  return fmaxf(m0, m1);
}

// Columns past `limit` (chunk-relative; may be negative) become -inf.
__device__ __forceinline__ void mask_chunk(uint32_t (&r)[32], int limit) {
#pragma unroll
  for (int i = 0; i < 32; ++i)
    if (i > limit) r[i] = 0xff800000u;
}

// 2^t for a pair with t ≤ 8 on the FMA pipe: t = n + f with n = floor(t) (the round-down add of
// 1.5·2^23 leaves n in the low mantissa bits), 2^f from the polynomial, n added to the exponent.
// t is clamped at -120 first: the polynomial's value at f = 0 sits just below 1 (exponent field
// 126), so the exponent add must stay well clear of the bottom of the range; 2^-120 is zero for
// any probability sum it joins (masked keys land here).
__device__ __forceinline__ float2 exp2_poly2(float2 t) {
  const float2 magic = make_float2(12582912.0f, 12582912.0f);
  t.x = fmaxf(t.x, -120.0f);
  t.y = fmaxf(t.y, -120.0f);
  const float2 r = __fadd2_rd(t, magic);
  const float2 fl = __fadd2_rn(r, make_float2(-12582912.0f, -12582912.0f));
  const float2 f = __ffma2_rn(fl, make_float2(-1.0f, -1.0f), t);
  float2 p = __ffma2_rn(make_float2(kExp2C3, kExp2C3), f, make_float2(kExp2C2, kExp2C2));
  p = __ffma2_rn(p, f, make_float2(kExp2C1, kExp2C1));
  p = __ffma2_rn(p, f, make_float2(kExp2C0, kExp2C0));
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(r.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(r.y) << 23)));
}

// 2^f on [0, 1) by a degree-2 polynomial for the FP8 kernel, whose P is rounded to e4m3 (3
// mantissa bits: steps of up to 6 %): fitted like the cubic above, max relative error 1.7e-3.
// Its value at f = 0 is above 1, so the exponent add needs no margin; the clamp stays. Measured
// on B200 (C4's per-GPU shape at degree 8, 5 heads × 75600): 2 pairs of 8 on it 1240 TFLOP/s
// against 1226 with the cubic; 4, 6, 8 pairs of 8: 1163, 1004, 917 (the FMA pipe, not the MUFU,
// limits there).
constexpr float kExp2Q0 = 1.00171638f;
constexpr float kExp2Q1 = 0.65764964f;
constexpr float kExp2Q2 = 0.33720079f;

__device__ __forceinline__ float2 exp2_poly2_quadratic(float2 t) {
  const float2 magic = make_float2(12582912.0f, 12582912.0f);
  t.x = fmaxf(t.x, -120.0f);
  t.y = fmaxf(t.y, -120.0f);
  const float2 r = __fadd2_rd(t, magic);
  const float2 fl = __fadd2_rn(r, make_float2(-12582912.0f, -12582912.0f));
  const float2 f = __ffma2_rn(fl, make_float2(-1.0f, -1.0f), t);
  float2 p = __ffma2_rn(make_float2(kExp2Q2, kExp2Q2), f, make_float2(kExp2Q1, kExp2Q1));
  p = __ffma2_rn(p, f, make_float2(kExp2Q0, kExp2Q0));
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(r.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(r.y) << 23)));
}

// 32 scores -> 32 probabilities 2^(s·scale - m) as 16 packed bf16 pairs, summed into `acc`.
__device__ __forceinline__ void exp_chunk(const uint32_t (&r)[32], float2 scale2, float2 negm2,
                                          float2& acc, uint32_t (&pk)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float2 sv = make_float2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
    const float2 t = __ffma2_rn(sv, scale2, negm2);
    float2 e;
    if ((i & 7) < kPolyPerEight) {
      e = exp2_poly2(t);
    } else {
      e = make_float2(ex2_approx(t.x), ex2_approx(t.y));
    }
    acc = __fadd2_rn(acc, e);
    pk[i] = pack_bf16x2(e.x, e.y);
  }
}

// ------------------------------------------------------------------------------ FP8 helpers
// P is stored as e4m3 codes of p·2^8: with the running max exact to within 2^0.5 (the FP8
// kernel rescales O whenever a row's max grows by more than that) every code is at most
// 2^8.5 ≈ 362 < 448, and values down to 2^-9·2^-8 stay representable.
constexpr float kPScaleLog2 = 8.0f;
constexpr float kRescaleLog2Fp8 = 0.5f;

// 32 scores (in TMEM order) times their keys' scales (32 consecutive floats).
__device__ __forceinline__ void scale_chunk(uint32_t (&r)[32], const float4* ks) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 k = ks[i];
    const float2 a = __fmul2_rn(make_float2(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1])),
                                make_float2(k.x, k.y));
    const float2 c = __fmul2_rn(make_float2(__uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3])),
                                make_float2(k.z, k.w));
    r[4 * i] = __float_as_uint(a.x);
    r[4 * i + 1] = __float_as_uint(a.y);
    r[4 * i + 2] = __float_as_uint(c.x);
    r[4 * i + 3] = __float_as_uint(c.y);
  }
}

// 32 scores -> 32 e4m3 codes of 2^(s·scale + bias) packed four to a word, summed into `acc`.
// (The MUFU unit's f16-pair form, ex2.approx.f16x2, was measured on B200 at the same 16 results
// per clock per SM as the fp32 form — two results an instruction at half the instruction rate —
// and an e4m3 P path through it ran 21 % slower: 1007 against 1270 TFLOP/s at C4's per-GPU
// shape.)
__device__ __forceinline__ void exp_chunk_fp8(const uint32_t (&r)[32], float2 scale2, float2 bias2,
                                              float2& acc, uint32_t* pk) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float2 e[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int k = 4 * i + 2 * h;
      const float2 sv = make_float2(__uint_as_float(r[k]), __uint_as_float(r[k + 1]));
      const float2 t = __ffma2_rn(sv, scale2, bias2);
      if (((2 * i + h) & 7) < kPolyPerEight) {
        e[h] = exp2_poly2_quadratic(t);
      } else {
        e[h] = make_float2(ex2_approx(t.x), ex2_approx(t.y));
      }
      acc = __fadd2_rn(acc, e[h]);
    }
    uint16_t lo, hi;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;" : "=h"(lo) : "f"(e[0].x), "f"(e[0].y));
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;" : "=h"(hi) : "f"(e[1].x), "f"(e[1].y));
    pk[i] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
  }
}

template <int HD, bool FP8, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
    attention_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const AttentionParams p) {
  using L = AttentionSmem<HD, FP8>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem + L::kQOffset;
  uint8_t* sKV = smem + L::kKVOffset;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;  // [block parity]: V_j and K_{j+1}
  uint64_t* kv_empty = bars + 3;
  uint64_t* s_full = bars + 3 + kStages;
  uint64_t* p_ready = s_full + 2;  // [tile][half]
  uint64_t* o_final = s_full + 6;
  uint64_t* drain = s_full + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOffset);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::kMiscOffset + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Work unit -> tile -> (query block, head, batch); for causal calls the walk starts at the
  // last query block: the heaviest tiles first.
  int part = -1, split_tile = 0;
  const int tile = SPLIT ? unit_tile(p, static_cast<int>(blockIdx.x), &part, &split_tile)
                         : static_cast<int>(blockIdx.x);
  const TileAt at = tile_at(p, tile);
  const int qb = at.qb, head = at.head, b = at.b;
  const int kv_head = (head + p.q_base) / p.group - p.kv_base;
  const int q0 = qb * (kQTiles * kBlockM);
  int kv_end = p.seq_k;
  if (p.causal) kv_end = min(p.seq_k, max(0, q0 + kQTiles * kBlockM + p.causal_offset));
  const int n_blocks = (kv_end + kBlockN - 1) / kBlockN;
  // this unit's key blocks: [kv_first, kv_first + n_kv), kv_first even (the softmax loop runs
  // over absolute block numbers and takes its barrier parity from them)
  int kv_first = 0, n_kv = n_blocks;
  if (SPLIT && part >= 0) {
    const int pairs = n_blocks / 2;
    kv_first = 2 * (part * pairs / p.parts);
    n_kv = (part + 1 == p.parts ? n_blocks : 2 * ((part + 1) * pairs / p.parts)) - kv_first;
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(&kv_full[0], 1);
    mbar_init(&kv_full[1], 1);
    for (int i = 0; i < kStages; ++i) mbar_init(&kv_empty[i], 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_ready[2 * s], kBlockM);
      mbar_init(&p_ready[2 * s + 1], kBlockM);
      mbar_init(&o_final[s], 1);
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 8) {
    tmem_alloc(tmem_slot, 512);
    tc_fence_before();
  }
  if (warp == 9 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 8) {
    // ------------------------------------------------------------------ softmax warpgroups
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    const int s = warp >> 2;
    const int quarter = warp & 3;
    const int q_row = q0 + s * kBlockM + quarter * 32 + lane;
    const uint32_t lane_bits = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_bits + static_cast<uint32_t>(s * kBlockN);
    const uint32_t tO = tmem + lane_bits + 256u + static_cast<uint32_t>(s * HD);
    const int visible = q_row + p.causal_offset;  // last key column this row sees (causal)
    // FP8: a row's scores carry its Q block scale; the columns' K scales are applied per key
    float scale = p.scale_log2;
    const float* k_scale_row = nullptr;
    if constexpr (FP8) {
      const long long qh = static_cast<long long>(b) * p.heads_q + head;
      scale *= (q_row < p.seq_q) ? p.q_scale[qh * p.scale_seq + q_row] : 0.f;
      k_scale_row = p.k_scale + (static_cast<long long>(b) * p.heads_kv + kv_head) * p.scale_seq;
    }
    float m = -INFINITY;  // running max, log2 domain, of the probabilities' reference point
    float l = 0.f;        // running row sum against m
    bool ok = true;
    // j: absolute key block; kv_first is even, so j & 1 is also the parity of the local count
    const int kv_stop = kv_first + n_kv;
    for (int j = kv_first; j < kv_stop; ++j) {
      if (!mbar_wait(&s_full[s], j & 1, abort, p.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t r0[32], r1[32], r2[32], r3[32];
      tmem_ld32(tS + 0, r0);
      tmem_ld32(tS + 32, r1);
      tmem_ld32(tS + 64, r2);
      tmem_ld32(tS + 96, r3);
      tmem_wait_ld();
      reg_fence(r0);
      reg_fence(r1);
      reg_fence(r2);
      reg_fence(r3);
      const int kv0 = walk_block(p, j, n_blocks) * kBlockN;
      // multipliers of the two 64-key halves (bf16: the softmax scale)
      float sc_lo = scale, sc_hi = scale;
      if constexpr (FP8) {
        bool split = false;
        for (int c = 0; c < p.n_cuts; ++c) {
          const int cut = p.cuts[c];
          split |= cut > kv0 && cut < kv0 + kBlockN && cut != kv0 + 64;
        }
        if (split) {  // a rank boundary inside a half: each key's own scale
          const float4* ks = reinterpret_cast<const float4*>(k_scale_row + kv0);
          scale_chunk(r0, ks);
          scale_chunk(r1, ks + 8);
          scale_chunk(r2, ks + 16);
          scale_chunk(r3, ks + 24);
        } else {  // one K block scale per half, folded into the exponent's multiplier
          sc_lo = scale * k_scale_row[kv0];
          sc_hi = scale * k_scale_row[kv0 + 64];
          // keys past the sequence have scale 0 and are masked: keep the multiplier positive
          if (!(sc_lo > 0.f)) sc_lo = scale;
          if (!(sc_hi > 0.f)) sc_hi = scale;
        }
      }
      const bool ragged = kv0 + kBlockN > p.seq_k;
      const bool diagonal = p.causal && kv0 + kBlockN - 1 > visible;
      if (ragged || diagonal) {
        const int limit = min(p.seq_k - 1, p.causal ? visible : p.seq_k - 1) - kv0;
        mask_chunk(r0, limit);
        mask_chunk(r1, limit - 32);
        mask_chunk(r2, limit - 64);
        mask_chunk(r3, limit - 96);
      }
      // row max: four independent 3-input chains, one per chunk, scaled per half
      const float mlo = fmaxf(chunk_max(r0), chunk_max(r1));
      const float mhi = fmaxf(chunk_max(r2), chunk_max(r3));
      const float mt = fmaxf(mlo == -INFINITY ? -INFINITY : mlo * sc_lo,
                             mhi == -INFINITY ? -INFINITY : mhi * sc_hi);
      const float m_new = fmaxf(m, mt);
      // Split kernel: a row whose max is still -inf has seen only masked keys or none yet (its
      // part's first block), its O is zero or not yet written (the first PV overwrites it), so
      // it takes the new max without a rescale. Whole-tile kernel: the first block sets the max.
      if (!SPLIT && j == 0) {
        m = m_new;
      } else if (__any_sync(0xffffffffu, (!SPLIT || m != -INFINITY) &&
                                             m_new > m + (FP8 ? kRescaleLog2Fp8 : kRescaleLog2))) {
        // O row rescale: this warp's rows, once PV of the previous tile completed (the commit
        // behind s_full covers every earlier MMA of the issuing thread).
        const float factor = (m == -INFINITY) ? 0.f : ex2_approx(m - m_new);
        l *= factor;
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
          reg_fence(o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
          tmem_st32(tO + c * 32, o);
        }
        m = m_new;
      }
      if (SPLIT && m == -INFINITY) m = m_new;
      const float mu = (m == -INFINITY) ? 0.f : m;
      const float2 scale_lo = make_float2(sc_lo, sc_lo), scale_hi = make_float2(sc_hi, sc_hi);
      float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
      if constexpr (FP8) {
        // P as e4m3 codes of 2^(t + 8) (≤ 256·2^0.5 < 448); the row sum carries the same 2^8
        const float2 negm2 = make_float2(kPScaleLog2 - mu, kPScaleLog2 - mu);
        uint32_t pk[16];
        exp_chunk_fp8(r0, scale_lo, negm2, acc0, pk);
        exp_chunk_fp8(r1, scale_lo, negm2, acc1, pk + 8);
        tmem_st16(tS + 0, pk);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_ready[2 * s]);
        exp_chunk_fp8(r2, scale_hi, negm2, acc0, pk);
        exp_chunk_fp8(r3, scale_hi, negm2, acc1, pk + 8);
        tmem_st16(tS + 16, pk);
      } else {
        const float2 negm2 = make_float2(-mu, -mu);
        uint32_t pk[16];
        // first half of P (keys 0..63): the MMA starts its product while the rest is formed
        exp_chunk(r0, scale_lo, negm2, acc0, pk);
        tmem_st16(tS + 0, pk);
        exp_chunk(r1, scale_lo, negm2, acc1, pk);
        tmem_st16(tS + 16, pk);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_ready[2 * s]);
        exp_chunk(r2, scale_hi, negm2, acc0, pk);
        tmem_st16(tS + 32, pk);
        exp_chunk(r3, scale_hi, negm2, acc1, pk);
        tmem_st16(tS + 48, pk);
      }
      const float2 acc = __fadd2_rn(acc0, acc1);
      l += acc.x + acc.y;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_ready[2 * s + 1]);
    }
    // ------------------------------------------------------------------------- epilogue
    // Everything the epilogue needs beyond (m, l, ok, n_kv) is derived again here, from fresh
    // index reads, so that it holds no register through the loop above.
    {
    const int e_tid = fresh_tid();
    const int e_s = e_tid >> 7;
    const int quarter = (e_tid >> 5) & 3;
    const int e_lane = e_tid & 31;
    int part = -1, split_tile = 0;
    const int e_tile =
        SPLIT ? unit_tile(p, fresh_ctaid(), &part, &split_tile) : fresh_ctaid();
    const TileAt e_at = tile_at(p, e_tile);
    const int head = e_at.head;
    const int b = e_at.b;
    const int kv_head = (head + p.q_base) / p.group - p.kv_base;
    const int q_row = e_at.qb * (kQTiles * kBlockM) +
                      e_s * kBlockM + quarter * 32 + e_lane;
    const uint32_t e_tO = *reinterpret_cast<volatile uint32_t*>(tmem_slot) +
                          (static_cast<uint32_t>(quarter * 32) << 16) + 256u +
                          static_cast<uint32_t>(e_s * HD);
    if (ok && n_kv > 0) {
      ok = mbar_wait(&o_final[e_s], 0, abort, p.status);
      tc_fence_after();
    }
    const bool valid = q_row < p.seq_q;
    __nv_bfloat16* dst;
    if (p.scatter) {
      // the row's owner: the rank whose sequence rows contain it (rows are contiguous per rank)
      int owner = 0;
      while (owner + 1 < p.world && q_row >= p.row_start[owner + 1]) ++owner;
      dst = p.outs[owner] + static_cast<long long>(b) * p.outs_strides[owner][2] +
            static_cast<long long>(q_row - p.row_start[owner]) * p.outs_strides[owner][0] +
            static_cast<long long>(head + p.head_offset) * p.outs_strides[owner][1];
    } else {
      dst = p.out + static_cast<long long>(b) * p.out_b +
            static_cast<long long>(q_row) * p.out_s + static_cast<long long>(head) * p.out_h;
    }
    // 32 fp32 columns of the row's O (against its row sum's reference) -> 16 bf16 pairs
    auto pack_chunk = [&](int c, const uint32_t (&o)[32], float inv, uint32_t (&packed)[16]) {
      if constexpr (FP8) {  // V's per-channel scales
        const float* vs = p.v_scale +
                          (static_cast<long long>(b) * p.heads_kv + kv_head) * HD + c * 32;
#pragma unroll
        for (int i = 0; i < 16; ++i)
          packed[i] = pack_bf16x2(__uint_as_float(o[2 * i]) * inv * vs[2 * i],
                                  __uint_as_float(o[2 * i + 1]) * inv * vs[2 * i + 1]);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          packed[i] = pack_bf16x2(__uint_as_float(o[2 * i]) * inv,
                                  __uint_as_float(o[2 * i + 1]) * inv);
      }
    };
    // ... straight to the row's destination, 16 bytes a store
    auto emit = [&](int c, const uint32_t (&o)[32], float inv) {
      uint32_t packed[16];
      pack_chunk(c, o, inv, packed);
      if (valid) {
        uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          d4[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2],
                             packed[4 * i + 3]);
      }
    };
    if (SPLIT && part >= 0) {
      // ------------------------------------------------- one part of a split tile
      // Leave this part's rows, then count in; the last part of the tile merges every part's
      // rows (each against the largest max) and writes the output. Every thread of the
      // warpgroup reaches both barriers, so none waits on a thread that gave up.
      const int row = quarter * 32 + e_lane;
      const long long slot0 = static_cast<long long>(split_tile) * p.parts * 2 + e_s;  // part 0
      if (ok) {
        const long long slot = slot0 + 2LL * part;
        // [HD/4 float4 columns][128 rows]: a warp's 32 rows are 512 contiguous bytes per access
        float4* wo = reinterpret_cast<float4*>(p.ws_o) + slot * (HD / 4) * kBlockM + row;
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(e_tO + c * 32, o);
          tmem_wait_ld();
          reg_fence(o);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            wo[(c * 8 + i) * kBlockM] = make_float4(__uint_as_float(o[4 * i]), __uint_as_float(o[4 * i + 1]),
                                        __uint_as_float(o[4 * i + 2]),
                                        __uint_as_float(o[4 * i + 3]));
        }
        p.ws_ml[slot * kBlockM + row] = make_float2(m, l);
        __threadfence();
      }
      // barriers 1 and 2: the warpgroups of query tiles 0 and 1
      const bool all_ok = e_s == 0 ? named_bar_and<1, kBlockM>(ok) : named_bar_and<2, kBlockM>(ok);
      volatile int* last_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOffset + 8) + e_s;
      if (quarter == 0 && e_lane == 0) {
        int last = 0;
        if (all_ok) {
          int* counter = p.counters + split_tile * 2 + e_s;
          last = atomicAdd(counter, 1) == p.parts - 1;
          if (last) atomicExch(counter, 0);
        }
        *last_flag = last;
      }
      if (e_s == 0) named_bar_sync<1, kBlockM>();
      else named_bar_sync<2, kBlockM>();
      if (*last_flag) {
        __threadfence();
        float mx = -INFINITY;
        for (int q = 0; q < p.parts; ++q)
          mx = fmaxf(mx, __ldcg(&p.ws_ml[(slot0 + 2LL * q) * kBlockM + row]).x);
        float sum = 0.f;
        for (int q = 0; q < p.parts; ++q) {
          const float2 ml = __ldcg(&p.ws_ml[(slot0 + 2LL * q) * kBlockM + row]);
          if (ml.x != -INFINITY) sum += ml.y * ex2_approx(ml.x - mx);
        }
        const float inv = (sum > 0.f && mx != -INFINITY) ? 1.f / sum : 0.f;
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          float acc[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[i] = 0.f;
          for (int q = 0; q < p.parts; ++q) {
            const long long slot = slot0 + 2LL * q;
            const float2 ml = __ldcg(&p.ws_ml[slot * kBlockM + row]);
            const float w = ml.x == -INFINITY ? 0.f : ex2_approx(ml.x - mx);
            const float4* src = reinterpret_cast<const float4*>(p.ws_o) +
                                (slot * (HD / 4) + c * 8) * kBlockM + row;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 x = __ldcg(src + i * kBlockM);
              acc[4 * i] = fmaf(w, x.x, acc[4 * i]);
              acc[4 * i + 1] = fmaf(w, x.y, acc[4 * i + 1]);
              acc[4 * i + 2] = fmaf(w, x.z, acc[4 * i + 2]);
              acc[4 * i + 3] = fmaf(w, x.w, acc[4 * i + 3]);
            }
          }
          uint32_t o[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(acc[i]);
          emit(c, o, inv);
        }
      }
    } else if (ok) {
      // rows that saw no key (bottom-right causal with seq_q > seq_k) are written as zeros
      const float inv = (l > 0.f && m != -INFINITY) ? 1.f / l : 0.f;
      // With a scatter most rows go to other GPUs' memory. A warp's 32 rows are staged in its
      // quarter of this tile's Q buffer (free: every MMA that read it completed before o_final,
      // and a bf16 Q tile is exactly the 128 rows × HD bf16 of the output tile)
      // and leave as whole rows, CPR lanes a row, so each store instruction writes whole 32-byte
      // sectors of RPI rows instead of one 16-byte piece of 32 rows.
      constexpr int CPR = HD / 8;  // 16-byte chunks a row
      constexpr int RPI = 32 / CPR;  // rows a store instruction
      // (bf16 only: the FP8 kernel's e4m3 Q tile is half the bytes of a bf16 output tile)
      const bool staged = !FP8 && p.scatter && n_kv > 0;
      uint8_t* stage = reinterpret_cast<uint8_t*>(
                           (reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                           ~static_cast<uintptr_t>(1023)) +
                       L::kQOffset + e_s * L::kTileBytes + quarter * (32 * HD * 2);
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t o[32];
        if (n_kv > 0) {
          tmem_ld32(e_tO + c * 32, o);
          tmem_wait_ld();
          reg_fence(o);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        if (staged) {
          uint32_t packed[16];
          pack_chunk(c, o, inv, packed);
          // chunk j of row r sits at chunk j ^ (r mod CPR): the row's writers and the
          // cooperative readers below both spread over the banks
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int j = c * 4 + i;
            *reinterpret_cast<uint4*>(stage + e_lane * (HD * 2) + ((j ^ (e_lane % CPR)) * 16)) =
                make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
          }
        } else {
          emit(c, o, inv);
        }
      }
      if (staged) {
        __syncwarp();
        const int sub = e_lane / CPR, ch = e_lane % CPR;
        const unsigned long long my_dst = reinterpret_cast<unsigned long long>(dst);
#pragma unroll 4
        for (int r0 = 0; r0 < 32; r0 += RPI) {
          const int r = r0 + sub;
          const unsigned long long row_dst = __shfl_sync(0xffffffffu, my_dst, r);
          const bool row_valid = __shfl_sync(0xffffffffu, valid, r);
          const uint4 v =
              *reinterpret_cast<const uint4*>(stage + r * (HD * 2) + ((ch ^ (r % CPR)) * 16));
          if (row_valid) reinterpret_cast<uint4*>(row_dst)[ch] = v;
        }
      }
    }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------------------ TMA producer
    // The whole warp walks the schedule (warp-uniform control flow); one elected lane issues.
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
    // Tiles in order K_0, V_0, K_1, V_1, ... of this unit's walk: tile i sits in ring slot
    // i % kStages. Q and K_0 complete q_full; walk step j's V_j and K_{j+1} complete
    // kv_full[j & 1] together, so the MMA warp waits once per step for both.
    auto tile_block = [&](int i) { return walk_block(p, kv_first + (i >> 1), n_blocks); };
    auto load_tile = [&](int i, uint64_t* bar) {
      const int stage = i % kStages;
      const CUtensorMap* map = (i & 1) ? &tm_v : &tm_k;
      for (int box = 0; box < L::kBoxes; ++box)
        tma_load_4d(sKV + stage * L::kTileBytes + box * L::kBoxBytes, map, bar, box * 64,
                    tile_block(i) * kBlockN, kv_head, b);
    };
    // Rows [r0, r1) resident: wait for each source not seen yet (warp-uniform; lane 0 polls),
    // then order the flag reads before the tensor copies that read the rows (async proxy).
    uint32_t seen = p.arrive != nullptr ? (1u << p.arrive_self) : 0xffffffffu;
    auto resident = [&](int r0, int r1) -> bool {
      uint32_t need = 0;
      for (int src = 0; src < p.n_src; ++src)
        if (p.src_start[src] < r1 && p.src_start[src + 1] > r0) need |= 1u << src;
      need &= ~seen;
      if (need == 0) return true;
      while (need != 0) {
        const int src = __ffs(need) - 1;
        bool arrived = true;
        if (lane == 0)
          arrived = wait_flag(p.arrive + src, p.arrive_seq, p.arrive_limit_ns, abort, p.status);
        if (!__shfl_sync(0xffffffffu, arrived, 0)) return false;
        seen |= 1u << src;
        need &= need - 1;
      }
      asm volatile("fence.proxy.async.global;" ::: "memory");
      return true;
    };
    bool issued_q = false;
    int pairs = 0;
    if (resident(q0, q0 + kQTiles * kBlockM) &&
        (n_kv == 0 || resident(tile_block(0) * kBlockN, tile_block(0) * kBlockN + kBlockN))) {
      if (elect_one()) {
        mbar_expect_tx(q_full, kQTiles * L::kTileBytes + (n_kv > 0 ? L::kTileBytes : 0));
        for (int s = 0; s < kQTiles; ++s)
          for (int box = 0; box < L::kBoxes; ++box)
            tma_load_4d(sQ + s * L::kTileBytes + box * L::kBoxBytes, &tm_q, q_full, box * 64,
                        q0 + s * kBlockM, head, b);
        if (n_kv > 0) load_tile(0, q_full);
      }
      __syncwarp();
      issued_q = true;
      for (int j = 0; j < n_kv; ++j) {
        const int iv = 2 * j + 1, ik = 2 * j + 2;
        const bool more = j + 1 < n_kv;
        // both slots free: the MMAs that read their previous tiles have completed
        if (iv >= kStages &&
            !warp_wait(&kv_empty[iv % kStages], ((iv / kStages) - 1) & 1, abort, p.status))
          break;
        if (more && ik >= kStages &&
            !warp_wait(&kv_empty[ik % kStages], ((ik / kStages) - 1) & 1, abort, p.status))
          break;
        const int bv = tile_block(iv) * kBlockN, bk = more ? tile_block(ik) * kBlockN : bv;
        if (!resident(bv, bv + kBlockN) || !resident(bk, bk + kBlockN)) break;
        if (elect_one()) {
          mbar_expect_tx(&kv_full[j & 1], (more ? 2 : 1) * L::kTileBytes);
          load_tile(iv, &kv_full[j & 1]);
          if (more) load_tile(ik, &kv_full[j & 1]);
        }
        __syncwarp();
        pairs = j + 1;
      }
    }
    // Every copy this CTA issued lands before the CTA unwinds (already true on the normal path,
    // where the MMA warp waited for each one).
    if (issued_q) drain_wait(q_full, 0, p.status);
    for (int j = max(0, pairs - 2); j < pairs; ++j)
      drain_wait(&kv_full[j & 1], (j >> 1) & 1, p.status);
    __syncwarp();
  } else if (warp == 9) {
    // ------------------------------------------------------------------------- MMA issuer
    // Warp-uniform schedule, one elected lane issuing every MMA and commit (a commit tracks
    // the MMAs of the thread that executes it, and elect.sync picks the same lane each time in
    // a converged warp). Descriptors are a base per operand plus compile-time offsets.
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
    if (n_kv > 0) {
      constexpr uint32_t kIdescQK =
          FP8 ? idesc_e4m3_f32(kBlockM, kBlockN, false) : idesc_bf16_f32(kBlockM, kBlockN, false);
      constexpr uint32_t kIdescPV =
          FP8 ? idesc_e4m3_f32(kBlockM, HD, true) : idesc_bf16_f32(kBlockM, HD, true);
      // one MMA takes 32 bytes of K: 16 bf16 or 32 e4m3 elements
      constexpr int kQKSteps = HD * L::kElem / 32;
      constexpr int kPVSteps = kBlockN * L::kElem / 32;
      constexpr int kPVRows = 32 / L::kElem;  // key rows per PV step
      const uint64_t dq = smem_desc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t dk = smem_desc_sw128(smem_u32(sKV), 16, 1024);
      const uint64_t dv = smem_desc_sw128(smem_u32(sKV), L::kBoxBytes, 1024);
      constexpr uint64_t kTileStep = L::kTileBytes >> 4;  // descriptor units (16 bytes)
      auto issue_qk = [&](int s, int stage) {
        const uint64_t qa = dq + static_cast<uint64_t>(s) * kTileStep;
        const uint64_t ka = dk + static_cast<uint64_t>(stage) * kTileStep;
#pragma unroll
        for (int kk = 0; kk < kQKSteps; ++kk) {
          // K-major 128-byte swizzle: each step moves 32 bytes inside a row's atom; every 4
          // steps move to the next box of 128-byte rows.
          const uint64_t off = static_cast<uint64_t>(((kk >> 2) * L::kBoxBytes + (kk & 3) * 32) >> 4);
          if constexpr (FP8) mma_ss_f8(tmem + s * kBlockN, qa + off, ka + off, kIdescQK, kk > 0 ? 1u : 0u);
          else mma_ss(tmem + s * kBlockN, qa + off, ka + off, kIdescQK, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int s, int stage, uint32_t accumulate, int half) {
        const uint64_t va = dv + static_cast<uint64_t>(stage) * kTileStep;
#pragma unroll
        for (int kk = half * (kPVSteps / 2); kk < (half + 1) * (kPVSteps / 2); ++kk) {
          // V is MN-major for this product: kPVRows key rows of 128 bytes per step; with bf16
          // the two 64-column halves of the head dimension are one box (16 KB) apart. P's
          // step is 8 TMEM columns either way (16 bf16 or 32 e4m3 codes a lane).
          const uint64_t vo = static_cast<uint64_t>((kk * kPVRows * 128) >> 4);
          if constexpr (FP8)
            mma_ts_f8(tmem + 256u + s * HD, tmem + s * kBlockN + kk * 8, va + vo, kIdescPV,
                      kk > 0 ? 1u : accumulate);
          else
            mma_ts(tmem + 256u + s * HD, tmem + s * kBlockN + kk * 8, va + vo, kIdescPV,
                   kk > 0 ? 1u : accumulate);
        }
      };
      bool ok = warp_wait(q_full, 0, abort, p.status);  // Q and K_0
      if (ok) {
        tc_fence_after();
        if (elect_one()) {
          issue_qk(0, 0);
          mma_commit(&s_full[0]);
          issue_qk(1, 0);
          mma_commit(&s_full[1]);
          mma_commit(&kv_empty[0]);
        }
        __syncwarp();
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        const int iv = 2 * j + 1, ik = 2 * j + 2;
        const int sv = iv % kStages, sk = ik % kStages;
        const bool more = j + 1 < n_kv;
        const uint32_t acc = j > 0 ? 1u : 0u;
        // V_j and K_{j+1}
        if (!(ok = warp_wait(&kv_full[j & 1], (j >> 1) & 1, abort, p.status))) break;
        if (!(ok = warp_wait(&p_ready[0], j & 1, abort, p.status))) break;
        tc_fence_after();
        if (elect_one()) issue_pv(0, sv, acc, 0);
        __syncwarp();
        if (!(ok = warp_wait(&p_ready[1], j & 1, abort, p.status))) break;
        tc_fence_after();
        if (elect_one()) {
          issue_pv(0, sv, acc, 1);
          if (!more) mma_commit(&o_final[0]);
          if (more) {
            issue_qk(0, sk);
            mma_commit(&s_full[0]);
          }
        }
        __syncwarp();
        if (!(ok = warp_wait(&p_ready[2], j & 1, abort, p.status))) break;
        tc_fence_after();
        if (elect_one()) issue_pv(1, sv, acc, 0);
        __syncwarp();
        if (!(ok = warp_wait(&p_ready[3], j & 1, abort, p.status))) break;
        tc_fence_after();
        if (elect_one()) {
          issue_pv(1, sv, acc, 1);
          mma_commit(&kv_empty[sv]);
          if (!more) mma_commit(&o_final[1]);
          if (more) {
            issue_qk(1, sk);
            mma_commit(&s_full[1]);
            mma_commit(&kv_empty[sk]);
          }
        }
        __syncwarp();
      }
      // Every MMA this warp issued completes before TMEM is released.
      if (elect_one()) mma_commit(drain);
      __syncwarp();
      drain_wait(drain, 0, p.status);
    }
    __syncwarp();
  } else {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------------- host side
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                 const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiled encode_tiled() {
  static EncodeTiled fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(ptr);
  }
  return fn;
}

// A 4-D tensor map over (head_dim, seq, heads, batch) with element strides
// (1, s_stride, h_stride, b_stride) and a box of 128 bytes × 128 rows in 128-byte swizzle:
// 64 bf16 or 128 e4m3 elements a row.
static int make_map(CUtensorMap* map, const void* base, int elem_bytes, int head_dim, int seq,
                    int heads, int batch, long long s_stride, long long h_stride,
                    long long b_stride) {
  EncodeTiled fn = encode_tiled();
  if (fn == nullptr) return cudaErrorNotSupported;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(seq),
                        static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(s_stride) * elem_bytes,
                           static_cast<cuuint64_t>(h_stride) * elem_bytes,
                           static_cast<cuuint64_t>(b_stride) * elem_bytes};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(128 / elem_bytes), 128, 1, 1};
  cuuint32_t elem[4] = {1, 1, 1, 1};
  const CUtensorMapDataType type =
      elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUresult r = fn(map, type, 4, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : cudaErrorInvalidValue;
}

// ------------------------------------------------------------------ split of the last wave
// A CTA owns a tile for its whole key range, so when the tiles are not a whole number of waves
// of one CTA per SM, the last wave leaves SMs idle (C2 at Ulysses degree 8: 390 tiles on 148
// SMs = 2.64 waves, the third 64 % full). The tiles past the last whole wave can instead run
// as `parts` CTAs each over a share of the keys, merged by the last one to finish. The plan
// minimises a wave count model in units of one key block's time per CTA, with a fixed cost per
// CTA (start-up, pipeline fill, epilogue) and per merged part.
constexpr double kUnitCost = 4.0;    // key blocks' worth of time a CTA spends outside its loop
constexpr double kMergeCost = 0.5;   // per part read back by the merging CTA
constexpr int kMaxParts = 16;
constexpr long long kMaxWholeWaves = 16;
constexpr size_t kMaxWorkspace = size_t(1) << 30;

struct SplitPlan {
  long long n_full;
  int parts;
  long long n_split;
};

static size_t split_bytes(long long n_split, int parts, int head_dim) {
  const size_t rows = static_cast<size_t>(n_split) * parts * kQTiles * kBlockM;
  const size_t counters = (static_cast<size_t>(n_split) * kQTiles * sizeof(int) + 255) & ~size_t(255);
  return counters + rows * sizeof(float2) + rows * head_dim * sizeof(float);
}

static SplitPlan plan_split(long long tiles, int n_blocks, int sms, int head_dim) {
  SplitPlan best = {tiles, 1, 0};
  const char* env = getenv("COZY_ATTENTION_SPLIT");
  if (env != nullptr && env[0] == '0' && env[1] == '\0') return best;
  if (sms <= 0 || n_blocks < 2 || tiles <= 0) return best;
  // Past many whole waves the SMs' finishing times have drifted apart by more than a tile, and
  // the ones that finish early absorb the partial wave: measured on B200 at the C2 shape, 21.08
  // waves gain nothing from a split (1185 vs 1191 TFLOP/s), 10.5 waves gain 2.8 %, 2.6 waves 12 %.
  if (tiles / sms >= kMaxWholeWaves) return best;
  const double unsplit = static_cast<double>((tiles + sms - 1) / sms) * (n_blocks + kUnitCost);
  // a clear gain only: a split costs workspace traffic the model leaves out
  double best_time = 0.95 * unsplit;
  const long long whole = tiles / sms;
  for (long long waves = whole; waves >= 0 && waves >= whole - 1; --waves) {
    const long long tail = tiles - waves * sms;
    if (tail <= 0) continue;
    // parts start on even key blocks: at least two blocks each
    for (int parts = 2; parts <= kMaxParts && parts <= n_blocks / 2; ++parts) {
      const long long units = tail * parts;
      const long long split_waves = (units + sms - 1) / sms;
      const int longest = 2 * ((n_blocks / 2 + parts - 1) / parts) + (n_blocks & 1);
      const double t = waves * (n_blocks + kUnitCost) +
                       split_waves * (longest + kUnitCost + kMergeCost * parts);
      if (t < best_time && split_bytes(tail, parts, head_dim) <= kMaxWorkspace) {
        best_time = t;
        best = {tiles - tail, parts, tail};
      }
    }
  }
  return best;
}

// Split workspace, one per (device, stream): launches on one stream run in order, so they can
// share it; launches on different streams may overlap and must not. Grows, never shrinks.
// A launch made while its stream is being captured into a graph never uses it (it runs
// unsplit): a graph keeps the address it was captured with and may be replayed on any stream,
// beside eager launches that share this workspace or after it has grown and been freed.
struct Workspace {
  void* ptr = nullptr;
  size_t bytes = 0;
};

static void* split_workspace(int device, cudaStream_t stream, size_t bytes) {
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &capture) != cudaSuccess ||
      capture != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return nullptr;
  }
  static std::mutex mutex;
  static std::map<std::pair<int, uintptr_t>, Workspace> spaces;
  std::lock_guard<std::mutex> lock(mutex);
  Workspace& w = spaces[{device, reinterpret_cast<uintptr_t>(stream)}];
  if (w.bytes >= bytes) return w.ptr;
  if (w.ptr != nullptr) {
    // earlier launches on this stream may still read the old buffer
    if (cudaStreamSynchronize(stream) != cudaSuccess || cudaFree(w.ptr) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    w = Workspace{};
  }
  const size_t want = std::max(bytes, size_t(64) << 20);
  if (cudaMalloc(&w.ptr, want) != cudaSuccess) {
    cudaGetLastError();
    w = Workspace{};
    return nullptr;
  }
  w.bytes = want;
  return w.ptr;
}

static int sm_count(int device) {
  static int counts[64] = {};
  if (device >= 64) return 0;
  if (counts[device] == 0)
    cudaDeviceGetAttribute(&counts[device], cudaDevAttrMultiProcessorCount, device);
  return counts[device];
}

// Where the split's workspace comes from: `given` (a caller's buffer of `given_bytes`; too
// small: the launch runs unsplit) or, with given == nullptr, the library's per-stream one.
struct WorkspaceChoice {
  void* given;
  size_t given_bytes;
};

template <int HD, bool FP8>
static int launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                  AttentionParams& p, bool allow_split, const WorkspaceChoice* choice,
                  cudaStream_t stream) {
  using L = AttentionSmem<HD, FP8>;
  static bool configured[64] = {};
  int device = 0;
  cudaGetDevice(&device);
  if (device < 64 && !configured[device]) {
    cudaError_t e = cudaFuncSetAttribute(attention_fwd_kernel<HD, FP8, false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(attention_fwd_kernel<HD, FP8, true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return e;
    configured[device] = true;
  }
  const long long tiles = static_cast<long long>(p.q_blocks) * p.heads_q * p.batch;
  SplitPlan plan = {tiles, 1, 0};
  // causal tiles differ in length and are ordered heaviest first: they are not split
  if (allow_split && !p.causal)
    plan = plan_split(tiles, (p.seq_k + kBlockN - 1) / kBlockN, sm_count(device), HD);
  p.n_full = static_cast<int>(plan.n_full);
  p.parts = plan.parts;
  p.ws_o = nullptr;
  p.ws_ml = nullptr;
  p.counters = nullptr;
  if (plan.n_split > 0) {
    const size_t need = split_bytes(plan.n_split, plan.parts, HD);
    uint8_t* ws = nullptr;
    if (choice != nullptr && choice->given != nullptr)
      ws = choice->given_bytes >= need ? static_cast<uint8_t*>(choice->given) : nullptr;
    else
      ws = static_cast<uint8_t*>(split_workspace(device, stream, need));
    if (ws == nullptr) {
      p.n_full = static_cast<int>(tiles);
      p.parts = 1;
      plan.n_split = 0;
    } else {
      const size_t rows = static_cast<size_t>(plan.n_split) * plan.parts * kQTiles * kBlockM;
      const size_t counter_bytes =
          (static_cast<size_t>(plan.n_split) * kQTiles * sizeof(int) + 255) & ~size_t(255);
      p.counters = reinterpret_cast<int*>(ws);
      p.ws_ml = reinterpret_cast<float2*>(ws + counter_bytes);
      p.ws_o = reinterpret_cast<float*>(ws + counter_bytes + rows * sizeof(float2));
      cudaError_t e = cudaMemsetAsync(p.counters, 0, counter_bytes, stream);
      if (e != cudaSuccess) return e;
    }
  }
  const long long units = p.n_full + plan.n_split * plan.parts;
  if (units > 0x7fffffffLL) return cudaErrorInvalidValue;
  if (plan.n_split > 0)
    attention_fwd_kernel<HD, FP8, true>
        <<<static_cast<unsigned>(units), kThreads, L::kAlloc, stream>>>(mq, mk, mv, p);
  else
    attention_fwd_kernel<HD, FP8, false>
        <<<static_cast<unsigned>(units), kThreads, L::kAlloc, stream>>>(mq, mk, mv, p);
  return cudaGetLastError();
}

struct Fp8Operands {
  const float* q_scale;
  const float* k_scale;
  const float* v_scale;
  long long scale_seq;
  const int* cuts;
  int n_cuts;
};

static int attention_launch(const void* q, const void* k, const void* v, void* out, int batch,
                            int seq_q, int seq_k, int heads_q, int heads_kv, int head_dim,
                            const long long* q_strides, const long long* k_strides,
                            const long long* v_strides, const long long* o_strides,
                            const CozyHeadMap* head_map, const CozyScatter* scatter, int causal,
                            float scale, int* status, const Fp8Operands* fp8, bool allow_split,
                            const Arrival* arrival, const WorkspaceChoice* choice,
                            cudaStream_t stream) {
  if (head_dim != 64 && head_dim != 128) return cudaErrorNotSupported;
  if (fp8 != nullptr && head_dim != 128) return cudaErrorNotSupported;
  if (batch <= 0 || seq_q <= 0 || seq_k <= 0 || heads_q <= 0 || heads_kv <= 0)
    return cudaErrorInvalidValue;
  CozyHeadMap map = {heads_q / heads_kv, 0, 0};
  if (head_map != nullptr) {
    map = *head_map;
  } else if (heads_q % heads_kv != 0) {
    return cudaErrorInvalidValue;
  }
  if (map.group <= 0) return cudaErrorInvalidValue;
  // every query head's key/value head must exist
  const int kv_first = (0 + map.q_base) / map.group - map.kv_base;
  const int kv_last = (heads_q - 1 + map.q_base) / map.group - map.kv_base;
  if (kv_first < 0 || kv_last >= heads_kv) return cudaErrorInvalidValue;
  if (batch > 65535 || heads_q > 65535) return cudaErrorInvalidValue;
  if (static_cast<long long>(batch) * heads_q * ((seq_q + 255) / 256) > 0x7fffffffLL)
    return cudaErrorInvalidValue;
  const void* ptrs[4] = {q, k, v, scatter ? q : out};
  for (const void* ptr : ptrs)
    if (ptr == nullptr || reinterpret_cast<uintptr_t>(ptr) % 16 != 0) return cudaErrorInvalidValue;
  // operand rows must start on 16-byte boundaries (TMA): 8 bf16 or 16 e4m3 elements
  const long long in_align = fp8 != nullptr ? 16 : 8;
  const long long* ins[3] = {q_strides, k_strides, v_strides};
  for (const long long* st : ins)
    for (int i = 0; i < 3; ++i)
      if (st[i] <= 0 || st[i] % in_align != 0) return cudaErrorInvalidValue;
  if (scatter == nullptr)
    for (int i = 0; i < 3; ++i)
      if (o_strides[i] <= 0 || o_strides[i] % 8 != 0) return cudaErrorInvalidValue;
  if (fp8 != nullptr) {
    if (!fp8->q_scale || !fp8->k_scale || !fp8->v_scale) return cudaErrorInvalidValue;
    if (fp8->n_cuts < 0 || fp8->n_cuts > COZY_MAX_PEERS || (fp8->n_cuts > 0 && !fp8->cuts))
      return cudaErrorInvalidValue;
    // the kernel reads K scales 128 keys at a time: the scale rows are padded to whole tiles
    if (fp8->scale_seq < ((seq_k + 127) / 128) * 128 || fp8->scale_seq < seq_q ||
        fp8->scale_seq % 4 != 0 || reinterpret_cast<uintptr_t>(fp8->k_scale) % 16)
      return cudaErrorInvalidValue;
  }
  if (scatter != nullptr) {
    if (scatter->world < 1 || scatter->world > COZY_MAX_PEERS || scatter->head_offset < 0)
      return cudaErrorInvalidValue;
    if (scatter->row_start[0] != 0 || scatter->row_start[scatter->world] != seq_q)
      return cudaErrorInvalidValue;
    for (int w = 0; w < scatter->world; ++w) {
      if (scatter->row_start[w + 1] < scatter->row_start[w]) return cudaErrorInvalidValue;
      if (scatter->row_start[w + 1] == scatter->row_start[w]) continue;
      if (scatter->out[w] == nullptr || reinterpret_cast<uintptr_t>(scatter->out[w]) % 16)
        return cudaErrorInvalidValue;
      for (int i = 0; i < 3; ++i)
        if (scatter->strides[w][i] <= 0 || scatter->strides[w][i] % 8) return cudaErrorInvalidValue;
    }
  }
  const int eb = fp8 != nullptr ? 1 : 2;
  CUtensorMap mq, mk, mv;
  int e;
  if ((e = make_map(&mq, q, eb, head_dim, seq_q, heads_q, batch, q_strides[0], q_strides[1],
                    q_strides[2])))
    return e;
  if ((e = make_map(&mk, k, eb, head_dim, seq_k, heads_kv, batch, k_strides[0], k_strides[1],
                    k_strides[2])))
    return e;
  if ((e = make_map(&mv, v, eb, head_dim, seq_k, heads_kv, batch, v_strides[0], v_strides[1],
                    v_strides[2])))
    return e;
  AttentionParams p;
  p.batch = batch;
  p.seq_q = seq_q;
  p.seq_k = seq_k;
  p.heads_q = heads_q;
  p.heads_kv = heads_kv;
  p.group = map.group;
  p.q_base = map.q_base;
  p.kv_base = map.kv_base;
  p.causal = causal ? 1 : 0;
  p.causal_offset = seq_k - seq_q;
  p.q_blocks = (seq_q + kQTiles * kBlockM - 1) / (kQTiles * kBlockM);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_s = o_strides ? o_strides[0] : 0;
  p.out_h = o_strides ? o_strides[1] : 0;
  p.out_b = o_strides ? o_strides[2] : 0;
  p.status = status;
  p.scatter = 0;
  p.world = 1;
  p.head_offset = 0;
  if (scatter != nullptr) {
    p.scatter = 1;
    p.world = scatter->world;
    p.head_offset = scatter->head_offset;
    for (int w = 0; w <= scatter->world; ++w) p.row_start[w] = scatter->row_start[w];
    for (int w = 0; w < scatter->world; ++w) {
      p.outs[w] = static_cast<__nv_bfloat16*>(scatter->out[w]);
      for (int i = 0; i < 3; ++i) p.outs_strides[w][i] = scatter->strides[w][i];
    }
  }
  // walk orders: the last query block first; key blocks upwards
  p.q_turn = p.q_blocks - 1;
  p.q_seg = p.q_blocks;
  p.kv_turn = -1;
  p.arrive = nullptr;
  p.arrive_seq = 0;
  p.arrive_limit_ns = 0;
  p.n_src = 0;
  p.arrive_self = 0;
  if (arrival != nullptr) {
    if (arrival->flags == nullptr || arrival->n_src < 1 || arrival->n_src > COZY_MAX_PEERS ||
        arrival->self < 0 || arrival->self >= arrival->n_src || arrival->limit_ns <= 0 ||
        reinterpret_cast<uintptr_t>(arrival->flags) % 8 != 0 || seq_q != seq_k)
      return cudaErrorInvalidValue;
    if (arrival->src_start[0] != 0 || arrival->src_start[arrival->n_src] != seq_k)
      return cudaErrorInvalidValue;
    for (int r = 0; r < arrival->n_src; ++r)
      if (arrival->src_start[r + 1] < arrival->src_start[r]) return cudaErrorInvalidValue;
    p.arrive = arrival->flags;
    p.arrive_seq = arrival->seq;
    p.arrive_limit_ns = arrival->limit_ns;
    p.n_src = arrival->n_src;
    p.arrive_self = arrival->self;
    for (int r = 0; r <= arrival->n_src; ++r) p.src_start[r] = arrival->src_start[r];
    // This GPU's own rows are resident first: every tile's keys start there and walk down
    // through the sources in the order they arrive (each source sends to the ranks after it in
    // turn, so source self - 1 lands first); non-causal query blocks start there too.
    const int lo = arrival->src_start[arrival->self], hi = arrival->src_start[arrival->self + 1];
    if (hi > lo) {
      p.kv_turn = (hi - 1) / kBlockN;
      if (!causal) {
        // every head's query blocks over this GPU's rows run first, then the next source's
        const int rows_q = kQTiles * kBlockM;
        p.q_turn = (hi - 1) / rows_q;
        p.q_seg = min(p.q_blocks, max(1, (hi - 1) / rows_q - lo / rows_q + 1));
      }
    }
  }
  p.q_scale = p.k_scale = p.v_scale = nullptr;
  p.scale_seq = 0;
  p.n_cuts = 0;
  if (fp8 != nullptr) {
    p.q_scale = fp8->q_scale;
    p.k_scale = fp8->k_scale;
    p.v_scale = fp8->v_scale;
    p.scale_seq = fp8->scale_seq;
    p.n_cuts = fp8->n_cuts;
    for (int c = 0; c < fp8->n_cuts; ++c) p.cuts[c] = fp8->cuts[c];
    return launch<128, true>(mq, mk, mv, p, allow_split, choice, stream);
  }
  if (head_dim == 128) return launch<128, false>(mq, mk, mv, p, allow_split, choice, stream);
  return launch<64, false>(mq, mk, mv, p, allow_split, choice, stream);
}

int attention_forward(const void* q, const void* k, const void* v, void* out, int batch,
                      int seq_q, int seq_k, int heads_q, int heads_kv, int head_dim,
                      const long long* q_strides, const long long* k_strides,
                      const long long* v_strides, const long long* o_strides,
                      const CozyHeadMap* head_map, const CozyScatter* scatter, int causal,
                      float scale, int* status, cudaStream_t stream) {
  return attention_launch(q, k, v, out, batch, seq_q, seq_k, heads_q, heads_kv, head_dim,
                          q_strides, k_strides, v_strides, o_strides, head_map, scatter, causal,
                          scale, status, nullptr, true, nullptr, nullptr, stream);
}

// The split plan attention_forward takes on the current device for a non-FP8 call of this shape
// (FP8 calls take the same plan): `whole` tiles of 256 query rows run in one CTA each, the
// remaining tiles in `parts` CTAs each (parts = 1: nothing is split).
// As attention_split_plan, for a GPU of `sms` SMs (host arithmetic only: no device is needed).
int attention_split_plan_for(int batch, int seq_q, int seq_k, int heads_q, int head_dim,
                             int causal, int sms, long long* whole, int* parts) {
  if (whole == nullptr || parts == nullptr || batch <= 0 || seq_q <= 0 || seq_k <= 0 ||
      heads_q <= 0 || sms <= 0 || (head_dim != 64 && head_dim != 128))
    return cudaErrorInvalidValue;
  const long long tiles =
      static_cast<long long>(batch) * heads_q * ((seq_q + kQTiles * kBlockM - 1) / (kQTiles * kBlockM));
  SplitPlan plan = {tiles, 1, 0};
  if (!causal) plan = plan_split(tiles, (seq_k + kBlockN - 1) / kBlockN, sms, head_dim);
  *whole = plan.n_full;
  *parts = plan.parts;
  return cudaSuccess;
}

int attention_split_plan(int batch, int seq_q, int seq_k, int heads_q, int head_dim, int causal,
                         long long* whole, int* parts) {
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  return attention_split_plan_for(batch, seq_q, seq_k, heads_q, head_dim, causal,
                                  sm_count(device), whole, parts);
}

// As attention_forward, without the split of the last wave (which needs a workspace this
// library allocates): allocates nothing.
int attention_forward_unsplit(const void* q, const void* k, const void* v, void* out, int batch,
                              int seq_q, int seq_k, int heads_q, int heads_kv, int head_dim,
                              const long long* q_strides, const long long* k_strides,
                              const long long* v_strides, const long long* o_strides,
                              const CozyHeadMap* head_map, const CozyScatter* scatter,
                              int causal, float scale, int* status, cudaStream_t stream) {
  return attention_launch(q, k, v, out, batch, seq_q, seq_k, heads_q, heads_kv, head_dim,
                          q_strides, k_strides, v_strides, o_strides, head_map, scatter, causal,
                          scale, status, nullptr, false, nullptr, nullptr, stream);
}

int attention_forward_fp8(const void* q, const void* k, const void* v, const float* q_scale,
                          const float* k_scale, const float* v_scale, long long scale_seq,
                          const int* cuts, int n_cuts, void* out, int batch, int seq_q, int seq_k, int heads_q, int heads_kv,
                          int head_dim, const long long* q_strides, const long long* k_strides,
                          const long long* v_strides, const long long* o_strides,
                          const CozyHeadMap* head_map, const CozyScatter* scatter, int causal,
                          float scale, int* status, cudaStream_t stream) {
  const Fp8Operands fp8 = {q_scale, k_scale, v_scale, scale_seq, cuts, n_cuts};
  return attention_launch(q, k, v, out, batch, seq_q, seq_k, heads_q, heads_kv, head_dim,
                          q_strides, k_strides, v_strides, o_strides, head_map, scatter, causal,
                          scale, status, &fp8, true, nullptr, nullptr, stream);
}

}  // namespace cozy

namespace cozy {

int attention_forward_ex(const void* q, const void* k, const void* v, void* out, int batch,
                         int seq_q, int seq_k, int heads_q, int heads_kv, int head_dim,
                         const long long* q_strides, const long long* k_strides,
                         const long long* v_strides, const long long* o_strides,
                         const CozyHeadMap* head_map, const CozyScatter* scatter, int causal,
                         float scale, int* status, const Arrival* arrival, void* workspace,
                         size_t workspace_bytes, cudaStream_t stream) {
  // a null workspace must not fall back to the library's own (it would allocate)
  static char none;
  const WorkspaceChoice choice = {workspace != nullptr ? workspace : &none,
                                  workspace != nullptr ? workspace_bytes : 0};
  return attention_launch(q, k, v, out, batch, seq_q, seq_k, heads_q, heads_kv, head_dim,
                          q_strides, k_strides, v_strides, o_strides, head_map, scatter, causal,
                          scale, status, nullptr, true, arrival, &choice, stream);
}

size_t attention_workspace_bytes(int batch, int seq_q, int seq_k, int heads_q, int head_dim,
                                 int causal, int sms) {
  if (batch <= 0 || seq_q <= 0 || seq_k <= 0 || heads_q <= 0 || sms <= 0 || causal ||
      (head_dim != 64 && head_dim != 128))
    return 0;
  const long long tiles = static_cast<long long>(batch) * heads_q *
                          ((seq_q + kQTiles * kBlockM - 1) / (kQTiles * kBlockM));
  const SplitPlan plan = plan_split(tiles, (seq_k + kBlockN - 1) / kBlockN, sms, head_dim);
  return plan.n_split > 0 ? split_bytes(plan.n_split, plan.parts, head_dim) : 0;
}

}  // namespace cozy
