/* C ABI of the B200-native Ulysses context-parallel attention path (libcozy_ulysses.so).
 *
 * Conventions (those of the reference's native modules, kernels/csrc/gemm.cpp:1-7 and
 * kernels/csrc/fa3.cpp:1-9 in cozy-runtime): arguments are raw device pointers, sizes, element
 * strides and a cudaStream_t passed as uintptr_t; the caller allocates every buffer it passes
 * (the exceptions, each stated at its entry point: the attention's split workspace, which the
 * library allocates once per (device, stream) outside stream capture and keeps, and the buffers
 * a CozyGroup maps when it is formed or reserved, never inside a layer call); each call
 * returns a cudaError_t value as an int (0 = queued on the stream; cudaErrorNotSupported = 801
 * when no kernel serves the shape; cudaErrorInvalidValue = 1 for bad arguments) and never
 * throws. `cozy_error_name` names a code. Kernels that wait report through a caller-owned
 * device status word (0 = fine, 1 = an on-chip wait timed out, 2 = a wait on a peer timed out).
 *
 * Every tensor is bf16 with its last (head) dimension contiguous unless stated otherwise.
 */
#ifndef COZY_ULYSSES_H
#define COZY_ULYSSES_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define COZY_MAX_PEERS 16

#if defined(__GNUC__)
#define COZY_API __attribute__((visibility("default")))
#else
#define COZY_API
#endif

/* How query heads map to key/value heads: query head h reads key/value head
 * (h + q_base) / group - kv_base. NULL selects group = heads_q / heads_kv, q_base = kv_base = 0
 * (torch's enable_gqa rule). A Ulysses rank that owns query heads [q_lo, q_lo + n) of a
 * grouped-query layer, and received key/value heads from kv_lo, passes {group, q_lo, kv_lo}. */
typedef struct CozyHeadMap {
  int group;
  int q_base;
  int kv_base;
} CozyHeadMap;

/* Where the attention writes its output rows when they go straight to their owners (the head->seq
 * crossing done by the attention's own stores over NVLink): output row r (global sequence
 * position) of batch b and local head h lands in owner p (row_start[p] <= r < row_start[p+1]) at
 * out[p] + b*strides[p][2] + (r - row_start[p])*strides[p][0] + (h + head_offset)*strides[p][1].
 * out[p] may be another GPU's memory (cozy_ipc_open). */
typedef struct CozyScatter {
  int world;
  int head_offset;
  int row_start[COZY_MAX_PEERS + 1];
  void* out[COZY_MAX_PEERS];
  long long strides[COZY_MAX_PEERS][3];
} CozyScatter;

/* Local attention over whole sequences: softmax(Q Kᵀ·scale) V for every (batch, query head),
 * query head h reading the key/value head `head_map` names. Causal masks align bottom-right
 * (key j visible to query i when j <= i + seq_k - seq_q).
 * Replaces the local kernel the reference's exchange calls as `compute` on a B200:
 * src/cozy_runtime/internal/attention_upstream.py:191-215 (`cudnn`, torch SDPA on cuDNN) and
 * :109-147 (`sdpa`), on [batch, seq, heads, dim] operands.
 * Strides are in elements, ordered {seq, head, batch}; each a multiple of 8; pointers 16-byte
 * aligned. head_dim 64 or 128. With `scatter` non-NULL the output goes where it says and
 * `out`/`o_strides` are ignored. */
COZY_API int cozy_attention_fwd(const void* q, const void* k, const void* v, void* out, int batch,
                       int seq_q, int seq_k, int heads_q, int heads_kv, int head_dim,
                       const long long* q_strides, const long long* k_strides,
                       const long long* v_strides, const long long* o_strides,
                       const CozyHeadMap* head_map, const CozyScatter* scatter, int causal,
                       float scale, int* status, uintptr_t stream);

/* How cozy_attention_fwd (and cozy_attention_fwd_fp8) schedule a call of this shape on the
 * current device. A CTA owns 256 query rows of one (batch, head) for the whole key range, so
 * tiles that fill no whole wave of one CTA per SM would leave SMs idle; instead, past the first
 * `*whole_tiles` tiles, each tile runs as `*parts` CTAs over consecutive shares of the keys,
 * whose partial rows the last CTA to finish merges (an atomic count, no waiting). `*parts` = 1
 * when nothing is split (always for causal calls). The split needs a workspace the library
 * allocates (cudaMalloc) at the first eager launch on a (device, stream) that needs it, and keeps
 * (it grows, never shrinks); launches on one stream share it in order. Launches made while the
 * stream is being captured into a graph never use it: they run unsplit, so a graph holds no
 * address of it. COZY_ATTENTION_SPLIT=0 in the environment turns the split off. */
COZY_API int cozy_attention_split_plan(int batch, int seq_q, int seq_k, int heads_q, int head_dim,
                                       int causal, long long* whole_tiles, int* parts);

/* The same plan for a GPU of `sms` SMs: host arithmetic only, no device needed. */
COZY_API int cozy_attention_split_plan_for(int batch, int seq_q, int seq_k, int heads_q,
                                           int head_dim, int causal, int sms,
                                           long long* whole_tiles, int* parts);

/* One tensor of the seq->head exchange's first stage (Q, K or V): this rank's rows
 * [batch, rows, heads, head_dim] (`src`, element strides {seq, head, batch}), optionally
 * RMS-normalised per head and rotated, written as the block each peer receives:
 * peer p gets heads [head_lo[p], head_lo[p] + head_n[p]) at dst[p] laid out
 * [rows][batch][head_n[p]][head_dim]. dst[p] may be a local send buffer (NCCL crossing) or
 * this rank's row offset inside peer p's receive buffer (peer stores over NVLink). */
typedef struct CozyPackTensor {
  const void* src;
  long long src_strides[3];
  int heads;
  int normalize;            /* per-head RMSNorm before RoPE */
  const float* norm_weight; /* [head_dim] fp32, or NULL for unit weight */
  float norm_offset;        /* weight + offset multiplies the normalised row */
  float norm_eps;
  int rotate;               /* apply RoPE (CozyRope) */
  void* dst[COZY_MAX_PEERS];
  int head_lo[COZY_MAX_PEERS];
  int head_n[COZY_MAX_PEERS];
} CozyPackTensor;

/* RoPE tables as the reference's `rope_tables` returns them
 * (src/cozy_runtime/accel/fusion/_kernels.py:497-517): fp32 cos and sin read at
 * token * stride_token + column * stride_channel. `token0` is the table row of this rank's
 * first row. The first `rotary` channels rotate: interleaved pairs (2i, 2i+1) read column i;
 * split-half pairs (j, j ± rotary/2) read column j. */
typedef struct CozyRope {
  const float* cos;
  const float* sin;
  long long stride_token;
  int stride_channel;
  long long token0;
  int rotary;
  int interleaved;
} CozyRope;

/* The fused first stage of the exchange for up to three tensors in one launch: per-head
 * RMSNorm + RoPE (the law of src/cozy_runtime/accel/fusion/_kernels.py:177-240
 * `head_norm_rope_kernel`, fp32 arithmetic rounded once) fused with the pack into per-peer
 * blocks that src/cozy_runtime/internal/parallel/ulysses.py:325-362 (`_pack`) performs. */
COZY_API int cozy_ulysses_pack(const CozyPackTensor* tensors, int count, int world, int rows, int batch,
                      int head_dim, const CozyRope* rope, uintptr_t stream);

/* Per-head RMSNorm (when `normalize`; weight NULL = unit, else weight + offset) then RoPE
 * (when `rope` is non-NULL) of x [batch, seq, heads, head_dim] into out of the same shape, any
 * strides ({seq, head, batch}, elements); fp32 arithmetic rounded once. The standalone form of
 * the first stage's law: a drop-in for src/cozy_runtime/accel/fusion/_kernels.py:459
 * (`head_norm_rope`, the Triton kernel at :177-240) and kernels/csrc/norm.cpp:41-107
 * (`rms_rope_split_half`). */
COZY_API int cozy_head_norm_rope(const void* x, void* out, int batch, int seq, int heads,
                                 int head_dim, const long long* x_strides,
                                 const long long* out_strides, const CozyRope* rope,
                                 int normalize, const float* weight, float offset, float eps,
                                 uintptr_t stream);

/* The last stage of the exchange: the attended rows returned by every rank, stacked by source
 * rank in `returned` ([world][rows][batch][head_n[p]][head_dim]), landed in this rank's output
 * `out` [batch, rows, heads, head_dim] (element strides {seq, head, batch}) at heads
 * head_lo[p] + j. Replaces src/cozy_runtime/internal/parallel/ulysses.py:435-457 (`_land`). */
COZY_API int cozy_ulysses_land(const void* returned, int world, int rows, int batch, int head_dim,
                      const int* head_lo, const int* head_n, void* out,
                      const long long* out_strides, uintptr_t stream);

/* ------------------------------------------------------------------------------- FP8 path
 * The FP8 recipe of the video configuration: K less its per-(batch, head) mean over the whole
 * sequence (the reference's narrow wire shifts K the same way, with one all-reduce:
 * src/cozy_runtime/internal/parallel/ulysses.py:588-604), Q and K as e4m3 with one fp32 scale
 * per 64-token × head block (max(absmax/448, 1e-12); blocks start at each rank's first row), V as
 * e4m3 with one fp32 scale per (batch, head, channel) over the whole sequence, P as e4m3,
 * (a block is 64 tokens of the whole sequence starting at a multiple of 64, cut where one rank's
 * rows end and the next rank's begin),
 * softmax and accumulation in fp32. The per-head law is src/cozy_runtime/internal/
 * attention_fp8.py:162-169 (`quantise_eager`); the reference's B200 FP8 kernel is FA4-fp8
 * (attention_upstream.py:293-317). head_dim 128. */

/* This rank's partial statistics: k_sum[b][h][d] += Σ_rows key, v_amax[b][h][d] = max(|value|)
 * (the caller zero-fills both and all-reduces them: SUM and MAX). The keys summed are the first
 * stage's keys: per-head RMSNorm (when `normalize`) then RoPE (when `rotate`, table row
 * rope.token0 + row) in fp32, rounded to bf16 — the keys the FP8 first stage quantises. */
typedef struct CozyFp8Stats {
  const void* key;
  const void* value;
  long long k_strides[3];
  long long v_strides[3];
  int rows, batch, heads, head_dim;
  float* k_sum;
  float* v_amax;
  int normalize;            /* K's per-head RMSNorm: weight NULL = unit, else weight + offset */
  const float* norm_weight;
  float norm_offset;
  float norm_eps;
  int rotate;               /* RoPE per `rope` */
  CozyRope rope;
} CozyFp8Stats;

/* One tensor of the FP8 first stage. Block mode (Q, K): `channel_scale` NULL; the per-token
 * scale of row r goes to scale_dst[p][(b * head_n[p] + h) * scale_seq + r] (point scale_dst[p]
 * at this rank's first row). Channel mode (V): codes = x / channel_scale[b][h][d], no per-token
 * scales. `mean_sum` (K): subtracts mean_sum[b][h][d] * mean_inv_count. `hadamard` (Q and K):
 * the row times the orthonormal Hadamard matrix (QKᵀ is unchanged; a channel outlier spreads over
 * the head before its block scale is taken), as the reference's FA4-fp8 path rotates Q and K
 * (src/cozy_runtime/internal/attention_upstream.py:276-317). Codes go to dst[p] as
 * [rows][batch][head_n[p]][128] bytes, as CozyPackTensor. `normalize` / `rotate` (Q and K): the
 * first stage's per-head RMSNorm and RoPE (CozyFp8Pack.rope, table row rope.token0 + row) come
 * first, in fp32, rounded to bf16 as the bf16 first stage rounds them; the FP8 recipe then
 * applies to those values, so RoPE, quantisation and the transpose are one pass over HBM. */
typedef struct CozyFp8Tensor {
  const void* src;
  long long src_strides[3];
  int heads;
  int hadamard;             /* rotate each row by the orthonormal Hadamard of order 128 first */
  const float* mean_sum;
  float mean_inv_count;
  const float* channel_scale;
  void* dst[COZY_MAX_PEERS];
  float* scale_dst[COZY_MAX_PEERS];
  long long scale_seq;
  int head_lo[COZY_MAX_PEERS];
  int head_n[COZY_MAX_PEERS];
  int normalize;
  const float* norm_weight;
  float norm_offset;
  float norm_eps;
  int rotate;
  const float* head_scale; /* per-head mode (Q, K): one descale per (batch, head) [batch][heads]
                              instead of the block scales; every row's per-token scale is it */
  float* head_amax;        /* cozy_fp8_head_amax's output [batch][heads] (caller zero-fills) */
} CozyFp8Tensor;

typedef struct CozyFp8Pack {
  CozyFp8Tensor t[3]; /* Q, K, V */
  int world, rows, batch, head_dim;
  int row0; /* this rank's first row in the whole sequence: blocks are [64i, 64i + 64) of the
               whole sequence, clipped to this rank's rows */
  int head_turn; /* the first head (of Q; K/V: the same fraction of theirs) the launch packs,
                    then the next ones round: a rank starting at its own heads writes to a
                    different peer than the other ranks at any moment */
  CozyRope rope; /* read by tensors with `rotate` */
  int per_head;  /* the reference's per-(batch, head) law (attention_fp8.py:134-169 after
                    attention_upstream.py:293-317 `fa4_fp8`): the Hadamard rotation as a bf16
                    matrix product (multiplier and result rounded to bf16), codes = x / descale
                    correctly rounded (head_scale for Q and K; V's channel_scale holds its
                    per-head descale broadcast over the channels), no K mean */
} CozyFp8Pack;

COZY_API int cozy_fp8_stats(const CozyFp8Stats* stats, uintptr_t stream);
COZY_API int cozy_fp8_pack(const CozyFp8Pack* pack, uintptr_t stream);
/* The per-head law's statistics: for every tensor with `head_amax`, the absmax over this rank's
 * rows of each (batch, head) after the transform cozy_fp8_pack applies (norm, RoPE, rotation),
 * atomically maxed into head_amax (the caller zero-fills it and all-reduces MAX). The reference
 * takes the same amax after the exchange, per head (attention_fp8.py:134-160). */
COZY_API int cozy_fp8_head_amax(const CozyFp8Pack* pack, uintptr_t stream);

/* cozy_attention_fwd on e4m3 operands: q/k/v codes with element (= byte) strides, each a
 * multiple of 16; q_scale/k_scale per token [batch][heads][scale_seq] (scale_seq ≥ seq_k
 * rounded up to 128, padding zero), v_scale [batch][heads_kv][128]. Output bf16.
 * K scales are constant over every 64-key block of the whole sequence except where one of the
 * `n_cuts` rows in `cuts` (the ranks' first rows, each > 0) falls inside it; the kernel takes
 * one scale per 64-key block elsewhere. */
COZY_API int cozy_attention_fwd_fp8(
    const void* q, const void* k, const void* v, const float* q_scale, const float* k_scale,
    const float* v_scale, long long scale_seq, const int* cuts, int n_cuts, void* out,
    int batch, int seq_q, int seq_k,
    int heads_q, int heads_kv, int head_dim, const long long* q_strides,
    const long long* k_strides, const long long* v_strides, const long long* o_strides,
    const CozyHeadMap* head_map, const CozyScatter* scatter, int causal, float scale,
    int* status, uintptr_t stream);

/* ------------------------------------------------------------ allocation-free degree-1 call
 * No counterpart in the reference: an addition for callers that must not allocate device memory
 * while they run — a stream being captured into a CUDA graph (cudaMalloc cannot be captured), a
 * serving loop that owns all device memory up front in a fixed arena, or a latency-bound host
 * thread (cudaMalloc can synchronize the device). Same result as the degree-1 first stage
 * (RoPE per `rope`, per-head RMSNorm with unit weight when `normalize`) followed by
 * cozy_attention_fwd, but the rotated Q and K live in a static device array of
 * COZY_NOALLOC_SCRATCH_BYTES that every GPU loading this library holds until the process exits.
 * The caller passes inputs and output; nothing is allocated. A call needing more than the array
 * ((heads_q + heads_kv) * seq * batch * head_dim * 2 bytes) returns cudaErrorInvalidValue.
 * Every call on a device shares the array: calls whose kernels overlap on the GPU race, so
 * serialize them. The first call on a device looks up the array's address; make it before any
 * stream capture. Strides as cozy_attention_fwd ({seq, head, batch}, elements). */
#define COZY_NOALLOC_SCRATCH_BYTES (64ull << 20)

COZY_API int cozy_rope_attention_fwd_noalloc(
    const void* q, const void* k, const void* v, void* out, int batch, int seq, int heads_q,
    int heads_kv, int head_dim, const long long* q_strides, const long long* k_strides,
    const long long* v_strides, const long long* o_strides, const CozyRope* rope, int normalize,
    float norm_eps, int causal, float scale, int* status, uintptr_t stream);

/* --------------------------------------------------------------------- the int8 wire
 * `exchange(..., narrow=True)`: rows of Q, K (less a shift every GPU shares) and V, and of the
 * attention's output, cross as int8 with one bf16 scale per row after a turn by the orthonormal
 * Hadamard matrix of the head dimension (64 or 128), and are turned back on arrival; the law of
 * src/cozy_runtime/internal/parallel/turn.py:60-82 (`law`, `law_back`):
 *   t = (x·H)·D^-1/2 - shift;  scale = bf16(max(max|t|·(1/127), 2^-126));
 *   code = sign(q)·floor(|q| + 1/2) of q = clamp(t / scale, -127, 127);
 *   back = bf16((code·H)·(scale·D^-1/2)). */

/* Adds this rank's column sums of K [batch, rows, heads, head_dim] (element strides {seq, head,
 * batch}) into `sum` [batch][heads][head_dim] fp32: the source of the shift after an all-reduce
 * (replaces `key.sum(1, dtype=torch.float32)` of src/cozy_runtime/internal/parallel/ulysses.py:
 * 588-604). */
COZY_API int cozy_key_sum(const void* key, const long long* strides, int rows, int batch,
                          int heads, int head_dim, float* sum, uintptr_t stream);

/* shift = turned(sum / count) per (batch, head): [batch][heads][head_dim] fp32, K's mean over
 * `count` rows turned (`_Shift.__call__`, ulysses.py:598-604). */
COZY_API int cozy_narrow_shift(const float* sum, long long count, int batch, int heads,
                               int head_dim, float* shift, uintptr_t stream);

/* One tensor of a narrow crossing: bf16 rows [batch, rows, heads, head_dim] (`src`, element
 * strides {seq, head, batch}), each turned (less `shift` [batch][heads][head_dim] when
 * non-NULL) and written as codes int8 [row_n[p]][batch][head_n[p]][head_dim] at dst[p] and
 * scales bf16 [row_n[p]][batch][head_n[p]] at scale_dst[p], for every destination p whose rows
 * [row_lo[p], +row_n[p]) and heads [head_lo[p], +head_n[p]) hold the row: by head for the first
 * stage, by row for the output's return. Replaces `turn.narrow` inside `ulysses._pack` (:325-362)
 * and `_returned` (:459-502). */
typedef struct CozyNarrowTensor {
  const void* src;
  long long src_strides[3];
  int heads;
  const float* shift;
  void* dst[COZY_MAX_PEERS];
  void* scale_dst[COZY_MAX_PEERS];
  int head_lo[COZY_MAX_PEERS];
  int head_n[COZY_MAX_PEERS];
  int row_lo[COZY_MAX_PEERS];
  int row_n[COZY_MAX_PEERS];
} CozyNarrowTensor;

COZY_API int cozy_narrow_pack(const CozyNarrowTensor* tensors, int count, int world, int rows,
                              int batch, int head_dim, uintptr_t stream);

/* Received codes [rows][batch][head_n][head_dim] int8 and scales [rows][batch][head_n] bf16 of
 * one source, to rows [row_lo, +rows) and heads [head_lo, +head_n) of `out`. */
typedef struct CozyWidenSource {
  const void* codes;
  const void* scales;
  int row_lo, rows, head_lo, head_n;
} CozyWidenSource;

/* `count` sources turned back into bf16 `out` [batch, ·, ·, head_dim] (element strides {seq,
 * head, batch}), bit for bit `turn.law_back`. Replaces `turn.widen` inside `ulysses._unpack`
 * (:420-432) and `_land` (:435-457). */
COZY_API int cozy_narrow_widen(const CozyWidenSource* sources, int count, int batch,
                               int head_dim, void* out, const long long* out_strides,
                               uintptr_t stream);

/* ---------------------------------------------------------------- peer memory (one node)
 * The NVLink exchange keeps its receive and landing buffers in memory every GPU of the group
 * maps. These replace the reference's copy-engine exchange buffers
 * (src/cozy_runtime/internal/parallel/copy_engine.py:136-251, mapped at group formation, never
 * inside a call). cozy_ipc_alloc zero-fills `bytes` of device memory and writes its IPC handle
 * (cozy_ipc_handle_bytes() bytes) to `handle`; another process opens it with cozy_ipc_open. */
COZY_API int cozy_ipc_alloc(unsigned long long bytes, void** ptr, void* handle);
COZY_API int cozy_ipc_open(const void* handle, void** ptr);
COZY_API int cozy_ipc_close(void* ptr);
COZY_API int cozy_ipc_free(void* ptr);
COZY_API int cozy_ipc_handle_bytes(void);

/* Arrival flags: `slot[i]` is this rank's 64-bit flag word in peer i's memory. cozy_peer_signal
 * fences this GPU's earlier writes at system scope and stores `seq` into every slot (release).
 * cozy_peer_wait blocks the stream until each of flags[0..count) reaches `seq` (acquire), or
 * gives up after `limit_ns` nanoseconds and sets *status to 2. Replaces the NCCL all-reduce
 * barriers of the copy-engine exchange (copy_engine.py:167). */
typedef struct CozyPeerSlots {
  int count;
  long long* slot[COZY_MAX_PEERS];
} CozyPeerSlots;

COZY_API int cozy_peer_signal(const CozyPeerSlots* slots, long long seq, uintptr_t stream);
COZY_API int cozy_peer_wait(const long long* flags, int count, long long seq, long long limit_ns,
                            int* status, uintptr_t stream);

/* ------------------------------------------------------------ the whole layer (one node)
 * One rank's group: what it maps for a Ulysses attention layer between the GPUs of one node —
 * receive and landing buffers (two sets, by call parity), arrival flags, a staging buffer for
 * the blocks it sends, the attention's split workspace — and a side stream for its copies.
 * Formed once per group and grown when a larger layer comes; no layer call allocates. Replaces
 * the reference's exchange (src/cozy_runtime/internal/parallel/ulysses.py:607-766) with its
 * group formation and mapped copy-engine buffers (copy_engine.py:408-449), for callers that run
 * the layer without Python.
 *
 * Formation (every rank of the group, together):
 *   cozy_group_create(rank, world, &g) on the rank's device (current);
 *   cozy_group_needs(g, &shape, &grow): whether the buffers must grow for this shape (all ranks
 *     answer alike); when they must: synchronize every rank's device and meet (a barrier over
 *     the caller's channel), then cozy_group_reserve(g, &shape, blob) (cozy_group_blob_bytes()
 *     bytes of IPC handles), exchange the blobs (all-gather, rank order) and cozy_group_open(g,
 *     blobs).
 * A call: cozy_ulysses_layer_fwd(g, &call, stream) on every rank; no other collective.
 * Errors: cudaError_t values; a wait on a peer that runs past call.wait_limit_ns sets *status
 * to 2 and the rank publishes nothing more. cozy_group_destroy releases everything (after the
 * group's last call on every rank). */
typedef struct CozyGroup CozyGroup;

typedef struct CozyLayerShape {
  int world;
  int rows[COZY_MAX_PEERS]; /* every rank's sequence rows, in rank order */
  int batch, heads_q, heads_kv, head_dim, causal;
} CozyLayerShape;

typedef struct CozyLayerCall {
  CozyLayerShape shape;
  /* this rank's rows [batch, rows[rank], heads, head_dim] bf16, element strides {seq, head,
   * batch} (each a multiple of 8); K and V have heads_kv heads */
  const void* q;
  const void* k;
  const void* v;
  long long q_strides[3], k_strides[3], v_strides[3];
  void* out; /* [batch, rows[rank], heads_q, head_dim] bf16, contiguous */
  float scale; /* 0: 1/sqrt(head_dim) */
  const CozyRope* rope; /* NULL: no RoPE; else tables over the whole sequence (token0 ignored) */
  int norm_q, norm_k;   /* per-head RMSNorm of Q / K before RoPE */
  const float* norm_q_weight;
  const float* norm_k_weight; /* NULL: unit weight */
  float norm_offset[2];       /* Q, K: weight + offset multiplies the normalised row */
  float norm_eps[2];          /* Q, K */
  long long wait_limit_ns; /* the longest a wait on another rank may take (0: 10 s) */
  int* status;             /* device status word (0 = fine) */
  int gate;                /* 0: the attention starts at once and waits per source inside the
                              kernel; 1: a wait kernel holds it until every source's rows have
                              landed (every rank then starts its attention at nearly the same
                              moment) */
  int cross;               /* 0: the first stage packs the other ranks' blocks into a staging
                              buffer and copy engines move them, beside the attention; 1: the
                              first stage stores them straight into their owners' receive
                              buffers over NVLink (SM stores), and one kernel sets the flags */
} CozyLayerCall;

COZY_API int cozy_group_create(int rank, int world, CozyGroup** group);
COZY_API int cozy_group_destroy(CozyGroup* group);
COZY_API int cozy_group_blob_bytes(void);
COZY_API int cozy_group_needs(const CozyGroup* group, const CozyLayerShape* shape, int* grow);
COZY_API int cozy_group_reserve(CozyGroup* group, const CozyLayerShape* shape, void* blob);
COZY_API int cozy_group_open(CozyGroup* group, const void* blobs);
/* One process holding every rank of a group on one GPU (tests): mark each group local before
 * its first reserve (blob may then be NULL), then connect them instead of opening blobs. */
COZY_API int cozy_group_make_local(CozyGroup* group);
COZY_API int cozy_group_connect_local(CozyGroup* const* groups, int world);
/* How arrival flags cross: 1 = a stream memory write (cuStreamWriteValue64, fenced), 2 = a copy
 * of a pinned host word behind the blocks on the same stream. */
COZY_API int cozy_group_flag_mode(const CozyGroup* group);
/* The last call number rank `src` published to this rank (kind 0: its Q/K/V blocks landed;
 * kind 1: its output rows landed); a synchronous read, for monitoring and tests. */
COZY_API int cozy_group_flag(const CozyGroup* group, int kind, int src, long long* value);
/* The latest call's crossing on this rank: milliseconds from its first copy to its last flag
 * write on the side stream, and the bytes its copies moved to the other ranks (for NVLink
 * bandwidth: bytes / ms). cudaErrorNotReady while that call's copies are still under way. */
COZY_API int cozy_group_crossing(CozyGroup* group, float* ms, unsigned long long* bytes);
/* The link probe of one ordered pair (this rank -> `dst`): `reps` back-to-back copies of this
 * rank's staging buffer (at least 8 MiB, whatever the layer shape: smaller copies measure the
 * copy's fixed cost) into dst's receive buffer (set 0), on the copy engines and side stream
 * the crossing uses; returns their time and bytes. It overwrites dst's receive set 0: call it
 * only while no layer call is in flight on any rank of the group (between barriers). Replaces
 * the reference's per-pair copy measurement (src/cozy_runtime/internal/parallel/links.py:
 * 394-519), which it takes inside the group's own processes and buffers. */
COZY_API int cozy_group_probe(CozyGroup* group, int dst, int reps, float* ms,
                              unsigned long long* bytes);

/* The layer: cozy_ulysses_layer_fwd = begin (first stage, copies and flags to every rank),
 * attend (the attention, waiting per source inside the kernel, output rows stored into their
 * owners' landing buffers; then "landed" flags), end (bounded wait for every rank's rows, copy
 * into out). The phases exist separately so one process can simulate all ranks on one GPU
 * (every rank's begin, then every rank's attend, then every rank's end). */
COZY_API int cozy_ulysses_layer_fwd(CozyGroup* group, const CozyLayerCall* call, uintptr_t stream);
COZY_API int cozy_ulysses_layer_begin(CozyGroup* group, const CozyLayerCall* call,
                                      uintptr_t stream);
COZY_API int cozy_ulysses_layer_attend(CozyGroup* group, const CozyLayerCall* call,
                                       uintptr_t stream);
COZY_API int cozy_ulysses_layer_end(CozyGroup* group, const CozyLayerCall* call, uintptr_t stream);

/* Name of a code returned above (a cudaError_t, or one of this library's). */
COZY_API const char* cozy_error_name(int code);

/* Library ABI version (major * 100 + minor). */
COZY_API int cozy_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* COZY_ULYSSES_H */
