// One Ulysses attention layer between the GPUs of one node, driven from C: the group a rank
// forms once (buffers every GPU of the group maps, arrival flags, a side stream for the copies)
// and the layer call itself.
//
// A call, on rank r of W (rows: every rank's sequence rows; heads padded and owned as the
// reference owns them, src/cozy_runtime/internal/parallel/ulysses.py:647):
//   1. first stage (one kernel, this GPU's memory only): RMSNorm + RoPE of Q and K, the
//      transpose into per-destination head blocks; r's own block goes straight into r's receive
//      buffer, the others into a staging buffer;
//   2. on the side stream, destination by destination (r+1, r+2, ...), the copy engines move each
//      block into the destination's receive buffer at r's row offset, and a stream memory write
//      (a system-scope fence, then the store) sets r's arrival flag in the destination's memory;
//   3. the attention starts at once on r's own rows: its producer warp waits for a source's flag
//      before its first load of that source's rows, and its key and query walks start at r's
//      own rows and go down through the sources in the order they arrive; its epilogue stores
//      every output row into its owner's landing buffer;
//   4. r publishes "my output rows have landed" to every rank, waits (bounded) until every rank
//      has, and copies its landing buffer into `out`.
// With `cross` set (SM crossing, the Python side's choice from degree 4), steps 1-2 become one:
// the first stage stores every block straight into its owner's receive buffer (bulk stores from
// shared memory) and one kernel fences at system scope and sets the flags. With `gate` set, a
// wait kernel holds the attention until every source has landed, and it runs with every row
// resident.
// Buffers are double-buffered by call parity: r writes call n into a peer only after every rank
// finished call n - 1 (step 4 of call n - 1), so every read of the set of call n - 2 is done. No
// SM is needed for the crossing itself, so the copies and the attention overlap.
//
// This replaces the reference's exchange over NCCL all-to-all or its copy-engine buffers
// (src/cozy_runtime/internal/parallel/ulysses.py:607-766, copy_engine.py:136-251).
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "../../include/cozy_ulysses.h"
#include "attention.h"
#include "sm100.cuh"

namespace cozy {
int ulysses_pack_to(const CozyPackTensor* tensors, int count, int world, int rows, int batch,
                    int head_dim, const CozyRope* rope, bool remote, cudaStream_t stream);
int peer_signal(const CozyPeerSlots* slots, long long seq, const int* status,
                cudaStream_t stream);
int peer_wait(const long long* flags, int count, long long seq, long long limit_ns, int* status,
              cudaStream_t stream);
}  // namespace cozy

namespace {

constexpr int kQKV = 0;  // flag kinds: a call's Q/K/V blocks have landed
constexpr int kOut = 1;  //             its output rows have landed
constexpr long long kDefaultWaitNs = 10000000000LL;
constexpr int kBuffers = 4;  // per set: q, k, v receive buffers and the landing buffer
// Streams the crossing spreads its destinations over. One stream ran the destinations one after
// another on one copy engine: 67 MB a rank at 237 GB/s at C2 degree 8, against 488 GB/s that a
// single pair reaches alone.
constexpr int kLanes = 7;
constexpr size_t kProbeBytes = 8u << 20;  // the link probe's copy size (see needed())

// Who owns what in one layer (ulysses.py:647 padding: ceil(H / W) query heads a rank; key/value
// heads as the owned query heads read them).
struct Plan {
  int world, total;
  int start[COZY_MAX_PEERS + 1];
  int q_lo[COZY_MAX_PEERS], q_n[COZY_MAX_PEERS], kv_lo[COZY_MAX_PEERS], kv_n[COZY_MAX_PEERS];
  int group;
};

bool make_plan(const CozyLayerShape& s, Plan* p) {
  if (s.world < 1 || s.world > COZY_MAX_PEERS || s.batch < 1 || s.heads_q < 1 ||
      s.heads_kv < 1 || s.heads_q % s.heads_kv != 0 || (s.head_dim != 64 && s.head_dim != 128))
    return false;
  p->world = s.world;
  p->group = s.heads_q / s.heads_kv;
  long long acc = 0;
  for (int r = 0; r < s.world; ++r) {
    if (s.rows[r] < 0) return false;
    p->start[r] = static_cast<int>(acc);
    acc += s.rows[r];
  }
  if (acc <= 0 || acc > (1LL << 30)) return false;
  p->start[s.world] = static_cast<int>(acc);
  p->total = static_cast<int>(acc);
  const int local = (s.heads_q + s.world - 1) / s.world;
  for (int r = 0; r < s.world; ++r) {
    const int lo = std::min(r * local, s.heads_q), hi = std::min((r + 1) * local, s.heads_q);
    p->q_lo[r] = lo;
    p->q_n[r] = hi - lo;
    p->kv_lo[r] = hi > lo ? lo / p->group : 0;
    p->kv_n[r] = hi > lo ? (hi - 1) / p->group - lo / p->group + 1 : 0;
  }
  return true;
}

// Buffer capacities (bytes) a shape needs; identical on every rank of the group, so all ranks
// decide alike whether to grow.
struct Caps {
  size_t q, kv, land, stage, workspace;
};

Caps needed(const CozyLayerShape& s, const Plan& p, int sms) {
  const size_t el = 2, d = static_cast<size_t>(s.head_dim), b = static_cast<size_t>(s.batch);
  int most_q = 0, most_kv = 0, most_rows = 0, sum_q = 0, sum_kv = 0;
  for (int r = 0; r < s.world; ++r) {
    most_q = std::max(most_q, p.q_n[r]);
    most_kv = std::max(most_kv, p.kv_n[r]);
    most_rows = std::max(most_rows, s.rows[r]);
    sum_q += p.q_n[r];
    sum_kv += p.kv_n[r];
  }
  Caps c;
  // The Q receive buffers and the staging buffer never shrink below kProbeBytes: the link probe
  // (cozy_group_probe) copies between them, and copies much smaller than this measure the
  // copy's fixed cost, not the link (67 KB copies read 18 GB/s over an NVLink pair that moves
  // 700 GB/s).
  c.q = std::max(static_cast<size_t>(p.total) * b * most_q * d * el, kProbeBytes);
  c.kv = static_cast<size_t>(p.total) * b * most_kv * d * el;
  c.land = b * most_rows * s.heads_q * d * el;
  c.stage = std::max(static_cast<size_t>(most_rows) * b * (sum_q + 2 * sum_kv) * d * el,
                     kProbeBytes);
  c.workspace = cozy::attention_workspace_bytes(s.batch, p.total, p.total, most_q, s.head_dim,
                                                s.causal, sms);
  return c;
}

using WriteValue64 = CUresult (*)(CUstream, CUdeviceptr, cuuint64_t, unsigned int);
using DeviceGet = CUresult (*)(CUdevice*, int);
using DeviceGetAttribute = CUresult (*)(int*, CUdevice_attribute, CUdevice);

template <typename Fn>
Fn driver_entry(const char* name) {
  void* ptr = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &ptr, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    return reinterpret_cast<Fn>(ptr);
  cudaGetLastError();
  return nullptr;
}

// Whether `device` takes 64-bit stream memory writes (cuStreamWriteValue64).
bool stream_mem_ops(int device) {
  const DeviceGet get = driver_entry<DeviceGet>("cuDeviceGet");
  const DeviceGetAttribute attr = driver_entry<DeviceGetAttribute>("cuDeviceGetAttribute");
  CUdevice dev;
  int value = 0;
  if (get == nullptr || attr == nullptr || get(&dev, device) != CUDA_SUCCESS ||
      attr(&value, CU_DEVICE_ATTRIBUTE_CAN_USE_64_BIT_STREAM_MEM_OPS, dev) != CUDA_SUCCESS)
    return false;
  return value != 0;
}

WriteValue64 write_value64() {
  static WriteValue64 fn = nullptr;
  static bool looked = false;
  if (!looked) {
    looked = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuStreamWriteValue64", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<WriteValue64>(ptr);
  }
  return fn;
}

struct Blob {
  cudaIpcMemHandle_t flags;
  cudaIpcMemHandle_t set[2][kBuffers];
};

}  // namespace

struct CozyGroup {
  int rank = 0, world = 1, device = 0, sms = 0;
  bool local = false;  // every rank in this process on one GPU (peer pointers, no IPC)
  bool opened = false;
  long long* flags = nullptr;  // [2 kinds][world], this GPU's memory
  void* mine[2][kBuffers] = {};
  void* stage = nullptr;
  void* workspace = nullptr;
  Caps caps = {0, 0, 0, 0, 0};
  long long* peer_flags[COZY_MAX_PEERS] = {};
  void* peer[COZY_MAX_PEERS][2][kBuffers] = {};
  std::vector<void*> imported;
  long long seq = 0;
  bool write_value = false;  // 64-bit stream memory writes available
  long long* ring = nullptr;  // pinned host words the flag copies read when they are not
  cudaStream_t side = nullptr;  // lane 0 of the crossing (and the link probe's stream)
  // more lanes: each destination's copies on its own stream, so several copy engines run at once
  cudaStream_t lanes[kLanes] = {};
  cudaEvent_t lane_done[kLanes] = {};
  cudaEvent_t packed = nullptr, sent = nullptr;
  // timing of the crossing: the side stream's copies and flags of the latest call
  cudaEvent_t cross_start = nullptr, cross_end = nullptr;
  unsigned long long cross_bytes = 0;
  std::mutex lock;
};

namespace {

constexpr int kRing = 64;

void release_sets(CozyGroup* g) {
  for (void* ptr : g->imported) cudaIpcCloseMemHandle(ptr);
  g->imported.clear();
  for (auto& set : g->mine)
    for (void*& ptr : set) {
      if (ptr != nullptr) cudaFree(ptr);
      ptr = nullptr;
    }
  if (g->stage != nullptr) cudaFree(g->stage);
  if (g->workspace != nullptr) cudaFree(g->workspace);
  g->stage = g->workspace = nullptr;
  memset(g->peer, 0, sizeof(g->peer));
  memset(g->peer_flags, 0, sizeof(g->peer_flags));
  g->caps = Caps{0, 0, 0, 0, 0};
  g->opened = false;
}

int check_call(const CozyGroup* g, const CozyLayerCall* c, Plan* plan) {
  if (g == nullptr || c == nullptr || !g->opened) return cudaErrorInvalidValue;
  if (c->shape.world != g->world || !make_plan(c->shape, plan)) return cudaErrorInvalidValue;
  const Caps need = needed(c->shape, *plan, g->sms);
  if (need.q > g->caps.q || need.kv > g->caps.kv || need.land > g->caps.land ||
      need.stage > g->caps.stage)
    return cudaErrorInvalidValue;  // the group was not reserved for this shape
  if (c->q == nullptr || c->k == nullptr || c->v == nullptr || c->out == nullptr ||
      c->status == nullptr)
    return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(c->out) % 16) return cudaErrorInvalidValue;
  if (c->rope != nullptr && (c->rope->cos == nullptr || c->rope->sin == nullptr))
    return cudaErrorInvalidValue;
  return cudaSuccess;
}

// Byte offset of rank `src`'s rows inside a receive buffer of head count n.
size_t row_offset(const Plan& p, const CozyLayerShape& s, int src, int n) {
  return static_cast<size_t>(p.start[src]) * s.batch * n * s.head_dim * 2;
}

}  // namespace

extern "C" {

int cozy_group_blob_bytes(void) { return static_cast<int>(sizeof(Blob)); }

int cozy_group_create(int rank, int world, CozyGroup** group) {
  if (group == nullptr || world < 1 || world > COZY_MAX_PEERS || rank < 0 || rank >= world)
    return cudaErrorInvalidValue;
  *group = nullptr;
  CozyGroup* g = new CozyGroup();
  g->rank = rank;
  g->world = world;
  cudaError_t e = cudaGetDevice(&g->device);
  if (e == cudaSuccess)
    e = cudaDeviceGetAttribute(&g->sms, cudaDevAttrMultiProcessorCount, g->device);
  g->write_value = e == cudaSuccess && stream_mem_ops(g->device) && write_value64() != nullptr;
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&g->flags), 2 * world * 8);
  if (e == cudaSuccess) e = cudaMemset(g->flags, 0, 2 * world * 8);
  if (e == cudaSuccess && !g->write_value)
    e = cudaHostAlloc(reinterpret_cast<void**>(&g->ring), kRing * sizeof(long long),
                      cudaHostAllocDefault);
  int least = 0, greatest = 0;
  if (e == cudaSuccess) e = cudaDeviceGetStreamPriorityRange(&least, &greatest);
  if (e == cudaSuccess)
    e = cudaStreamCreateWithPriority(&g->side, cudaStreamNonBlocking, greatest);
  g->lanes[0] = g->side;
  for (int l = 1; l < kLanes && e == cudaSuccess; ++l) {
    e = cudaStreamCreateWithPriority(&g->lanes[l], cudaStreamNonBlocking, greatest);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&g->lane_done[l], cudaEventDisableTiming);
  }
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&g->packed, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&g->sent, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreate(&g->cross_start);
  if (e == cudaSuccess) e = cudaEventCreate(&g->cross_end);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cozy_group_destroy(g);
    return e;
  }
  *group = g;
  return cudaSuccess;
}

int cozy_group_destroy(CozyGroup* g) {
  if (g == nullptr) return cudaSuccess;
  cudaError_t e = cudaDeviceSynchronize();
  release_sets(g);
  if (g->flags != nullptr) cudaFree(g->flags);
  if (g->ring != nullptr) cudaFreeHost(g->ring);
  if (g->packed != nullptr) cudaEventDestroy(g->packed);
  if (g->sent != nullptr) cudaEventDestroy(g->sent);
  if (g->cross_start != nullptr) cudaEventDestroy(g->cross_start);
  if (g->cross_end != nullptr) cudaEventDestroy(g->cross_end);
  for (int l = 1; l < kLanes; ++l) {
    if (g->lanes[l] != nullptr) cudaStreamDestroy(g->lanes[l]);
    if (g->lane_done[l] != nullptr) cudaEventDestroy(g->lane_done[l]);
  }
  if (g->side != nullptr) cudaStreamDestroy(g->side);
  delete g;
  return e;
}

int cozy_group_needs(const CozyGroup* g, const CozyLayerShape* shape, int* grow) {
  Plan plan;
  if (g == nullptr || shape == nullptr || grow == nullptr || shape->world != g->world ||
      !make_plan(*shape, &plan))
    return cudaErrorInvalidValue;
  const Caps need = needed(*shape, plan, g->sms);
  *grow = !g->opened || need.q > g->caps.q || need.kv > g->caps.kv ||
          need.land > g->caps.land || need.stage > g->caps.stage ||
          need.workspace > g->caps.workspace;
  return cudaSuccess;
}

int cozy_group_reserve(CozyGroup* g, const CozyLayerShape* shape, void* blob) {
  Plan plan;
  if (g == nullptr || shape == nullptr || shape->world != g->world || !make_plan(*shape, &plan))
    return cudaErrorInvalidValue;
  if (blob == nullptr && !g->local) return cudaErrorInvalidValue;
  std::lock_guard<std::mutex> guard(g->lock);
  const Caps need = needed(*shape, plan, g->sms);
  Caps grown = {std::max(need.q, g->caps.q), std::max(need.kv, g->caps.kv),
                std::max(need.land, g->caps.land), std::max(need.stage, g->caps.stage),
                std::max(need.workspace, g->caps.workspace)};
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return e;
  release_sets(g);
  const size_t sizes[kBuffers] = {grown.q, grown.kv, grown.kv, grown.land};
  Blob b;
  memset(&b, 0, sizeof(b));
  for (int s = 0; s < 2 && e == cudaSuccess; ++s)
    for (int i = 0; i < kBuffers && e == cudaSuccess; ++i) {
      e = cudaMalloc(&g->mine[s][i], std::max<size_t>(sizes[i], 256));
      if (e == cudaSuccess) e = cudaMemset(g->mine[s][i], 0, std::max<size_t>(sizes[i], 256));
      if (e == cudaSuccess && !g->local) e = cudaIpcGetMemHandle(&b.set[s][i], g->mine[s][i]);
    }
  if (e == cudaSuccess) e = cudaMalloc(&g->stage, std::max<size_t>(grown.stage, 256));
  if (e == cudaSuccess && grown.workspace > 0) e = cudaMalloc(&g->workspace, grown.workspace);
  if (e == cudaSuccess && !g->local) e = cudaIpcGetMemHandle(&b.flags, g->flags);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    release_sets(g);
    return e;
  }
  g->caps = grown;
  if (blob != nullptr) memcpy(blob, &b, sizeof(b));
  return cudaSuccess;
}

int cozy_group_open(CozyGroup* g, const void* blobs) {
  if (g == nullptr || blobs == nullptr || g->local || g->mine[0][0] == nullptr)
    return cudaErrorInvalidValue;
  std::lock_guard<std::mutex> guard(g->lock);
  const Blob* all = static_cast<const Blob*>(blobs);
  cudaError_t e = cudaSuccess;
  for (int r = 0; r < g->world && e == cudaSuccess; ++r) {
    if (r == g->rank) {
      g->peer_flags[r] = g->flags;
      for (int s = 0; s < 2; ++s)
        for (int i = 0; i < kBuffers; ++i) g->peer[r][s][i] = g->mine[s][i];
      continue;
    }
    void* ptr = nullptr;
    e = cudaIpcOpenMemHandle(&ptr, all[r].flags, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) break;
    g->imported.push_back(ptr);
    g->peer_flags[r] = static_cast<long long*>(ptr);
    for (int s = 0; s < 2 && e == cudaSuccess; ++s)
      for (int i = 0; i < kBuffers && e == cudaSuccess; ++i) {
        e = cudaIpcOpenMemHandle(&ptr, all[r].set[s][i], cudaIpcMemLazyEnablePeerAccess);
        if (e == cudaSuccess) {
          g->imported.push_back(ptr);
          g->peer[r][s][i] = ptr;
        }
      }
  }
  if (e != cudaSuccess) return e;
  g->opened = true;
  return cudaSuccess;
}

int cozy_group_connect_local(CozyGroup* const* groups, int world) {
  if (groups == nullptr || world < 1 || world > COZY_MAX_PEERS) return cudaErrorInvalidValue;
  for (int r = 0; r < world; ++r)
    if (groups[r] == nullptr || groups[r]->world != world || groups[r]->rank != r ||
        groups[r]->mine[0][0] == nullptr)
      return cudaErrorInvalidValue;
  for (int r = 0; r < world; ++r) {
    CozyGroup* g = groups[r];
    g->local = true;
    for (int q = 0; q < world; ++q) {
      g->peer_flags[q] = groups[q]->flags;
      for (int s = 0; s < 2; ++s)
        for (int i = 0; i < kBuffers; ++i) g->peer[q][s][i] = groups[q]->mine[s][i];
    }
    g->opened = true;
  }
  return cudaSuccess;
}

// Marks a group formed for one process's simulation of every rank on one GPU before its first
// reserve (buffers are plain allocations, not exported).
int cozy_group_make_local(CozyGroup* g) {
  if (g == nullptr || g->mine[0][0] != nullptr) return cudaErrorInvalidValue;
  g->local = true;
  return cudaSuccess;
}

int cozy_group_flag(const CozyGroup* g, int kind, int src, long long* value) {
  if (g == nullptr || value == nullptr || kind < 0 || kind > 1 || src < 0 || src >= g->world ||
      g->flags == nullptr)
    return cudaErrorInvalidValue;
  return cudaMemcpy(value, g->flags + kind * g->world + src, sizeof(long long),
                    cudaMemcpyDeviceToHost);
}

int cozy_group_crossing(CozyGroup* g, float* ms, unsigned long long* bytes) {
  if (g == nullptr || ms == nullptr || bytes == nullptr) return cudaErrorInvalidValue;
  std::lock_guard<std::mutex> guard(g->lock);
  if (g->seq == 0) return cudaErrorNotReady;
  const cudaError_t e = cudaEventElapsedTime(ms, g->cross_start, g->cross_end);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return e;
  }
  *bytes = g->cross_bytes;
  return cudaSuccess;
}

int cozy_group_probe(CozyGroup* g, int dst, int reps, float* ms, unsigned long long* bytes) {
  if (g == nullptr || ms == nullptr || bytes == nullptr || reps < 1) return cudaErrorInvalidValue;
  std::lock_guard<std::mutex> guard(g->lock);
  if (!g->opened || dst < 0 || dst >= g->world || dst == g->rank) return cudaErrorInvalidValue;
  void* to = g->peer[dst][0][0];
  const size_t n = std::min(g->caps.stage, g->caps.q);
  if (to == nullptr || g->stage == nullptr || n == 0) return cudaErrorInvalidValue;
  cudaEvent_t start, end;
  cudaError_t e = cudaEventCreate(&start);
  if (e != cudaSuccess) return e;
  if ((e = cudaEventCreate(&end)) != cudaSuccess) {
    cudaEventDestroy(start);
    return e;
  }
  // the same copy engines and stream the crossing uses, `reps` times back to back
  e = cudaEventRecord(start, g->side);
  for (int i = 0; i < reps && e == cudaSuccess; ++i)
    e = cudaMemcpyAsync(to, g->stage, n, cudaMemcpyDeviceToDevice, g->side);
  if (e == cudaSuccess) e = cudaEventRecord(end, g->side);
  if (e == cudaSuccess) e = cudaEventSynchronize(end);
  if (e == cudaSuccess) e = cudaEventElapsedTime(ms, start, end);
  cudaEventDestroy(start);
  cudaEventDestroy(end);
  *bytes = static_cast<unsigned long long>(n) * reps;
  return e;
}

int cozy_group_flag_mode(const CozyGroup* g) {
  if (g == nullptr) return -1;
  return g->write_value ? 1 : 2;
}

// Sets `flag` (this GPU's or a peer's) to `seq` behind `stream`'s earlier work: a stream memory
// write (a system-scope fence, then the store), or the copy of a pinned host word where the
// device lacks 64-bit stream writes.
static int write_flag(CozyGroup* g, long long* flag, long long seq, cudaStream_t stream) {
  if (g->write_value) {
    const CUresult r = write_value64()(reinterpret_cast<CUstream>(stream),
                                       reinterpret_cast<CUdeviceptr>(flag),
                                       static_cast<cuuint64_t>(seq), 0);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorLaunchFailure;
  }
  long long* word = g->ring + (seq % kRing);
  *word = seq;
  return cudaMemcpyAsync(flag, word, sizeof(long long), cudaMemcpyHostToDevice, stream);
}

int cozy_ulysses_layer_begin(CozyGroup* g, const CozyLayerCall* c, uintptr_t stream_handle) {
  Plan plan;
  int e = check_call(g, c, &plan);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> guard(g->lock);
  const cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_handle);
  const CozyLayerShape& s = c->shape;
  const int me = g->rank, world = g->world;
  const long long seq = ++g->seq;
  const int set = static_cast<int>(seq & 1);
  const size_t el = 2, d = static_cast<size_t>(s.head_dim), b = static_cast<size_t>(s.batch);
  const size_t mine = static_cast<size_t>(s.rows[me]);
  const bool sm_cross = c->cross && world > 1;
  // the staging buffer is free once the previous call's copies have left
  if ((e = cudaStreamWaitEvent(stream, g->sent, 0)) != cudaSuccess) return e;
  if (sm_cross && (e = cudaEventRecord(g->cross_start, stream)) != cudaSuccess) return e;
  // 1. first stage: own block into own receive buffer, the others into staging (copy-engine
  //    crossing) or straight into their owners' receive buffers (SM crossing; destinations
  //    listed from this rank on, so the ranks write to different peers at any moment)
  CozyPackTensor t[3];
  memset(t, 0, sizeof(t));
  const void* src[3] = {c->q, c->k, c->v};
  const long long* strides[3] = {c->q_strides, c->k_strides, c->v_strides};
  const int heads[3] = {s.heads_q, s.heads_kv, s.heads_kv};
  size_t stage_off = 0;
  size_t block_off[3][COZY_MAX_PEERS] = {};
  for (int i = 0; i < 3; ++i) {
    t[i].src = src[i];
    for (int k = 0; k < 3; ++k) t[i].src_strides[k] = strides[i][k];
    t[i].heads = heads[i];
    t[i].rotate = c->rope != nullptr && i < 2;
    t[i].normalize = i == 0 ? c->norm_q : (i == 1 ? c->norm_k : 0);
    t[i].norm_weight = i == 0 ? c->norm_q_weight : (i == 1 ? c->norm_k_weight : nullptr);
    t[i].norm_offset = i < 2 ? c->norm_offset[i] : 0.f;
    t[i].norm_eps = i < 2 ? c->norm_eps[i] : 0.f;
    for (int p = 0; p < world; ++p) {
      if (sm_cross) {
        const int q = (me + p) % world;
        const int n = i == 0 ? plan.q_n[q] : plan.kv_n[q];
        t[i].head_lo[p] = i == 0 ? plan.q_lo[q] : plan.kv_lo[q];
        t[i].head_n[p] = n;
        t[i].dst[p] = n == 0 ? nullptr
                             : static_cast<uint8_t*>(g->peer[q][set][i]) +
                                   row_offset(plan, s, me, n);
        continue;
      }
      const int n = i == 0 ? plan.q_n[p] : plan.kv_n[p];
      t[i].head_lo[p] = i == 0 ? plan.q_lo[p] : plan.kv_lo[p];
      t[i].head_n[p] = n;
      if (p == me) {
        t[i].dst[p] = static_cast<uint8_t*>(g->mine[set][i]) + row_offset(plan, s, me, n);
      } else {
        block_off[i][p] = stage_off;
        t[i].dst[p] = static_cast<uint8_t*>(g->stage) + stage_off;
        stage_off += mine * b * n * d * el;
      }
      if (n == 0) t[i].dst[p] = nullptr;
    }
  }
  CozyRope rope;
  if (c->rope != nullptr) {
    rope = *c->rope;
    rope.token0 = plan.start[me];
  }
  if (mine > 0 &&
      (e = cozy::ulysses_pack_to(t, 3, world, s.rows[me], s.batch, s.head_dim,
                                 c->rope != nullptr ? &rope : nullptr, sm_cross, stream)) !=
          cudaSuccess)
    return e;
  if (sm_cross) {
    // 2. the flags: every block stored (the pack's bulk stores complete before it ends), one
    //    kernel fences at system scope and sets this rank's flag in every rank's memory
    //    (its own too, which the gate waits on)
    CozyPeerSlots slots;
    memset(&slots, 0, sizeof(slots));
    slots.count = world;
    for (int p = 0; p < world; ++p) slots.slot[p] = g->peer_flags[p] + kQKV * world + me;
    if ((e = cozy::peer_signal(&slots, seq, c->status, stream)) != cudaSuccess) return e;
    g->cross_bytes = 0;
    for (int p = 0; p < world; ++p)
      if (p != me)
        g->cross_bytes += mine * b * (plan.q_n[p] + 2 * plan.kv_n[p]) * d * el;
    if ((e = cudaEventRecord(g->cross_end, stream)) != cudaSuccess) return e;
    return cudaEventRecord(g->sent, stream);
  }
  if ((e = cudaEventRecord(g->packed, stream)) != cudaSuccess) return e;
  if (c->gate && world > 1 && (e = write_flag(g, g->flags + kQKV * world + me, seq, stream)) !=
                                  cudaSuccess)
    return e;
  // 2. the crossing: copy engines, destination by destination, each followed by its flag
  const int used = std::min(world - 1, kLanes);
  for (int l = 0; l < std::max(used, 1); ++l)
    if ((e = cudaStreamWaitEvent(g->lanes[l], g->packed, 0)) != cudaSuccess) return e;
  if ((e = cudaEventRecord(g->cross_start, g->side)) != cudaSuccess) return e;
  g->cross_bytes = 0;
  for (int step = 1; step < world; ++step) {
    const int p = (me + step) % world;
    const cudaStream_t lane = g->lanes[(step - 1) % kLanes];
    for (int i = 0; i < 3; ++i) {
      const int n = i == 0 ? plan.q_n[p] : plan.kv_n[p];
      const size_t bytes = mine * b * n * d * el;
      if (bytes == 0) continue;
      g->cross_bytes += bytes;
      uint8_t* dst = static_cast<uint8_t*>(g->peer[p][set][i]) + row_offset(plan, s, me, n);
      if ((e = cudaMemcpyAsync(dst, static_cast<uint8_t*>(g->stage) + block_off[i][p], bytes,
                               cudaMemcpyDeviceToDevice, lane)) != cudaSuccess)
        return e;
    }
    if ((e = write_flag(g, g->peer_flags[p] + kQKV * world + me, seq, lane)) != cudaSuccess)
      return e;
  }
  // lane 0 joins the others: `sent` and the crossing's end cover every lane
  for (int l = 1; l < used; ++l) {
    if ((e = cudaEventRecord(g->lane_done[l], g->lanes[l])) != cudaSuccess) return e;
    if ((e = cudaStreamWaitEvent(g->side, g->lane_done[l], 0)) != cudaSuccess) return e;
  }
  if ((e = cudaEventRecord(g->cross_end, g->side)) != cudaSuccess) return e;
  return cudaEventRecord(g->sent, g->side);
}

int cozy_ulysses_layer_attend(CozyGroup* g, const CozyLayerCall* c, uintptr_t stream_handle) {
  Plan plan;
  int e = check_call(g, c, &plan);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> guard(g->lock);
  const cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_handle);
  const CozyLayerShape& s = c->shape;
  const int me = g->rank, world = g->world;
  const long long seq = g->seq;
  const int set = static_cast<int>(seq & 1);
  const int qn = plan.q_n[me], kvn = plan.kv_n[me];
  const bool gate = c->gate && world > 1;
  if (gate) {  // every source's rows (this rank's own flag set after its pack) before the attention
    const long long limit = c->wait_limit_ns > 0 ? c->wait_limit_ns : kDefaultWaitNs;
    if ((e = cozy::peer_wait(g->flags + kQKV * world, world, seq, limit, c->status, stream)) !=
        cudaSuccess)
      return e;
  }
  if (qn > 0) {
    const long long b = s.batch, d = s.head_dim;
    const long long qs[3] = {b * qn * d, d, qn * d};
    const long long ks[3] = {b * kvn * d, d, kvn * d};
    const CozyHeadMap map = {plan.group, plan.q_lo[me], plan.kv_lo[me]};
    CozyScatter sc;
    memset(&sc, 0, sizeof(sc));
    sc.world = world;
    sc.head_offset = plan.q_lo[me];
    for (int p = 0; p <= world; ++p) sc.row_start[p] = plan.start[p];
    for (int p = 0; p < world; ++p) {
      sc.out[p] = g->peer[p][set][3];
      sc.strides[p][0] = static_cast<long long>(s.heads_q) * d;
      sc.strides[p][1] = d;
      sc.strides[p][2] = static_cast<long long>(s.rows[p]) * s.heads_q * d;
    }
    cozy::Arrival arrival;
    memset(&arrival, 0, sizeof(arrival));
    arrival.flags = g->flags + kQKV * world;
    arrival.seq = seq;
    arrival.limit_ns = c->wait_limit_ns > 0 ? c->wait_limit_ns : kDefaultWaitNs;
    arrival.n_src = world;
    arrival.self = me;
    for (int p = 0; p <= world; ++p) arrival.src_start[p] = plan.start[p];
    const float scale = c->scale > 0.f ? c->scale : 1.f / sqrtf(static_cast<float>(d));
    e = cozy::attention_forward_ex(g->mine[set][0], g->mine[set][1], g->mine[set][2], nullptr,
                                   s.batch, plan.total, plan.total, qn, kvn, s.head_dim, qs, ks,
                                   ks, nullptr, &map, &sc, s.causal, scale, c->status,
                                   world > 1 && !gate ? &arrival : nullptr, g->workspace,
                                   g->caps.workspace, stream);
    if (e != cudaSuccess) return e;
  }
  // 4a. every owner's rows from this rank have landed (skipped after a timeout on this GPU)
  CozyPeerSlots slots;
  memset(&slots, 0, sizeof(slots));
  slots.count = world;
  for (int p = 0; p < world; ++p) slots.slot[p] = g->peer_flags[p] + kOut * world + me;
  return cozy::peer_signal(&slots, seq, c->status, stream);
}

int cozy_ulysses_layer_end(CozyGroup* g, const CozyLayerCall* c, uintptr_t stream_handle) {
  Plan plan;
  int e = check_call(g, c, &plan);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> guard(g->lock);
  const cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_handle);
  const CozyLayerShape& s = c->shape;
  const long long seq = g->seq;
  const int set = static_cast<int>(seq & 1);
  const long long limit = c->wait_limit_ns > 0 ? c->wait_limit_ns : kDefaultWaitNs;
  if ((e = cozy::peer_wait(g->flags + kOut * g->world, g->world, seq, limit, c->status,
                           stream)) != cudaSuccess)
    return e;
  const size_t bytes =
      static_cast<size_t>(s.batch) * s.rows[g->rank] * s.heads_q * s.head_dim * 2;
  if (bytes == 0) return cudaSuccess;
  return cudaMemcpyAsync(c->out, g->mine[set][3], bytes, cudaMemcpyDeviceToDevice, stream);
}

int cozy_ulysses_layer_fwd(CozyGroup* g, const CozyLayerCall* c, uintptr_t stream) {
  int e = cozy_ulysses_layer_begin(g, c, stream);
  if (e == cudaSuccess) e = cozy_ulysses_layer_attend(g, c, stream);
  if (e == cudaSuccess) e = cozy_ulysses_layer_end(g, c, stream);
  return e;
}

}  // extern "C"
