// Peer memory for the in-kernel NVLink exchange: buffers shared between the GPUs of one node
// through CUDA IPC, and the arrival flags the ranks signal each other through.
//
// A flag is a 64-bit word in the receiving rank's memory, one per (kind, source rank). A source
// publishes "call `seq` of kind k has landed in your buffers" by storing seq into it with release
// semantics at system scope, after a system-scope fence; the receiver waits (bounded) until every
// source's word reaches seq with acquire loads. Sequence numbers only grow, so flags are never
// reset.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "../../include/cozy_ulysses.h"
#include "sm100.cuh"

namespace cozy {

__global__ void peer_signal_kernel(CozyPeerSlots slots, long long seq, const int* status) {
  const int i = threadIdx.x;
  __threadfence_system();
  // after a timed-out wait on this GPU nothing more is published to the peers
  if (status != nullptr && *reinterpret_cast<const volatile int*>(status) != kStatusOk) return;
  if (i < slots.count) {
    long long* slot = slots.slot[i];
    asm volatile("st.release.sys.global.s64 [%0], %1;" ::"l"(slot), "l"(seq) : "memory");
  }
}

__global__ void peer_wait_kernel(const long long* flags, int count, long long seq,
                                 long long limit_ns, int* status) {
  const int i = threadIdx.x;
  if (i < count) {
    const long long* flag = flags + i;
    const uint64_t start = global_timer_ns();
    for (uint32_t spin = 0;; ++spin) {
      long long v;
      asm volatile("ld.acquire.sys.global.s64 %0, [%1];" : "=l"(v) : "l"(flag) : "memory");
      if (v >= seq) break;
      if ((spin & 255u) == 255u) {
        if (status != nullptr && *reinterpret_cast<volatile int*>(status) != kStatusOk) break;
        if (global_timer_ns() - start > static_cast<uint64_t>(limit_ns)) {
          if (status != nullptr) atomicCAS(status, kStatusOk, kStatusPeerTimeout);
          break;
        }
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  __threadfence_system();
}

int peer_signal(const CozyPeerSlots* slots, long long seq, const int* status,
                cudaStream_t stream) {
  if (slots == nullptr || slots->count < 0 || slots->count > COZY_MAX_PEERS)
    return cudaErrorInvalidValue;
  for (int i = 0; i < slots->count; ++i)
    if (slots->slot[i] == nullptr || reinterpret_cast<uintptr_t>(slots->slot[i]) % 8)
      return cudaErrorInvalidValue;
  peer_signal_kernel<<<1, 32, 0, stream>>>(*slots, seq, status);
  return cudaGetLastError();
}

int peer_wait(const long long* flags, int count, long long seq, long long limit_ns, int* status,
              cudaStream_t stream) {
  if (flags == nullptr || count < 0 || count > COZY_MAX_PEERS || limit_ns <= 0)
    return cudaErrorInvalidValue;
  peer_wait_kernel<<<1, 32, 0, stream>>>(flags, count, seq, limit_ns, status);
  return cudaGetLastError();
}

}  // namespace cozy

extern "C" {

int cozy_ipc_alloc(unsigned long long bytes, void** ptr, void* handle) {
  if (ptr == nullptr || handle == nullptr || bytes == 0) return cudaErrorInvalidValue;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return e;
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return e;
  }
  *ptr = p;
  return cudaSuccess;
}

int cozy_ipc_open(const void* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return cudaErrorInvalidValue;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

int cozy_ipc_close(void* ptr) { return cudaIpcCloseMemHandle(ptr); }

int cozy_ipc_free(void* ptr) { return cudaFree(ptr); }

int cozy_ipc_handle_bytes(void) { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }

int cozy_peer_signal(const CozyPeerSlots* slots, long long seq, uintptr_t stream) {
  return cozy::peer_signal(slots, seq, nullptr, reinterpret_cast<cudaStream_t>(stream));
}

int cozy_peer_wait(const long long* flags, int count, long long seq, long long limit_ns,
                   int* status, uintptr_t stream) {
  return cozy::peer_wait(flags, count, seq, limit_ns, status,
                         reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
