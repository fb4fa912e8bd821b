// Internal interface of the attention kernel's launcher for the library's own callers (the
// layer entry in layer.cu): the crossing-aware launch and the split workspace size. Not part of
// the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include "../../include/cozy_ulysses.h"

namespace cozy {

// Rows that are still crossing from other GPUs when the attention starts: rows
// [src_start[s], src_start[s + 1]) of the (whole-sequence) operands come from source s and are
// resident once flags[s] (this GPU's memory, written by source s) reaches `seq`. Row block
// `self` is resident at launch. The kernel waits per source, at most `limit_ns`, then reports a
// peer timeout in the status word and returns.
struct Arrival {
  const long long* flags;
  long long seq;
  long long limit_ns;
  int n_src;
  int self;
  int src_start[COZY_MAX_PEERS + 1];
};

// cozy_attention_fwd with an optional arrival (nullptr: every row resident) and the split's
// workspace given by the caller (`workspace` of `workspace_bytes`; nullptr: the launch runs
// unsplit). Allocates nothing.
int attention_forward_ex(const void* q, const void* k, const void* v, void* out, int batch,
                         int seq_q, int seq_k, int heads_q, int heads_kv, int head_dim,
                         const long long* q_strides, const long long* k_strides,
                         const long long* v_strides, const long long* o_strides,
                         const CozyHeadMap* head_map, const CozyScatter* scatter, int causal,
                         float scale, int* status, const Arrival* arrival, void* workspace,
                         size_t workspace_bytes, cudaStream_t stream);

// Bytes of split workspace a call of this shape takes on a GPU of `sms` SMs (0: it runs unsplit).
size_t attention_workspace_bytes(int batch, int seq_q, int seq_k, int heads_q, int head_dim,
                                 int causal, int sms);

}  // namespace cozy
