"""The allocation-free degree-1 entry point against the library's ordinary path.

`cozy_rope_attention_fwd_noalloc` serves callers that cannot allocate device memory while they
run (a stream under CUDA-graph capture, a serving loop with a fixed memory arena, a
latency-bound host thread): it keeps the rotated Q and K in a static device array instead of a
buffer. Its output must match the ordinary entry points — the first stage `cozy_ulysses_pack`
into an allocated buffer followed by `cozy_attention_fwd`, which `ulysses.exchange` runs at
degree 1 — at the bf16 tolerance the other GPU tests use (max-abs 2e-2, mean-abs 2e-3), on two
calls in a row (the second call reuses the array the first one left behind), and against the CPU
oracle's RMSNorm/RoPE and attention laws on the same inputs.

This file is collected last so a failure here never hides the rest of the suite.
"""

import ctypes
import math

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _strides(t):
    return (ctypes.c_longlong * 3)(t.stride(1), t.stride(2), t.stride(0))


def _noalloc(lib, q, k, v, out, spec, *, normalize, causal):
    from cozy_runtime_b200 import _lib, attention

    rope = _lib.Rope()
    rope.cos = spec.cos.data_ptr()
    rope.sin = spec.sin.data_ptr()
    rope.stride_token = spec.stride_token
    rope.stride_channel = spec.stride_channel
    rope.token0 = 0
    rope.rotary = spec.rotary
    rope.interleaved = int(spec.interleaved)
    batch, seq, hq, dim = q.shape
    return lib.cozy_rope_attention_fwd_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), batch, seq, hq, k.shape[2],
        dim, _strides(q), _strides(k), _strides(v), _strides(out), ctypes.byref(rope),
        int(normalize), 1e-6, int(causal), 1.0 / math.sqrt(dim),
        attention.status_word(q.device).data_ptr(), torch.cuda.current_stream().cuda_stream,
    )


@pytest.mark.parametrize(
    "batch,seq,hq,hkv,dim,causal,normalize,kind",
    [(1, 1000, 4, 2, 128, True, False, "llama"), (2, 300, 3, 3, 64, False, True, "axial")],
)
def test_noalloc_matches_ordinary_path(batch, seq, hq, hkv, dim, causal, normalize, kind):
    from cozy_runtime_b200 import _lib, attention, rope, ulysses

    lib = _lib.load()
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    if kind == "llama":
        spec = rope.llama(seq, dim)
    else:
        spec = rope.axial((3, 10, 10), (dim // 4, dim // 8 * 3, dim // 8 * 3))
    spec = spec.to(device)
    g = torch.Generator(device=device).manual_seed(seq + hq)
    q = torch.randn(batch, seq, hq, dim, generator=g, device=device).to(torch.bfloat16)
    k = torch.randn(batch, seq, hkv, dim, generator=g, device=device).to(torch.bfloat16)
    v = torch.randn(batch, seq, hkv, dim, generator=g, device=device).to(torch.bfloat16)
    norm = ulysses.Norm(eps=1e-6) if normalize else None
    want = ulysses.exchange(q, k, v, None, None, causal=causal, rope=spec, norm_q=norm,
                            norm_k=norm)
    for _ in range(2):
        got = torch.empty_like(q)
        code = _noalloc(lib, q, k, v, got, spec, normalize=normalize, causal=causal)
        assert code == 0, _lib.error_name(code)
        torch.cuda.synchronize()
        attention.check_status(device)
        err = (got.float() - want.float()).abs()
        assert err.max().item() <= MAX_ABS, f"max-abs {err.max().item():.3e}"
        assert err.mean().item() <= MEAN_ABS, f"mean-abs {err.mean().item():.3e}"
    # and on its own against the CPU oracle's law: RMSNorm/RoPE, then fp32 attention
    cos, sin = spec.cos.cpu(), spec.sin.cpu()
    tables = cos.reshape(-1, spec.stride_token), sin.reshape(-1, spec.stride_token)
    rot = [oracle.head_norm_rope(t.float().cpu(), *tables, rotary=spec.rotary,
                                 interleaved=spec.interleaved, normalize=normalize,
                                 stride_channel=spec.stride_channel).to(torch.bfloat16)
           for t in (q, k)]
    law = oracle.attention_fp32(rot[0], rot[1], v.cpu(), causal=causal)
    err = (got.float().cpu() - law).abs()
    assert err.max().item() <= MAX_ABS, f"oracle max-abs {err.max().item():.3e}"
    assert err.mean().item() <= MEAN_ABS, f"oracle mean-abs {err.mean().item():.3e}"


def test_noalloc_refuses_more_than_its_array():
    from cozy_runtime_b200 import _lib, rope

    lib = _lib.load()
    device = torch.device("cuda", 0)
    seq, heads, dim = 65536, 4, 128  # (4 + 4) * 65536 * 128 * 2 bytes = 128 MiB > 64 MiB
    spec = rope.llama(16, dim).to(device)
    x = torch.zeros(1, seq, heads, dim, dtype=torch.bfloat16, device=device)
    out = torch.empty_like(x)
    code = _noalloc(lib, x, x, x, out, spec, normalize=False, causal=False)
    assert code == _lib.INVALID_VALUE


def test_noalloc_refusal_launches_nothing():
    """A call the attention would refuse (3 query heads over 2 key/value heads) is refused
    before the first stage runs: no kernel is launched, so the shared array keeps what the
    last accepted call left in it."""
    from torch.profiler import ProfilerActivity, profile

    from cozy_runtime_b200 import _lib, rope

    lib = _lib.load()
    device = torch.device("cuda", 0)
    spec = rope.llama(64, 128).to(device)
    q = torch.zeros(1, 64, 3, 128, dtype=torch.bfloat16, device=device)
    kv = torch.zeros(1, 64, 2, 128, dtype=torch.bfloat16, device=device)
    out = torch.empty_like(q)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        code = _noalloc(lib, q, kv, kv, out, spec, normalize=False, causal=False)
        torch.cuda.synchronize()
    assert code == _lib.INVALID_VALUE
    launched = [e.name for e in prof.events() if "cozy" in e.name]
    assert not launched, launched
