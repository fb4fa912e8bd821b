"""The drop-in boundary on the GPU: the Diffusers-signature backend call and the exchange with a
caller's own `compute`, as the reference's callers use them.

`attention_ulysses.function(name)` builds the backend call (the reference's
src/cozy_runtime/internal/attention_ulysses.py:184-272): without a parallel config it runs the
kernel directly; with one it runs the exchange on the config's process group (here a one-rank
NCCL group, installed with `serve`). Sparse producers call `exchange(q, k, v, group, compute)`
with their own head-local compute (internal/producers.py:121-132). Checked against the CPU
oracle at the path's bf16 bar (max-abs ≤ 2e-2, mean-abs ≤ 2e-3).
"""

import socket

import pytest
import torch
import torch.distributed as dist

import oracle

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _check(got, want):
    err = (got.float().cpu() - want.float()).abs()
    assert err.max().item() <= MAX_ABS, f"max-abs {err.max().item():.3e}"
    assert err.mean().item() <= MEAN_ABS, f"mean-abs {err.mean().item():.3e}"


def _inputs(seq=700, hq=4, hkv=2, dim=128, seed=21):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, seq, hq, dim, generator=g).to(torch.bfloat16)
    k = torch.randn(1, seq, hkv, dim, generator=g).to(torch.bfloat16)
    v = torch.randn(1, seq, hkv, dim, generator=g).to(torch.bfloat16)
    return q, k, v


@pytest.fixture()
def one_rank_group():
    """A one-rank NCCL process group on cuda:0 (the group a parallel config names)."""
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0,
                            world_size=1, device_id=device)
    try:
        yield dist.group.WORLD
    finally:
        dist.destroy_process_group()


def test_backend_call_without_parallel_config():
    from cozy_runtime_b200 import attention_ulysses

    call = attention_ulysses.function("cozy_b200")
    q, k, v = _inputs()
    got = call(q.cuda(), k.cuda(), v.cuda(), is_causal=True, enable_gqa=True)
    torch.cuda.synchronize()
    assert got.shape == q.shape and got.dtype == q.dtype
    _check(got, oracle.attention_fp32(q, k, v, causal=True))


def test_backend_call_with_parallel_config(one_rank_group):
    from cozy_runtime_b200 import attention_ulysses

    class Config:  # what Diffusers passes as _parallel_config
        pass

    attention_ulysses.serve(lambda config: one_rank_group)
    try:
        call = attention_ulysses.function("cozy_b200")
        q, k, v = _inputs(seq=901, hq=6, hkv=6, seed=22)
        got = call(q.cuda(), k.cuda(), v.cuda(), scale=0.07, _parallel_config=Config())
        torch.cuda.synchronize()
        _check(got, oracle.attention_fp32(q, k, v, scale=0.07))
        # the refusals the reference makes under Ulysses stand
        with pytest.raises(ValueError):
            call(q.cuda(), k.cuda(), v.cuda(), attn_mask=torch.ones(1, device="cuda"),
                 _parallel_config=Config())
    finally:
        attention_ulysses.serve(None)


def test_exchange_with_callable_compute(one_rank_group):
    """The bf16 exchange with a caller's compute: it gets [B, S, h, D] views of whole sequences
    and returns the same shape; grouped K/V heads arrive replicated to the query heads."""
    from cozy_runtime_b200 import attention_ulysses

    seen = []

    def compute(qq, kk, vv):
        seen.append((tuple(qq.shape), tuple(kk.shape)))
        o = torch.nn.functional.scaled_dot_product_attention(
            qq.transpose(1, 2).float(), kk.transpose(1, 2).float(), vv.transpose(1, 2).float())
        return o.transpose(1, 2).to(qq.dtype)

    q, k, v = _inputs(seq=513, hq=4, hkv=2, seed=23)
    got = attention_ulysses.exchange(q.cuda(), k.cuda(), v.cuda(), one_rank_group, compute)
    torch.cuda.synchronize()
    assert seen == [((1, 513, 4, 128), (1, 513, 4, 128))]
    _check(got, oracle.attention_fp32(q, k, v))
