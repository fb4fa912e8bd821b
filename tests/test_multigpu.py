"""The exchange between GPU processes (one per GPU) over both transports — in-kernel NVLink peer
stores and NCCL all-to-all — against the reference's golden outputs and the oracle. Needs two or
more GPUs; skipped otherwise.

Each case spawns W processes (W ≤ visible GPUs), every rank passes its `tensor_split` rows and
the rows come from the store meeting (no `rows` argument), as the reference's exchange does.
NVLS is off (`NCCL_NVLS_ENABLE=0`), as the reference's group formation sets it.
"""

import os
import socket
import tempfile

import pytest
import torch

import oracle
from tests._golden import load, narrow_cases, tensor, ulysses_cases

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _gpus() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _sdpa_compute(qq, kk, vv):
    """A caller's own head-local compute: torch SDPA in fp32 on [B, S, h, D] views."""
    o = torch.nn.functional.scaled_dot_product_attention(
        qq.transpose(1, 2).float(), kk.transpose(1, 2).float(), vv.transpose(1, 2).float())
    return o.transpose(1, 2).to(qq.dtype)


def _rank(rank, world, port, inputs, causal, outdir, rope_args, transport, fp8=False,
          narrow=False, compute=False):
    import torch.distributed as dist

    from cozy_runtime_b200 import rope as rope_mod
    from cozy_runtime_b200 import ulysses

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group(
        "nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
        device_id=device,
    )
    q, k, v = (torch.tensor_split(t, world, dim=1)[rank].contiguous().to(device) for t in inputs)
    spec = None
    if rope_args is not None:
        spec = rope_mod.axial(rope_args[0], (44, 42, 42), after=rope_args[1]).to(device)
    outs = [
        ulysses.exchange(q, k, v, dist.group.WORLD, _sdpa_compute if compute else None,
                         causal=causal, rope=spec, transport=transport, fp8=fp8, narrow=narrow)
        for _ in range(3)
    ]
    torch.cuda.synchronize()
    from cozy_runtime_b200 import attention

    attention.check_status(device)
    out = outs[0]
    assert all(torch.equal(out, o) for o in outs[1:]), "repeated calls differ"
    torch.save(out.cpu(), os.path.join(outdir, f"{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def _run(inputs, world, causal=False, rope_args=None, transport="peer", fp8=False,
         narrow=False, compute=False):
    import torch.multiprocessing as mp

    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_rank, args=(world, _port(), inputs, causal, tmp, rope_args, transport, fp8,
                              narrow, compute),
                 nprocs=world, join=True)
        return torch.cat([torch.load(os.path.join(tmp, f"{r}.pt")) for r in range(world)], dim=1)


def _check(got, want):
    err = (got.float() - want.float()).abs()
    assert err.max().item() <= MAX_ABS, f"max-abs {err.max().item():.3e}"
    assert err.mean().item() <= MEAN_ABS, f"mean-abs {err.mean().item():.3e}"


@pytest.mark.parametrize("transport", ["peer", "nccl"])
@pytest.mark.parametrize("name", ulysses_cases())
def test_exchange_matches_reference_golden(name, transport):
    case = load(name)
    world = int(case["world"])
    if world < 2 or world > _gpus():
        pytest.skip(f"needs {world} GPUs")
    inputs = tuple(tensor(case[key]) for key in ("q", "k", "v"))
    got = _run(inputs, world, causal=bool(case["causal"]), transport=transport)
    _check(got, tensor(case["out"]).float())


@pytest.mark.parametrize(
    "world,hq,hkv,causal,rotate",
    [(2, 8, 8, False, True), (4, 8, 2, True, False), (8, 8, 8, False, True), (8, 32, 8, True, False),
     (3, 5, 5, False, True)],
)
@pytest.mark.parametrize("transport", ["peer", "nccl"])
def test_exchange_against_oracle(world, hq, hkv, causal, rotate, transport):
    if world > _gpus():
        pytest.skip(f"needs {world} GPUs")
    from cozy_runtime_b200 import rope as rope_mod

    g = torch.Generator().manual_seed(world + hq)
    grid, text = (2, 6, 10), 17
    seq = 2 * 6 * 10 + text
    q = torch.randn(1, seq, hq, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(1, seq, hkv, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(1, seq, hkv, 128, generator=g).to(torch.bfloat16)
    got = _run((q, k, v), world, causal=causal, rope_args=(grid, text) if rotate else None,
               transport=transport)
    if rotate:
        spec = rope_mod.axial(grid, (44, 42, 42), after=text)
        q, k = (oracle.head_norm_rope(t.float(), spec.cos, spec.sin, rotary=128, interleaved=True,
                                      normalize=False).to(torch.bfloat16) for t in (q, k))
    _check(got, oracle.attention_fp32(q, k, v, causal=causal))


@pytest.mark.parametrize("world,hq,hkv,causal", [(2, 4, 4, False), (8, 16, 16, False), (4, 8, 2, True)])
def test_fp8_exchange_peer_against_law(world, hq, hkv, causal):
    """The FP8 path over the NVLink transport (statistics all-reduced, e4m3 codes and scales
    stored into the owners' buffers) against the oracle's FP8 law and exact attention."""
    if world > _gpus():
        pytest.skip(f"needs {world} GPUs")
    g = torch.Generator().manual_seed(world * 7 + hq)
    seq = 1000
    q = torch.randn(1, seq, hq, 128, generator=g)
    k = torch.randn(1, seq, hkv, 128, generator=g)
    v = torch.randn(1, seq, hkv, 128, generator=g)
    k = torch.where(torch.rand(k.shape, generator=g) < 0.01, k * 8, k)
    q, k, v = (t.to(torch.bfloat16) for t in (q, k, v))
    got = _run((q, k, v), world, causal=causal, fp8=True).float()
    rows = [t.shape[0] for t in torch.tensor_split(torch.empty(seq), world)]
    law = oracle.fp8_attention_law(*(torch.split(t, rows, dim=1) for t in (q, k, v)), causal=causal)

    def cos(a, b):
        a = a.permute(0, 2, 1, 3).reshape(a.shape[2], -1)
        b = b.permute(0, 2, 1, 3).reshape(b.shape[2], -1)
        return torch.nn.functional.cosine_similarity(a, b, dim=1).min().item()

    assert cos(got, law) >= 0.999
    assert cos(got, oracle.attention_fp32(q, k, v, causal=causal)) >= 0.995


@pytest.mark.parametrize("transport", ["peer", "nccl"])
@pytest.mark.parametrize("name", narrow_cases())
def test_narrow_exchange_matches_reference_golden(name, transport):
    """The int8 wire between GPU processes against the reference's own narrow exchange."""
    case = load(name)
    world = int(case["world"])
    if world < 2 or world > _gpus():
        pytest.skip(f"needs {world} GPUs")
    inputs = tuple(tensor(case[key]) for key in ("q", "k", "v"))
    got = _run(inputs, world, causal=bool(case["causal"]), transport=transport, narrow=True)
    _check(got, tensor(case["out"]).float())


@pytest.mark.parametrize("world,hq,hkv,causal", [(2, 4, 4, False), (4, 8, 2, True), (8, 16, 16, False)])
@pytest.mark.parametrize("transport", ["peer", "nccl"])
def test_narrow_exchange_against_oracle(world, hq, hkv, causal, transport):
    if world > _gpus():
        pytest.skip(f"needs {world} GPUs")
    g = torch.Generator().manual_seed(world * 31 + hq)
    seq = 1000 + world
    q = torch.randn(1, seq, hq, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(1, seq, hkv, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(1, seq, hkv, 128, generator=g).to(torch.bfloat16)
    got = _run((q, k, v), world, causal=causal, transport=transport, narrow=True)
    parts = [torch.tensor_split(t, world, dim=1) for t in (q, k, v)]
    want = torch.cat(oracle.exchange_narrow(
        *parts, lambda a, b, c: oracle.attention_fp32(a, b, c, causal=causal)), dim=1)
    _check(got, want.float())


@pytest.mark.parametrize("world", [2, 4])
def test_exchange_with_callable_compute(world):
    """The bf16 exchange with a caller's own compute (sparse producers' use) across processes:
    NCCL crossing, [B, S, h, D] operands, against the oracle."""
    if world > _gpus():
        pytest.skip(f"needs {world} GPUs")
    g = torch.Generator().manual_seed(40 + world)
    q, k, v = (torch.randn(1, 803, 8, 128, generator=g).to(torch.bfloat16) for _ in range(3))
    got = _run((q, k, v), world, compute=True)
    _check(got, oracle.attention_fp32(q, k, v))
