"""The exchange between GPU processes (one per GPU) over both transports — the NVLink layer
(copy-engine crossing overlapped with the attention) and NCCL all-to-all — against the
reference's golden outputs and the oracle. Needs two or more GPUs; skipped otherwise.

Every rank passes its `tensor_split` rows and the rows come from the store meeting (no `rows`
argument), as the reference's exchange does. NVLS is off (`NCCL_NVLS_ENABLE=0`), as the
reference's group formation sets it. To keep process start-up and NCCL formation out of every
case, the cases of one degree W run in one set of W processes (started once, on the first test
that needs that degree); each case's inputs are rebuilt in every process from a small
description, each case runs three times (the repeats must agree bit for bit), and the tests
then check what the processes saved.
"""

import os
import socket
import tempfile
import traceback

import pytest
import torch

import oracle
from tests._golden import load, narrow_cases, tensor, ulysses_cases

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

MAX_ABS, MEAN_ABS = 2e-2, 2e-3
GRID, TEXT = (2, 6, 10), 17


def _gpus() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# ----------------------------------------------------------------------------- the cases
def _random_inputs(seed, seq, hq, hkv, outliers=False):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, seq, hq, 128, generator=g)
    k = torch.randn(1, seq, hkv, 128, generator=g)
    v = torch.randn(1, seq, hkv, 128, generator=g)
    if outliers:
        k = torch.where(torch.rand(k.shape, generator=g) < 0.01, k * 8, k)
    return tuple(t.to(torch.bfloat16) for t in (q, k, v))


def inputs_of(case: dict):
    """The whole [B, S, H, D] Q, K, V of a case (every process rebuilds them alike)."""
    if "golden" in case:
        data = load(case["golden"])
        return tuple(tensor(data[key]) for key in ("q", "k", "v"))
    return _random_inputs(case["seed"], case["seq"], case["hq"], case["hkv"],
                          case.get("outliers", False))


def _cases() -> list[dict]:
    out = []
    for name in ulysses_cases():
        world = int(load(name)["world"])
        for transport in ("peer", "nccl"):
            out.append({"id": f"golden-{name}-{transport}", "world": world, "golden": name,
                        "causal": bool(load(name)["causal"]), "transport": transport})
    for world, hq, hkv, causal, rotate in [(2, 8, 8, False, True), (4, 8, 2, True, False),
                                           (8, 8, 8, False, True), (8, 32, 8, True, False),
                                           (3, 5, 5, False, True), (7, 32, 8, True, False)]:
        for transport in ("peer", "nccl"):
            out.append({"id": f"oracle-w{world}-{hq}-{hkv}-{causal}-{rotate}-{transport}",
                        "world": world, "seed": world + hq, "seq": 2 * 6 * 10 + TEXT, "hq": hq,
                        "hkv": hkv, "causal": causal, "rotate": rotate, "transport": transport})
    for world, hq, hkv, causal, transport in [(2, 4, 4, False, "peer"), (8, 16, 16, False, "peer"),
                                              (4, 8, 2, True, "peer"), (2, 4, 4, False, "nccl"),
                                              (4, 8, 2, True, "nccl"), (8, 16, 16, False, "nccl")]:
        out.append({"id": f"fp8-w{world}-{hq}-{hkv}-{causal}-{transport}", "world": world,
                    "seed": world * 7 + hq, "seq": 1000, "hq": hq, "hkv": hkv, "causal": causal,
                    "outliers": True, "fp8": True, "transport": transport})
    for world, transport in [(2, "peer"), (4, "nccl")]:  # the reference's per-head FP8 row
        out.append({"id": f"fp8head-w{world}-{transport}", "world": world, "seed": 70 + world,
                    "seq": 1000, "hq": 8, "hkv": 8, "causal": False, "outliers": True,
                    "fp8": "head", "transport": transport})
    for world, transport in [(2, "peer"), (4, "nccl"), (8, "peer")]:  # RoPE in the e4m3 stage
        out.append({"id": f"fp8rope-w{world}-{transport}", "world": world, "seed": 60 + world,
                    "seq": 2 * 6 * 10 + TEXT, "hq": 8, "hkv": 8, "causal": False,
                    "rotate": True, "fp8": True, "transport": transport})
    for name in narrow_cases():
        world = int(load(name)["world"])
        for transport in ("peer", "nccl"):
            out.append({"id": f"narrowgolden-{name}-{transport}", "world": world,
                        "golden": name, "causal": bool(load(name)["causal"]), "narrow": True,
                        "transport": transport})
    for world, hq, hkv, causal in [(2, 4, 4, False), (4, 8, 2, True), (8, 16, 16, False)]:
        for transport in ("peer", "nccl"):
            out.append({"id": f"narrow-w{world}-{hq}-{hkv}-{causal}-{transport}", "world": world,
                        "seed": world * 31 + hq, "seq": 1000 + world, "hq": hq, "hkv": hkv,
                        "causal": causal, "narrow": True, "transport": transport})
    for world in (2, 4, 8):
        out.append({"id": f"compute-w{world}", "world": world, "seed": 40 + world, "seq": 803,
                    "hq": 8, "hkv": 8, "causal": False, "compute": True, "transport": "nccl"})
    return out


CASES = {c["id"]: c for c in _cases()}


# ----------------------------------------------------------------------- the processes
def _sdpa_compute(qq, kk, vv):
    """A caller's own head-local compute: torch SDPA in fp32 on [B, S, h, D] views."""
    o = torch.nn.functional.scaled_dot_product_attention(
        qq.transpose(1, 2).float(), kk.transpose(1, 2).float(), vv.transpose(1, 2).float())
    return o.transpose(1, 2).to(qq.dtype)


def _batch_rank(rank, world, port, cases, outdir):
    import torch.distributed as dist

    from cozy_runtime_b200 import attention, ulysses
    from cozy_runtime_b200 import rope as rope_mod

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    from datetime import timedelta

    dist.init_process_group(
        "nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
        device_id=device, timeout=timedelta(seconds=120),
    )
    for case in cases:
        path = os.path.join(outdir, f"{case['id']}.{rank}")
        try:
            q, k, v = (torch.tensor_split(t, world, dim=1)[rank].contiguous().to(device)
                       for t in inputs_of(case))
            spec = None
            if case.get("rotate"):
                spec = rope_mod.axial(GRID, (44, 42, 42), after=TEXT).to(device)
            outs = [
                ulysses.exchange(
                    q, k, v, dist.group.WORLD, _sdpa_compute if case.get("compute") else None,
                    causal=case["causal"], rope=spec, transport=case["transport"],
                    fp8=case.get("fp8", False), narrow=case.get("narrow", False))
                for _ in range(3)
            ]
            torch.cuda.synchronize()
            attention.check_status(device)
            if not all(torch.equal(outs[0], o) for o in outs[1:]):
                raise AssertionError("repeated calls differ")
            torch.save(outs[0].cpu(), path + ".pt")
            with open(path + ".transport", "w") as fh:
                fh.write(ulysses.transport_of(dist.group.WORLD, device)
                         if case["transport"] == "peer" else "nccl")
        except Exception:  # noqa: BLE001 - recorded for the test that owns the case
            with open(path + ".err", "w") as fh:
                fh.write(traceback.format_exc())
    dist.barrier()
    dist.destroy_process_group()


_RUNS: dict[int, str] = {}
_TMP = tempfile.TemporaryDirectory()


def _result(case_id: str) -> torch.Tensor:
    """The whole output of a case (its degree's processes run once, on first need)."""
    case = CASES[case_id]
    world = case["world"]
    if world < 2 or world > _gpus():
        pytest.skip(f"needs {world} GPUs")
    if world not in _RUNS:
        import torch.multiprocessing as mp

        outdir = os.path.join(_TMP.name, f"w{world}")
        os.makedirs(outdir, exist_ok=True)
        todo = [c for c in CASES.values() if c["world"] == world]
        mp.spawn(_batch_rank, args=(world, _port(), todo, outdir), nprocs=world, join=True)
        _RUNS[world] = outdir
    outdir = _RUNS[world]
    parts = []
    for rank in range(world):
        path = os.path.join(outdir, f"{case_id}.{rank}")
        if os.path.exists(path + ".err"):
            raise AssertionError(f"rank {rank}:\n" + open(path + ".err").read())
        parts.append(torch.load(path + ".pt"))
        if CASES[case_id]["transport"] == "peer":
            assert open(path + ".transport").read() == "peer", "the peer transport did not form"
    return torch.cat(parts, dim=1)


def _check(got, want):
    err = (got.float() - want.float()).abs()
    assert err.max().item() <= MAX_ABS, f"max-abs {err.max().item():.3e}"
    assert err.mean().item() <= MEAN_ABS, f"mean-abs {err.mean().item():.3e}"


# ---------------------------------------------------------------------------- the tests
@pytest.mark.parametrize("case_id", [c for c in CASES if c.startswith("golden-")])
def test_exchange_matches_reference_golden(case_id):
    got = _result(case_id)
    _check(got, tensor(load(CASES[case_id]["golden"])["out"]).float())


@pytest.mark.parametrize("case_id", [c for c in CASES if c.startswith("oracle-")])
def test_exchange_against_oracle(case_id):
    from cozy_runtime_b200 import rope as rope_mod

    case = CASES[case_id]
    got = _result(case_id)
    q, k, v = inputs_of(case)
    if case["rotate"]:
        spec = rope_mod.axial(GRID, (44, 42, 42), after=TEXT)
        q, k = (oracle.head_norm_rope(t.float(), spec.cos, spec.sin, rotary=128, interleaved=True,
                                      normalize=False).to(torch.bfloat16) for t in (q, k))
    _check(got, oracle.attention_fp32(q, k, v, causal=case["causal"]))


@pytest.mark.parametrize("case_id", [c for c in CASES if c.startswith("fp8")])
def test_fp8_exchange_against_law(case_id):
    """The FP8 path between processes (statistics all-reduced; e4m3 codes and scales stored
    into the owners' buffers over NVLink, or crossing by NCCL all-to-all), with RoPE fused into
    the e4m3 first stage in the `fp8rope` cases, against the oracle's FP8 law and exact
    attention over the first stage's output."""
    from cozy_runtime_b200 import rope as rope_mod

    case = CASES[case_id]
    got = _result(case_id).float()
    q, k, v = inputs_of(case)
    if case.get("rotate"):
        spec = rope_mod.axial(GRID, (44, 42, 42), after=TEXT)
        q, k = (oracle.head_norm_rope(t.float(), spec.cos, spec.sin, rotary=128, interleaved=True,
                                      normalize=False).to(torch.bfloat16) for t in (q, k))
    rows = [t.shape[0] for t in torch.tensor_split(torch.empty(case["seq"]), case["world"])]
    law = oracle.fp8_attention_law(*(torch.split(t, rows, dim=1) for t in (q, k, v)),
                                   causal=case["causal"],
                                   law="head" if case["fp8"] == "head" else "block")

    def cos(a, b):
        a = a.permute(0, 2, 1, 3).reshape(a.shape[2], -1)
        b = b.permute(0, 2, 1, 3).reshape(b.shape[2], -1)
        return torch.nn.functional.cosine_similarity(a, b, dim=1).min().item()

    assert cos(got, law) >= 0.999
    assert cos(got, oracle.attention_fp32(q, k, v, causal=case["causal"])) >= 0.995


@pytest.mark.parametrize("case_id", [c for c in CASES if c.startswith("narrowgolden-")])
def test_narrow_exchange_matches_reference_golden(case_id):
    """The int8 wire between GPU processes against the reference's own narrow exchange."""
    got = _result(case_id)
    _check(got, tensor(load(CASES[case_id]["golden"])["out"]).float())


@pytest.mark.parametrize("case_id", [c for c in CASES if c.startswith("narrow-w")])
def test_narrow_exchange_against_oracle(case_id):
    case = CASES[case_id]
    got = _result(case_id)
    q, k, v = inputs_of(case)
    parts = [torch.tensor_split(t, case["world"], dim=1) for t in (q, k, v)]
    want = torch.cat(oracle.exchange_narrow(
        *parts, lambda a, b, c: oracle.attention_fp32(a, b, c, causal=case["causal"])), dim=1)
    _check(got, want.float())


@pytest.mark.parametrize("case_id", [c for c in CASES if c.startswith("compute-")])
def test_exchange_with_callable_compute(case_id):
    """The bf16 exchange with a caller's own compute (sparse producers' use) across processes:
    NCCL crossing, [B, S, h, D] operands, against the oracle."""
    got = _result(case_id)
    q, k, v = inputs_of(CASES[case_id])
    _check(got, oracle.attention_fp32(q, k, v))
