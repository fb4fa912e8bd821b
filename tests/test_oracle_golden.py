"""The oracle pinned against golden vectors from the reference's own code (no GPU)."""

import numpy as np
import pytest
import torch

import oracle
from tests._golden import load, narrow_cases, rope_cases, tensor, ulysses_cases


@pytest.mark.parametrize("name", ulysses_cases())
def test_exchange_matches_reference(name):
    case = load(name)
    q, k, v = (tensor(case[key]) for key in ("q", "k", "v"))
    world, causal = int(case["world"]), bool(case["causal"])
    rows = oracle.sequence_rows(q.shape[1], world)
    assert rows == [int(r) for r in case["rows"]]
    parts = [torch.tensor_split(t, world, dim=1) for t in (q, k, v)]
    outs = oracle.exchange(
        *parts, lambda a, b, c: oracle.attention_fp32(a, b, c, causal=causal)
    )
    got = torch.cat(outs, dim=1)
    want = tensor(case["out"]).float()
    if str(case["dtype"]) == "bfloat16":  # the reference computed in bf16: its own rounding
        assert (got - want).abs().max() < 2e-2
    else:
        assert (got - want).abs().max() < 2e-5


@pytest.mark.parametrize("name", rope_cases())
def test_rope_law_matches_reference(name):
    case = load(name)
    x = tensor(case["x"]).float()
    weight = tensor(case["weight"]) if int(case["has_weight"]) else None
    cos, sin = torch.from_numpy(case["cos"]), torch.from_numpy(case["sin"])
    cols = int(case["stride_token"])
    got = oracle.head_norm_rope(
        x,
        cos.reshape(-1, cols),
        sin.reshape(-1, cols),
        rotary=int(case["rotary"]),
        interleaved=bool(case["interleaved"]),
        weight=weight,
        offset=float(case["offset"]),
        eps=float(case["eps"]),
        stride_channel=int(case["stride_channel"]),
    )
    want = torch.from_numpy(case["want"])
    assert (got - want).abs().max() < 1e-12


def test_fp8_per_head_law_matches_reference():
    case = load("fp8_quantise.npz")
    x = tensor(case["x"])
    codes, descale = oracle.quantise_e4m3_per_head(x)
    assert np.array_equal(codes.view(torch.uint8).numpy(), case["codes"])
    assert np.array_equal(descale.numpy(), case["descale"])


def test_fp8_head_rotation_matches_reference():
    """`rotate_bf16` against the reference's `_hadamard` on bf16 (attention_upstream.py:276):
    equal except where the two fp32 sums, added in another order, straddle a bf16 rounding
    tie (at most 1e-4 of the elements, one bf16 step apart)."""
    case = load("fp8_head.npz")
    for name in ("q", "k"):
        got = oracle.rotate_bf16(tensor(case[name])).float()
        want = tensor(case["r" + name]).float()
        off = got != want
        assert off.float().mean().item() <= 1e-4, name
        step = want.abs()[off] * 2.0 ** -7  # one bf16 step (8 significant bits)
        assert ((got - want).abs()[off] <= step + 1e-30).all(), name


def test_fp8_head_quantise_matches_reference():
    """The per-head law on the reference's rotated Q and K and on V: codes and descales equal
    the reference's `quantise_eager` bit for bit (fixture of its FP8 row, `fa4_fp8`)."""
    case = load("fp8_head.npz")
    for name, src in (("q", "rq"), ("k", "rk"), ("v", "v")):
        codes, descale = oracle.quantise_e4m3_per_head(tensor(case[src]))
        assert np.array_equal(codes.view(torch.uint8).numpy(), case[name + "_codes"]), name
        assert np.array_equal(descale.numpy(), case[name + "_descale"]), name


def test_sequence_rows_is_tensor_split():
    for total in (1, 7, 250, 33272, 131071):
        for world in (1, 2, 3, 4, 7, 8):
            want = [t.shape[0] for t in torch.tensor_split(torch.empty(total), world)]
            assert oracle.sequence_rows(total, world) == want


def test_owned_heads_cover_each_head_once():
    for heads in (5, 7, 24, 32, 40):
        for world in (1, 2, 3, 4, 7, 8):
            seen = [h for r in range(world) for h in oracle.owned_heads(heads, world, r)]
            assert seen == list(range(heads))


def test_fp8_block_law_is_per_head_law_at_whole_sequence():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(1, 64, 2, 16, generator=g)
    codes, descale = oracle.quantise_fp8_blocks(x, block=64)
    amax = x.abs().amax(dim=(1, 3))
    assert torch.allclose(descale[:, 0], amax / 448.0)
    back = codes.float() * descale[:, 0][:, None, :, None]
    assert (back - x).abs().max() <= amax.max() / 448.0 * 16


@pytest.mark.parametrize("dim", [64, 128])
def test_turn_law_matches_reference(dim):
    """The int8 wire's law, bit for bit: codes, bf16 scales and the rows back, without and with
    K's turned mean as the shift."""
    case = load(f"turn_d{dim}.npz")
    x, key = tensor(case["x"]), tensor(case["key"])
    codes, scale = oracle.narrow_law(x)
    assert np.array_equal(codes.numpy(), case["codes"])
    assert torch.equal(scale, tensor(case["scale"]))
    assert torch.equal(oracle.narrow_law_back(codes, scale), tensor(case["back"]))
    shift = oracle.turned(key.sum(1, dtype=torch.float32) / key.shape[1])
    assert torch.equal(shift, torch.from_numpy(case["shift"]))
    kcodes, kscale = oracle.narrow_law(key, shift[:, None])
    assert np.array_equal(kcodes.numpy(), case["kcodes"])
    assert torch.equal(kscale, tensor(case["kscale"]))
    assert torch.equal(oracle.narrow_law_back(kcodes, kscale), tensor(case["kback"]))


@pytest.mark.parametrize("name", narrow_cases())
def test_narrow_exchange_matches_reference(name):
    """The whole narrow exchange against the reference's, bit for bit, both running torch SDPA on
    the bf16 operands as the compute (the reference's CPU `sdpa` calls it)."""
    case = load(name)
    q, k, v = (tensor(case[key]) for key in ("q", "k", "v"))
    world, causal = int(case["world"]), bool(case["causal"])
    assert oracle.sequence_rows(q.shape[1], world) == [int(r) for r in case["rows"]]
    parts = [torch.tensor_split(t, world, dim=1) for t in (q, k, v)]

    def sdpa_bf16(a, b, c):  # the reference's compute here: torch SDPA on the bf16 operands
        out = torch.nn.functional.scaled_dot_product_attention(
            a.transpose(1, 2), b.transpose(1, 2), c.transpose(1, 2), is_causal=causal
        )
        return out.transpose(1, 2)

    outs = oracle.exchange_narrow(*parts, sdpa_bf16)
    got = torch.cat(outs, dim=1).float()
    want = tensor(case["out"]).float()
    assert torch.equal(got, want)


def _exchange_group_rank(rank, world, port, outdir, case_name):
    import os

    import torch.distributed as dist

    case = load(case_name)
    causal = bool(case["causal"])
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    parts = [torch.tensor_split(tensor(case[key]), world, dim=1)[rank].contiguous()
             for key in ("q", "k", "v")]
    out = oracle.exchange_group(
        *parts, dist.group.WORLD, lambda a, b, c: oracle.attention_fp32(a, b, c, causal=causal))
    torch.save(out, os.path.join(outdir, f"{rank}.pt"))
    dist.destroy_process_group()


@pytest.mark.parametrize("name", ["ulysses_w2_causal_gqa.npz", "ulysses_w3_padheads.npz",
                                  "ulysses_w4_padheads.npz"])
def test_exchange_over_gloo_matches_reference(name):
    """The oracle's exchange with real crossings (W gloo processes: the reference's own CPU path,
    which the bench's reference arm times) against the reference's outputs."""
    import os
    import socket
    import tempfile

    import torch.multiprocessing as mp

    case = load(name)
    world = int(case["world"])
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_exchange_group_rank, args=(world, port, tmp, name), nprocs=world, join=True)
        got = torch.cat([torch.load(os.path.join(tmp, f"{r}.pt")) for r in range(world)], dim=1)
    want = tensor(case["out"]).float()
    tol = 2e-2 if str(case["dtype"]) == "bfloat16" else 2e-5
    assert (got.float() - want).abs().max() < tol
