"""The oracle pinned against golden vectors from the reference's own code (no GPU)."""

import numpy as np
import pytest
import torch

import oracle
from tests._golden import load, rope_cases, tensor, ulysses_cases


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
