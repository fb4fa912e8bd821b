"""The golden fixtures discriminate: each test plants one plausible mistake in a copy of an oracle
law (on the CPU) and checks that the reference's own outputs reject it, so a pass of the real
law against them means something."""

import numpy as np
import torch

import oracle
from tests._golden import load, tensor


def test_turn_golden_rejects_an_unrounded_scale():
    """The wire's scale is rounded to bf16 before the codes are formed; dividing by the fp32
    scale instead moves codes."""
    case = load("turn_d128.npz")
    x = tensor(case["x"])
    t = oracle.turned(x)
    scale32 = (t.abs().amax(-1, keepdim=True) * (1.0 / 127)).clamp(min=torch.finfo(x.dtype).tiny)
    q = (t / scale32).clamp(-127, 127)
    wrong = (q.sign() * (q.abs() + 0.5).floor()).to(torch.int8)
    assert not np.array_equal(wrong.numpy(), case["codes"])
    right, _ = oracle.narrow_law(x)
    assert np.array_equal(right.numpy(), case["codes"])


def test_fp8_golden_rejects_the_full_range_target():
    """The reference maps a head's amax onto 440, not e4m3's 448."""
    case = load("fp8_quantise.npz")
    x = tensor(case["x"]).float()
    amax = x.abs().amax(dim=(1, 3), keepdim=True)
    descale = torch.clamp(amax / 448.0, min=1e-12)
    wrong = torch.clamp(x / descale, -448, 448).to(torch.float8_e4m3fn)
    assert not np.array_equal(wrong.view(torch.uint8).numpy(), case["codes"])


def test_rope_golden_rejects_the_other_pairing():
    """Interleaved pairs (2i, 2i+1) and split-half pairs (j, j ± R/2) give different rows."""
    case = load("rope_interleaved_full.npz")
    x = tensor(case["x"]).float()
    cols = int(case["stride_token"])
    cos = torch.from_numpy(case["cos"]).reshape(-1, cols)
    sin = torch.from_numpy(case["sin"]).reshape(-1, cols)
    kwargs = dict(rotary=int(case["rotary"]), weight=None, offset=float(case["offset"]),
                  eps=float(case["eps"]), stride_channel=int(case["stride_channel"]))
    want = torch.from_numpy(case["want"])
    right = oracle.head_norm_rope(x, cos, sin, interleaved=True, **kwargs)
    assert (right - want).abs().max() < 1e-12
    # the same frequencies paired split-half (a split-half table has a column per channel)
    wide = {**kwargs, "stride_channel": 1}
    wrong = oracle.head_norm_rope(x, torch.cat([cos, cos], 1), torch.cat([sin, sin], 1),
                                  interleaved=False, **wide)
    assert (wrong - want).abs().max() > 1e-3


def test_exchange_golden_rejects_top_left_causal():
    """Bottom-right causal alignment is what the reference computes when a rank's queries are a
    suffix of the keys; top-left alignment on the same rows differs."""
    case = load("ulysses_w2_causal_gqa.npz")
    q, k, v = (tensor(case[key]) for key in ("q", "k", "v"))
    want = tensor(case["out"]).float()
    right = oracle.attention_fp32(q, k, v, causal=True)
    assert (right - want).abs().max() < 2e-5
    # queries of the second half only, against every key: top-left would hide later keys
    half = q.shape[1] // 2
    tail = oracle.attention_fp32(q[:, half:], k, v, causal=True)
    assert (tail - want[:, half:]).abs().max() < 2e-5  # bottom-right: the same rows as above
    s_q, s_k = q.shape[1] - half, k.shape[1]
    top_left = torch.ones(s_q, s_k, dtype=torch.bool).tril()
    group = q.shape[2] // k.shape[2]
    kk, vv = k.repeat_interleave(group, dim=2), v.repeat_interleave(group, dim=2)
    scores = torch.einsum("bqhd,bkhd->bhqk", q[:, half:].float(), kk.float()) / q.shape[3] ** 0.5
    scores = scores.masked_fill(~top_left, float("-inf"))
    wrong = torch.einsum("bhqk,bkhd->bqhd", scores.softmax(-1), vv.float())
    assert (wrong - want[:, half:]).abs().max() > 1e-2


def test_fp8_head_golden_rejects_an_unrotated_quantiser():
    """The reference's FP8 row rotates Q and K by the Hadamard before the per-head scale is
    taken: quantising the unrotated keys gives other codes and descales."""
    case = load("fp8_head.npz")
    codes, descale = oracle.quantise_e4m3_per_head(tensor(case["k"]))
    assert not np.array_equal(codes.view(torch.uint8).numpy(), case["k_codes"])
    assert not np.array_equal(descale.numpy(), case["k_descale"])


def test_fp8_head_golden_rejects_an_fp32_rotation():
    """The reference's rotation is a bf16 matrix product (result rounded to bf16): an fp32
    rotation with the exact 1/sqrt(128) moves many of the rotated values off the fixture."""
    case = load("fp8_head.npz")
    x = tensor(case["q"]).float()
    exact = x @ oracle.hadamard_matrix(x.shape[-1])
    want = tensor(case["rq"]).float()
    assert (exact != want).float().mean().item() > 0.5
    assert (oracle.rotate_bf16(tensor(case["q"])).float() != want).float().mean().item() < 1e-4
