"""Parity of the sm_100a attention kernel (cozy_attention_fwd, through the C ABI) with the oracle.

Tolerance (the path's bf16 bar): max-abs ≤ 2e-2 and mean-abs ≤ 2e-3 against the fp32 oracle on
the same bf16 inputs.
"""

import math

import pytest
import torch

import oracle
from tests._golden import load, tensor, ulysses_cases

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _randn(shape, g, scale=1.0):
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


def _check(got: torch.Tensor, want: torch.Tensor) -> None:
    err = (got.float().cpu() - want.float()).abs()
    assert torch.isfinite(got.float()).all()
    assert err.max().item() <= MAX_ABS, f"max-abs {err.max().item():.3e}"
    assert err.mean().item() <= MEAN_ABS, f"mean-abs {err.mean().item():.3e}"


CASES = [
    # batch, seq_q, seq_k, heads_q, heads_kv, dim, causal, input scale
    (1, 256, 256, 2, 2, 128, False, 1.0),
    (1, 1000, 1000, 2, 2, 128, False, 1.0),
    (2, 77, 77, 3, 3, 128, False, 1.0),
    (1, 700, 700, 4, 1, 128, True, 1.0),
    (1, 513, 513, 2, 2, 64, False, 1.0),
    (1, 1024, 1024, 2, 2, 64, True, 1.0),
    (1, 2048, 2048, 1, 1, 128, True, 1.0),
    (1, 384, 384, 2, 2, 128, False, 4.0),  # large logits: exercises the O rescale
    (1, 257, 300, 2, 2, 128, True, 1.0),  # cross lengths, causal bottom-right
    (1, 1, 130, 1, 1, 128, False, 1.0),  # one query row
]


@pytest.mark.parametrize("batch,sq,sk,hq,hkv,dim,causal,amp", CASES)
def test_attention_matches_oracle(batch, sq, sk, hq, hkv, dim, causal, amp):
    from cozy_runtime_b200 import attention

    g = torch.Generator().manual_seed(20261017 + sq + hq)
    q = _randn((batch, sq, hq, dim), g, amp)
    k = _randn((batch, sk, hkv, dim), g, amp)
    v = _randn((batch, sk, hkv, dim), g)
    got = attention.forward(
        q.cuda(), k.cuda(), v.cuda(), is_causal=causal, enable_gqa=hq != hkv
    )
    torch.cuda.synchronize()
    attention.check_status(got.device)
    want = oracle.attention_fp32(q, k, v, causal=causal)
    _check(got, want)


def test_attention_rows_without_keys_are_zero():
    """Bottom-right causal with more queries than keys: the first Sq - Sk rows see no key. The
    kernel writes zeros there (torch's SDPA gives NaN); every other row matches the oracle."""
    from cozy_runtime_b200 import attention

    g = torch.Generator().manual_seed(3)
    q = _randn((1, 300, 2, 128), g)
    k = _randn((1, 257, 2, 128), g)
    v = _randn((1, 257, 2, 128), g)
    got = attention.forward(q.cuda(), k.cuda(), v.cuda(), is_causal=True).float().cpu()
    assert torch.equal(got[:, :43], torch.zeros_like(got[:, :43]))
    want = oracle.attention_fp32(q, k, v, causal=True)
    _check(got[:, 43:], want[:, 43:])


def test_attention_strided_layouts():
    """[S, B, H, D] storage (the exchange's receive layout) read through strides."""
    from cozy_runtime_b200 import attention

    g = torch.Generator().manual_seed(5)
    base = [_randn((600, 2, 3, 128), g) for _ in range(3)]
    q, k, v = (t.cuda().permute(1, 0, 2, 3) for t in base)  # [B, S, H, D] views
    out = torch.empty(600, 2, 3, 128, dtype=torch.bfloat16, device="cuda").permute(1, 0, 2, 3)
    attention.attention_into(out, q, k, v)
    torch.cuda.synchronize()
    want = oracle.attention_fp32(*(t.permute(1, 0, 2, 3) for t in base))
    _check(out, want)


def test_attention_head_map():
    """A rank's slice of a grouped-query layer: query heads 5..9 of group 4 read K/V heads 1, 2
    held locally as heads 0, 1."""
    from cozy_runtime_b200 import attention

    g = torch.Generator().manual_seed(11)
    q = _randn((1, 200, 5, 128), g)
    k = _randn((1, 200, 2, 128), g)
    v = _randn((1, 200, 2, 128), g)
    out = torch.empty_like(q).cuda()
    attention.attention_into(out, q.cuda(), k.cuda(), v.cuda(), causal=True, head_map=(4, 5, 1))
    torch.cuda.synchronize()
    idx = torch.tensor([(5 + i) // 4 - 1 for i in range(5)])
    want = oracle.attention_fp32(q, k[:, :, idx], v[:, :, idx], causal=True)
    _check(out, want)


def test_attention_refuses_unserved():
    from cozy_runtime_b200 import attention

    q = torch.zeros(1, 8, 1, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        attention.forward(q, q, q, dropout_p=0.1)
    with pytest.raises(ValueError):
        attention.forward(q.float(), q.float(), q.float())
    with pytest.raises(ValueError):
        attention.forward(q, q[:, :, :0], q[:, :, :0])


@pytest.mark.parametrize("name", [n for n in ulysses_cases() if "_w1" in n or n == "ulysses_w1.npz"])
def test_attention_matches_reference_golden_w1(name):
    """Degree 1: the kernel against the reference's own output."""
    from cozy_runtime_b200 import attention

    case = load(name)
    q, k, v = (tensor(case[key]) for key in ("q", "k", "v"))
    got = attention.forward(q.cuda(), k.cuda(), v.cuda(), is_causal=bool(case["causal"]))
    torch.cuda.synchronize()
    _check(got, tensor(case["out"]).float())


def test_attention_large_sequence_property():
    """At a long sequence the output of attention to identical keys is the mean of V."""
    from cozy_runtime_b200 import attention

    s = 33272
    g = torch.Generator().manual_seed(2)
    q = _randn((1, s, 1, 128), g).cuda()
    k = torch.ones(1, s, 1, 128, dtype=torch.bfloat16, device="cuda")
    v = _randn((1, s, 1, 128), g).cuda()
    got = attention.forward(q, k, v)
    want = v.float().mean(dim=1, keepdim=True).expand_as(got)
    err = (got.float() - want).abs()
    assert err.max().item() < 2e-2
    assert math.isfinite(err.mean().item())
