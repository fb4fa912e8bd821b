"""The split of the last wave: tiles past the last whole wave of one CTA per SM run as several
CTAs over shares of the keys, and the last one to finish merges their rows.

Checked against the fp32 oracle at sizes it finishes in seconds (the path's bf16 bar: max-abs
≤ 2e-2, mean-abs ≤ 2e-3), and at the full C2 degree-8 shape (3 heads × 33272 tokens, whose 390
tiles fill 2.64 waves of 148 SMs) against an fp32 torch reference on the GPU for rows of split
and of whole tiles, plus split against unsplit (COZY_ATTENTION_SPLIT=0) output: relative L2
≤ 1e-2 (bf16 rounding of the output is 2^-9 relative).
"""

import os

import pytest
import torch

import oracle
from tests.test_gpu_attention import _check, _randn

pytestmark = pytest.mark.gpu


def _unsplit(fn):
    old = os.environ.get("COZY_ATTENTION_SPLIT")
    os.environ["COZY_ATTENTION_SPLIT"] = "0"
    try:
        return fn()
    finally:
        if old is None:
            del os.environ["COZY_ATTENTION_SPLIT"]
        else:
            os.environ["COZY_ATTENTION_SPLIT"] = old


def _sms() -> int:
    return torch.cuda.get_device_properties(0).multi_processor_count


def test_split_plan():
    from cozy_runtime_b200 import attention

    sms = _sms()
    whole, parts = attention.split_plan(1, 33272, 33272, 3, 128, False)  # C2 at degree 8
    tiles = 3 * 130
    assert parts > 1 and whole % sms == 0 and whole < tiles
    # causal calls are never split; a whole number of waves needs no split
    assert attention.split_plan(1, 33272, 33272, 3, 128, True) == (tiles, 1)
    assert attention.split_plan(1, 256 * sms, 256 * sms, 1, 128, False)[1] == 1
    os.environ["COZY_ATTENTION_SPLIT"] = "0"
    try:
        assert attention.split_plan(1, 33272, 33272, 3, 128, False) == (tiles, 1)
    finally:
        del os.environ["COZY_ATTENTION_SPLIT"]


SPLIT_CASES = [
    # batch, seq_q, seq_k, heads_q, heads_kv, dim, input scale
    (1, 4000, 4000, 2, 2, 128, 1.0),  # ragged last key block inside the last part
    (2, 3000, 3000, 3, 3, 64, 1.0),
    (1, 2000, 2000, 4, 1, 128, 1.0),  # grouped-query heads
    (1, 1500, 2900, 2, 2, 128, 4.0),  # cross lengths; large logits (rescale inside parts)
]


@pytest.mark.parametrize("batch,sq,sk,hq,hkv,dim,amp", SPLIT_CASES)
def test_split_matches_oracle(batch, sq, sk, hq, hkv, dim, amp):
    from cozy_runtime_b200 import attention

    assert attention.split_plan(batch, sq, sk, hq, dim, False)[1] > 1
    g = torch.Generator().manual_seed(7 + sq + hq)
    q = _randn((batch, sq, hq, dim), g, amp)
    k = _randn((batch, sk, hkv, dim), g, amp)
    v = _randn((batch, sk, hkv, dim), g)
    got = attention.forward(q.cuda(), k.cuda(), v.cuda(), enable_gqa=hq != hkv)
    torch.cuda.synchronize()
    attention.check_status(got.device)
    _check(got, oracle.attention_fp32(q, k, v))
    # twice in a row on the same stream: the counters start from zero every launch
    again = attention.forward(q.cuda(), k.cuda(), v.cuda(), enable_gqa=hq != hkv)
    torch.cuda.synchronize()
    assert torch.equal(got, again)


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm()).item()


def _exact_rows(q, k, v, head, rows):
    """fp32 attention on the GPU for query rows `rows` of `head` (non-causal, scale 1/√D)."""
    qh = q[0, rows, head].float()
    kh, vh = k[0, :, head].float(), v[0, :, head].float()
    s = (qh @ kh.T) / qh.shape[-1] ** 0.5
    return torch.softmax(s, dim=-1) @ vh


def test_split_at_c2_degree8_shape():
    from cozy_runtime_b200 import attention

    s, h, d = 33272, 3, 128
    whole, parts = attention.split_plan(1, s, s, h, d, False)
    assert parts > 1
    g = torch.Generator(device="cuda").manual_seed(8)
    q, k, v = (
        (torch.randn(1, s, h, d, generator=g, device="cuda") * 0.5).to(torch.bfloat16)
        for _ in range(3)
    )
    got = attention.forward(q, k, v)
    plain = _unsplit(lambda: attention.forward(q, k, v))
    torch.cuda.synchronize()
    attention.check_status(got.device)
    # tile t: query block (q_blocks - 1 - t % q_blocks) of head t // q_blocks
    q_blocks = (s + 255) // 256
    first_split = whole
    split_head = first_split // q_blocks
    split_block = q_blocks - 1 - first_split % q_blocks  # highest split query block of that head
    rows = torch.arange(0, min(2048, (split_block + 1) * 256), device="cuda")
    want = _exact_rows(q, k, v, split_head, rows)
    assert _rel(got[0, rows, split_head], want) <= 1e-2
    whole_rows = torch.arange(s - 2048, s, device="cuda")  # head 0's last block: a whole tile
    assert _rel(got[0, whole_rows, 0], _exact_rows(q, k, v, 0, whole_rows)) <= 1e-2
    assert _rel(got, plain) <= 1e-2
    assert torch.isfinite(got.float()).all()


def test_split_fp8():
    """The FP8 kernel takes the same split. Split and unsplit outputs are both e4m3 roundings
    of P, each part's against its own running max, so they are compared with the oracle's FP8
    law (cosine ≥ 0.999, mean-abs ≤ 2.5e-3) and exact attention (cosine ≥ 0.995), the FP8
    path's own bars, rather than with each other."""
    from cozy_runtime_b200 import attention
    from tests.test_gpu_fp8 import _cosine_per_head, _inputs, simulate_fp8

    batch, seq, heads, world = 1, 3000, 4, 2
    # each simulated rank attends its 2 heads over the whole sequence
    assert attention.split_plan(batch, seq, seq, heads // world, 128, False)[1] > 1
    q, k, v = _inputs(batch, seq, heads, heads, 12)
    got = simulate_fp8(q, k, v, world)
    attention.check_status(torch.device("cuda"))
    rows = [t.shape[0] for t in torch.tensor_split(torch.empty(seq), world)]
    law = oracle.fp8_attention_law(*(torch.split(t, rows, dim=1) for t in (q, k, v)))
    assert (got - law).abs().mean().item() <= 2.5e-3
    assert _cosine_per_head(got, law).min().item() >= 0.999
    assert _cosine_per_head(got, oracle.attention_fp32(q, k, v)).min().item() >= 0.995


def test_captured_launch_never_uses_the_split_workspace():
    """A launch captured into a CUDA graph runs unsplit, so the graph holds no workspace
    address: growing (freeing and reallocating) the stream's workspace with a larger eager call
    after the capture, then replaying the graph, still gives the unsplit result bit for bit."""
    from cozy_runtime_b200 import attention

    batch, sq, hq, dim = 1, 4000, 2, 128
    assert attention.split_plan(batch, sq, sq, hq, dim, False)[1] > 1
    g = torch.Generator().manual_seed(31)
    q, k, v = (_randn((batch, sq, hq, dim), g).cuda() for _ in range(3))
    attention.status_word(q.device)
    want = _unsplit(lambda: attention.forward(q, k, v))
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        attention.forward(q, k, v)  # eager on this stream: its workspace exists before capture
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            captured = attention.forward(q, k, v)
        # a larger split call on the capture stream grows its workspace
        big = 3 * 130 * 256
        g2 = torch.Generator(device="cuda").manual_seed(5)
        qb, kb, vb = (torch.randn(1, big // 3, 3, dim, generator=g2, device="cuda")
                      .to(torch.bfloat16) for _ in range(3))
        assert attention.split_plan(1, big // 3, big // 3, 3, dim, False)[1] > 1
        attention.forward(qb, kb, vb)
        captured.zero_()
        graph.replay()
    torch.cuda.synchronize()
    attention.check_status(q.device)
    assert torch.equal(captured, want)
    _check(captured, oracle.attention_fp32(q.cpu(), k.cpu(), v.cpu()))
