"""The NVLink layer entry (`cozy_ulysses_layer_*`, the default multi-GPU path) with every rank
simulated on one GPU.

W `CozyGroup`s live in this process on one device, connected directly (no IPC): each rank's
first stage writes its own block into its receive buffer and the rest into staging, its side
stream's copy engines move the blocks into the other ranks' receive buffers and set their
arrival flags, its attention waits per source inside the kernel, walks keys from its own rows
on and stores every output row into its owner's landing buffer; then flags and the copy out.
This is the code the multi-GPU runs execute, with peer addresses that happen to be local. The
phases run rank by rank (every rank's begin, then every attend, then every end), so no kernel
ever waits for a kernel launched after it.

Checked against the reference's own exchange outputs (golden vectors) and the CPU oracle at the
path's bf16 bar (max-abs ≤ 2e-2, mean-abs ≤ 2e-3), and at the BASELINE configurations' full
sequence lengths against fp32 attention computed on the GPU for a subset of heads and rows.
"""

import math

import pytest
import torch

import oracle
from tests._golden import load, tensor, ulysses_cases

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def simulate_layer(q, k, v, world, *, causal=False, rope=None, norm=None, rows=None,
                   skip=(), wait_limit_ns=0):
    """Every rank's layer call on this GPU; returns ([B, S, H, D] output, the groups). Ranks in
    `skip` make no call at all (a peer that never comes)."""
    from cozy_runtime_b200 import attention, peer, ulysses

    dev = torch.device("cuda")
    batch, total, heads, dim = q.shape
    rows = rows or ulysses.tensor_split_rows(total, world)
    shape = peer.layer_shape(rows, batch, heads, k.shape[2], dim, causal)
    groups = peer.local_layer_groups(world, dev, shape)
    starts = [sum(rows[:r]) for r in range(world)]
    parts = [[t[:, starts[r]:starts[r] + rows[r]].contiguous().to(dev) for t in (q, k, v)]
             for r in range(world)]
    outs = [torch.zeros(batch, rows[r], heads, dim, dtype=torch.bfloat16, device=dev)
            for r in range(world)]
    status = attention.status_word(dev)
    calls = [ulysses._layer_call(*parts[r], outs[r], rows, causal, None, rope, norm, norm,
                                 status.data_ptr(), wait_limit_ns) for r in range(world)]
    stream = torch.cuda.current_stream(dev).cuda_stream
    for phase in ("begin", "attend", "end"):
        for r in range(world):
            if r not in skip:
                groups[r].run(phase, calls[r][0], stream)
    torch.cuda.synchronize()
    return torch.cat(outs, dim=1), groups


def _close(groups):
    for g in groups:
        g.close()


def _check(got, want):
    err = (got.float().cpu() - want.float().cpu()).abs()
    assert torch.isfinite(got.float()).all()
    assert err.max().item() <= MAX_ABS, f"max-abs {err.max().item():.3e}"
    assert err.mean().item() <= MEAN_ABS, f"mean-abs {err.mean().item():.3e}"


@pytest.mark.parametrize("name", ulysses_cases())
def test_layer_matches_reference_golden(name):
    from cozy_runtime_b200 import attention

    case = load(name)
    world = int(case["world"])
    q, k, v = (tensor(case[key]) for key in ("q", "k", "v"))
    got, groups = simulate_layer(q, k, v, world, causal=bool(case["causal"]))
    attention.check_status(torch.device("cuda"))
    _check(got, tensor(case["out"]).float())
    _close(groups)


@pytest.mark.parametrize(
    "world,batch,seq,hq,hkv,dim,causal",
    [
        (2, 1, 3001, 4, 4, 128, False),
        (3, 2, 1100, 5, 5, 64, False),  # padded heads, batch 2, head dim 64
        (7, 1, 2000, 32, 8, 128, True),  # C5's uneven rows and head groups at degree 7
        (8, 1, 4159 * 2, 24, 24, 128, False),  # C2's layout at degree 8 (shorter sequence)
        (4, 1, 1500, 8, 2, 128, True),  # GQA groups that span ranks
    ],
)
def test_layer_matches_oracle(world, batch, seq, hq, hkv, dim, causal):
    from cozy_runtime_b200 import attention

    g = torch.Generator().manual_seed(seq + world + hq)
    q = torch.randn(batch, seq, hq, dim, generator=g).to(torch.bfloat16)
    k = torch.randn(batch, seq, hkv, dim, generator=g).to(torch.bfloat16)
    v = torch.randn(batch, seq, hkv, dim, generator=g).to(torch.bfloat16)
    got, groups = simulate_layer(q, k, v, world, causal=causal)
    attention.check_status(torch.device("cuda"))
    heads = list(range(0, hq, max(1, hq // 4)))
    group = hq // hkv
    want = oracle.attention_fp32(q[:, :, heads], k[:, :, [h // group for h in heads]],
                                 v[:, :, [h // group for h in heads]], causal=causal)
    _check(got[:, :, heads], want)
    _close(groups)


@pytest.mark.parametrize("world,seq,hq,hkv,causal", [(3, 1100, 5, 5, False),
                                                     (8, 4159 * 2, 24, 24, False),
                                                     (4, 1500, 8, 2, True)])
@pytest.mark.parametrize("cross", ["ce", "sm"])
def test_layer_gate_matches_oracle(monkeypatch, world, seq, hq, hkv, causal, cross):
    """The gated layer (`CozyLayerCall.gate`: a wait kernel holds the attention until every
    source's rows have landed, then it runs with every row resident) against the oracle."""
    from cozy_runtime_b200 import attention

    monkeypatch.setenv("COZY_LAYER_GATE", "1")
    monkeypatch.setenv("COZY_LAYER_CROSS", cross)
    g = torch.Generator().manual_seed(seq + 3 * world)
    q = torch.randn(1, seq, hq, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(1, seq, hkv, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(1, seq, hkv, 128, generator=g).to(torch.bfloat16)
    got, groups = simulate_layer(q, k, v, world, causal=causal)
    attention.check_status(torch.device("cuda"))
    heads = list(range(0, hq, max(1, hq // 4)))
    group = hq // hkv
    want = oracle.attention_fp32(q[:, :, heads], k[:, :, [h // group for h in heads]],
                                 v[:, :, [h // group for h in heads]], causal=causal)
    _check(got[:, :, heads], want)
    _close(groups)


@pytest.mark.parametrize("world,seq,hq,hkv,causal", [(3, 1100, 5, 5, False),
                                                     (8, 4159 * 2, 24, 24, False),
                                                     (7, 2000, 32, 8, True)])
def test_layer_sm_crossing_matches_oracle(monkeypatch, world, seq, hq, hkv, causal):
    """The SM crossing (`CozyLayerCall.cross`: the first stage stores every block straight
    into its owner's receive buffer, one kernel sets the flags) with the attention's in-kernel
    waits, against the oracle."""
    from cozy_runtime_b200 import attention

    monkeypatch.setenv("COZY_LAYER_CROSS", "sm")
    monkeypatch.setenv("COZY_LAYER_GATE", "0")
    g = torch.Generator().manual_seed(seq + 5 * world)
    q = torch.randn(1, seq, hq, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(1, seq, hkv, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(1, seq, hkv, 128, generator=g).to(torch.bfloat16)
    got, groups = simulate_layer(q, k, v, world, causal=causal)
    attention.check_status(torch.device("cuda"))
    heads = list(range(0, hq, max(1, hq // 4)))
    group = hq // hkv
    want = oracle.attention_fp32(q[:, :, heads], k[:, :, [h // group for h in heads]],
                                 v[:, :, [h // group for h in heads]], causal=causal)
    _check(got[:, :, heads], want)
    _close(groups)


def test_layer_twice_uses_both_buffer_sets():
    """Two calls in a row on the same groups (call parity picks the other set of receive and
    landing buffers) give identical outputs."""
    from cozy_runtime_b200 import attention, peer, ulysses

    dev = torch.device("cuda")
    world, batch, seq, heads, dim = 3, 1, 1537, 6, 128
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(batch, seq, heads, dim, generator=g).to(torch.bfloat16)
               for _ in range(3))
    rows = ulysses.tensor_split_rows(seq, world)
    shape = peer.layer_shape(rows, batch, heads, heads, dim, False)
    groups = peer.local_layer_groups(world, dev, shape)
    starts = [sum(rows[:r]) for r in range(world)]
    parts = [[t[:, starts[r]:starts[r] + rows[r]].contiguous().to(dev) for t in (q, k, v)]
             for r in range(world)]
    status = attention.status_word(dev)
    results = []
    for _ in range(3):
        outs = [torch.zeros(batch, rows[r], heads, dim, dtype=torch.bfloat16, device=dev)
                for r in range(world)]
        calls = [ulysses._layer_call(*parts[r], outs[r], rows, False, None, None, None, None,
                                     status.data_ptr()) for r in range(world)]
        stream = torch.cuda.current_stream(dev).cuda_stream
        for phase in ("begin", "attend", "end"):
            for r in range(world):
                groups[r].run(phase, calls[r][0], stream)
        torch.cuda.synchronize()
        results.append(torch.cat(outs, dim=1))
    attention.check_status(dev)
    assert torch.equal(results[0], results[1]) and torch.equal(results[0], results[2])
    assert [groups[0].flag(0, r) for r in range(world)] == [0, 3, 3]  # Q/K/V from the others
    assert [groups[0].flag(1, r) for r in range(world)] == [3, 3, 3]  # output rows from all
    _check(results[0], oracle.attention_fp32(q, k, v))
    _close(groups)


def test_layer_with_rope_and_norm():
    """RMSNorm (unit weight) and 2-D axial RoPE in the first stage, at C3's layout (batch 2,
    image tokens after text) at degree 4, against the oracle's laws."""
    from cozy_runtime_b200 import attention
    from cozy_runtime_b200 import rope as rope_mod
    from cozy_runtime_b200 import ulysses

    grid, text = (1, 12, 12), 32
    spec = rope_mod.axial(grid, (16, 56, 56), before=text)
    seq = 12 * 12 + text
    g = torch.Generator().manual_seed(11)
    q, k, v = (torch.randn(2, seq, 8, 128, generator=g).to(torch.bfloat16) for _ in range(3))
    got, groups = simulate_layer(q, k, v, 4, rope=spec.to(torch.device("cuda")),
                                 norm=ulysses.Norm())
    attention.check_status(torch.device("cuda"))
    rot = [oracle.head_norm_rope(t.float(), spec.cos, spec.sin, rotary=128, interleaved=True,
                                 normalize=True).to(torch.bfloat16) for t in (q, k)]
    _check(got, oracle.attention_fp32(rot[0], rot[1], v))
    _close(groups)


def _exact_rows(q, k, v, head, kv_head, rows, causal):
    """fp32 attention on the GPU for query rows `rows` of one head (scale 1/sqrt(D))."""
    qh = q[0, rows, head].float()
    kh, vh = k[0, :, kv_head].float(), v[0, :, kv_head].float()
    s = (qh @ kh.T) / math.sqrt(qh.shape[-1])
    if causal:
        offset = k.shape[1] - q.shape[1]
        cols = torch.arange(k.shape[1], device=q.device)
        s = s.masked_fill(cols[None, :] > rows[:, None] + offset, float("-inf"))
    return torch.softmax(s, dim=-1) @ vh


def _sample_rows(rows, starts, picks=3):
    """Row indices at the start, middle and end of every rank's block."""
    out = []
    for r, n in enumerate(rows):
        s0 = starts[r]
        out += [s0, s0 + n // 2, s0 + n - 1][:picks]
    return out


@pytest.mark.parametrize("config", ["c2_w8", "c5_w7"])
def test_layer_at_full_baseline_length(config):
    """BASELINE's C2 (S = 33272, 24 heads, degree 8; its 3-head ranks take the split of the last
    wave) and C5 (S = 131071, causal, 32 query over 8 key/value heads, degree 7: rows
    18725/18724, 5 query heads a rank and a 2-head last rank) at full sequence length, with a
    subset of heads on the larger one. Rows at the start, middle and end of every rank's block
    are checked against fp32 attention on the GPU (relative L2 ≤ 1e-2: bf16 output rounding is
    2^-9), and the whole output's rows stay finite."""
    from cozy_runtime_b200 import attention, ulysses

    dev = torch.device("cuda")
    if config == "c2_w8":
        world, seq, hq, hkv, causal, amp = 8, 33272, 24, 24, False, 0.5
    else:
        world, seq, hq, hkv, causal, amp = 7, 131071, 32, 8, True, 1.0
    g = torch.Generator(device=dev).manual_seed(seq)
    q = (torch.randn(1, seq, hq, 128, generator=g, device=dev) * amp).to(torch.bfloat16)
    k = (torch.randn(1, seq, hkv, 128, generator=g, device=dev) * amp).to(torch.bfloat16)
    v = (torch.randn(1, seq, hkv, 128, generator=g, device=dev) * amp).to(torch.bfloat16)
    got, groups = simulate_layer(q, k, v, world, causal=causal)
    attention.check_status(dev)
    rows = ulysses.tensor_split_rows(seq, world)
    starts = [sum(rows[:r]) for r in range(world)]
    pick = torch.tensor(_sample_rows(rows, starts), device=dev)
    group = hq // hkv
    for head in (0, hq // 2 + 1, hq - 1):
        want = _exact_rows(q, k, v, head, head // group, pick, causal)
        have = got[0, pick, head].float()
        rel = ((have - want).norm() / want.norm()).item()
        assert rel <= 1e-2, (head, rel)
    assert torch.isfinite(got.float()).all()
    _close(groups)


def test_layer_peer_timeout_publishes_nothing():
    """A rank whose peer never sends: its attention's wait on that source runs out (a short
    limit), the status word says so (2), it publishes no "rows landed" flag and writes no
    output row into its peer's landing buffer; the device keeps working afterwards."""
    from cozy_runtime_b200 import attention

    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(1, 600, 2, 128, generator=g).to(torch.bfloat16) for _ in range(3))
    status = attention.status_word(dev)
    status.zero_()
    got, groups = simulate_layer(q, k, v, 2, skip=(1,), wait_limit_ns=200_000_000)
    assert int(status.item()) == 2
    assert groups[1].flag(1, 0) == 0  # rank 0 never said its rows landed on rank 1
    assert groups[1].flag(0, 0) == 1  # (its Q/K/V blocks did land: that came before)
    # the attention gave up before its epilogue: no output row went to any owner (rank 0's own
    # landing buffer, copied into its output, still holds the zeros it was formed with)
    assert torch.count_nonzero(got[:, :300]).item() == 0
    status.zero_()
    _close(groups)
    # the context still runs work
    again, groups = simulate_layer(q, k, v, 2)
    attention.check_status(dev)
    _check(again, oracle.attention_fp32(q, k, v))
    _close(groups)
