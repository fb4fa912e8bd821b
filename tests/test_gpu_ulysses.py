"""The Ulysses exchange's kernels (pack, attention on receive buffers, land) on one GPU.

W ranks run as W `RankStep`s in one process; the crossings between them are device copies of
exactly the blocks NCCL's all-to-all moves (the same split sizes and offsets `exchange` hands it).
The assembled output is compared with the reference's own exchange output (golden vectors from
`tests/golden/make_golden.py`) at the path's bf16 tolerance: max-abs ≤ 2e-2, mean-abs ≤ 2e-3.
"""

import numpy as np
import pytest
import torch

import oracle
from tests._golden import load, rope_cases, tensor, ulysses_cases

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _offsets(sizes):
    return np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(int).tolist()


def simulate(q, k, v, world, *, causal=False, rope=None, norm_q=None, norm_k=None, rows=None):
    """Every rank's exchange on this GPU; returns the concatenated [B, S, H, D] output."""
    from cozy_runtime_b200 import ulysses

    total = q.shape[1]
    rows = rows or ulysses.tensor_split_rows(total, world)
    layout = ulysses.plan(rows, q.shape[2], k.shape[2])
    starts = _offsets(rows)
    steps = []
    for r in range(world):
        part = [t[:, starts[r] : starts[r] + rows[r]].contiguous().cuda() for t in (q, k, v)]
        steps.append(
            ulysses.RankStep(*part, layout, r, rope=rope, norm_q=norm_q, norm_k=norm_k)
        )
    for st in steps:
        st.pack()
    recvs = [st.receive_buffers() if world > 1 else (st.q_send, st.k_send, st.v_send) for st in steps]
    if world > 1:
        for idx, (send_name, out_name, in_name) in enumerate(
            [("q_send", "q_sizes", "q_in"), ("k_send", "kv_sizes", "kv_in"), ("v_send", "kv_sizes", "kv_in")]
        ):
            for d in range(world):
                for s in range(world):
                    out_sizes = getattr(steps[s], out_name)
                    in_sizes = getattr(steps[d], in_name)
                    n = out_sizes[d]
                    assert n == in_sizes[s]
                    src = getattr(steps[s], send_name)[_offsets(out_sizes)[d] :][:n]
                    recvs[d][idx][_offsets(in_sizes)[s] :][:n].copy_(src)
    o_sends = [st.attend(*recvs[r], None, causal, None) for r, st in enumerate(steps)]
    outs = []
    for d, st in enumerate(steps):
        if world == 1:
            returned = o_sends[0]
        else:
            returned = torch.empty(sum(st.back_sizes), dtype=q.dtype, device="cuda")
            for s in range(world):
                n = st.back_sizes[s]
                assert n == steps[s].back_in[d]
                src = o_sends[s][_offsets(steps[s].back_in)[d] :][:n]
                returned[_offsets(st.back_sizes)[s] :][:n].copy_(src)
        outs.append(st.land(returned))
    torch.cuda.synchronize()
    return torch.cat(outs, dim=1)


def _check(got, want):
    err = (got.float().cpu() - want.float()).abs()
    assert err.max().item() <= MAX_ABS, f"max-abs {err.max().item():.3e}"
    assert err.mean().item() <= MEAN_ABS, f"mean-abs {err.mean().item():.3e}"


@pytest.mark.parametrize("name", ulysses_cases())
def test_exchange_matches_reference_golden(name):
    case = load(name)
    q, k, v = (tensor(case[key]) for key in ("q", "k", "v"))
    got = simulate(q, k, v, int(case["world"]), causal=bool(case["causal"]))
    _check(got, tensor(case["out"]).float())


@pytest.mark.parametrize(
    "world,batch,seq,hq,hkv,dim,causal",
    [
        (8, 1, 4159 * 8, 24, 24, 128, False),  # C2 layout at degree 8 (shorter sequence below)
        (7, 1, 2000, 32, 8, 128, True),  # C5's uneven split and head groups at degree 7
        (4, 2, 1152, 24, 24, 128, False),  # C3 batch 2
        (3, 1, 1001, 5, 5, 64, False),
    ],
)
def test_exchange_matches_oracle(world, batch, seq, hq, hkv, dim, causal):
    if seq > 20000:
        seq = 4159 * 2  # keep the CPU oracle to seconds; the layout is the same
    g = torch.Generator().manual_seed(seq + world)
    q = torch.randn(batch, seq, hq, dim, generator=g).to(torch.bfloat16)
    k = torch.randn(batch, seq, hkv, dim, generator=g).to(torch.bfloat16)
    v = torch.randn(batch, seq, hkv, dim, generator=g).to(torch.bfloat16)
    got = simulate(q, k, v, world, causal=causal)
    heads = list(range(0, hq, max(1, hq // 4)))  # the oracle on a subset of heads
    groups = hq // hkv
    kv_heads = [h // groups for h in heads]
    want = oracle.attention_fp32(q[:, :, heads], k[:, :, kv_heads], v[:, :, kv_heads], causal=causal)
    _check(got[:, :, heads], want)


@pytest.mark.parametrize("name", rope_cases())
def test_pack_rope_matches_reference_law(name):
    """Stage 1 alone (degree 1): per-head RMSNorm + RoPE against the reference's own checker law
    (`internal/bench/kernels.py:819` `_fused_rope`, recorded in the golden vectors)."""
    from cozy_runtime_b200 import ulysses
    from cozy_runtime_b200.rope import RopeSpec

    case = load(name)
    x = tensor(case["x"])  # [1, seq, heads, dim] bf16
    batch, seq, heads, dim = x.shape
    cols = int(case["stride_token"])
    rope = RopeSpec(
        torch.from_numpy(case["cos"]).reshape(-1).cuda(),
        torch.from_numpy(case["sin"]).reshape(-1).cuda(),
        cols, int(case["stride_channel"]), int(case["rotary"]), bool(case["interleaved"]),
    )
    weight = torch.from_numpy(case["weight"]).float().cuda() if int(case["has_weight"]) else None
    norm = ulysses.Norm(weight, float(case["offset"]), float(case["eps"]))
    layout = ulysses.plan([seq], heads, heads)
    xd = x.cuda()
    step = ulysses.RankStep(xd, xd, xd, layout, 0, rope=rope, norm_q=norm, norm_k=norm)
    step.pack()
    torch.cuda.synchronize()
    got = step.q_send.view(seq, batch, heads, dim).permute(1, 0, 2, 3).float().cpu()
    want = torch.from_numpy(case["want"]).float()
    err = (got - want).abs()
    assert (err <= 1e-2 + 8e-3 * want.abs()).all(), f"max err {err.max().item():.3e}"
    # V is packed untouched
    v_got = step.v_send.view(seq, batch, heads, dim).permute(1, 0, 2, 3).cpu()
    assert torch.equal(v_got, x)


def test_exchange_with_rope_matches_oracle():
    """Stage 1 with 3-D axial RoPE at degree 4, end to end against the oracle law + attention."""
    from cozy_runtime_b200 import rope as rope_mod

    grid, text = (3, 5, 8), 16
    spec = rope_mod.axial(grid, (44, 42, 42), after=text)
    seq = 3 * 5 * 8 + text
    g = torch.Generator().manual_seed(9)
    q, k, v = (torch.randn(1, seq, 4, 128, generator=g).to(torch.bfloat16) for _ in range(3))
    got = simulate(q, k, v, 4, rope=spec.to(torch.device("cuda")))
    qr = oracle.head_norm_rope(q.float(), spec.cos, spec.sin, rotary=128, interleaved=True,
                               normalize=False).to(torch.bfloat16)
    kr = oracle.head_norm_rope(k.float(), spec.cos, spec.sin, rotary=128, interleaved=True,
                               normalize=False).to(torch.bfloat16)
    want = oracle.attention_fp32(qr, kr, v)
    _check(got, want)
