"""The int8 wire (`exchange(..., narrow=True)`) on one GPU, through the C ABI.

Kernel law: `cozy_narrow_widen` equals the reference's `turn.law_back` bit for bit (the codes'
turn is exact in fp32); `cozy_narrow_pack` equals `turn.law` except where the fp32 sums of the
turn round differently from the reference's matrix product, which can move a row's scale by one
bf16 step or a code by one (at most 0.5 % of codes, none by more than one, here).

Exchange: W ranks run as W `NarrowStep`s on one GPU, each writing into every rank's receive and
landing blocks at the addresses the NVLink transport would give it; compared with the
reference's own narrow exchange (golden fixtures: it ran torch SDPA in bf16) under the path's bf16
bar (max-abs ≤ 2e-2, mean-abs ≤ 2e-3), and at larger sizes with the oracle's narrow exchange
around fp32 attention.
"""

import numpy as np
import pytest
import torch

import oracle
from tests._golden import load, narrow_cases, tensor

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _pack_one(x: torch.Tensor, shift: torch.Tensor | None):
    """x [B, S, H, D] narrowed into one destination holding every row and head."""
    from cozy_runtime_b200 import narrow

    b, s, h, d = x.shape
    codes = torch.zeros(s * b * h * d, dtype=torch.int8, device="cuda")
    scales = torch.zeros(s * b * h, dtype=torch.bfloat16, device="cuda")
    t = narrow._tensor(x, shift, [(codes.data_ptr(), scales.data_ptr())], [0], [h], [0], [s])
    narrow.pack([t], 1, s, x)
    torch.cuda.synchronize()
    # [S][B][H][D] -> [B, S, H, D]
    return (codes.view(s, b, h, d).permute(1, 0, 2, 3).cpu(),
            scales.view(s, b, h, 1).permute(1, 0, 2, 3).cpu())


@pytest.mark.parametrize("dim", [64, 128])
def test_narrow_pack_and_widen_match_law(dim):
    from cozy_runtime_b200 import narrow

    case = load(f"turn_d{dim}.npz")
    x, key = tensor(case["x"]).cuda(), tensor(case["key"]).cuda()
    for src, shift_want, codes_key, scale_key in (
        (x, None, "codes", "scale"), (key, case["shift"], "kcodes", "kscale"),
    ):
        shift = None
        if shift_want is not None:
            k_sum = torch.zeros(key.shape[0], key.shape[2], dim, device="cuda")
            narrow.key_sum_into(src, k_sum)
            shift = narrow.turned_mean(k_sum, src.shape[1])
            torch.testing.assert_close(shift.cpu(), torch.from_numpy(shift_want), rtol=1e-5,
                                       atol=1e-6)
            shift = torch.from_numpy(shift_want).cuda()  # the law's own shift: codes comparable
        codes, scales = _pack_one(src, shift)
        want_codes = torch.from_numpy(case[codes_key])
        diff = (codes.int() - want_codes.int()).abs()
        assert diff.max().item() <= 1
        assert diff.ne(0).float().mean().item() <= 5e-3
        want_scale = tensor(case[scale_key])
        rel = ((scales.float() - want_scale.float()).abs() / want_scale.float()).max().item()
        assert rel <= 2 ** -7  # one bf16 step at most
    # widen is law_back bit for bit
    for codes_key, scale_key, back_key in (("codes", "scale", "back"), ("kcodes", "kscale", "kback")):
        codes = torch.from_numpy(case[codes_key])  # [B, S, H, D]
        scale = tensor(case[scale_key])  # [B, S, H, 1]
        b, s, h, d = codes.shape
        c = codes.permute(1, 0, 2, 3).contiguous().cuda()  # [S][B][H][D]
        sc = scale.permute(1, 0, 2, 3).contiguous().cuda()
        out = torch.empty(b, s, h, d, dtype=torch.bfloat16, device="cuda")
        narrow.widen([(c.data_ptr(), sc.data_ptr(), 0, s, 0, h)], out)
        torch.cuda.synchronize()
        assert torch.equal(out.cpu(), tensor(case[back_key]))


def simulate_narrow(q, k, v, world, *, causal=False):
    """W ranks' narrow stages on one GPU, the peer transport's addresses; returns the output."""
    from cozy_runtime_b200 import narrow, ulysses

    batch, total, heads, dim = q.shape
    hkv = k.shape[2]
    rows = ulysses.tensor_split_rows(total, world)
    layout = ulysses.plan(rows, heads, hkv)
    dev = torch.device("cuda")
    starts = [layout.start(r) for r in range(world)]
    steps = [
        narrow.NarrowStep(*(t[:, starts[r]: starts[r] + rows[r]].contiguous().to(dev)
                            for t in (q, k, v)), layout, r)
        for r in range(world)
    ]
    k_sum = torch.zeros(batch, hkv, dim, device=dev)
    for st in steps:  # the all-reduce
        narrow.key_sum_into(st.key, k_sum)
    shift = narrow.turned_mean(k_sum, total)
    i8, bf = torch.int8, torch.bfloat16
    recv = [{
        kind: (torch.zeros(total * batch * n * dim, dtype=i8, device=dev),
               torch.zeros(total * batch * n, dtype=bf, device=dev))
        for kind, n in (("q", layout.q_n[p]), ("k", layout.kv_n[p]), ("v", layout.kv_n[p]))
    } for p in range(world)]
    landing = [(torch.zeros(rows[p] * batch * heads * dim, dtype=i8, device=dev),
                torch.zeros(rows[p] * batch * heads, dtype=bf, device=dev)) for p in range(world)]

    def first(p, kind, n, r):
        codes, scales = recv[p][kind]
        return narrow.scale_ptr(codes.data_ptr(), scales.data_ptr(), starts[r] * batch * n * dim, dim)

    for r, st in enumerate(steps):
        st.pack_to(
            shift,
            [first(p, "q", layout.q_n[p], r) for p in range(world)],
            [first(p, "k", layout.kv_n[p], r) for p in range(world)],
            [first(p, "v", layout.kv_n[p], r) for p in range(world)],
        )
    for r, st in enumerate(steps):
        qn, kvn = layout.q_n[r], layout.kv_n[r]
        if not qn:
            continue
        ops = [st.operands(*recv[r][kind], n) for kind, n in (("q", qn), ("k", kvn), ("v", kvn))]
        attended = ulysses._attend_operands(*ops, layout, r, None, causal, None)
        back = []
        for p in range(world):
            at = sum(rows[p] * batch * layout.q_n[u] * dim for u in range(r))
            back.append(narrow.scale_ptr(landing[p][0].data_ptr(), landing[p][1].data_ptr(), at, dim))
        st.return_to(attended, back)
    outs = [st.land(*landing[r]) for r, st in enumerate(steps)]
    torch.cuda.synchronize()
    return torch.cat(outs, dim=1).float().cpu()


def _check(got, want):
    err = (got - want.float()).abs()
    assert torch.isfinite(got).all()
    assert err.max().item() <= MAX_ABS, f"max-abs {err.max().item():.3e}"
    assert err.mean().item() <= MEAN_ABS, f"mean-abs {err.mean().item():.3e}"


@pytest.mark.parametrize("name", narrow_cases())
def test_narrow_exchange_matches_reference_golden(name):
    from cozy_runtime_b200 import attention

    case = load(name)
    q, k, v = (tensor(case[key]) for key in ("q", "k", "v"))
    world, causal = int(case["world"]), bool(case["causal"])
    got = simulate_narrow(q, k, v, world, causal=causal)
    attention.check_status(torch.device("cuda"))
    _check(got, tensor(case["out"]))


@pytest.mark.parametrize(
    "world,batch,seq,hq,hkv,dim,causal",
    [(4, 1, 1000, 8, 8, 128, False), (3, 2, 700, 5, 5, 64, False), (8, 1, 1300, 8, 2, 128, True),
     (7, 1, 900, 7, 7, 128, False)],
)
def test_narrow_exchange_matches_oracle(world, batch, seq, hq, hkv, dim, causal):
    from cozy_runtime_b200 import attention

    g = torch.Generator().manual_seed(seq + world)
    q = torch.randn(batch, seq, hq, dim, generator=g).to(torch.bfloat16)
    k = torch.randn(batch, seq, hkv, dim, generator=g).to(torch.bfloat16)
    v = torch.randn(batch, seq, hkv, dim, generator=g).to(torch.bfloat16)
    got = simulate_narrow(q, k, v, world, causal=causal)
    attention.check_status(torch.device("cuda"))
    parts = [torch.tensor_split(t, world, dim=1) for t in (q, k, v)]
    want = torch.cat(oracle.exchange_narrow(
        *parts, lambda a, b, c: oracle.attention_fp32(a, b, c, causal=causal)), dim=1)
    _check(got, want)
    # and the wire's loss stays small against exact attention
    exact = oracle.attention_fp32(q, k, v, causal=causal)
    cos = torch.nn.functional.cosine_similarity(got.flatten(), exact.flatten(), dim=0).item()
    assert cos >= 0.999, cos


def test_narrow_public_call_degree1():
    """`ulysses.exchange(..., narrow=True)` at degree 1 (the reference narrows there too),
    with a callable `narrow` deciding on the total."""
    from cozy_runtime_b200 import attention, ulysses

    case = load("narrow_w1.npz")
    q, k, v = (tensor(case[key]).cuda() for key in ("q", "k", "v"))
    seen = []

    def decide(total):
        seen.append(total)
        return True

    got = ulysses.exchange(q, k, v, None, None, narrow=decide)
    torch.cuda.synchronize()
    attention.check_status(got.device)
    assert seen == [q.shape[1]]
    _check(got.float().cpu(), tensor(case["out"]))
    wide = ulysses.exchange(q, k, v, None, None, narrow=False)
    assert not torch.equal(wide, got)  # the wire's law was applied


def test_narrow_with_rope_and_compute():
    """RoPE/RMSNorm before the wire, and a callable `compute` on the widened operands."""
    from cozy_runtime_b200 import rope, ulysses

    g = torch.Generator().manual_seed(5)
    s, h, d = 600, 4, 128
    q, k, v = (torch.randn(1, s, h, d, generator=g).to(torch.bfloat16) for _ in range(3))
    tables = rope.llama(s, d)
    norm = ulysses.Norm()
    got = ulysses.exchange(q.cuda(), k.cuda(), v.cuda(), None, None, narrow=True,
                           rope=tables.to(torch.device("cuda")), norm_q=norm, norm_k=norm)

    def sdpa(a, b, c):
        return torch.nn.functional.scaled_dot_product_attention(
            a.transpose(1, 2), b.transpose(1, 2), c.transpose(1, 2)).transpose(1, 2)

    via_compute = ulysses.exchange(q.cuda(), k.cuda(), v.cuda(), None, sdpa, narrow=True,
                                   rope=tables.to(torch.device("cuda")), norm_q=norm, norm_k=norm)
    torch.cuda.synchronize()
    rq = oracle.head_norm_rope(q.float(), tables.cos, tables.sin, rotary=d, interleaved=False,
                               weight=None, offset=0.0, eps=1e-6).to(torch.bfloat16)
    rk = oracle.head_norm_rope(k.float(), tables.cos, tables.sin, rotary=d, interleaved=False,
                               weight=None, offset=0.0, eps=1e-6).to(torch.bfloat16)
    want = oracle.exchange_narrow([rq], [rk], [v], oracle.attention_fp32)[0]
    _check(got.float().cpu(), want)
    _check(via_compute.float().cpu(), want)
    assert np.isfinite(got.float().cpu().numpy()).all()
