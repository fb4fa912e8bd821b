"""The stages on their own: the standalone RMSNorm + RoPE entry point against the reference's
law (golden vectors of the reference's own checker), and the bounded peer wait running out."""

import pytest
import torch

from tests._golden import load, rope_cases, tensor

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", rope_cases())
def test_head_norm_rope_matches_reference_law(name):
    """`cozy_head_norm_rope` (drop-in for the reference's `head_norm_rope`) against the law
    recorded from the reference's checker `internal/bench/kernels.py:819`."""
    from cozy_runtime_b200 import rope

    case = load(name)
    x = tensor(case["x"]).cuda()
    spec = rope.RopeSpec(
        torch.from_numpy(case["cos"]).reshape(-1).cuda(),
        torch.from_numpy(case["sin"]).reshape(-1).cuda(),
        int(case["stride_token"]), int(case["stride_channel"]), int(case["rotary"]),
        bool(case["interleaved"]),
    )
    weight = torch.from_numpy(case["weight"]).cuda() if int(case["has_weight"]) else None
    got = rope.head_norm_rope(x, spec, weight=weight, offset=float(case["offset"]),
                              eps=float(case["eps"]))
    torch.cuda.synchronize()
    want = torch.from_numpy(case["want"]).float()
    err = (got.float().cpu() - want).abs()
    assert (err <= 1e-2 + 8e-3 * want.abs()).all(), f"max err {err.max().item():.3e}"


def test_head_norm_rope_strided_batch2():
    """Batch 2, a strided [S, B, H, D] input view, 3-D axial tables, against the oracle law."""
    import oracle
    from cozy_runtime_b200 import rope

    spec = rope.axial((2, 3, 5), (44, 42, 42), after=4)
    seq = 2 * 3 * 5 + 4
    g = torch.Generator().manual_seed(4)
    base = torch.randn(seq, 2, 3, 128, generator=g).to(torch.bfloat16)
    x = base.cuda().permute(1, 0, 2, 3)
    got = rope.head_norm_rope(x, spec.to(torch.device("cuda")), normalize=True)
    want = oracle.head_norm_rope(base.permute(1, 0, 2, 3).float(), spec.cos, spec.sin,
                                 rotary=128, interleaved=True, normalize=True)
    err = (got.float().cpu() - want.float()).abs()
    assert (err <= 1e-2 + 8e-3 * want.abs().float()).all()


def test_peer_wait_times_out_into_status():
    """A flag no peer ever sets: the bounded wait gives up after its limit, reports status 2
    (a peer timeout) and the context stays usable. No GPU fault is involved."""
    from cozy_runtime_b200 import _lib, attention

    lib = _lib.load()
    device = torch.device("cuda", 0)
    flags = torch.zeros(4, dtype=torch.int64, device=device)
    status = attention.status_word(device)
    status.zero_()
    code = lib.cozy_peer_wait(flags.data_ptr(), 4, 1, 200_000_000, status.data_ptr(),
                              torch.cuda.current_stream().cuda_stream)
    assert code == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 2
    with pytest.raises(RuntimeError, match="peer"):
        attention.check_status(device)
    # the context still runs work, and a wait on flags already set returns at once
    flags.fill_(5)
    code = lib.cozy_peer_wait(flags.data_ptr(), 4, 5, 200_000_000, status.data_ptr(),
                              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert code == 0 and int(status.item()) == 0
    assert torch.ones(3, device=device).sum().item() == 3.0


def test_exchange_raises_after_a_timeout():
    """A wait that ran out (a flag nothing sets, 0.2 s) leaves status 2; the exchange sees it
    without synchronizing (the status word is copied to the host behind each call) and the
    call after the one that copied it raises, once; later calls work."""
    from cozy_runtime_b200 import _lib, attention, ulysses

    lib = _lib.load()
    device = torch.device("cuda", 0)
    g = torch.Generator(device=device).manual_seed(2)
    q, k, v = (torch.randn(1, 300, 2, 128, generator=g, device=device).to(torch.bfloat16)
               for _ in range(3))
    status = attention.status_word(device)
    status.zero_()
    ulysses.exchange(q, k, v, None)  # a watch exists
    torch.cuda.synchronize()
    flags = torch.zeros(1, dtype=torch.int64, device=device)
    assert lib.cozy_peer_wait(flags.data_ptr(), 1, 1, 200_000_000, status.data_ptr(),
                              torch.cuda.current_stream().cuda_stream) == 0
    ulysses.exchange(q, k, v, None)  # queued behind the timed-out wait: copies status 2
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="peer"):
        ulysses.exchange(q, k, v, None)
    out = ulysses.exchange(q, k, v, None)
    torch.cuda.synchronize()
    assert int(status.item()) == 0 and torch.isfinite(out.float()).all()
