"""Every BASELINE configuration at its full size, through the public exchange.

C1 (fp32, D = 64, S = 1024) is served by casting to bf16 (the kernels compute in bf16 with fp32
softmax and accumulation) and back: checked against fp32 attention with the path's bf16 bar.
C2 (video DiT, S = 33272, 3-D RoPE), C3 (Flux, B = 2, S = 4608, RMSNorm + 2-D RoPE) and C5
(causal GQA prefill, S = 131071, 1-D RoPE) run at degree 1 on one GPU, C3 also at degree 4
simulated through the NVLink layer (the degree-8 C2 and degree-7 C5 layouts are in
test_gpu_layer.py, C4's FP8 degree 8 in test_gpu_fp8.py). The reference is fp32 attention on
the GPU over the RoPE/RMSNorm law of the CPU oracle (the reference's own checker law, pinned to
its fixtures), for three heads and rows at the start, middle and end of the sequence; bar:
relative L2 ≤ 1e-2 per head (bf16 output rounding is 2^-9) and max-abs ≤ 2e-2.
"""

import math

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _rows(seq: int) -> torch.Tensor:
    picks = list(range(0, 256)) + list(range(seq // 2 - 128, seq // 2 + 128)) + list(
        range(seq - 256, seq))
    return torch.tensor(sorted(set(picks)))


def _rotate(x: torch.Tensor, spec, norm: bool) -> torch.Tensor:
    """The first stage's law (oracle, fp64 on the CPU) on [B, S, H, D] bf16, back in bf16."""
    cos = spec.cos.cpu().reshape(-1, spec.stride_token) if spec is not None else None
    if spec is None:
        y = x.double()
        if norm:
            y = y * torch.rsqrt(y.pow(2).mean(-1, keepdim=True) + 1e-6)
        return y.to(torch.bfloat16)
    sin = spec.sin.cpu().reshape(-1, spec.stride_token)
    return oracle.head_norm_rope(x.cpu(), cos, sin, rotary=spec.rotary,
                                 interleaved=spec.interleaved, normalize=norm,
                                 stride_channel=spec.stride_channel).to(torch.bfloat16)


def _check_heads(got, q, k, v, heads, causal, rows):
    """fp32 attention on the GPU for `rows` of each head in `heads` against `got`."""
    dev = got.device
    group = q.shape[2] // k.shape[2]
    sel = rows.to(dev)
    for b in range(q.shape[0]):
        for h in heads:
            qh = q[b, rows.to(q.device), h].to(dev).float()
            kh = k[b, :, h // group].to(dev).float()
            vh = v[b, :, h // group].to(dev).float()
            s = (qh @ kh.T) / math.sqrt(q.shape[3])
            if causal:
                cols = torch.arange(k.shape[1], device=dev)
                s = s.masked_fill(cols[None, :] > sel[:, None] + (k.shape[1] - q.shape[1]),
                                  float("-inf"))
            want = torch.softmax(s, dim=-1) @ vh
            have = got[b, sel, h].float()
            rel = ((have - want).norm() / want.norm()).item()
            assert rel <= 1e-2, (b, h, rel)
            assert (have - want).abs().max().item() <= 2e-2, (b, h)


def test_c1_fp32_degree1():
    """C1: B=1, H=12, S=1024, D=64, fp32 N(0,1), no mask, degree 1 (the reference's CPU case)."""
    from cozy_runtime_b200 import attention, ulysses

    g = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn(1, 1024, 12, 64, generator=g) for _ in range(3))
    got = ulysses.exchange(*(t.cuda() for t in (q, k, v)), None)
    torch.cuda.synchronize()
    attention.check_status(got.device)
    assert got.dtype == torch.float32 and got.shape == q.shape
    want = oracle.attention_fp32(q, k, v)
    err = (got.cpu() - want).abs()
    assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3


@pytest.mark.parametrize("config", ["c2", "c5"])
def test_full_length_degree1(config):
    from cozy_runtime_b200 import attention, ulysses
    from cozy_runtime_b200 import rope as rope_mod

    dev = torch.device("cuda")
    if config == "c2":
        seq, hq, hkv, causal, amp = 33272, 24, 24, False, 0.5
        spec = rope_mod.axial((21, 30, 52), (44, 42, 42), after=512)
    else:
        seq, hq, hkv, causal, amp = 131071, 32, 8, True, 1.0
        spec = rope_mod.llama(seq, 128, 500000.0)
    g = torch.Generator(device=dev).manual_seed(seq)
    q = (torch.randn(1, seq, hq, 128, generator=g, device=dev) * amp).to(torch.bfloat16)
    k = (torch.randn(1, seq, hkv, 128, generator=g, device=dev) * amp).to(torch.bfloat16)
    v = (torch.randn(1, seq, hkv, 128, generator=g, device=dev) * amp).to(torch.bfloat16)
    got = ulysses.exchange(q, k, v, None, None, causal=causal, rope=spec.to(dev))
    torch.cuda.synchronize()
    attention.check_status(dev)
    heads = [0, hq // 2 + 1, hq - 1]
    group = hq // hkv
    qr = _rotate(q[:, :, heads].cpu(), spec, False)
    kr = _rotate(k[:, :, sorted({h // group for h in heads})].cpu(), spec, False)
    kv_index = {kh: i for i, kh in enumerate(sorted({h // group for h in heads}))}
    for i, h in enumerate(heads):
        sub_v = v[:, :, [h // group]]
        _check_heads(got[:, :, [h]], qr[:, :, [i]], kr[:, :, [kv_index[h // group]]], sub_v,
                     [0], causal, _rows(seq))


def test_c3_full_degree1_and_degree4():
    """C3: B=2, H=24, S=512 text + 64x64 image = 4608, per-head RMSNorm (unit weight) on Q and K
    then 2-D axial RoPE (16/56/56, theta 10000) on the image tokens; degree 1 through the public
    call and degree 4 simulated through the NVLink layer."""
    from cozy_runtime_b200 import attention, ulysses
    from cozy_runtime_b200 import rope as rope_mod
    from tests.test_gpu_layer import simulate_layer

    dev = torch.device("cuda")
    spec = rope_mod.axial((1, 64, 64), (16, 56, 56), 10000.0, before=512)
    g = torch.Generator(device=dev).manual_seed(3)
    q, k, v = (torch.randn(2, 4608, 24, 128, generator=g, device=dev).to(torch.bfloat16)
               for _ in range(3))
    norm = ulysses.Norm()
    one = ulysses.exchange(q, k, v, None, None, rope=spec.to(dev), norm_q=norm, norm_k=norm)
    four, groups = simulate_layer(q, k, v, 4, rope=spec.to(dev), norm=norm)
    torch.cuda.synchronize()
    attention.check_status(dev)
    for g_ in groups:
        g_.close()
    qr, kr = _rotate(q.cpu(), spec, True), _rotate(k.cpu(), spec, True)
    for got in (one, four):
        _check_heads(got, qr, kr, v, [0, 13, 23], False, _rows(4608))
