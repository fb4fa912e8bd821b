"""Rotary tables for the fused first stage, in the layout the reference's kernels read.

A table is `(cos, sin, stride_token, stride_channel)` fp32, as
`src/cozy_runtime/accel/fusion/_kernels.py:497-517` (`rope_tables`) returns it: channel pair /
column `col` of token `t` is read at `t * stride_token + col * stride_channel`. The builders
below make the tables the benchmark configurations name (1-D RoPE for an LLM, 2-D and 3-D axial
RoPE for image and video DiTs); a model that brings its own tables passes them through
`rope_tables`-style tuples unchanged.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor


@dataclass(frozen=True)
class RopeSpec:
    """A rotary operand for `ulysses.exchange`: tables over the WHOLE sequence (row = global
    token position), the rotated channel count and the pairing convention."""

    cos: Tensor
    sin: Tensor
    stride_token: int
    stride_channel: int
    rotary: int
    interleaved: bool

    def to(self, device: torch.device) -> RopeSpec:
        return RopeSpec(
            self.cos.to(device), self.sin.to(device), self.stride_token, self.stride_channel,
            self.rotary, self.interleaved,
        )

    def struct(self, token0: int):
        """The `CozyRope` a first stage reads: table row `token0` is its first row's."""
        from cozy_runtime_b200 import _lib

        r = _lib.Rope()
        r.cos, r.sin = self.cos.data_ptr(), self.sin.data_ptr()
        r.stride_token, r.stride_channel = self.stride_token, self.stride_channel
        r.token0, r.rotary, r.interleaved = token0, self.rotary, int(self.interleaved)
        return r


def _freqs(dim: int, theta: float) -> Tensor:
    return 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))


def axial(
    grid: tuple[int, ...],
    dims: tuple[int, ...],
    theta: float = 10000.0,
    *,
    before: int = 0,
    after: int = 0,
) -> RopeSpec:
    """Interleaved axial RoPE over a token grid (video t×h×w, image h×w): each axis a rotates
    `dims[a]` channels (dims[a]/2 pairs) by position × theta^(-2i/dims[a]); the axes' pairs are
    concatenated in order, the grid flattened row-major. `before`/`after` unrotated tokens
    (text) sit before/after the grid with identity rows (cos 1, sin 0)."""
    if len(grid) != len(dims) or any(d % 2 for d in dims):
        raise ValueError("one even channel count per grid axis")
    axes = torch.meshgrid(*(torch.arange(n, dtype=torch.float64) for n in grid), indexing="ij")
    angles = torch.cat(
        [pos.reshape(-1, 1) * _freqs(d, theta)[None, :] for pos, d in zip(axes, dims, strict=True)],
        dim=1,
    )
    pairs = sum(dims) // 2
    ident = torch.zeros(1, pairs, dtype=torch.float64)
    angles = torch.cat([ident.expand(before, -1), angles, ident.expand(after, -1)], dim=0)
    cos = torch.cos(angles).float().contiguous()
    sin = torch.sin(angles).float().contiguous()
    sin[:before] = 0.0
    cos[:before] = 1.0
    if after:
        sin[-after:] = 0.0
        cos[-after:] = 1.0
    return RopeSpec(cos, sin, pairs, 1, sum(dims), True)


def llama(seq: int, dim: int, theta: float = 500000.0) -> RopeSpec:
    """1-D split-half RoPE (channel j pairs with j ± dim/2): tables [seq, dim] with each
    frequency repeated for both halves, the layout Diffusers/transformers split-half uses."""
    pos = torch.arange(seq, dtype=torch.float64)[:, None]
    angles = pos * _freqs(dim, theta)[None, :]
    angles = torch.cat([angles, angles], dim=1)
    return RopeSpec(
        torch.cos(angles).float().contiguous(), torch.sin(angles).float().contiguous(),
        dim, 1, dim, False,
    )


def head_norm_rope(
    x: Tensor,
    tables: RopeSpec | None,
    *,
    weight: Tensor | None = None,
    offset: float = 0.0,
    eps: float = 1e-6,
    normalize: bool = True,
    out: Tensor | None = None,
    token0: int = 0,
) -> Tensor:
    """Per-head RMSNorm then RoPE of [batch, seq, heads, head_dim] bf16 `x` (one launch of
    `cozy_head_norm_rope`): the drop-in for src/cozy_runtime/accel/fusion/_kernels.py:459
    (`head_norm_rope(launch, entry, x, weight, eps, tables, dtype)`, law :177-240) with the
    tables as `rope_tables` lays them out (`RopeSpec`; row = token of `x`'s sequence).
    `weight`: fp32 [head_dim] or None (unit); `normalize=False` rotates only; `token0`: the
    table row of `x`'s first token (a rank's rows of a longer sequence)."""
    import ctypes

    import torch

    from cozy_runtime_b200 import _lib

    if x.dtype != torch.bfloat16 or not x.is_cuda:
        raise ValueError("head_norm_rope serves bf16 CUDA tensors")
    batch, seq, heads, dim = x.shape
    out = torch.empty_like(x) if out is None else out
    rope_arg = None if tables is None else tables.struct(token0)
    w = None
    if weight is not None:
        w = weight.to(device=x.device, dtype=torch.float32).contiguous()
    code = _lib.load().cozy_head_norm_rope(
        x.data_ptr(), out.data_ptr(), batch, seq, heads, dim,
        _lib.strides3((x.stride(1), x.stride(2), x.stride(0))),
        _lib.strides3((out.stride(1), out.stride(2), out.stride(0))),
        None if rope_arg is None else ctypes.byref(rope_arg), int(normalize),
        None if w is None else w.data_ptr(), float(offset), float(eps),
        torch.cuda.current_stream(x.device).cuda_stream,
    )
    _lib.check("cozy_head_norm_rope", code)
    return out
