"""The int8 wire of the exchange (`exchange(..., narrow=True)`), stage by stage.

The reference's law (src/cozy_runtime/internal/parallel/turn.py:60-82): every row of a head's
Q, K (less K's mean over the whole sequence, turned: `_Shift`, ulysses.py:588-604) and V, and of
the attention's output, crosses as int8 after a turn by the orthonormal Hadamard matrix of the
head dimension, with one bf16 scale per row, and is turned back on arrival. Here the turn,
scale and codes of a row are one warp's work in `cozy_narrow_pack`, which writes them straight
into every destination (a peer's receive buffer over NVLink, or a local send block for NCCL);
`cozy_narrow_widen` turns them back into the attention's operands or the caller's output.

Block layouts (all row-major):
  first stage, to peer p:  codes [rows_mine][B][n_p][D] int8, scales [rows_mine][B][n_p] bf16,
                           at row `start_mine` of p's [total][B][n_p][D] receive buffers;
  return, to owner p:      codes [rows_p][B][qn_mine][D], scales [rows_p][B][qn_mine], at
                           block `mine` of p's landing buffers, stacked by source rank.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch
from torch import Tensor

from cozy_runtime_b200 import _lib

ORDERS = (64, 128)


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def key_sum_into(key: Tensor, out: Tensor) -> None:
    """Add the column sums of `key` [B, S, H, D] (bf16) into `out` [B, H, D] fp32."""
    code = _lib.load().cozy_key_sum(
        key.data_ptr(), _lib.strides3((key.stride(1), key.stride(2), key.stride(0))),
        key.shape[1], key.shape[0], key.shape[2], key.shape[3], out.data_ptr(),
        _stream(key.device),
    )
    _lib.check("cozy_key_sum", code)


def turned_mean(k_sum: Tensor, total: int) -> Tensor:
    """The shift: (k_sum / total) turned, [B, H, D] fp32 (`_Shift.__call__`)."""
    shift = torch.empty_like(k_sum)
    batch, heads, dim = (int(n) for n in k_sum.shape)
    code = _lib.load().cozy_narrow_shift(
        k_sum.data_ptr(), total, batch, heads, dim, shift.data_ptr(), _stream(k_sum.device)
    )
    _lib.check("cozy_narrow_shift", code)
    return shift


def _tensor(
    src: Tensor,
    shift: Tensor | None,
    dst: Sequence[tuple[int, int]],
    head_lo: Sequence[int],
    head_n: Sequence[int],
    row_lo: Sequence[int],
    row_n: Sequence[int],
) -> _lib.NarrowTensor:
    t = _lib.NarrowTensor()
    t.src = src.data_ptr()
    t.src_strides[:] = [src.stride(1), src.stride(2), src.stride(0)]
    t.heads = src.shape[2]
    t.shift = None if shift is None else shift.data_ptr()
    for p, (codes, scales) in enumerate(dst):
        t.dst[p], t.scale_dst[p] = codes, scales
        t.head_lo[p], t.head_n[p] = head_lo[p], head_n[p]
        t.row_lo[p], t.row_n[p] = row_lo[p], row_n[p]
    return t


def pack(tensors: Sequence[_lib.NarrowTensor], world: int, rows: int, like: Tensor) -> None:
    arr = (_lib.NarrowTensor * len(tensors))(*tensors)
    code = _lib.load().cozy_narrow_pack(
        arr, len(tensors), world, rows, like.shape[0], like.shape[3], _stream(like.device)
    )
    _lib.check("cozy_narrow_pack", code)


def widen(sources: Sequence[tuple[int, int, int, int, int, int]], out: Tensor) -> None:
    """Sources (codes ptr, scales ptr, row_lo, rows, head_lo, head_n) turned back into `out`
    [B, S, H, D] bf16 (any strides)."""
    arr = (_lib.WidenSource * len(sources))()
    for i, (codes, scales, row_lo, rows, head_lo, head_n) in enumerate(sources):
        arr[i].codes, arr[i].scales = codes, scales
        arr[i].row_lo, arr[i].rows, arr[i].head_lo, arr[i].head_n = row_lo, rows, head_lo, head_n
    code = _lib.load().cozy_narrow_widen(
        arr, len(sources), out.shape[0], out.shape[3], out.data_ptr(),
        _lib.strides3((out.stride(1), out.stride(2), out.stride(0))), _stream(out.device),
    )
    _lib.check("cozy_narrow_widen", code)


class NarrowStep:
    """One rank's narrow stages of one exchange (`ulysses.Plan` layout `layout`, `rank`)."""

    def __init__(self, query: Tensor, key: Tensor, value: Tensor, layout, rank: int) -> None:
        if query.shape[3] not in ORDERS:
            raise ValueError(f"the int8 wire serves head_dim {ORDERS}")
        self.query, self.key, self.value = query, key, value
        self.layout, self.rank = layout, rank
        self.batch, self.mine, self.heads, self.dim = (int(n) for n in query.shape)
        self.heads_kv = int(key.shape[2])
        self.start = layout.start(rank)

    # ---------------------------------------------------------------- block sizes (elements)
    def first_block(self, p: int, kind: str) -> int:
        """Codes this rank sends peer p for Q ("q") or K/V ("kv")."""
        n = self.layout.q_n[p] if kind == "q" else self.layout.kv_n[p]
        return self.mine * self.batch * n * self.dim

    def return_block(self, p: int) -> int:
        """Codes of owner p's rows this rank sends back: all its query heads."""
        return self.layout.rows[p] * self.batch * self.layout.q_n[self.rank] * self.dim

    def landing_block(self, s: int) -> int:
        """Codes source s sends this rank back: its query heads of this rank's rows."""
        return self.mine * self.batch * self.layout.q_n[s] * self.dim

    # ------------------------------------------------------------------------- stages
    def shift(self, k_sum: Tensor) -> Tensor:
        return turned_mean(k_sum, self.layout.total)

    def pack_to(
        self,
        shift: Tensor,
        q_dst: Sequence[tuple[int, int]],
        k_dst: Sequence[tuple[int, int]],
        v_dst: Sequence[tuple[int, int]],
    ) -> None:
        """Q, K less `shift`, V narrowed into every peer's block: (codes, scales) addresses per
        peer; one launch."""
        lay, world = self.layout, self.layout.world
        every = [0] * world, [self.mine] * world
        pack(
            [
                _tensor(self.query, None, q_dst, lay.q_lo, lay.q_n, *every),
                _tensor(self.key, shift, k_dst, lay.kv_lo, lay.kv_n, *every),
                _tensor(self.value, None, v_dst, lay.kv_lo, lay.kv_n, *every),
            ],
            world, self.mine, self.query,
        )

    def return_to(self, attended: Tensor, dst: Sequence[tuple[int, int]]) -> None:
        """The attention's rows [B, total, qn, D] narrowed to their owners by row."""
        lay, world = self.layout, self.layout.world
        qn = lay.q_n[self.rank]
        if not qn:
            return
        starts = [lay.start(p) for p in range(world)]
        pack(
            [_tensor(attended, None, dst, [0] * world, [qn] * world, starts, list(lay.rows))],
            world, lay.total, attended,
        )

    def operands(self, codes: Tensor, scales: Tensor, n: int) -> Tensor:
        """Received [total][B][n][D] codes and [total][B][n] scales widened into the attention's
        operand buffer, returned as its [B, total, n, D] view."""
        total = self.layout.total
        out = torch.empty(total, self.batch, n, self.dim, dtype=torch.bfloat16,
                          device=self.query.device)
        view = out.permute(1, 0, 2, 3)
        if n:
            widen([(codes.data_ptr(), scales.data_ptr(), 0, total, 0, n)], view)
        return view

    def land(self, codes: Tensor, scales: Tensor) -> Tensor:
        """The returned blocks (stacked by source rank) widened into [B, rows, H, D]."""
        lay, world = self.layout, self.layout.world
        out = torch.empty(self.batch, self.mine, self.heads, self.dim, dtype=torch.bfloat16,
                          device=self.query.device)
        sources, at = [], 0
        for s in range(world):
            if lay.q_n[s] and self.mine:
                sources.append((codes.data_ptr() + at, scales.data_ptr() + 2 * (at // self.dim),
                                0, self.mine, lay.q_lo[s], lay.q_n[s]))
            at += self.landing_block(s)
        if sources:
            widen(sources, out)
        return out


def scale_ptr(codes_base: int, scales_base: int, code_offset: int, dim: int) -> tuple[int, int]:
    """(codes, scales) addresses of a block `code_offset` codes into a buffer pair: the scales
    of a block of codes sit at the same row offset, one bf16 per row of `dim` codes."""
    return codes_base + code_offset, scales_base + 2 * (code_offset // dim)


__all__ = ["NarrowStep", "key_sum_into", "turned_mean", "pack", "widen", "scale_ptr", "ORDERS"]
