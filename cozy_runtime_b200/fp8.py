"""The FP8 variant of the exchange's stages (the FP8 video configuration's recipe).

Per rank and call: partial statistics of its rows (K sums, V channel absmax; `cozy_fp8_stats`),
made global by the caller (one all-reduce each: SUM, MAX — the reference's `_Shift` does the
K mean the same way, `src/cozy_runtime/internal/parallel/ulysses.py:588-604`); the first stage
(`cozy_fp8_pack`; per-head RMSNorm and RoPE first when asked, rounded to bf16 as the bf16 first
stage leaves them, so RoPE, quantisation and the transpose are one pass) writes e4m3 codes of Q
and K (one scale per 64-token × head block — 64 tokens
of the whole sequence from a multiple of 64, cut at rank boundaries — K less the
global mean, both rotated by the orthonormal Hadamard of order 128 first, as the reference's
FA4-fp8 row does, `src/cozy_runtime/internal/attention_upstream.py:276-317`) and V (one scale per
channel) into every peer's receive buffers with Q/K's
per-token scales beside them; the attention (`cozy_attention_fwd_fp8`) reads the codes in place
and writes bf16 output rows to their owners.
"""

from __future__ import annotations

import ctypes
import math
from collections.abc import Sequence
from dataclasses import dataclass

import torch
from torch import Tensor

from cozy_runtime_b200 import _lib, attention

E4M3_MAX = 448.0
#: The per-head law maps a head's amax onto 440, not 448 (attention_fp8.py:31-34).
E4M3_TARGET = 440.0
SCALE_FLOOR = 1e-12
BLOCK = 64
#: The recipes: "block" (BASELINE's FP8 configuration: 64-token block scales on Hadamard-rotated
#: Q and K less its mean, V per channel) and "head" (the reference's own FP8 row, `fa4_fp8`:
#: Hadamard-rotated Q and K, one scale per (batch, head) of Q, K and V, target 440).
LAWS = ("block", "head")


def _norm_fields(t, norm) -> None:
    """A per-head RMSNorm's fields (`ulysses.Norm` or None) into an FP8 stage descriptor."""
    t.normalize = int(norm is not None)
    if norm is not None:
        t.norm_weight = norm.weight.data_ptr() if norm.weight is not None else None
        t.norm_offset = float(norm.offset)
        t.norm_eps = float(norm.eps)


def scale_seq(total: int) -> int:
    """Per-token scale rows are padded to whole 128-key tiles (the kernel reads them so)."""
    return -(-total // 128) * 128


@dataclass
class Fp8Scales:
    """The global statistics one call's first stage quantises with. Block law: K's sums over the
    whole sequence [B, Hkv, 128] (its mean is subtracted) and V's per-channel scales. Per-head
    law: Q's and K's descales [B, H] / [B, Hkv] and V's per-head descales broadcast over its
    channels [B, Hkv, 128]."""

    v_scale: Tensor
    k_sum: Tensor | None = None
    q_head: Tensor | None = None
    k_head: Tensor | None = None


class Fp8Step:
    """One rank's FP8 stages of one exchange (`ulysses.Plan` layout, `rank`)."""

    def __init__(self, query: Tensor, key: Tensor, value: Tensor, layout, rank: int, *,
                 rope=None, norm_q=None, norm_k=None, law: str = "block") -> None:
        if query.shape[3] != 128:
            raise ValueError("the FP8 path serves head_dim 128")
        if law not in LAWS:
            raise ValueError(f"FP8 law {law!r}: one of {LAWS}")
        self.law = law
        self.query, self.key, self.value = query, key, value
        self.layout, self.rank = layout, rank
        # the first stage's law (per-head RMSNorm, then RoPE by global position) before the
        # recipe: `rope` a RopeSpec over the whole sequence, `norm_*` ulysses.Norm or None
        self.rope, self.norm_q, self.norm_k = rope, norm_q, norm_k
        self.batch, self.mine, self.heads, self.dim = (int(n) for n in query.shape)
        self.heads_kv = int(key.shape[2])
        self.total = layout.total
        self.sseq = scale_seq(self.total)

    # --------------------------------------------------------------- statistics
    def stats_into(self, k_sum: Tensor, v_amax: Tensor) -> None:
        """Add this rank's K sums into `k_sum` and max its |V| into `v_amax` ([B, Hkv, 128] fp32)."""
        st = _lib.Fp8Stats()
        st.key = self.key.data_ptr()
        st.value = self.value.data_ptr()
        st.k_strides[:] = [self.key.stride(1), self.key.stride(2), self.key.stride(0)]
        st.v_strides[:] = [self.value.stride(1), self.value.stride(2), self.value.stride(0)]
        st.rows, st.batch, st.heads, st.head_dim = self.mine, self.batch, self.heads_kv, self.dim
        st.k_sum, st.v_amax = k_sum.data_ptr(), v_amax.data_ptr()
        _norm_fields(st, self.norm_k)
        if self.rope is not None:
            st.rotate, st.rope = 1, self.rope.struct(self.layout.start(self.rank))
        code = _lib.load().cozy_fp8_stats(
            ctypes.byref(st), torch.cuda.current_stream(self.query.device).cuda_stream
        )
        _lib.check("cozy_fp8_stats", code)

    @staticmethod
    def channel_scale(v_amax: Tensor) -> Tensor:
        """V's per-channel scale from its global absmax: max(amax / 448, 1e-12)."""
        return (v_amax / E4M3_MAX).clamp_(min=SCALE_FLOOR)

    # --------------------------------------------------------------- per-head law
    def head_amax_into(self, q_amax: Tensor, k_amax: Tensor, v_amax: Tensor) -> None:
        """Max this rank's per-(batch, head) absmax of the rotated Q and K and of V into
        `q_amax` [B, H] and `k_amax`, `v_amax` [B, Hkv] (fp32; the caller zero-fills them and
        all-reduces MAX)."""
        pk = self._pack_struct([None] * self.layout.world, [None] * self.layout.world,
                               [None] * self.layout.world, None, None)
        for i, amax in enumerate((q_amax, k_amax, v_amax)):
            pk.t[i].head_amax = amax.data_ptr()
        code = _lib.load().cozy_fp8_head_amax(
            ctypes.byref(pk), torch.cuda.current_stream(self.query.device).cuda_stream
        )
        _lib.check("cozy_fp8_head_amax", code)

    @staticmethod
    def head_scales(q_amax: Tensor, k_amax: Tensor, v_amax: Tensor) -> tuple[Tensor, Tensor, Tensor]:
        """The per-head law's descales from the global amax: max(amax / 440, 1e-12)
        (attention_fp8.py:169); V's broadcast over its 128 channels, the form the attention
        reads."""
        # amax / 440 correctly rounded, as the reference divides on the host (a CUDA tensor
        # divided by a scalar may be multiplied by its reciprocal instead)
        q, k, v = ((a.double() / E4M3_TARGET).float().clamp_(min=SCALE_FLOOR)
                   for a in (q_amax, k_amax, v_amax))
        return q.contiguous(), k.contiguous(), v[..., None].expand(*v.shape, 128).contiguous()

    # --------------------------------------------------------------- first stage
    def _pack_struct(self, q_dst, k_dst, v_dst, qs_dst, ks_dst, *, k_sum=None, v_scale=None,
                     q_head=None, k_head=None, scale_rows=None) -> _lib.Fp8Pack:
        lay = self.layout
        pk = _lib.Fp8Pack()
        pk.world, pk.rows, pk.batch, pk.head_dim = lay.world, self.mine, self.batch, self.dim
        pk.row0 = lay.start(self.rank)
        # start at this rank's own heads: the ranks then write to different peers at a time
        pk.head_turn = lay.q_lo[self.rank] if lay.q_n[self.rank] else 0
        pk.per_head = int(self.law == "head")
        if self.rope is not None:
            pk.rope = self.rope.struct(lay.start(self.rank))
        block = self.law == "block"
        specs = [
            (self.query, lay.q_lo, lay.q_n, q_dst, qs_dst, None, None, q_head),
            (self.key, lay.kv_lo, lay.kv_n, k_dst, ks_dst, k_sum if block else None, None, k_head),
            (self.value, lay.kv_lo, lay.kv_n, v_dst, None, None, v_scale, None),
        ]
        for i, (src, lo, n, dst, sdst, mean, chan, head) in enumerate(specs):
            t = pk.t[i]
            t.src = src.data_ptr()
            t.src_strides[:] = [src.stride(1), src.stride(2), src.stride(0)]
            t.heads = src.shape[2]
            t.hadamard = int(i < 2)  # Q and K, as the reference's FA4-fp8 row rotates them
            t.mean_sum = mean.data_ptr() if mean is not None else None
            t.mean_inv_count = 1.0 / self.total
            t.channel_scale = chan.data_ptr() if chan is not None else None
            t.head_scale = head.data_ptr() if head is not None else None
            t.scale_seq = self.sseq if scale_rows is None else scale_rows
            if i < 2:
                _norm_fields(t, self.norm_q if i == 0 else self.norm_k)
                t.rotate = int(self.rope is not None)
            for p in range(lay.world):
                t.dst[p] = dst[p]
                t.scale_dst[p] = sdst[p] if sdst is not None else None
                t.head_lo[p] = lo[p]
                t.head_n[p] = n[p]
        return pk

    def pack_to(
        self,
        scales: Fp8Scales,
        q_dst: Sequence[int],
        k_dst: Sequence[int],
        v_dst: Sequence[int],
        qs_dst: Sequence[int],
        ks_dst: Sequence[int],
        scale_rows: int | None = None,
    ) -> None:
        """Codes into every peer's receive buffers (addresses of this rank's first row there)
        and Q/K per-token scales into their scale arrays (addresses of this rank's first token;
        a head's scales are `scale_rows` apart, default the padded whole sequence)."""
        pk = self._pack_struct(q_dst, k_dst, v_dst, qs_dst, ks_dst, k_sum=scales.k_sum,
                               v_scale=scales.v_scale, q_head=scales.q_head,
                               k_head=scales.k_head, scale_rows=scale_rows)
        code = _lib.load().cozy_fp8_pack(
            ctypes.byref(pk), torch.cuda.current_stream(self.query.device).cuda_stream
        )
        _lib.check("cozy_fp8_pack", code)

    def scales(self, handle=None) -> Fp8Scales:
        """This call's global statistics (this rank's, all-reduced over `handle` when given)."""
        import torch.distributed as dist

        dev, b = self.query.device, self.batch
        if self.law == "block":
            k_sum = torch.zeros(b, self.heads_kv, self.dim, dtype=torch.float32, device=dev)
            v_amax = torch.zeros(b, self.heads_kv, self.dim, dtype=torch.float32, device=dev)
            self.stats_into(k_sum, v_amax)
            if handle is not None:
                dist.all_reduce(k_sum, op=dist.ReduceOp.SUM, group=handle)
                dist.all_reduce(v_amax, op=dist.ReduceOp.MAX, group=handle)
            return Fp8Scales(v_scale=self.channel_scale(v_amax), k_sum=k_sum)
        flat = torch.zeros(b * (self.heads + 2 * self.heads_kv), dtype=torch.float32, device=dev)
        q_amax = flat[: b * self.heads].view(b, self.heads)
        k_amax = flat[b * self.heads : b * (self.heads + self.heads_kv)].view(b, self.heads_kv)
        v_amax = flat[b * (self.heads + self.heads_kv) :].view(b, self.heads_kv)
        self.head_amax_into(q_amax, k_amax, v_amax)
        if handle is not None:
            dist.all_reduce(flat, op=dist.ReduceOp.MAX, group=handle)
        q, k, v = self.head_scales(q_amax, k_amax, v_amax)
        return Fp8Scales(v_scale=v, q_head=q, k_head=k)

    # --------------------------------------------------------------- attention
    def attend(
        self,
        q8: Tensor,
        k8: Tensor,
        v8: Tensor,
        qs: Tensor,
        ks: Tensor,
        v_scale_local: Tensor,
        *,
        causal: bool,
        scale: float | None,
        scatter: _lib.Scatter | None = None,
        into: Tensor | None = None,
    ) -> None:
        """Attention over this rank's heads from its receive buffers (uint8 codes
        [total][B][n][128], per-token scales [B][n][scale_seq], V scales [B][n_kv][128] of this
        rank's K/V heads) into `into` ([B, total, n, 128] view) or to the owners (`scatter`)."""
        lay, rank = self.layout, self.rank
        qn, kvn = lay.q_n[rank], lay.kv_n[rank]
        if not qn:
            return
        total, batch, dim = self.total, self.batch, self.dim
        qv = q8[: total * batch * qn * dim].view(total, batch, qn, dim).permute(1, 0, 2, 3)
        kv = k8[: total * batch * kvn * dim].view(total, batch, kvn, dim).permute(1, 0, 2, 3)
        vv = v8[: total * batch * kvn * dim].view(total, batch, kvn, dim).permute(1, 0, 2, 3)

        def strides(t: Tensor):
            return _lib.strides3((t.stride(1), t.stride(2), t.stride(0)))

        head_map = _lib.HeadMap(lay.group, lay.q_lo[rank], lay.kv_lo[rank])
        sc = 1.0 / math.sqrt(dim) if scale is None else float(scale)
        cuts = [lay.start(r) for r in range(1, lay.world) if 0 < lay.start(r) < total]
        cut_arr = (ctypes.c_int * max(1, len(cuts)))(*cuts)
        code = _lib.load().cozy_attention_fwd_fp8(
            qv.data_ptr(), kv.data_ptr(), vv.data_ptr(), qs.data_ptr(), ks.data_ptr(),
            v_scale_local.data_ptr(), self.sseq, cut_arr, len(cuts),
            None if into is None else into.data_ptr(),
            batch, total, total, qn, kvn, dim,
            strides(qv), strides(kv), strides(vv), None if into is None else strides(into),
            ctypes.byref(head_map), None if scatter is None else ctypes.byref(scatter),
            int(causal), sc, attention.status_word(self.query.device).data_ptr(),
            torch.cuda.current_stream(self.query.device).cuda_stream,
        )
        _lib.check("cozy_attention_fwd_fp8", code)

    def local_v_scale(self, v_scale: Tensor) -> Tensor:
        """V scales of this rank's K/V heads, contiguous [B, n_kv, 128]."""
        lo, n = self.layout.kv_lo[self.rank], self.layout.kv_n[self.rank]
        return v_scale[:, lo : lo + n].contiguous()
