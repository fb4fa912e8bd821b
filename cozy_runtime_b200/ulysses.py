"""The Ulysses exchange around head-local attention, B200-native.

`exchange(query, key, value, handle, compute, site, narrow)` has the signature and the result of
the reference's `src/cozy_runtime/internal/parallel/ulysses.py:607` (`exchange`, installed behind
`attention_ulysses.exchange`): every rank passes its sequence rows [B, S_r, H, D] and gets back
its rows of the attention over the whole sequence, for every head. Differences of mechanism:

* The first stage is one fused kernel (`cozy_ulysses_pack`): RoPE and per-head RMSNorm (when
  asked), the transpose into per-peer head blocks, for Q, K and V in one launch.
* Q, K and V cross by the kernels' own stores into the peers' receive buffers over NVLink
  (`peer.PeerGroup`, the default on one node once its formation check passes), or with NCCL
  all-to-all (the reference's default wire, ulysses.py:207-246).
* `narrow=True` takes the reference's int8 wire (turn.py): one warp per row turns, scales and
  quantizes it into every destination, and one widens it back (`narrow.NarrowStep`).
* With `compute=None` the native sm_100a attention reads the receive buffers in place
  ([S, B, h, D], no unpack) and writes its output straight into the return send buffer; a
  callable `compute` gets [B, S, h, D] views and is served the reference's way.
* Heads are owned per rank as the reference pads them (ulysses.py:647): rank p attends over
  heads [p·⌈H/W⌉, (p+1)·⌈H/W⌉) ∩ [0, H); padded heads are never computed or sent. Grouped-query
  K/V heads cross only to the ranks whose query heads read them.
* The landing of the returned rows is one kernel (`cozy_ulysses_land`).

Row ownership follows `torch.tensor_split` (the reference's Diffusers split with
`ulysses_anything=True`, src/cozy_runtime/internal/parallel/cp.py:166-174). Every rank's row count
comes from a store meeting per call, as the reference's (ulysses.py:89-133), unless the caller
passes `rows`.
"""

from __future__ import annotations

import ctypes
import json
import math
import os
import threading
import weakref
from collections.abc import Callable, Sequence
from dataclasses import dataclass

import torch
import torch.distributed as dist
from torch import Tensor

from cozy_runtime_b200 import _lib, attention, peer
from cozy_runtime_b200 import fp8 as fp8_mod
from cozy_runtime_b200 import links as links_mod
from cozy_runtime_b200 import narrow as narrow_mod
from cozy_runtime_b200 import rope as rope_mod
from cozy_runtime_b200.rope import RopeSpec

Compute = Callable[[Tensor, Tensor, Tensor], Tensor]


@dataclass(frozen=True)
class Norm:
    """Per-head RMSNorm applied in the first stage: `x·rsqrt(mean(x²)+eps)·(weight+offset)`
    (weight None: unit), the law of src/cozy_runtime/accel/fusion/_kernels.py:78-86."""

    weight: Tensor | None = None
    offset: float = 0.0
    eps: float = 1e-6


@dataclass(frozen=True)
class Plan:
    """Who holds what in one exchange of `world` ranks."""

    rows: tuple[int, ...]
    heads: int
    heads_kv: int
    q_lo: tuple[int, ...]
    q_n: tuple[int, ...]
    kv_lo: tuple[int, ...]
    kv_n: tuple[int, ...]

    @property
    def world(self) -> int:
        return len(self.rows)

    @property
    def total(self) -> int:
        return sum(self.rows)

    @property
    def group(self) -> int:
        return self.heads // self.heads_kv

    def start(self, rank: int) -> int:
        return sum(self.rows[:rank])


def plan(rows: Sequence[int], heads: int, heads_kv: int) -> Plan:
    """Head ownership for rows `rows` (one entry per rank): query heads as the reference's padded
    blocks (ulysses.py:647, :325-362), key/value heads as the query heads read them."""
    world = len(rows)
    if heads % heads_kv:
        raise ValueError("query heads must be a multiple of key/value heads")
    group = heads // heads_kv
    local = (heads + (-heads % world)) // world
    q_lo, q_n, kv_lo, kv_n = [], [], [], []
    for rank in range(world):
        lo = min(rank * local, heads)
        hi = min((rank + 1) * local, heads)
        q_lo.append(lo)
        q_n.append(hi - lo)
        if hi > lo:
            kv_lo.append(lo // group)
            kv_n.append((hi - 1) // group - lo // group + 1)
        else:
            kv_lo.append(0)
            kv_n.append(0)
    return Plan(tuple(rows), heads, heads_kv, tuple(q_lo), tuple(q_n), tuple(kv_lo), tuple(kv_n))


def destination_order(rank: int, world: int) -> list[int]:
    """The order a rank's first stage fills its peers' blocks in: from itself onwards. The
    kernel fills destinations in list order (one grid row of CTAs per peer); so ordered, the
    ranks write to a different peer each at any moment (a permutation), instead of all into peer
    0's memory first, then peer 1's, which would put every sender behind one receiver's NVLink
    ingress at a time."""
    return [(rank + i) % world for i in range(world)]


def tensor_split_rows(total: int, world: int) -> list[int]:
    """`torch.tensor_split` row counts (cp.py:166-174)."""
    base, extra = divmod(total, world)
    return [base + (1 if r < extra else 0) for r in range(world)]


# --------------------------------------------------------------------------- store meeting
class _Meeting:
    """One metadata round per call over the group's store: every rank's rows and site. Ranks
    whose sites differ made different calls; each raises (ulysses.py:103-133)."""

    def __init__(self, handle) -> None:
        from torch.distributed.distributed_c10d import _get_process_group_store

        base = _get_process_group_store(handle)
        name = getattr(handle, "group_name", "") or "world"
        self.store = dist.PrefixStore(f"cozy-b200.ulysses/{name}/", base)
        self.rank = dist.get_rank(handle)
        self.world = dist.get_world_size(handle)
        self.sequence = 0
        self.lock = threading.Lock()

    def gather(self, value: dict) -> list[dict]:
        self.sequence += 1
        keys = [f"{self.sequence}/{rank}" for rank in range(self.world)]
        self.store.set(keys[self.rank], json.dumps(value))
        self.store.wait(keys)
        rows = [json.loads(self.store.get(key)) for key in keys]
        if self.sequence > 1:
            self.store.delete_key(f"{self.sequence - 1}/{self.rank}")
        sites = [row["site"] for row in rows]
        if len(set(sites)) > 1:
            raise RuntimeError(
                f"Ulysses call {self.sequence} is not one call: "
                + ", ".join(f"GPU {rank} at {site}" for rank, site in enumerate(sites))
            )
        return rows


_MEETINGS: weakref.WeakKeyDictionary = weakref.WeakKeyDictionary()
_MEETINGS_LOCK = threading.Lock()


def _meeting(handle) -> _Meeting:
    with _MEETINGS_LOCK:
        found = _MEETINGS.get(handle)
        if found is None:
            found = _MEETINGS[handle] = _Meeting(handle)
        return found


# ------------------------------------------------------------------------------- clock
class _Clock:
    """Device-event spans of this process's exchanges (the reference's `_Clock`,
    ulysses.py:507-577): the whole exchange, the attention inside it; exposed = the rest."""

    def __init__(self) -> None:
        self.pending: list[tuple] = []
        self.totals = self._zero()
        self.lock = threading.Lock()

    @staticmethod
    def _zero() -> dict:
        return {"calls": 0, "exchange": 0.0, "attention": 0.0, "before": 0.0, "crossed": 0}

    @staticmethod
    def mark(on: Tensor):
        if not on.is_cuda or torch.cuda.is_current_stream_capturing():
            return None
        event = torch.cuda.Event(enable_timing=True)
        event.record()
        return event

    def add(self, marks: tuple, crossed: int) -> None:
        if any(m is None for m in marks):
            return
        with self.lock:
            self.pending.append((marks, crossed))
            if len(self.pending) > 256:
                self._fold(wait=False)

    def _fold(self, *, wait: bool) -> None:
        while self.pending:
            (began, first, last, ended), crossed = self.pending[0]
            if wait:
                ended.synchronize()
            elif not ended.query():
                return
            self.pending.pop(0)
            self.totals["calls"] += 1
            self.totals["exchange"] += began.elapsed_time(ended)
            self.totals["attention"] += first.elapsed_time(last)
            self.totals["before"] += began.elapsed_time(first)
            self.totals["crossed"] += crossed

    def take(self) -> dict:
        with self.lock:
            self._fold(wait=True)
            t, self.totals = self.totals, self._zero()
        return {
            "calls": t["calls"],
            "crossed_gb": round(t["crossed"] / 1e9, 3),
            "exchange_ms": round(t["exchange"], 3),
            "attention_ms": round(t["attention"], 3),
            "exposed_ms": round(t["exchange"] - t["attention"], 3),
            # exposed before the attention (first stage, crossing, arrival) and after it
            "before_ms": round(t["before"], 3),
            "after_ms": round(t["exchange"] - t["attention"] - t["before"], 3),
        }


_CLOCK = _Clock()


def taken() -> dict:
    """What this process's exchanges moved and took since the last take (ulysses.py:580)."""
    return _CLOCK.take()


# ------------------------------------------------------------------------------ exchange
def _pack_tensor(
    src: Tensor,
    sends: list[int],
    lo: Sequence[int],
    n: Sequence[int],
    *,
    rotate: bool,
    norm: Norm | None,
) -> _lib.PackTensor:
    t = _lib.PackTensor()
    t.src = src.data_ptr()
    t.src_strides[:] = [src.stride(1), src.stride(2), src.stride(0)]
    t.heads = src.shape[2]
    t.rotate = int(rotate)
    t.normalize = int(norm is not None)
    if norm is not None:
        t.norm_weight = norm.weight.data_ptr() if norm.weight is not None else None
        t.norm_offset = float(norm.offset)
        t.norm_eps = float(norm.eps)
    for p, ptr in enumerate(sends):
        t.dst[p] = ptr
        t.head_lo[p] = lo[p]
        t.head_n[p] = n[p]
    return t


def _rope_struct(rope: RopeSpec, token0: int) -> _lib.Rope:
    return rope.struct(token0)


def pack(
    tensors: Sequence[tuple[Tensor, Sequence[int], Sequence[int], Sequence[int], bool, Norm | None]],
    rows: int,
    rope: RopeSpec | None,
    token0: int,
) -> None:
    """One `cozy_ulysses_pack` launch: each entry (src, dst pointers per peer, head_lo, head_n,
    rotate, norm)."""
    src0 = tensors[0][0]
    arr = (_lib.PackTensor * len(tensors))(
        *(_pack_tensor(s, d, lo, n, rotate=r, norm=nm) for s, d, lo, n, r, nm in tensors)
    )
    rope_arg = None
    if rope is not None:
        rope_arg = _rope_struct(rope, token0)
    code = _lib.load().cozy_ulysses_pack(
        arr, len(tensors), len(tensors[0][1]), rows, src0.shape[0], src0.shape[3],
        None if rope_arg is None else rope_arg, torch.cuda.current_stream(src0.device).cuda_stream,
    )
    _lib.check("cozy_ulysses_pack", code)


def land(
    returned: Tensor, out: Tensor, lo: Sequence[int], n: Sequence[int]
) -> None:
    """One `cozy_ulysses_land` launch: `returned` stacked by source rank into `out`'s heads."""
    world = len(lo)
    code = _lib.load().cozy_ulysses_land(
        returned.data_ptr(), world, out.shape[1], out.shape[0], out.shape[3],
        (_lib.c_int * world)(*lo), (_lib.c_int * world)(*n), out.data_ptr(),
        _lib.strides3((out.stride(1), out.stride(2), out.stride(0))),
        torch.cuda.current_stream(out.device).cuda_stream,
    )
    _lib.check("cozy_ulysses_land", code)


def _offsets(sizes: Sequence[int]) -> list[int]:
    out, acc = [], 0
    for s in sizes:
        out.append(acc)
        acc += s
    return out


class RankStep:
    """One rank's part of one exchange, phase by phase, so a crossing can be NCCL's
    (`exchange`) or any other transport that moves the same blocks: `send` buffers hold this
    rank's block for peer p at `send_offsets[p]`; `receive` buffers take source p's block at
    `receive_offsets[p]`."""

    def __init__(
        self,
        query: Tensor,
        key: Tensor,
        value: Tensor,
        layout: Plan,
        rank: int,
        *,
        rope: RopeSpec | None = None,
        norm_q: Norm | None = None,
        norm_k: Norm | None = None,
    ) -> None:
        self.query, self.key, self.value = query, key, value
        self.layout, self.rank = layout, rank
        self.rope, self.norm_q, self.norm_k = rope, norm_q, norm_k
        batch, mine, heads, dim = (int(n) for n in query.shape)
        self.batch, self.mine, self.heads, self.dim = batch, mine, heads, dim
        world, rows = layout.world, layout.rows
        self.qn, self.kvn = layout.q_n[rank], layout.kv_n[rank]
        self.q_sizes = [mine * batch * layout.q_n[p] * dim for p in range(world)]
        self.kv_sizes = [mine * batch * layout.kv_n[p] * dim for p in range(world)]
        self.q_in = [r * batch * self.qn * dim for r in rows]
        self.kv_in = [r * batch * self.kvn * dim for r in rows]
        self.back_sizes = list(self.q_sizes)  # O returns as Q left: my rows, peer p's heads
        self.back_in = list(self.q_in)
        self.q_send = self.k_send = self.v_send = None

    def receive_buffers(self) -> tuple[Tensor, Tensor, Tensor]:
        total, dev, dt = self.layout.total, self.query.device, self.query.dtype
        return (
            torch.empty(total * self.batch * self.qn * self.dim, dtype=dt, device=dev),
            torch.empty(total * self.batch * self.kvn * self.dim, dtype=dt, device=dev),
            torch.empty(total * self.batch * self.kvn * self.dim, dtype=dt, device=dev),
        )

    def pack(self) -> None:
        """Stage 1 into local send blocks (an NCCL crossing follows): norm/RoPE/transposition
        of Q, K, V in one launch."""
        el = self.query.element_size()
        dev, dt = self.query.device, self.query.dtype
        self.q_send = torch.empty(sum(self.q_sizes), dtype=dt, device=dev)
        self.k_send = torch.empty(sum(self.kv_sizes), dtype=dt, device=dev)
        self.v_send = torch.empty(sum(self.kv_sizes), dtype=dt, device=dev)

        def ptrs(buf: Tensor, sizes: Sequence[int]) -> list[int]:
            return [buf.data_ptr() + off * el for off in _offsets(sizes)]

        self.pack_to(
            ptrs(self.q_send, self.q_sizes),
            ptrs(self.k_send, self.kv_sizes),
            ptrs(self.v_send, self.kv_sizes),
        )

    def pack_to(self, q_dst: Sequence[int], k_dst: Sequence[int], v_dst: Sequence[int]) -> None:
        """Stage 1 into the given per-peer block addresses (local, or in the peers' own receive
        buffers over NVLink): one launch for Q, K and V."""
        lay, rotate = self.layout, self.rope is not None
        order = destination_order(self.rank, lay.world)

        def turned(seq):
            return [seq[p] for p in order]

        pack(
            [
                (self.query, turned(q_dst), turned(lay.q_lo), turned(lay.q_n), rotate,
                 self.norm_q),
                (self.key, turned(k_dst), turned(lay.kv_lo), turned(lay.kv_n), rotate,
                 self.norm_k),
                (self.value, turned(v_dst), turned(lay.kv_lo), turned(lay.kv_n), False, None),
            ],
            self.mine,
            self.rope,
            lay.start(self.rank),
        )

    def attend(
        self,
        q_recv: Tensor,
        k_recv: Tensor,
        v_recv: Tensor,
        compute: Compute | None,
        causal: bool,
        scale: float | None,
        into: Tensor | None = None,
        scatter: _lib.Scatter | None = None,
    ) -> Tensor:
        """Attention over this rank's heads of the whole sequence, read in place from the
        receive buffers ([total][B][n][D]); returns the O send buffer in the same layout, or
        writes `into` ([B, total, n, D], any strides; degree 1: the output itself)."""
        lay, total, batch, dim = self.layout, self.layout.total, self.batch, self.dim
        qn, kvn = self.qn, self.kvn
        if scatter is not None:
            o_send, ov = None, None
        elif into is None:
            o_send = torch.empty(
                total * batch * qn * dim, dtype=self.query.dtype, device=self.query.device
            )
            ov = o_send.view(total, batch, qn, dim).permute(1, 0, 2, 3) if qn else None
        else:
            o_send, ov = into, into
        if not qn:
            return o_send
        qv = q_recv.view(total, batch, qn, dim).permute(1, 0, 2, 3)
        kv = k_recv.view(total, batch, kvn, dim).permute(1, 0, 2, 3)
        vv = v_recv.view(total, batch, kvn, dim).permute(1, 0, 2, 3)
        if compute is None:
            head_map = (lay.group, lay.q_lo[self.rank], lay.kv_lo[self.rank])
            attention.attention_into(
                None if scatter is not None else ov, qv, kv, vv, causal=causal, scale=scale,
                head_map=head_map, scatter=scatter,
            )
            return o_send
        if kvn != qn or lay.group != 1:
            idx = torch.tensor(
                [(lay.q_lo[self.rank] + i) // lay.group - lay.kv_lo[self.rank] for i in range(qn)],
                device=self.query.device,
            )
            kv, vv = kv.index_select(2, idx), vv.index_select(2, idx)
        attended = compute(qv, kv, vv)
        if attended.shape != (batch, total, qn, dim) or attended.dtype != self.query.dtype:
            raise ValueError("Ulysses attention returned incompatible output")
        ov.copy_(attended)
        return o_send

    def land(self, returned: Tensor) -> Tensor:
        """Stage 3: the returned rows of every source rank into [B, S_r, H, D]."""
        out = torch.empty(
            (self.batch, self.mine, self.heads, self.dim), dtype=self.query.dtype,
            device=self.query.device,
        )
        land(returned, out, self.layout.q_lo, self.layout.q_n)
        return out

    def moved(self) -> int:
        """Bytes this rank sent to other ranks (Q, K, V in; O back)."""
        r = self.rank
        el = self.query.element_size()
        return el * (
            sum(self.q_sizes) - self.q_sizes[r] + 2 * (sum(self.kv_sizes) - self.kv_sizes[r])
            + sum(self.back_in) - self.back_in[r]
        )


def exchange(
    query: Tensor,
    key: Tensor,
    value: Tensor,
    handle,
    compute: Compute | None = None,
    site: str = "",
    narrow: bool | Callable[[int], bool] = False,
    **options,
) -> Tensor:
    """Sequence shards -> whole sequences per head subset -> attention -> back (keywords: those
    of `_exchange`). fp32 and fp16 inputs with the native attention cross and multiply as bf16
    and come back in their own dtype. Raises when an earlier call on this device reported a
    timed-out wait, seen without synchronizing: the status word is copied to the host behind
    every call."""
    if query.is_cuda and compute is None and query.dtype in (torch.float32, torch.float16):
        # the kernels compute in bf16 (fp32 softmax and accumulation): other floating inputs
        # cross and multiply as bf16 and the output returns in the query's dtype
        wide = query.dtype
        out = exchange(query.to(torch.bfloat16), key.to(torch.bfloat16),
                       value.to(torch.bfloat16), handle, None, site, narrow, **options)
        return out.to(wide)
    if query.is_cuda:
        attention.raise_if_failed(query.device)
    out = _exchange(query, key, value, handle, compute, site, narrow, **options)
    if query.is_cuda:
        attention.watch_after_call(query.device)
    return out


def _exchange(
    query: Tensor,
    key: Tensor,
    value: Tensor,
    handle,
    compute: Compute | None = None,
    site: str = "",
    narrow: bool | Callable[[int], bool] = False,
    *,
    rows: Sequence[int] | None = None,
    causal: bool = False,
    scale: float | None = None,
    rope: RopeSpec | None = None,
    norm_q: Norm | None = None,
    norm_k: Norm | None = None,
    transport: str | None = None,
    fp8: bool | str = False,
) -> Tensor:
    """Sequence shards -> whole sequences per head subset -> attention -> back.

    The first seven arguments are the reference's (`attention_ulysses.Exchange`); `compute=None`
    takes the native attention with `causal`/`scale`. `rows`: every rank's row count, when the
    caller knows them (skips the store meeting). `rope`: tables over the whole sequence, applied
    to Q and K by global position in the first stage; `norm_q`/`norm_k`: per-head RMSNorm before
    it. `transport`: "peer" (in-kernel NVLink stores between the GPUs of one node) or "nccl"
    (NCCL all-to-all); default `COZY_ULYSSES_TRANSPORT`, else "peer" for native attention on a
    CUDA group of one node. `fp8`: Q, K and V cross and multiply as e4m3 (`fp8.Fp8Step`: K less
    its global mean, Q/K Hadamard-rotated with 64-token block scales, V per-channel scales, P as
    e4m3; head_dim 128, native attention, either transport; RMSNorm/RoPE fused into the e4m3
    first stage); `fp8="head"`: the reference's own FP8 row instead (`fa4_fp8`: Hadamard-rotated
    Q and K, one e4m3 scale per (batch, head) of Q, K and V, target 440). `narrow` (or
    `narrow(total)`): Q, K less its turned global mean, V and the output cross as int8 with a
    bf16 scale per row after a Hadamard turn (`narrow.NarrowStep`, the reference's wire; head
    dims 64 and 128; any dimension that is not a power of two stays wide, as in the reference).
    Returns [B, S_r, H, D] in the query's dtype.
    """
    if not query.is_cuda:
        raise ValueError("cozy-b200 exchange serves CUDA tensors only")
    if query.dtype != torch.bfloat16:
        raise ValueError(f"cozy-b200 exchange serves bf16, not {query.dtype}")
    world = dist.get_world_size(handle) if handle is not None else 1
    rank = dist.get_rank(handle) if handle is not None else 0
    batch, mine, heads, dim = (int(n) for n in query.shape)
    heads_kv = int(key.shape[2])
    if key.shape != value.shape or key.shape[:2] != query.shape[:2] or key.shape[3] != dim:
        raise ValueError("Q, K and V must share batch, rows and head dim; K and V one shape")
    if rows is None:
        if world == 1:
            rows = [mine]
        else:
            meet = _meeting(handle)
            with meet.lock:
                proposals = meet.gather(
                    {"rows": mine, "site": f"{site or 'attention'} [{batch} x {heads} x {dim}]"}
                )
            rows = [int(p["rows"]) for p in proposals]
    rows = [int(r) for r in rows]
    if len(rows) != world or rows[rank] != mine:
        raise ValueError(f"rows {rows} do not match rank {rank}'s {mine} rows of {world}")
    layout = plan(rows, heads, heads_kv)
    began = _Clock.mark(query)
    # The int8 wire, decided on the agreed total as the reference does (ulysses.py:691): its
    # Hadamard turn needs a power-of-two head dimension, else the exchange stays wide. The FP8
    # path's own e4m3 wire is narrower still and takes precedence.
    total = layout.total
    wanted = bool(narrow(total) if callable(narrow) else narrow)
    if wanted and not fp8 and dim & (dim - 1) == 0:
        if dim not in narrow_mod.ORDERS:
            raise NotImplementedError(f"the int8 wire serves head_dim {narrow_mod.ORDERS}")
        return _exchange_narrow(
            query, key, value, handle, layout, rank, began, compute, causal, scale, rope,
            norm_q, norm_k, transport,
        )

    if fp8:
        if fp8 is not True and fp8 not in fp8_mod.LAWS:
            raise ValueError(f"fp8={fp8!r}: True (the block recipe) or one of {fp8_mod.LAWS}")
        if compute is not None:
            raise NotImplementedError("the FP8 path serves the native e4m3 attention only")
        over_peer = world > 1 and (_transport(handle, transport) == "peer"
                                   and _peer_ready(handle, query.device))
        return _exchange_fp8(query, key, value, handle, layout, rank, began, causal, scale,
                             rope=rope, norm_q=norm_q, norm_k=norm_k, over_peer=over_peer,
                             law="head" if fp8 == "head" else "block")
    if world == 1 and rope is None and norm_q is None and norm_k is None and compute is None:
        out = torch.empty((batch, mine, heads, dim), dtype=query.dtype, device=query.device)
        first = _Clock.mark(query)
        attention.attention_into(out, query, key, value, causal=causal, scale=scale)
        _CLOCK.add((began, first, _Clock.mark(query), _Clock.mark(query)), 0)
        return out

    if (world > 1 and compute is None and _transport(handle, transport) == "peer"
            and _peer_ready(handle, query.device)):
        return _exchange_peer(
            query, key, value, handle, layout, rank, began, causal, scale, rope, norm_q, norm_k
        )
    step = RankStep(query, key, value, layout, rank, rope=rope, norm_q=norm_q, norm_k=norm_k)
    step.pack()
    with _Crossing(handle) as crossing:
        if world == 1:
            q_recv, k_recv, v_recv = step.q_send, step.k_send, step.v_send
        else:
            q_recv, k_recv, v_recv = step.receive_buffers()
            crossing.crossed = True
            dist.all_to_all_single(q_recv, step.q_send, step.q_in, step.q_sizes, group=handle)
            dist.all_to_all_single(k_recv, step.k_send, step.kv_in, step.kv_sizes, group=handle)
            dist.all_to_all_single(v_recv, step.v_send, step.kv_in, step.kv_sizes, group=handle)
        if world == 1:  # degree 1: attention writes the output itself, nothing lands
            out = torch.empty((batch, mine, heads, dim), dtype=query.dtype, device=query.device)
            first = _Clock.mark(query)
            step.attend(q_recv, k_recv, v_recv, compute, causal, scale, into=out)
            last = _Clock.mark(query)
        else:
            first = _Clock.mark(query)
            o_send = step.attend(q_recv, k_recv, v_recv, compute, causal, scale)
            last = _Clock.mark(query)
            returned = torch.empty(sum(step.back_sizes), dtype=query.dtype, device=query.device)
            dist.all_to_all_single(returned, o_send, step.back_sizes, step.back_in, group=handle)
            out = step.land(returned)
    _CLOCK.add((began, first, last, _Clock.mark(query)), step.moved())
    return out


_FORMED: weakref.WeakKeyDictionary = weakref.WeakKeyDictionary()


def _peer_ready(handle, device: torch.device) -> bool:
    """Whether the group's NVLink transport passed its formation check (run once per group, on
    every rank together): one small exchange over the peer transport and over NCCL must give the
    same bytes on every rank, as the reference checks its copy-engine exchange against NCCL
    before using it (src/cozy_runtime/internal/parallel/copy_engine.py:408-449). A failed check
    leaves the group on NCCL."""
    state = _FORMED.get(handle)
    if state is None:
        _FORMED[handle] = "checking"  # the check's own exchanges take the peer path
        state = _FORMED[handle] = _form_check(handle, device)
    return state is not False


def _form_check(handle, device: torch.device) -> bool:
    world, rank = dist.get_world_size(handle), dist.get_rank(handle)
    gen = torch.Generator(device=device).manual_seed(977 + rank)
    rows = tensor_split_rows(64 * world + 3, world)
    heads = 2 * world
    q, k, v = (
        torch.randn(1, rows[rank], heads, 128, generator=gen, device=device).to(torch.bfloat16)
        for _ in range(3)
    )
    ok = True
    try:
        over_peer = exchange(q, k, v, handle, None, rows=rows, transport="peer")
        over_nccl = exchange(q, k, v, handle, None, rows=rows, transport="nccl")
        torch.cuda.synchronize(device)
        # The NVLink layer walks each tile's keys from this rank's own rows on, the NCCL path
        # from row 0: the sums differ in order, so the outputs agree to bf16 rounding, not bit
        # for bit. A transport that moved wrong or stale bytes misses by far more.
        diff = (over_peer.float() - over_nccl.float()).abs()
        ok = bool(diff.max().item() <= 1e-2 and diff.mean().item() <= 1e-3) and not int(
            attention.status_word(device).item()
        )
    except RuntimeError:
        ok = False
    agreed = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
    dist.all_reduce(agreed, op=dist.ReduceOp.MIN, group=handle)
    if not agreed.item():
        return False
    # the bytes are right; now the links: every ordered pair measured over the layer's own copy
    # engines (the reference's per-pair probe, links.py:394-519), the route from the pairs
    found = links_mod.measure(peer.layer_group_for(handle, device), handle, device)
    _LINKS[handle] = found
    return found.exchange == "peer"


_LINKS: weakref.WeakKeyDictionary = weakref.WeakKeyDictionary()


def links_of(handle):
    """The measured links of a group whose NVLink layer formed (`links.Links`), else None."""
    return _LINKS.get(handle) if handle is not None else None


def transport_of(handle, device: torch.device | None = None) -> str:
    """Which transport `exchange` takes on `handle` with native attention: "local" (one rank),
    "peer" (the NVLink layer, once its formation check passed) or "nccl"."""
    if handle is None or dist.get_world_size(handle) == 1:
        return "local"
    if _transport(handle, None) != "peer":
        return "nccl"
    state = _FORMED.get(handle)
    if state is None and device is not None:
        state = _peer_ready(handle, device)
    return "peer" if state is True else "nccl"


def _transport(handle, asked: str | None) -> str:
    choice = asked or os.environ.get("COZY_ULYSSES_TRANSPORT", "") or "peer"
    if choice not in ("peer", "nccl"):
        raise ValueError(f"unknown Ulysses transport {choice!r} (peer or nccl)")
    if choice == "peer" and dist.get_backend(handle) != "nccl":
        return "nccl"  # a CPU/gloo group has no device peers
    return choice


def _layer_call(
    query: Tensor, key: Tensor, value: Tensor, out: Tensor, rows: Sequence[int], causal: bool,
    scale: float | None, rope: RopeSpec | None, norm_q: Norm | None, norm_k: Norm | None,
    status: int, wait_limit_ns: int = 0,
) -> tuple[_lib.LayerCall, list]:
    """`CozyLayerCall` for this rank's tensors, and the objects it points into (keep them alive
    until the call is queued)."""
    batch, _, heads, dim = (int(n) for n in query.shape)
    call = _lib.LayerCall()
    call.shape = peer.layer_shape(rows, batch, heads, int(key.shape[2]), dim, causal)
    call.q, call.k, call.v = query.data_ptr(), key.data_ptr(), value.data_ptr()
    for field, t in (("q_strides", query), ("k_strides", key), ("v_strides", value)):
        if t.stride(3) != 1:
            raise ValueError("the head dimension must be contiguous")
        getattr(call, field)[:] = [t.stride(1), t.stride(2), t.stride(0)]
    call.out = out.data_ptr()
    call.scale = 1.0 / math.sqrt(dim) if scale is None else float(scale)
    keep: list = []
    if rope is not None:
        r = _rope_struct(rope, 0)
        keep.append(r)
        call.rope = ctypes.pointer(r)
    for i, norm in enumerate((norm_q, norm_k)):
        if norm is None:
            continue
        setattr(call, "norm_q" if i == 0 else "norm_k", 1)
        if norm.weight is not None:
            w = norm.weight.to(device=query.device, dtype=torch.float32).contiguous()
            keep.append(w)
            setattr(call, "norm_q_weight" if i == 0 else "norm_k_weight", w.data_ptr())
        call.norm_offset[i] = float(norm.offset)
        call.norm_eps[i] = float(norm.eps)
    call.wait_limit_ns = int(wait_limit_ns)
    call.status = status
    call.gate = int(layer_gate(len(rows)))
    call.cross = int(layer_cross(len(rows)) == "sm")
    return call, keep


def layer_cross(world: int) -> str:
    """How the NVLink layer's blocks cross (`CozyLayerCall.cross`): "ce" (copy engines from a
    staging buffer, beside the attention) or "sm" (the first stage stores straight into the
    owners' buffers). `COZY_LAYER_CROSS` forces either."""
    forced = os.environ.get("COZY_LAYER_CROSS", "")
    if forced in ("ce", "sm"):
        return forced
    # Measured at C2 on one B200 node: degree 8, SM stores cross 67 MB a rank at 518 GB/s
    # (1.709 ms layer) against 234 GB/s on the copy engines (1.846 ms; seven streams at once
    # were no faster than one); degree 2, the copy engines' crossing (444 GB/s) hides under the
    # attention's own-rows work and the layer matched the SM-store design (6.02-6.09 against
    # 5.91-6.06 ms).
    return "sm" if world >= 4 else "ce"


def layer_gate(world: int) -> bool:
    """Whether the NVLink layer holds the attention until every source's rows have landed
    (`CozyLayerCall.gate`) instead of letting it start at once and wait per source inside the
    kernel. `COZY_LAYER_GATE` = 1 / 0 forces either."""
    forced = os.environ.get("COZY_LAYER_GATE", "")
    if forced in ("0", "1"):
        return forced == "1"
    return False


def _exchange_peer(
    query: Tensor,
    key: Tensor,
    value: Tensor,
    handle,
    layout: Plan,
    rank: int,
    began,
    causal: bool,
    scale: float | None,
    rope: RopeSpec | None,
    norm_q: Norm | None,
    norm_k: Norm | None,
) -> Tensor:
    """The exchange over NVLink through the C layer entry (`cozy_ulysses_layer_*` on this
    rank's `peer.LayerGroup`): the first stage writes this rank's own block into its receive
    buffer and the others into staging, the copy engines move them to their owners with an
    arrival flag each, the attention starts on this rank's own rows at once and waits per source
    inside the kernel, its epilogue stores every output row into its owner's landing buffer,
    and flags say when a call's rows have landed."""
    batch, mine, heads, dim = (int(n) for n in query.shape)
    device = query.device
    lg = peer.layer_group_for(handle, device)
    out = torch.empty((batch, mine, heads, dim), dtype=query.dtype, device=device)
    call, keep = _layer_call(
        query, key, value, out, layout.rows, causal, scale, rope, norm_q, norm_k,
        attention.status_word(device).data_ptr(),
    )
    stream = torch.cuda.current_stream(device).cuda_stream
    with lg.lock:
        lg.ensure(call.shape)
        lg.run("begin", call, stream)
        first = _Clock.mark(query)
        lg.run("attend", call, stream)
        last = _Clock.mark(query)
        lg.run("end", call, stream)
    del keep
    step = RankStep(query, key, value, layout, rank)
    _CLOCK.add((began, first, last, _Clock.mark(query)), step.moved())
    return out


def _first_law(x: Tensor, rope: RopeSpec | None, norm: Norm | None, token0: int) -> Tensor:
    """Per-head RMSNorm and RoPE of a rank's rows (global positions from `token0`), as the
    first stage applies them, into a new tensor: the narrow wire turns the result."""
    if rope is None and norm is None:
        return x
    weight = None if norm is None or norm.weight is None else norm.weight
    return rope_mod.head_norm_rope(
        x, rope, weight=weight, offset=0.0 if norm is None else norm.offset,
        eps=1e-6 if norm is None else norm.eps, normalize=norm is not None, token0=token0,
    )


def _attend_operands(
    qv: Tensor, kv: Tensor, vv: Tensor, layout: Plan, rank: int, compute: Compute | None,
    causal: bool, scale: float | None,
) -> Tensor:
    """This rank's heads attended over the whole sequence from [B, total, n, D] operands:
    [B, total, qn, D] rows in a [total][B][qn][D] buffer (the return's source layout)."""
    batch, total, qn, dim = qv.shape
    o = torch.empty(total, batch, qn, dim, dtype=qv.dtype, device=qv.device)
    ov = o.permute(1, 0, 2, 3)
    if compute is None:
        head_map = (layout.group, layout.q_lo[rank], layout.kv_lo[rank])
        attention.attention_into(ov, qv, kv, vv, causal=causal, scale=scale, head_map=head_map)
        return ov
    if kv.shape[2] != qn or layout.group != 1:
        idx = torch.tensor(
            [(layout.q_lo[rank] + i) // layout.group - layout.kv_lo[rank] for i in range(qn)],
            device=qv.device,
        )
        kv, vv = kv.index_select(2, idx), vv.index_select(2, idx)
    attended = compute(qv, kv, vv)
    if attended.shape != (batch, total, qn, dim) or attended.dtype != qv.dtype:
        raise ValueError("Ulysses attention returned incompatible output")
    ov.copy_(attended)
    return ov


def _exchange_narrow(
    query: Tensor,
    key: Tensor,
    value: Tensor,
    handle,
    layout: Plan,
    rank: int,
    began,
    compute: Compute | None,
    causal: bool,
    scale: float | None,
    rope: RopeSpec | None,
    norm_q: Norm | None,
    norm_k: Norm | None,
    transport: str | None,
) -> Tensor:
    """The exchange over the int8 wire (the reference's `narrow=True`, ulysses.py:704-766): K's
    sums all-reduced and turned into the shift, Q/K/V narrowed into every peer's receive
    blocks, widened into the operands, attended, the output rows narrowed back to their owners
    and widened into [B, S_r, H, D]. Crosses over NCCL or the peer transport; at degree 1 the
    rows still take the wire's law, as the reference's exchange does."""
    batch, mine, heads, dim = (int(n) for n in query.shape)
    heads_kv = int(key.shape[2])
    device = query.device
    world, total, rows = layout.world, layout.total, layout.rows
    start = layout.start(rank)
    query = _first_law(query, rope, norm_q, start)
    key = _first_law(key, rope, norm_k, start)
    step = narrow_mod.NarrowStep(query, key, value, layout, rank)
    k_sum = torch.zeros(batch, heads_kv, dim, dtype=torch.float32, device=device)
    narrow_mod.key_sum_into(key, k_sum)
    with _Crossing(handle) as crossing:
        if world > 1:
            crossing.crossed = True
            dist.all_reduce(k_sum, op=dist.ReduceOp.SUM, group=handle)
        shift = step.shift(k_sum)
        qn, kvn = layout.q_n[rank], layout.kv_n[rank]
        i8, bf = torch.int8, torch.bfloat16
        moved = sum(
            step.first_block(p, "q") + 2 * step.first_block(p, "kv") + step.return_block(p)
            for p in range(world) if p != rank
        ) * (1 + 2 / dim)
        if (world > 1 and _transport(handle, transport) == "peer"
                and _peer_ready(handle, device)):
            pg = peer.group_for(handle, device)
            status = attention.status_word(device).data_ptr()
            most_q, most_kv = max(layout.q_n), max(layout.kv_n)
            sizes = {
                "nqc": total * batch * most_q * dim, "nqs": total * batch * most_q * 2,
                "nkc": total * batch * most_kv * dim, "nks": total * batch * most_kv * 2,
                "nvc": total * batch * most_kv * dim, "nvs": total * batch * most_kv * 2,
                "nlc": max(rows) * batch * heads * dim, "nls": max(rows) * batch * heads * 2,
            }
            with pg.lock:
                pg.ensure(sizes)
                seq = pg.next_seq()
                s = seq & 1

                def first(p: int, kind: str, n: int) -> tuple[int, int]:
                    at = start * batch * n * dim
                    return narrow_mod.scale_ptr(
                        pg.peer(p, s, f"n{kind}c"), pg.peer(p, s, f"n{kind}s"), at, dim
                    )

                r = range(world)
                step.pack_to(
                    shift,
                    [first(p, "q", layout.q_n[p]) for p in r],
                    [first(p, "k", layout.kv_n[p]) for p in r],
                    [first(p, "v", layout.kv_n[p]) for p in r],
                )
                pg.signal(peer.QKV, seq)
                pg.wait(peer.QKV, seq, status)
                q_op = step.operands(pg.view(s, "nqc", i8), pg.view(s, "nqs", bf), qn)
                k_op = step.operands(pg.view(s, "nkc", i8), pg.view(s, "nks", bf), kvn)
                v_op = step.operands(pg.view(s, "nvc", i8), pg.view(s, "nvs", bf), kvn)
                first_mark = _Clock.mark(query)
                attended = _attend_operands(q_op, k_op, v_op, layout, rank, compute, causal,
                                            scale) if qn else None
                last = _Clock.mark(query)
                if attended is not None:
                    # owner p's landing block from this rank: after the blocks of ranks below it
                    back = []
                    for p in r:
                        at = sum(rows[p] * batch * layout.q_n[u] * dim for u in range(rank))
                        back.append(narrow_mod.scale_ptr(
                            pg.peer(p, s, "nlc"), pg.peer(p, s, "nls"), at, dim))
                    step.return_to(attended, back)
                pg.signal(peer.OUT, seq)
                pg.wait(peer.OUT, seq, status)
                out = step.land(pg.view(s, "nlc", i8), pg.view(s, "nls", bf))
            _CLOCK.add((began, first_mark, last, _Clock.mark(query)), round(moved))
            return out

        # NCCL crossing (and degree 1: the send blocks are the receive blocks)
        def blocks(sizes: list[int]) -> tuple[Tensor, Tensor, list[tuple[int, int]]]:
            codes = torch.empty(sum(sizes), dtype=i8, device=device)
            scales = torch.empty(sum(sizes) // dim, dtype=bf, device=device)
            ptrs = [narrow_mod.scale_ptr(codes.data_ptr(), scales.data_ptr(), off, dim)
                    for off in _offsets(sizes)]
            return codes, scales, ptrs

        q_sizes = [step.first_block(p, "q") for p in range(world)]
        kv_sizes = [step.first_block(p, "kv") for p in range(world)]
        qs, ks, vs = blocks(q_sizes), blocks(kv_sizes), blocks(kv_sizes)
        step.pack_to(shift, qs[2], ks[2], vs[2])
        received = []
        for sent, sizes, n in ((qs, q_sizes, qn), (ks, kv_sizes, kvn), (vs, kv_sizes, kvn)):
            if world == 1:
                received.append((sent[0], sent[1]))
                continue
            arriving = [rr * batch * n * dim for rr in rows]
            codes = torch.empty(sum(arriving), dtype=i8, device=device)
            scales = torch.empty(sum(arriving) // dim, dtype=bf, device=device)
            dist.all_to_all_single(codes, sent[0], arriving, sizes, group=handle)
            dist.all_to_all_single(scales, sent[1], [a // dim for a in arriving],
                                   [z // dim for z in sizes], group=handle)
            received.append((codes, scales))
        q_op = step.operands(*received[0], qn)
        k_op = step.operands(*received[1], kvn)
        v_op = step.operands(*received[2], kvn)
        first_mark = _Clock.mark(query)
        attended = _attend_operands(q_op, k_op, v_op, layout, rank, compute, causal,
                                    scale) if qn else None
        last = _Clock.mark(query)
        back_sizes = [step.return_block(p) for p in range(world)]
        o_codes, o_scales, o_ptrs = blocks(back_sizes)
        if attended is not None:
            step.return_to(attended, o_ptrs)
        if world == 1:
            returned = (o_codes, o_scales)
        else:
            land_in = [step.landing_block(u) for u in range(world)]
            codes = torch.empty(sum(land_in), dtype=i8, device=device)
            scales = torch.empty(sum(land_in) // dim, dtype=bf, device=device)
            dist.all_to_all_single(codes, o_codes, land_in, back_sizes, group=handle)
            dist.all_to_all_single(scales, o_scales, [a // dim for a in land_in],
                                   [z // dim for z in back_sizes], group=handle)
            returned = (codes, scales)
        out = step.land(*returned)
    _CLOCK.add((began, first_mark, last, _Clock.mark(query)), round(moved))
    return out


def _exchange_fp8(
    query: Tensor,
    key: Tensor,
    value: Tensor,
    handle,
    layout: Plan,
    rank: int,
    began,
    causal: bool,
    scale: float | None,
    *,
    rope: RopeSpec | None = None,
    norm_q: Norm | None = None,
    norm_k: Norm | None = None,
    over_peer: bool = True,
    law: str = "block",
) -> Tensor:
    """The FP8 exchange: statistics all-reduced (block law: K sums and V channel absmax;
    per-head law: Q, K, V absmax per head), e4m3 codes and their scales written into every
    owner's receive buffers (peer transport; local at degree 1) or into per-destination send
    blocks crossing by NCCL all-to-all, the e4m3 attention, bf16 rows to their owners. RMSNorm /
    RoPE, when given, run inside the e4m3 first stage."""
    batch, mine, heads, dim = (int(n) for n in query.shape)
    device = query.device
    world, total, rows = layout.world, layout.total, layout.rows
    step = fp8_mod.Fp8Step(query, key, value, layout, rank, rope=rope, norm_q=norm_q,
                           norm_k=norm_k, law=law)
    scales = step.scales(handle if world > 1 else None)
    v_local = step.local_v_scale(scales.v_scale)
    sseq = step.sseq
    qn, kvn = layout.q_n[rank], layout.kv_n[rank]
    if world == 1:
        u8, f32 = torch.uint8, torch.float32
        q8 = torch.empty(total * batch * qn * dim, dtype=u8, device=device)
        k8 = torch.empty(total * batch * kvn * dim, dtype=u8, device=device)
        v8 = torch.empty(total * batch * kvn * dim, dtype=u8, device=device)
        qs = torch.zeros(batch * qn * sseq, dtype=f32, device=device)
        ks = torch.zeros(batch * kvn * sseq, dtype=f32, device=device)
        step.pack_to(scales, [q8.data_ptr()], [k8.data_ptr()], [v8.data_ptr()],
                     [qs.data_ptr()], [ks.data_ptr()])
        out = torch.empty((batch, mine, heads, dim), dtype=query.dtype, device=device)
        first = _Clock.mark(query)
        step.attend(q8, k8, v8, qs, ks, v_local, causal=causal, scale=scale, into=out)
        _CLOCK.add((began, first, _Clock.mark(query), _Clock.mark(query)), 0)
        return out
    if not over_peer:
        return _exchange_fp8_nccl(step, scales, v_local, handle, began, causal, scale)
    sizes = {
        "q8": total * batch * max(layout.q_n) * dim,
        "k8": total * batch * max(layout.kv_n) * dim,
        "v8": total * batch * max(layout.kv_n) * dim,
        "qs": batch * max(layout.q_n) * sseq * 4,
        "ks": batch * max(layout.kv_n) * sseq * 4,
        "land": batch * max(rows) * heads * dim * query.element_size(),
    }
    pg = peer.group_for(handle, device)
    status = attention.status_word(device).data_ptr()
    with pg.lock:
        pg.ensure(sizes)
        seq = pg.next_seq()
        s = seq & 1
        start = layout.start(rank)
        r = range(world)
        step.pack_to(
            scales,
            [pg.peer(p, s, "q8") + start * batch * layout.q_n[p] * dim for p in r],
            [pg.peer(p, s, "k8") + start * batch * layout.kv_n[p] * dim for p in r],
            [pg.peer(p, s, "v8") + start * batch * layout.kv_n[p] * dim for p in r],
            [pg.peer(p, s, "qs") + start * 4 for p in r],
            [pg.peer(p, s, "ks") + start * 4 for p in r],
        )
        pg.signal(peer.QKV, seq)
        pg.wait(peer.QKV, seq, status)
        first = _Clock.mark(query)
        if qn:
            scatter = _scatter(layout, rank, heads, dim, lambda p: pg.peer(p, s, "land"))
            step.attend(
                pg.view(s, "q8"), pg.view(s, "k8"), pg.view(s, "v8"),
                pg.view(s, "qs", torch.float32), pg.view(s, "ks", torch.float32), v_local,
                causal=causal, scale=scale, scatter=scatter,
            )
        last = _Clock.mark(query)
        pg.signal(peer.OUT, seq)
        pg.wait(peer.OUT, seq, status)
        out = torch.empty((batch, mine, heads, dim), dtype=query.dtype, device=device)
        land = pg.view(s, "land", query.dtype)[: batch * mine * heads * dim]
        out.copy_(land.view(batch, mine, heads, dim))
    _CLOCK.add((began, first, last, _Clock.mark(query)), 0)
    return out


def _exchange_fp8_nccl(step, scales, v_local: Tensor, handle, began, causal: bool,
                       scale: float | None) -> Tensor:
    """The FP8 exchange over NCCL: the e4m3 first stage writes per-destination send blocks
    (codes [rows][B][n_p][128]; block scales [B][n_p][rows]), four all-to-alls move codes and
    scales, the scales are laid out per head over the whole sequence, and the bf16 output returns
    as the bf16 path's does (all-to-all, then `land`)."""
    query = step.query
    lay, rank, device = step.layout, step.rank, query.device
    batch, mine, dim = step.batch, step.mine, step.dim
    world, total = lay.world, lay.total
    qn, kvn = lay.q_n[rank], lay.kv_n[rank]
    u8, f32 = torch.uint8, torch.float32
    q_sizes = [mine * batch * lay.q_n[p] * dim for p in range(world)]
    kv_sizes = [mine * batch * lay.kv_n[p] * dim for p in range(world)]
    qs_sizes = [batch * lay.q_n[p] * mine for p in range(world)]
    ks_sizes = [batch * lay.kv_n[p] * mine for p in range(world)]
    q_send = torch.empty(sum(q_sizes), dtype=u8, device=device)
    k_send = torch.empty(sum(kv_sizes), dtype=u8, device=device)
    v_send = torch.empty(sum(kv_sizes), dtype=u8, device=device)
    qs_send = torch.empty(sum(qs_sizes), dtype=f32, device=device)
    ks_send = torch.empty(sum(ks_sizes), dtype=f32, device=device)

    def at(buf: Tensor, sizes: Sequence[int]) -> list[int]:
        return [buf.data_ptr() + off * buf.element_size() for off in _offsets(sizes)]

    sseq = step.sseq
    # send blocks hold this rank's rows only: a head's scales are `mine` apart there
    step.pack_to(scales, at(q_send, q_sizes), at(k_send, kv_sizes), at(v_send, kv_sizes),
                 at(qs_send, qs_sizes), at(ks_send, ks_sizes), scale_rows=mine)
    rows = lay.rows
    q_in = [r * batch * qn * dim for r in rows]
    kv_in = [r * batch * kvn * dim for r in rows]
    q8 = torch.empty(sum(q_in), dtype=u8, device=device)
    k8 = torch.empty(sum(kv_in), dtype=u8, device=device)
    v8 = torch.empty(sum(kv_in), dtype=u8, device=device)
    qs_in = [batch * qn * r for r in rows]
    ks_in = [batch * kvn * r for r in rows]
    qs_got = torch.empty(sum(qs_in), dtype=f32, device=device)
    ks_got = torch.empty(sum(ks_in), dtype=f32, device=device)
    with _Crossing(handle) as crossing:
        crossing.crossed = True
        dist.all_to_all_single(q8, q_send, q_in, q_sizes, group=handle)
        dist.all_to_all_single(k8, k_send, kv_in, kv_sizes, group=handle)
        dist.all_to_all_single(v8, v_send, kv_in, kv_sizes, group=handle)
        dist.all_to_all_single(qs_got, qs_send, qs_in, qs_sizes, group=handle)
        dist.all_to_all_single(ks_got, ks_send, ks_in, ks_sizes, group=handle)

        def whole(got: Tensor, n: int, sizes: Sequence[int]) -> Tensor:
            # source blocks [B][n][rows_s] side by side -> [B][n][scale_seq], padding zero
            out = torch.zeros(batch, max(n, 1), sseq, dtype=f32, device=device)
            if n:
                parts = [t.view(batch, n, r) for t, r in zip(torch.split(got, sizes), rows,
                                                              strict=True)]
                out[:, :, :total] = torch.cat(parts, dim=2)
            return out.view(-1)

        qs, ks = whole(qs_got, qn, qs_in), whole(ks_got, kvn, ks_in)
        o_send = torch.empty(total * batch * qn * dim, dtype=query.dtype, device=device)
        first = _Clock.mark(query)
        if qn:
            ov = o_send.view(total, batch, qn, dim).permute(1, 0, 2, 3)
            step.attend(q8, k8, v8, qs, ks, v_local, causal=causal, scale=scale, into=ov)
        last = _Clock.mark(query)
        back = RankStep(query, step.key, step.value, lay, rank)
        returned = torch.empty(sum(back.back_sizes), dtype=query.dtype, device=device)
        dist.all_to_all_single(returned, o_send, back.back_sizes, back.back_in, group=handle)
        out = back.land(returned)
    moved = (sum(q_sizes) - q_sizes[rank] + 2 * (sum(kv_sizes) - kv_sizes[rank])
             + 4 * (sum(qs_sizes) - qs_sizes[rank] + sum(ks_sizes) - ks_sizes[rank])
             + query.element_size() * (sum(back.back_in) - back.back_in[rank]))
    _CLOCK.add((began, first, last, _Clock.mark(query)), moved)
    return out


def _scatter(layout: Plan, rank: int, heads: int, dim: int, landing) -> _lib.Scatter:
    """Where each output row goes: owner p's landing buffer [B][rows_p][H][D] at `landing(p)`."""
    sc = _lib.Scatter()
    sc.world = layout.world
    sc.head_offset = layout.q_lo[rank]
    acc = 0
    for p in range(layout.world):
        sc.row_start[p] = acc
        acc += layout.rows[p]
        sc.out[p] = landing(p)
        sc.strides[p][0] = heads * dim
        sc.strides[p][1] = dim
        sc.strides[p][2] = layout.rows[p] * heads * dim
    sc.row_start[layout.world] = acc
    return sc


def _abort(handle) -> None:
    """After crossing began, a failing rank ends its group so peers blocked in collectives raise
    (the reference's `abort_process_group`, src/cozy_runtime/internal/parallel/group.py:360-372,
    called at ulysses.py:754-758): the group's own abort where its backend has one (NCCL), else
    torch's process-group abort; a group without either (gloo) is left to its timeout, as in the
    reference."""
    abort = getattr(handle, "abort", None)
    try:
        if callable(abort):
            abort()
            return
        import torch.distributed.distributed_c10d as c10d

        whole = getattr(c10d, "_abort_process_group", None)
        if whole is not None:
            whole(handle)
    except Exception:  # noqa: BLE001 - the original error is what the caller sees
        pass


class _Crossing:
    """The part of an exchange after its first crossing began: an exception raised inside ends
    the group before it propagates, so peers waiting in a collective raise instead of waiting
    for this rank. `crossed` is set once the first crossing is under way."""

    def __init__(self, handle) -> None:
        self.handle = handle
        self.crossed = False

    def __enter__(self) -> _Crossing:
        return self

    def __exit__(self, kind, exc, tb) -> bool:
        if kind is not None and self.crossed:
            _abort(self.handle)
        return False
