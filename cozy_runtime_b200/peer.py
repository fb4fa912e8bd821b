"""The in-kernel NVLink exchange of one process group: buffers every GPU of the node maps, and the
arrival flags the ranks signal each other through.

It replaces the reference's copy-engine exchange (`src/cozy_runtime/internal/parallel/
copy_engine.py:136-251`: a mapped receive buffer per GPU, NCCL all-reduce barriers around DMA
copies) with stores issued by the kernels themselves: the first stage writes each peer's heads
straight into that peer's receive buffer, the attention writes each output row straight into its
owner's landing buffer, and a 64-bit flag per (kind, source) in the receiver's memory says that a
call's writes have landed (`cozy_peer_signal` / `cozy_peer_wait`, bounded waits).

Receive and landing buffers are double-buffered by call parity. A rank writes call n into a
peer's set n % 2 only after it saw every rank's first-stage flag of call n, so every peer has
finished call n - 1, and with it every read of set n % 2 from call n - 2: no extra barrier.

Buffers are mapped when a group first runs a shape (all ranks together: they agree on sizes,
which follow from the agreed rows) and grow, never shrink, as shapes grow.
"""

from __future__ import annotations

import ctypes
import threading
import weakref

import torch
import torch.distributed as dist

from cozy_runtime_b200 import _lib

#: How long a rank waits for its peers' writes before it reports a peer timeout (status 2).
WAIT_LIMIT_NS = 10_000_000_000
#: flag kinds: a call's Q/K/V have landed; its output rows have landed
QKV, OUT = 0, 1


class _Ptr:
    """A CUDA array interface over raw device memory, to view it as a torch tensor."""

    def __init__(self, ptr: int, nbytes: int) -> None:
        self.__cuda_array_interface__ = {
            "shape": (nbytes,),
            "typestr": "|u1",
            "data": (ptr, False),
            "version": 3,
            "strides": None,
            "stream": None,
        }


def _tensor(ptr: int, nbytes: int, device: torch.device) -> torch.Tensor:
    """Bytes at `ptr` as a uint8 tensor (callers `.view()` the dtype they store)."""
    return torch.as_tensor(_Ptr(ptr, nbytes), device=device)


class _Alloc:
    """One IPC-shareable allocation of this rank."""

    def __init__(self, nbytes: int) -> None:
        lib = _lib.load()
        self.ptr = ctypes.c_void_p()
        self.handle = ctypes.create_string_buffer(lib.cozy_ipc_handle_bytes())
        _lib.check("cozy_ipc_alloc", lib.cozy_ipc_alloc(nbytes, ctypes.byref(self.ptr), self.handle))
        self.nbytes = nbytes

    def free(self) -> None:
        if self.ptr.value:
            _lib.load().cozy_ipc_free(self.ptr)
            self.ptr = ctypes.c_void_p()


class PeerGroup:
    """One rank's view of a group's mapped buffers."""

    def __init__(self, handle, device: torch.device) -> None:
        self.handle = handle
        self.device = device
        self.rank = dist.get_rank(handle)
        self.world = dist.get_world_size(handle)
        self.seq = 0
        self.lock = threading.Lock()
        self.sizes: dict[str, int] = {}  # bytes per named buffer (one of each per set)
        self.local: dict[tuple[int, str], _Alloc] = {}
        self.peer_ptrs: dict[tuple[int, int, str], int] = {}  # (peer, set, name) -> address
        self.opened: list[ctypes.c_void_p] = []
        self.views: dict[tuple[int, str], torch.Tensor] = {}
        self.flags = _Alloc(2 * self.world * 8)
        self.peer_flags = self._exchange_handles({("flags", 0): self.flags})

    # ------------------------------------------------------------------ mapping
    def _exchange_handles(self, allocs: dict) -> dict:
        """All-gather this rank's handles; open every peer's; return {(peer, key): address}."""
        mine = {key: bytes(a.handle.raw) for key, a in allocs.items()}
        gathered: list = [None] * self.world
        dist.all_gather_object(gathered, mine, group=self.handle)
        lib = _lib.load()
        out = {}
        for peer, handles in enumerate(gathered):
            for key, raw in handles.items():
                if peer == self.rank:
                    out[(peer, key)] = allocs[key].ptr.value
                    continue
                ptr = ctypes.c_void_p()
                buf = ctypes.create_string_buffer(raw, len(raw))
                _lib.check("cozy_ipc_open", lib.cozy_ipc_open(buf, ctypes.byref(ptr)))
                self.opened.append(ptr)
                out[(peer, key)] = ptr.value
        return out

    def ensure(self, sizes: dict[str, int]) -> None:
        """Map two sets of buffers named as `sizes` (bytes; at least that large) on every rank.
        Every rank calls with sizes that follow from the same agreed rows, so all decide alike;
        a set only grows."""
        if all(self.sizes.get(name, -1) >= n for name, n in sizes.items()):
            return
        grow = dict(self.sizes)
        for name, n in sizes.items():
            grow[name] = max(n, grow.get(name, 0))
        torch.cuda.synchronize(self.device)
        self._release_sets()
        dist.barrier(group=self.handle)
        allocs = {}
        for s in (0, 1):
            for name, n in sorted(grow.items()):
                allocs[(name, s)] = self.local[(s, name)] = _Alloc(max(256, -(-n // 256) * 256))
        ptrs = self._exchange_handles(allocs)
        for (peer, (name, s)), addr in ptrs.items():
            self.peer_ptrs[(peer, s, name)] = addr
        for (s, name), alloc in self.local.items():
            self.views[(s, name)] = _tensor(alloc.ptr.value, grow[name], self.device)
        self.sizes = grow

    def _release_sets(self) -> None:
        lib = _lib.load()
        keep = []
        flag_addrs = {addr for (_, key), addr in self.peer_flags.items()}
        for ptr in self.opened:
            if ptr.value in flag_addrs:
                keep.append(ptr)
            else:
                lib.cozy_ipc_close(ptr)
        self.opened = keep
        self.peer_ptrs.clear()
        self.views.clear()
        for alloc in self.local.values():
            alloc.free()
        self.local.clear()

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        self._release_sets()
        lib = _lib.load()
        for ptr in self.opened:
            lib.cozy_ipc_close(ptr)
        self.opened = []
        self.flags.free()

    # ------------------------------------------------------------------ calls
    def next_seq(self) -> int:
        self.seq += 1
        return self.seq

    def peer(self, peer: int, s: int, kind: str) -> int:
        return self.peer_ptrs[(peer, s, kind)]

    def view(self, s: int, kind: str, dtype: torch.dtype = torch.uint8) -> torch.Tensor:
        """This rank's buffer `kind` of set `s` as a flat tensor of `dtype`."""
        return self.views[(s, kind)].view(dtype)

    def signal(self, kind: int, seq: int) -> None:
        """Store `seq` into this rank's flag of `kind` in every rank's memory."""
        slots = _lib.PeerSlots()
        slots.count = self.world
        for p in range(self.world):
            slots.slot[p] = self.peer_flags[(p, ("flags", 0))] + (kind * self.world + self.rank) * 8
        code = _lib.load().cozy_peer_signal(
            ctypes.byref(slots), seq, torch.cuda.current_stream(self.device).cuda_stream
        )
        _lib.check("cozy_peer_signal", code)

    def wait(self, kind: int, seq: int, status_ptr: int) -> None:
        """The stream waits until every rank's flag of `kind` here reaches `seq`."""
        base = self.flags.ptr.value + kind * self.world * 8
        code = _lib.load().cozy_peer_wait(
            base, self.world, seq, WAIT_LIMIT_NS, status_ptr,
            torch.cuda.current_stream(self.device).cuda_stream,
        )
        _lib.check("cozy_peer_wait", code)


_GROUPS: weakref.WeakKeyDictionary = weakref.WeakKeyDictionary()
_GROUPS_LOCK = threading.Lock()


def group_for(handle, device: torch.device) -> PeerGroup:
    """This rank's mapped buffers for `handle` (formed on first use; collective)."""
    with _GROUPS_LOCK:
        found = _GROUPS.get(handle)
        if found is None:
            found = _GROUPS[handle] = PeerGroup(handle, device)
        return found


def close(handle) -> None:
    """Unmap and free the group's buffers (collective with the group's other ranks)."""
    with _GROUPS_LOCK:
        found = _GROUPS.pop(handle, None)
    if found is not None:
        found.close()
        dist.barrier(group=handle)


# ------------------------------------------------------------------ the C-side layer group
def layer_shape(rows, batch: int, heads: int, heads_kv: int, dim: int, causal: bool
                ) -> _lib.LayerShape:
    """`CozyLayerShape` of a layer: every rank's rows and the head layout."""
    shape = _lib.LayerShape()
    shape.world = len(rows)
    for r, n in enumerate(rows):
        shape.rows[r] = int(n)
    shape.batch, shape.heads_q, shape.heads_kv = batch, heads, heads_kv
    shape.head_dim, shape.causal = dim, int(causal)
    return shape


class LayerGroup:
    """One rank's `CozyGroup`: the buffers, flags and side stream the C layer entry
    (`cozy_ulysses_layer_fwd`) runs one node's Ulysses layer with. Formed on first use of a
    process group (collective) and grown when a larger layer comes, as `PeerGroup` is."""

    def __init__(self, handle, device: torch.device, *, rank: int | None = None,
                 world: int | None = None, local: bool = False) -> None:
        lib = _lib.load()
        self.handle, self.device, self.local = handle, device, local
        self.rank = dist.get_rank(handle) if rank is None else rank
        self.world = dist.get_world_size(handle) if world is None else world
        self.lock = threading.Lock()
        ptr = ctypes.c_void_p()
        with torch.cuda.device(device):
            _lib.check("cozy_group_create", lib.cozy_group_create(self.rank, self.world,
                                                                  ctypes.byref(ptr)))
        self.ptr = ptr
        if local:
            _lib.check("cozy_group_make_local", lib.cozy_group_make_local(self.ptr))

    def needs(self, shape: _lib.LayerShape) -> bool:
        grow = ctypes.c_int(0)
        _lib.check("cozy_group_needs", _lib.load().cozy_group_needs(self.ptr, ctypes.byref(shape),
                                                                    ctypes.byref(grow)))
        return bool(grow.value)

    def ensure(self, shape: _lib.LayerShape) -> None:
        """Grow the buffers for `shape` on every rank together (all ranks agree: the decision
        follows from the agreed rows)."""
        if not self.needs(shape):
            return
        lib = _lib.load()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.handle)  # no rank still writes into the buffers about to go
        blob = ctypes.create_string_buffer(lib.cozy_group_blob_bytes())
        with torch.cuda.device(self.device):
            _lib.check("cozy_group_reserve", lib.cozy_group_reserve(self.ptr, ctypes.byref(shape),
                                                                    blob))
        gathered: list = [None] * self.world
        dist.all_gather_object(gathered, bytes(blob.raw), group=self.handle)
        blobs = ctypes.create_string_buffer(b"".join(gathered), len(blob.raw) * self.world)
        with torch.cuda.device(self.device):
            _lib.check("cozy_group_open", lib.cozy_group_open(self.ptr, blobs))

    def flag_mode(self) -> str:
        mode = _lib.load().cozy_group_flag_mode(self.ptr)
        return {1: "stream write", 2: "host word copy"}.get(mode, str(mode))

    def flag(self, kind: int, src: int) -> int:
        """The last call number rank `src` published here (0: Q/K/V landed, 1: output rows)."""
        value = ctypes.c_longlong(0)
        _lib.check("cozy_group_flag", _lib.load().cozy_group_flag(self.ptr, kind, src,
                                                                  ctypes.byref(value)))
        return value.value

    def crossing(self) -> tuple[float, int] | None:
        """(ms, bytes) of the latest call's crossing on this rank (copies to the other ranks and
        their flags, on the side stream), or None while it is under way."""
        ms, nbytes = ctypes.c_float(0), ctypes.c_ulonglong(0)
        code = _lib.load().cozy_group_crossing(self.ptr, ctypes.byref(ms), ctypes.byref(nbytes))
        if code != _lib.SUCCESS:
            return None
        return ms.value, nbytes.value

    def probe(self, dst: int, reps: int = 8) -> tuple[float, int]:
        """(ms, bytes) of `reps` copies from this rank's staging buffer into `dst`'s receive
        buffer over the crossing's copy engines (`cozy_group_probe`; no call in flight)."""
        ms, nbytes = ctypes.c_float(0), ctypes.c_ulonglong(0)
        _lib.check("cozy_group_probe", _lib.load().cozy_group_probe(
            self.ptr, dst, reps, ctypes.byref(ms), ctypes.byref(nbytes)))
        return ms.value, nbytes.value

    def run(self, phase: str, call: _lib.LayerCall, stream: int) -> None:
        entry = f"cozy_ulysses_layer_{phase}"
        _lib.check(entry, getattr(_lib.load(), entry)(self.ptr, ctypes.byref(call), stream))

    def close(self) -> None:
        if self.ptr is not None and self.ptr.value:
            torch.cuda.synchronize(self.device)
            _lib.load().cozy_group_destroy(self.ptr)
        self.ptr = None


def local_layer_groups(world: int, device: torch.device, shape: _lib.LayerShape
                       ) -> list[LayerGroup]:
    """Every rank of a `world`-rank group in this process, on one GPU: buffers are plain
    allocations the ranks address directly (tests simulate the layer with them: every rank's
    begin, then every rank's attend, then every rank's end)."""
    groups = [LayerGroup(None, device, rank=r, world=world, local=True) for r in range(world)]
    lib = _lib.load()
    with torch.cuda.device(device):
        for g in groups:
            _lib.check("cozy_group_reserve", lib.cozy_group_reserve(g.ptr, ctypes.byref(shape),
                                                                    None))
        ptrs = (ctypes.c_void_p * world)(*(g.ptr.value for g in groups))
        _lib.check("cozy_group_connect_local", lib.cozy_group_connect_local(ptrs, world))
    return groups


_LAYER_GROUPS: weakref.WeakKeyDictionary = weakref.WeakKeyDictionary()


def layer_group_for(handle, device: torch.device) -> LayerGroup:
    """This rank's layer group for `handle` (formed on first use; collective)."""
    with _GROUPS_LOCK:
        found = _LAYER_GROUPS.get(handle)
        if found is None:
            found = _LAYER_GROUPS[handle] = LayerGroup(handle, device)
        return found


def close_layer(handle) -> None:
    """Release the layer group of `handle` (collective with the group's other ranks)."""
    with _GROUPS_LOCK:
        found = _LAYER_GROUPS.pop(handle, None)
    if found is not None:
        found.close()
        dist.barrier(group=handle)
