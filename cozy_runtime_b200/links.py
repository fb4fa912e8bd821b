"""The measured links between a group's GPUs, and the route its Ulysses exchange takes.

Mirrors the reference's src/cozy_runtime/internal/parallel/links.py: nothing about a pair's speed
is inferred from a topology table; every ordered pair is measured by copying over it, and the
group's route follows from the pairs (`Links.exchange`, :123-132). There the measurement runs in
a child process once per boot and a second group of processes checks NCCL and the copy engines;
here it runs inside the group's own processes, on the very buffers, copy engines and side stream
the NVLink layer crosses with (`cozy_group_probe`), right after the formation check has proved
that those buffers carry the right bytes (`ulysses._form_check`, the reference's verified
copy). All ranks copy at once, each to a different peer, step by step: the pattern of the
exchange itself.

Route: the NVLink layer ("peer") where every ordered pair is direct — peer-mapped and copying at
NVLink class rates (`DIRECT_GBS`) — else NCCL, which the reference also takes where peer memory
works for NCCL but not for its own copies (`peer_route`, :108-110). NVML's active NVLink link
count per GPU is recorded beside the rates (read-only queries; -1 where NVML is absent).
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass

#: A pair copying below this (GB/s) is not NVLink class: PCIe 5.0 x16 moves about 50 GB/s a
#: direction, one NVLink 5 link 50 GB/s, a B200's eighteen 900 GB/s.
DIRECT_GBS = 100.0
#: Copies per measured pair (each of the layer's 8 MiB probe size: 64 MiB, ~0.1 ms on NVLink).
REPS = 8


@dataclass(frozen=True)
class Pair:
    """One ordered pair as measured: `src` copied to `dst` at `gbs` (0: not measured)."""

    src: int
    dst: int
    gbs: float
    peer: bool = True

    @property
    def direct(self) -> bool:
        return self.peer and self.gbs >= DIRECT_GBS


@dataclass(frozen=True)
class Links:
    pairs: tuple[Pair, ...]
    nvlink: tuple[int, ...] = ()
    reason: str = ""

    @property
    def all_peers(self) -> bool:
        return bool(self.pairs) and all(p.peer for p in self.pairs)

    @property
    def all_direct(self) -> bool:
        return bool(self.pairs) and all(p.direct for p in self.pairs)

    @property
    def exchange(self) -> str:
        """What carries the group's exchange: "peer" (the NVLink layer) or "nccl"."""
        return "peer" if self.all_direct and not self.reason else "nccl"

    def why(self) -> str:
        if self.reason:
            return self.reason
        slow = [p for p in self.pairs if not p.direct]
        if slow:
            p = slow[0]
            return (f"GPU pair {p.src}->{p.dst} copies at {p.gbs:.1f} GB/s, below the "
                    f"{DIRECT_GBS:.0f} GB/s of an NVLink-class link: the exchange stays on NCCL")
        return f"every pair direct (slowest {min(p.gbs for p in self.pairs):.0f} GB/s)"

    def summary(self) -> dict:
        rates = [p.gbs for p in self.pairs]
        return {
            "route": self.exchange,
            "pairs": len(self.pairs),
            "min_gbs": round(min(rates), 1) if rates else None,
            "max_gbs": round(max(rates), 1) if rates else None,
            "nvlink_links": list(self.nvlink),
            "why": self.why(),
        }


def decide(rates: Sequence[Sequence[float]], nvlink: Sequence[int] = (),
           peers: Sequence[Sequence[bool]] | None = None) -> Links:
    """Links from a measured rate matrix (`rates[src][dst]`, GB/s; the diagonal is ignored)."""
    world = len(rates)
    pairs = tuple(
        Pair(s, d, float(rates[s][d]), True if peers is None else bool(peers[s][d]))
        for s in range(world) for d in range(world) if s != d
    )
    return Links(pairs, tuple(int(n) for n in nvlink))


def nvlink_links(index: int, nvml=None) -> int:
    """Active NVLink links of the GPU with CUDA index `index` (NVML, read-only), -1 if unknown.
    `nvml`: the `pynvml` module or a stand-in with the same calls."""
    try:
        if nvml is None:
            import pynvml as nvml  # nvidia_ml_py
        nvml.nvmlInit()
        handle = nvml.nvmlDeviceGetHandleByIndex(index)
        active = 0
        for link in range(getattr(nvml, "NVML_NVLINK_MAX_LINKS", 18)):
            try:
                if nvml.nvmlDeviceGetNvLinkState(handle, link) == nvml.NVML_FEATURE_ENABLED:
                    active += 1
            except Exception:  # noqa: BLE001 - a link index past the device's own
                break
        return active
    except Exception:  # noqa: BLE001 - no NVML here: unknown
        return -1


def measure(layer_group, handle, device, reps: int = REPS) -> Links:
    """Every ordered pair of the group measured over the layer's copy engines (collective; no
    layer call may be in flight): in step s each rank copies to rank + s, all at once."""
    import torch
    import torch.distributed as dist

    world, rank = dist.get_world_size(handle), dist.get_rank(handle)
    mine = [0.0] * world
    reason = ""
    for step in range(1, world):
        dst = (rank + step) % world
        dist.barrier(group=handle)
        try:
            ms, nbytes = layer_group.probe(dst, reps)
            mine[dst] = nbytes / (ms * 1e-3) / 1e9 if ms > 0 else 0.0
        except RuntimeError as exc:  # keep stepping with the others; the route says why
            reason = reason or f"rank {rank} could not copy to rank {dst}: {exc}"
    dist.barrier(group=handle)
    index = device.index
    if index is None:
        index = torch.cuda.current_device() if device.type == "cuda" else -1
    links = nvlink_links(index) if index >= 0 else -1
    row = torch.tensor(mine + [float(links)], dtype=torch.float64, device=device)
    rows = [torch.empty_like(row) for _ in range(world)]
    dist.all_gather(rows, row, group=handle)
    # the failure flag travels too: every rank must decide alike
    failed = torch.tensor([1 if reason else 0], dtype=torch.int32, device=device)
    dist.all_reduce(failed, op=dist.ReduceOp.MAX, group=handle)
    rates = [r[:world].tolist() for r in rows]
    found = decide(rates, [int(r[world].item()) for r in rows])
    if failed.item():
        found = Links(found.pairs, found.nvlink, reason or "a rank could not copy to a peer")
    return found
