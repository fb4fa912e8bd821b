"""The context-parallel types a parallel config carries to the attention backend.

Mirrors `src/cozy_runtime/internal/parallel/cp.py:25-77`: `CpComms` holds the group's
communication facts explicitly (the group, this process's rank in it, its device) so that a
backend never reads the default process group ambiently, and `GroupMesh` is the mesh a
Diffusers-style `ParallelConfig` exposes as `context_parallel_config._ulysses_mesh`: one Ulysses
axis of `size` ranks over that group, and a ring axis of degree 1 that refuses to hand out a
group. `attention_ulysses.group(config)` reads a config built from these.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


class ContextParallelUnavailable(ValueError):
    """This generation cannot be sharded as asked (the reference's `GroupRefusal` code
    `context_parallel_unavailable`)."""

    code = "context_parallel_unavailable"


@dataclass(slots=True)
class CpComms:
    """A group's communication facts, passed explicitly. `pg` is replaced when the group forms
    again; whatever holds these reads it per collective."""

    pg: object | None  # torch.distributed.ProcessGroup
    rank: int
    device: torch.device | str


class GroupMesh:
    """The mesh a parallel config's `setup` reads: the Ulysses axis of `size` ranks over
    `comms.pg`; the ring axis has degree 1 and refuses to name a group."""

    def __init__(self, comms: CpComms, size: int, local_rank: int, *,
                 axis: str = "ulysses") -> None:
        self._comms, self._size, self._local_rank, self._axis = comms, int(size), int(local_rank), axis

    def size(self) -> int:
        return self._size

    def get_local_rank(self) -> int:
        return self._local_rank

    def get_group(self):
        if self._axis == "ring":
            raise ContextParallelUnavailable(
                "ring attention is not served: the B200 path is Ulysses sequence parallelism "
                "only (ring_degree=1)")
        return self._comms.pg

    def __getitem__(self, key: str | tuple[str, ...]) -> GroupMesh:
        if isinstance(key, tuple) or key == "ulysses":
            return GroupMesh(self._comms, self._size, self._local_rank)
        if key == "ring":
            return GroupMesh(self._comms, 1, 0, axis="ring")
        raise KeyError(key)
