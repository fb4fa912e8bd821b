"""The drop-in boundary: the reference's backend-call wrapper with the B200 kernel and exchange.

Mirrors `src/cozy_runtime/internal/attention_ulysses.py`: `Local` (:48-75) describes a head-local
kernel, `function(backend, local)` (:184) makes its Diffusers-style backend call (`BackendCall`,
:94-109), which without a parallel config calls the kernel and with one runs `exchange`
(:233-272) through the torch side `serve`d at import (:168). `CANDIDATE` is the selection row a
B200 (`tcgen05` family) attention table names for this kernel (`internal/attention.py:117-236`).

Relative to the reference, the B200 row serves what the benchmark configurations need under
Ulysses: causal attention (bottom-right) and grouped-query K/V heads, both of which the
reference's wrapper refuses (:259-262) but its exchange does not depend on.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass, field
from typing import Protocol

from torch import Tensor

from cozy_runtime_b200 import attention, ulysses


class Options(dict):
    """The keyword options every `Local.forward` takes (attention_ulysses.py:38-45)."""


@dataclass(frozen=True, slots=True)
class Local:
    """A forward-only kernel over [batch, sequence, heads, dim] (attention_ulysses.py:48-75)."""

    forward: Callable[..., Tensor]
    impl: Callable[[Tensor, Tensor, Tensor, dict], str]
    head_local: bool = True
    rows: int = 0
    refusal: Callable[[Tensor, Tensor, dict], str] | None = None
    instead: tuple[str, Local] | None = None
    narrow: bool = False
    #: options the kernel serves under Ulysses (the reference serves neither)
    ulysses_causal: bool = False
    ulysses_gqa: bool = False


class BackendCall(Protocol):
    def __call__(
        self,
        query: Tensor,
        key: Tensor,
        value: Tensor,
        attn_mask: Tensor | None = None,
        dropout_p: float = 0.0,
        is_causal: bool = False,
        scale: float | None = None,
        enable_gqa: bool = False,
        return_lse: bool = False,
        _parallel_config: object = None,
    ) -> Tensor: ...


#: The B200 kernel as a `Local`.
COZY_B200 = Local(
    forward=attention.forward,
    impl=attention.implementation,
    head_local=True,
    rows=256,
    refusal=attention.refusal,
    ulysses_causal=True,
    ulysses_gqa=True,
)


@dataclass(frozen=True)
class Candidate:
    """The selection row for this kernel (internal/attention.py:117 `Candidate`)."""

    name: str = "cozy-b200"
    backend: str = "cozy_b200"
    local: Local = COZY_B200
    families: frozenset = field(default_factory=lambda: frozenset({"tcgen05"}))
    dtypes: tuple = ("bfloat16",)
    head_dims: tuple = (64, 128)
    causal: bool = True
    gqa: bool = True
    masks: bool = False
    level: int = 16


CANDIDATE = Candidate()

_FUNCTIONS: dict[str, BackendCall] = {}
_GROUP: Callable[[object], object] | None = None


def serve(group_of: Callable[[object], object]) -> None:
    """Install how a parallel config names its process group (attention_ulysses.py:168)."""
    global _GROUP
    _GROUP = group_of


def group(config: object):
    """The Ulysses process group of a parallel config; ring is refused (ulysses.py:73-86)."""
    if _GROUP is not None:
        return _GROUP(config)
    cp = getattr(config, "context_parallel_config", config)
    if getattr(cp, "ring_degree", 1) != 1:
        raise ValueError("ring attention needs LSE merging; only Ulysses is served")
    mesh = getattr(cp, "_ulysses_mesh", None)
    handle = getattr(cp, "group", None) if mesh is None else mesh.get_group()
    if handle is None:
        raise ValueError("the Ulysses configuration is not initialized")
    return handle


def function(backend: str, local: Local = COZY_B200) -> BackendCall:
    """`backend`'s call, made once per process (attention_ulysses.py:184-190)."""
    found = _FUNCTIONS.get(backend)
    if found is None:
        found = _FUNCTIONS[backend] = _dispatch(backend, local)
    return found


def exchange(query, key, value, handle, compute, site: str = "", narrow=False) -> Tensor:
    """The reference's `attention_ulysses.exchange` (:363-376), served by the B200 exchange."""
    return ulysses.exchange(query, key, value, handle, compute, site, narrow)


def _dispatch(backend: str, local: Local) -> BackendCall:
    def attention_call(
        query: Tensor,
        key: Tensor,
        value: Tensor,
        attn_mask: Tensor | None = None,
        dropout_p: float = 0.0,
        is_causal: bool = False,
        scale: float | None = None,
        enable_gqa: bool = False,
        return_lse: bool = False,
        _parallel_config: object = None,
    ) -> Tensor:
        if return_lse:
            raise ValueError(f"{backend} does not return log-sum-exp")
        options = {
            "attn_mask": attn_mask,
            "dropout_p": dropout_p,
            "is_causal": is_causal,
            "scale": scale,
            "enable_gqa": enable_gqa,
        }
        if _parallel_config is None:
            return local.forward(query, key, value, **options)
        if not local.head_local:
            raise ValueError(f"{backend} reduces across heads and does not serve Ulysses")
        unequal = query.shape[2] != key.shape[2]
        if (
            attn_mask is not None
            or (is_causal and not local.ulysses_causal)
            or (unequal and not (local.ulysses_gqa and enable_gqa))
        ):
            raise ValueError(
                f"{backend} under Ulysses serves unmasked attention"
                + ("" if local.ulysses_causal else ", noncausal")
                + ("" if local.ulysses_gqa else ", with equal heads")
            )
        handle = group(_parallel_config)
        if local is COZY_B200:
            if dropout_p != 0.0:
                raise ValueError(f"{backend} is an inference kernel and does not support dropout")
            return ulysses.exchange(
                query, key, value, handle, None, causal=is_causal, scale=scale
            )
        return ulysses.exchange(
            query,
            key,
            value,
            handle,
            lambda q, k, v: local.forward(q, k, v, **options),
            narrow=local.narrow,
        )

    return attention_call
