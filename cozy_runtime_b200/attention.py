"""The B200 local attention kernel as a `Local`-style forward over [batch, seq, heads, dim].

`forward` is what the reference's exchange calls as `compute` on each rank (the reference's B200
row is `src/cozy_runtime/internal/attention_upstream.py:191-215` `cudnn`; its option checks are
:71-95 `_options`, `_heads`, `_output`). It runs `cozy_attention_fwd` from libcozy_ulysses.so;
there is no other implementation behind it.
"""

from __future__ import annotations

import ctypes
import math

import torch
from torch import Tensor

from cozy_runtime_b200 import _lib

_STATUS: dict[int, Tensor] = {}


def status_word(device: torch.device) -> Tensor:
    """This device's status word the kernels report timeouts through (int32, 0 = fine)."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    found = _STATUS.get(index)
    if found is None:
        found = _STATUS[index] = torch.zeros(1, dtype=torch.int32, device=device)
    return found


def check_status(device: torch.device) -> None:
    """Raise if a kernel on `device` reported a timed-out wait (synchronizes the device)."""
    word = int(status_word(device).item())
    if word:
        status_word(device).zero_()
        raise RuntimeError(f"attention kernel reported: {_lib.STATUS_NAMES.get(word, word)}")


class _Watch:
    """A watch on a device's status word that never synchronizes: after each call the word is
    copied into pinned host memory behind the call's work; the next call reads it once that copy
    has completed (an event query) and raises if a wait timed out."""

    def __init__(self) -> None:
        self.host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.event: torch.cuda.Event | None = None

    def after(self, word: Tensor, stream: torch.cuda.Stream) -> None:
        with torch.cuda.stream(stream):
            self.host.copy_(word, non_blocking=True)
        self.event = torch.cuda.Event()
        self.event.record(stream)

    def failed(self) -> int:
        if self.event is None or not self.event.query():
            return 0
        return int(self.host[0])


_WATCHES: dict[int, _Watch] = {}


def watch_after_call(device: torch.device) -> None:
    """Queue the copy of `device`'s status word behind the call just enqueued (no sync)."""
    if torch.cuda.is_current_stream_capturing():
        return
    index = device.index if device.index is not None else torch.cuda.current_device()
    watch = _WATCHES.get(index)
    if watch is None:
        watch = _WATCHES[index] = _Watch()
    watch.after(status_word(device), torch.cuda.current_stream(device))


def raise_if_failed(device: torch.device) -> None:
    """Raise if an earlier call on `device` reported a timed-out wait, as far as the watch has
    seen without synchronizing (the reference raises after any failure of an exchange,
    src/cozy_runtime/internal/parallel/ulysses.py:754-758). The word is cleared, so the error is
    raised once. While a stream is being captured into a CUDA graph nothing is checked (an
    event query is not allowed then); the watch resumes with the next eager call."""
    if torch.cuda.is_current_stream_capturing():
        return
    index = device.index if device.index is not None else torch.cuda.current_device()
    watch = _WATCHES.get(index)
    word = watch.failed() if watch is not None else 0
    if word:
        watch.host.zero_()
        watch.event = None
        status_word(device).zero_()
        raise RuntimeError(
            f"an earlier attention call on {device} reported: {_lib.STATUS_NAMES.get(word, word)}"
        )


def _strides(t: Tensor) -> ctypes.Array:
    """Element strides {seq, head, batch} of a [batch, seq, heads, dim] view."""
    if t.stride(3) != 1:
        raise ValueError("the head dimension must be contiguous")
    return _lib.strides3((t.stride(1), t.stride(2), t.stride(0)))


def refusal(query: Tensor, key: Tensor, options: dict) -> str:
    """Why this kernel does not serve a call, or "" (the reference's `Local.refusal`)."""
    if options.get("attn_mask") is not None:
        return "masks are not served"
    if options.get("dropout_p", 0.0) != 0.0:
        return "dropout is not served"
    if query.dtype != torch.bfloat16:
        return f"{query.dtype} is not served (bf16 only)"
    if query.shape[-1] not in (64, 128):
        return f"head dim {query.shape[-1]} is not served (64 or 128)"
    if not query.is_cuda:
        return "operands are not on a CUDA device"
    return ""


def attention_into(
    out: Tensor | None,
    query: Tensor,
    key: Tensor,
    value: Tensor,
    *,
    causal: bool = False,
    scale: float | None = None,
    head_map: tuple[int, int, int] | None = None,
    scatter: _lib.Scatter | None = None,
) -> None:
    """softmax(QKᵀ·scale)V of [B, Sq, Hq, D] queries over [B, Sk, Hkv, D] keys/values, into
    `out` ([B, Sq, Hq, D], any strides with D contiguous), on the current stream.
    `head_map` = (group, q_base, kv_base): query head h reads key head (h+q_base)//group-kv_base.
    `scatter`: rows go to their owners' outputs instead (`out` is then None)."""
    batch, sq, hq, dim = query.shape
    sk, hkv = key.shape[1], key.shape[2]
    scale = 1.0 / math.sqrt(dim) if scale is None else float(scale)
    mapping = None if head_map is None else ctypes.byref(_lib.HeadMap(*head_map))
    code = _lib.load().cozy_attention_fwd(
        query.data_ptr(), key.data_ptr(), value.data_ptr(),
        None if out is None else out.data_ptr(),
        batch, sq, sk, hq, hkv, dim,
        _strides(query), _strides(key), _strides(value),
        None if out is None else _strides(out),
        mapping, None if scatter is None else ctypes.byref(scatter), int(causal), scale,
        status_word(query.device).data_ptr(),
        torch.cuda.current_stream(query.device).cuda_stream,
    )
    _lib.check("cozy_attention_fwd", code)


def forward(
    query: Tensor,
    key: Tensor,
    value: Tensor,
    *,
    attn_mask: Tensor | None = None,
    dropout_p: float = 0.0,
    is_causal: bool = False,
    scale: float | None = None,
    enable_gqa: bool = False,
) -> Tensor:
    """Attention over [batch, seq, heads, dim] with the reference's local-kernel options
    (`attention_ulysses.Options`), causal aligned bottom-right; returns the query's shape and
    dtype on its device."""
    if dropout_p != 0.0:
        raise ValueError("cozy-b200 is an inference kernel and does not support dropout")
    if scale is not None and not math.isfinite(scale):
        raise ValueError("attention scale must be finite")
    if query.shape[2] != key.shape[2] and not enable_gqa:
        raise ValueError("unequal Q/KV head counts require enable_gqa=True")
    why = refusal(query, key, {"attn_mask": attn_mask, "dropout_p": dropout_p})
    if why:
        raise ValueError(f"cozy-b200 attention: {why}")
    raise_if_failed(query.device)
    out = torch.empty(query.shape, dtype=query.dtype, device=query.device)
    attention_into(out, query, key, value, causal=is_causal, scale=scale)
    watch_after_call(query.device)
    return out


def implementation(query: Tensor, key: Tensor, value: Tensor, options: dict) -> str:
    """The reference's `Local.impl`: the concrete implementation serving these operands."""
    return "cozy-b200-tcgen05"


def split_plan(
    batch: int, seq_q: int, seq_k: int, heads_q: int, head_dim: int, causal: bool
) -> tuple[int, int]:
    """(whole tiles, parts): how a call of this shape is scheduled on the current CUDA device
    (`cozy_attention_split_plan`). Past the first `whole` 256-row tiles, each tile runs as
    `parts` CTAs over shares of the keys, merged by the last to finish; parts 1 = no split."""
    import ctypes

    from cozy_runtime_b200 import _lib

    whole, parts = ctypes.c_longlong(0), ctypes.c_int(0)
    code = _lib.load().cozy_attention_split_plan(
        batch, seq_q, seq_k, heads_q, head_dim, int(causal), ctypes.byref(whole),
        ctypes.byref(parts),
    )
    _lib.check("cozy_attention_split_plan", code)
    return whole.value, parts.value
