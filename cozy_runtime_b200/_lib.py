"""ctypes binding of libcozy_ulysses.so (the C ABI declared in include/cozy_ulysses.h).

The library is built in-tree (`cozy_runtime_b200.build`). There is no fallback: if the library
is missing or fails to load, every entry point raises, so a GPU run can never silently take a
CPU or eager path.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, Structure, c_char_p, c_float, c_int, c_longlong, c_uint64, c_void_p
from pathlib import Path

MAX_PEERS = 16
LIBRARY = Path(__file__).resolve().parent / "libcozy_ulysses.so"

#: cudaError_t values the library returns itself
SUCCESS = 0
INVALID_VALUE = 1
NOT_SUPPORTED = 801

#: device status words (include/cozy_ulysses.h)
STATUS_NAMES = {0: "ok", 1: "on-chip wait timed out", 2: "wait on a peer timed out"}


class PackTensor(Structure):
    """`CozyPackTensor`."""

    _fields_ = [
        ("src", c_void_p),
        ("src_strides", c_longlong * 3),
        ("heads", c_int),
        ("normalize", c_int),
        ("norm_weight", c_void_p),
        ("norm_offset", c_float),
        ("norm_eps", c_float),
        ("rotate", c_int),
        ("dst", c_void_p * MAX_PEERS),
        ("head_lo", c_int * MAX_PEERS),
        ("head_n", c_int * MAX_PEERS),
    ]


class Rope(Structure):
    """`CozyRope`."""

    _fields_ = [
        ("cos", c_void_p),
        ("sin", c_void_p),
        ("stride_token", c_longlong),
        ("stride_channel", c_int),
        ("token0", c_longlong),
        ("rotary", c_int),
        ("interleaved", c_int),
    ]


class HeadMap(Structure):
    """`CozyHeadMap`."""

    _fields_ = [("group", c_int), ("q_base", c_int), ("kv_base", c_int)]


class Scatter(Structure):
    """`CozyScatter`."""

    _fields_ = [
        ("world", c_int),
        ("head_offset", c_int),
        ("row_start", c_int * (MAX_PEERS + 1)),
        ("out", c_void_p * MAX_PEERS),
        ("strides", (c_longlong * 3) * MAX_PEERS),
    ]


class PeerSlots(Structure):
    """`CozyPeerSlots`."""

    _fields_ = [("count", c_int), ("slot", c_void_p * MAX_PEERS)]


class Fp8Stats(Structure):
    """`CozyFp8Stats`."""

    _fields_ = [
        ("key", c_void_p),
        ("value", c_void_p),
        ("k_strides", c_longlong * 3),
        ("v_strides", c_longlong * 3),
        ("rows", c_int),
        ("batch", c_int),
        ("heads", c_int),
        ("head_dim", c_int),
        ("k_sum", c_void_p),
        ("v_amax", c_void_p),
        ("normalize", c_int),
        ("norm_weight", c_void_p),
        ("norm_offset", c_float),
        ("norm_eps", c_float),
        ("rotate", c_int),
        ("rope", Rope),
    ]


class Fp8Tensor(Structure):
    """`CozyFp8Tensor`."""

    _fields_ = [
        ("src", c_void_p),
        ("src_strides", c_longlong * 3),
        ("heads", c_int),
        ("hadamard", c_int),
        ("mean_sum", c_void_p),
        ("mean_inv_count", c_float),
        ("channel_scale", c_void_p),
        ("dst", c_void_p * MAX_PEERS),
        ("scale_dst", c_void_p * MAX_PEERS),
        ("scale_seq", c_longlong),
        ("head_lo", c_int * MAX_PEERS),
        ("head_n", c_int * MAX_PEERS),
        ("normalize", c_int),
        ("norm_weight", c_void_p),
        ("norm_offset", c_float),
        ("norm_eps", c_float),
        ("rotate", c_int),
        ("head_scale", c_void_p),
        ("head_amax", c_void_p),
    ]


class Fp8Pack(Structure):
    """`CozyFp8Pack`."""

    _fields_ = [
        ("t", Fp8Tensor * 3),
        ("world", c_int),
        ("rows", c_int),
        ("batch", c_int),
        ("head_dim", c_int),
        ("row0", c_int),
        ("head_turn", c_int),
        ("rope", Rope),
        ("per_head", c_int),
    ]


class NarrowTensor(Structure):
    """`CozyNarrowTensor`."""

    _fields_ = [
        ("src", c_void_p),
        ("src_strides", c_longlong * 3),
        ("heads", c_int),
        ("shift", c_void_p),
        ("dst", c_void_p * MAX_PEERS),
        ("scale_dst", c_void_p * MAX_PEERS),
        ("head_lo", c_int * MAX_PEERS),
        ("head_n", c_int * MAX_PEERS),
        ("row_lo", c_int * MAX_PEERS),
        ("row_n", c_int * MAX_PEERS),
    ]


class WidenSource(Structure):
    """`CozyWidenSource`."""

    _fields_ = [
        ("codes", c_void_p),
        ("scales", c_void_p),
        ("row_lo", c_int),
        ("rows", c_int),
        ("head_lo", c_int),
        ("head_n", c_int),
    ]


class LayerShape(Structure):
    """`CozyLayerShape`."""

    _fields_ = [
        ("world", c_int),
        ("rows", c_int * MAX_PEERS),
        ("batch", c_int),
        ("heads_q", c_int),
        ("heads_kv", c_int),
        ("head_dim", c_int),
        ("causal", c_int),
    ]


class LayerCall(Structure):
    """`CozyLayerCall`."""

    _fields_ = [
        ("shape", LayerShape),
        ("q", c_void_p),
        ("k", c_void_p),
        ("v", c_void_p),
        ("q_strides", c_longlong * 3),
        ("k_strides", c_longlong * 3),
        ("v_strides", c_longlong * 3),
        ("out", c_void_p),
        ("scale", c_float),
        ("rope", POINTER(Rope)),
        ("norm_q", c_int),
        ("norm_k", c_int),
        ("norm_q_weight", c_void_p),
        ("norm_k_weight", c_void_p),
        ("norm_offset", c_float * 2),
        ("norm_eps", c_float * 2),
        ("wait_limit_ns", c_longlong),
        ("status", c_void_p),
        ("gate", c_int),
        ("cross", c_int),
    ]


class CudaCallError(RuntimeError):
    """A library entry point returned a non-zero cudaError_t."""

    def __init__(self, entry: str, code: int, name: str) -> None:
        super().__init__(f"{entry} returned {code} ({name})")
        self.code = code


_LIB: ctypes.CDLL | None = None
_LOAD_ERROR: str = ""

#: entry point -> (argtypes, restype); the exported symbols `include/cozy_ulysses.h` declares
SIGNATURES = {
    "cozy_attention_fwd": (
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
         POINTER(c_longlong), POINTER(c_longlong), POINTER(c_longlong), POINTER(c_longlong),
         POINTER(HeadMap), POINTER(Scatter), c_int, c_float, c_void_p, c_uint64],
        c_int,
    ),
    "cozy_attention_split_plan": (
        [c_int, c_int, c_int, c_int, c_int, c_int, POINTER(c_longlong), POINTER(c_int)],
        c_int,
    ),
    "cozy_attention_split_plan_for": (
        [c_int, c_int, c_int, c_int, c_int, c_int, c_int, POINTER(c_longlong), POINTER(c_int)],
        c_int,
    ),
    "cozy_key_sum": (
        [c_void_p, POINTER(c_longlong), c_int, c_int, c_int, c_int, c_void_p, c_uint64], c_int,
    ),
    "cozy_narrow_shift": (
        [c_void_p, c_longlong, c_int, c_int, c_int, c_void_p, c_uint64], c_int,
    ),
    "cozy_narrow_pack": (
        [POINTER(NarrowTensor), c_int, c_int, c_int, c_int, c_int, c_uint64], c_int,
    ),
    "cozy_narrow_widen": (
        [POINTER(WidenSource), c_int, c_int, c_int, c_void_p, POINTER(c_longlong), c_uint64],
        c_int,
    ),
    "cozy_ulysses_pack": (
        [POINTER(PackTensor), c_int, c_int, c_int, c_int, c_int, POINTER(Rope), c_uint64],
        c_int,
    ),
    "cozy_ulysses_land": (
        [c_void_p, c_int, c_int, c_int, c_int, POINTER(c_int), POINTER(c_int), c_void_p,
         POINTER(c_longlong), c_uint64],
        c_int,
    ),
    "cozy_ipc_alloc": ([ctypes.c_ulonglong, POINTER(c_void_p), c_void_p], c_int),
    "cozy_ipc_open": ([c_void_p, POINTER(c_void_p)], c_int),
    "cozy_ipc_close": ([c_void_p], c_int),
    "cozy_ipc_free": ([c_void_p], c_int),
    "cozy_ipc_handle_bytes": ([], c_int),
    "cozy_peer_signal": ([POINTER(PeerSlots), c_longlong, c_uint64], c_int),
    "cozy_peer_wait": ([c_void_p, c_int, c_longlong, c_longlong, c_void_p, c_uint64], c_int),
    "cozy_rope_attention_fwd_noalloc": (
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
         POINTER(c_longlong), POINTER(c_longlong), POINTER(c_longlong), POINTER(c_longlong),
         POINTER(Rope), c_int, c_float, c_int, c_float, c_void_p, c_uint64],
        c_int,
    ),
    "cozy_head_norm_rope": (
        [c_void_p, c_void_p, c_int, c_int, c_int, c_int, POINTER(c_longlong),
         POINTER(c_longlong), POINTER(Rope), c_int, c_void_p, c_float, c_float, c_uint64],
        c_int,
    ),
    "cozy_fp8_stats": ([POINTER(Fp8Stats), c_uint64], c_int),
    "cozy_fp8_head_amax": ([POINTER(Fp8Pack), c_uint64], c_int),
    "cozy_fp8_pack": ([POINTER(Fp8Pack), c_uint64], c_int),
    "cozy_attention_fwd_fp8": (
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_longlong,
         POINTER(c_int), c_int, c_void_p,
         c_int, c_int, c_int, c_int, c_int, c_int,
         POINTER(c_longlong), POINTER(c_longlong), POINTER(c_longlong), POINTER(c_longlong),
         POINTER(HeadMap), POINTER(Scatter), c_int, c_float, c_void_p, c_uint64],
        c_int,
    ),
    "cozy_group_create": ([c_int, c_int, POINTER(c_void_p)], c_int),
    "cozy_group_destroy": ([c_void_p], c_int),
    "cozy_group_blob_bytes": ([], c_int),
    "cozy_group_needs": ([c_void_p, POINTER(LayerShape), POINTER(c_int)], c_int),
    "cozy_group_reserve": ([c_void_p, POINTER(LayerShape), c_void_p], c_int),
    "cozy_group_open": ([c_void_p, c_void_p], c_int),
    "cozy_group_make_local": ([c_void_p], c_int),
    "cozy_group_connect_local": ([POINTER(c_void_p), c_int], c_int),
    "cozy_group_flag_mode": ([c_void_p], c_int),
    "cozy_group_flag": ([c_void_p, c_int, c_int, POINTER(c_longlong)], c_int),
    "cozy_group_crossing": ([c_void_p, POINTER(c_float), POINTER(ctypes.c_ulonglong)], c_int),
    "cozy_group_probe": ([c_void_p, c_int, c_int, POINTER(c_float), POINTER(ctypes.c_ulonglong)],
                         c_int),
    "cozy_ulysses_layer_fwd": ([c_void_p, POINTER(LayerCall), c_uint64], c_int),
    "cozy_ulysses_layer_begin": ([c_void_p, POINTER(LayerCall), c_uint64], c_int),
    "cozy_ulysses_layer_attend": ([c_void_p, POINTER(LayerCall), c_uint64], c_int),
    "cozy_ulysses_layer_end": ([c_void_p, POINTER(LayerCall), c_uint64], c_int),
    "cozy_error_name": ([c_int], c_char_p),
    "cozy_abi_version": ([], c_int),
}


def load() -> ctypes.CDLL:
    """The loaded library; raises RuntimeError when it is missing or does not load."""
    global _LIB, _LOAD_ERROR
    if _LIB is not None:
        return _LIB
    if not LIBRARY.exists():
        raise RuntimeError(
            f"{LIBRARY.name} is not built: run `python -m cozy_runtime_b200.build` "
            "(the CUDA path has no fallback)"
        )
    try:
        lib = ctypes.CDLL(str(LIBRARY))
    except OSError as exc:
        _LOAD_ERROR = str(exc)
        raise RuntimeError(f"{LIBRARY.name} failed to load: {exc}") from exc
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _LIB = lib
    return lib


def error_name(code: int) -> str:
    return load().cozy_error_name(code).decode()


def check(entry: str, code: int) -> None:
    if code != SUCCESS:
        raise CudaCallError(entry, code, error_name(code))


def strides3(values) -> ctypes.Array:
    return (c_longlong * 3)(*(int(v) for v in values))
