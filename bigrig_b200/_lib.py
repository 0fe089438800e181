"""ctypes binding of libbigrig_b200.so, the C-ABI library declared in include/bigrig_b200.h.

There is no fallback: if the library is missing or fails to load, every compute
entry point raises.  ``load()`` builds it first when the CUDA sources are newer
than the library and nvcc is available (never on the hot path: the first call
loads, later calls return the cached handle).
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

OK = 0
ERR_INVALID = -1
ERR_CUDA = -2
ERR_UNSUPPORTED = -3
ERR_WORKSPACE = -4

F32, F16, BF16 = 0, 1, 2
SOFTMAX_TOPK, TOPK_SOFTMAX = 0, 1

EXPORTS = (
    "bigrig_version", "bigrig_last_error", "bigrig_check_layout", "bigrig_moe_workspace_bytes",
    "bigrig_dequant", "bigrig_router_logits", "bigrig_router_topk", "bigrig_moe_permute",
    "bigrig_switch_glu", "bigrig_combine", "bigrig_moe_forward", "bigrig_workspace_errors",
    "bigrig_timing_enable", "bigrig_timing_read", "bigrig_launch_counts", "bigrig_kernel_name",
    "bigrig_set_path", "bigrig_get_path", "bigrig_moe_layer", "bigrig_switch_glu_noalloc", "bigrig_copy_regions",
    "bigrig_moe_layer_routed", "bigrig_test_grid_barrier", "bigrig_widen_expert",
    "bigrig_peer_buffer_bytes", "bigrig_peer_alloc", "bigrig_peer_free", "bigrig_peer_open",
    "bigrig_peer_close", "bigrig_peer_workspace_bytes", "bigrig_peer_layer", "bigrig_peer_errors",
)
NOALLOC_SCRATCH_BYTES = 4 << 20
KERNELS = {"router_logits": 0, "router_topk": 1, "permute": 2, "gate_up": 3, "down": 4,
           "combine": 5, "dequant": 6, "gemm_gate_up": 7, "gemm_down": 8, "route": 9,
           "down_combine": 10, "decode_layer": 11, "decode_split": 12, "peer_gather": 13,
           "peer_localize": 14, "peer_scatter": 15, "peer_combine": 16}
PATHS = {"auto": 0, "gemv": 1, "gemm": 2, "chain": 3, "tiled": 4, "split": 5}


class ExpertLayout(ctypes.Structure):
    """Mirror of ``bigrig_expert_layout`` (include/bigrig_b200.h)."""
    _fields_ = [
        ("hidden", ctypes.c_int32), ("inter", ctypes.c_int32), ("bits", ctypes.c_int32),
        ("group_size", ctypes.c_int32), ("scale_dtype", ctypes.c_int32),
        ("flags", ctypes.c_int32), ("bytes_per_expert", ctypes.c_int64),
        ("slot_stride", ctypes.c_int64), ("weight_off", ctypes.c_int64 * 3),
        ("scales_off", ctypes.c_int64 * 3), ("biases_off", ctypes.c_int64 * 3),
        ("bias_off", ctypes.c_int64 * 3),
    ]


PEER_MAX_RANKS = 8
PEER_HANDLE_BYTES = 64


class PeerGroup(ctypes.Structure):
    """Mirror of ``bigrig_peer_group`` (include/bigrig_b200.h)."""
    _fields_ = [
        ("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("tokens", ctypes.c_int32),
        ("hidden", ctypes.c_int32), ("top_k", ctypes.c_int32), ("wait_ms", ctypes.c_int32),
        ("base", ctypes.c_void_p * PEER_MAX_RANKS),
    ]


class LibraryError(RuntimeError):
    """The CUDA library could not be loaded; there is no CPU path to fall back on."""


_lock = threading.Lock()
_lib = None

_P = ctypes.c_void_p
_I = ctypes.c_int
_SIG = {
    "bigrig_version": (ctypes.c_char_p, []),
    "bigrig_last_error": (ctypes.c_char_p, []),
    "bigrig_check_layout": (_I, [ctypes.POINTER(ExpertLayout)]),
    "bigrig_moe_workspace_bytes": (ctypes.c_size_t, [_I, _I, _I, ctypes.POINTER(ExpertLayout)]),
    "bigrig_dequant": (_I, [_P, ctypes.POINTER(ExpertLayout), _I, _I, _P, _P]),
    "bigrig_router_logits": (_I, [_P, _P, _P, _P, _I, _I, _I, _P]),
    "bigrig_router_topk": (_I, [_P, _I, _I, _I, _I, _I, _I, _P, _P, _P]),
    "bigrig_moe_permute": (_I, [_P, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P]),
    "bigrig_switch_glu": (_I, [_P, _P, _I, _I, _I, _P, _P, ctypes.POINTER(ExpertLayout), _P, _P,
                              ctypes.c_size_t, _P]),
    "bigrig_combine": (_I, [_P, _P, _I, _I, _I, _P, _P]),
    "bigrig_moe_forward": (_I, [_P, _P, _I, _I, _I, _I, _I, _I, _P, _P,
                               ctypes.POINTER(ExpertLayout), _P, _P, _P, _P, ctypes.c_size_t, _P]),
    "bigrig_workspace_errors": (_I, [_P, _P, _P]),
    "bigrig_copy_regions": (_I, [_P, _P, _P, _I, _P]),
    "bigrig_timing_enable": (_I, [_I]),
    "bigrig_timing_read": (_I, [_I, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64)]),
    "bigrig_launch_counts": (_I, [ctypes.POINTER(ctypes.c_int64)]),
    "bigrig_kernel_name": (ctypes.c_char_p, [_I]),
    "bigrig_set_path": (_I, [_I, _I]),
    "bigrig_get_path": (_I, [_P, _P]),
    "bigrig_moe_layer": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _P, _P, ctypes.POINTER(ExpertLayout),
                              _P, _P, _P, _P, _P, ctypes.c_size_t, _P]),
    "bigrig_test_grid_barrier": (_I, [_I, ctypes.c_uint]),
    "bigrig_widen_expert": (_I, [_P, _P, ctypes.POINTER(ExpertLayout), _I, _P]),
    "bigrig_moe_layer_routed": (_I, [_P, _P, _P, _I, _I, _I, _P, _P, ctypes.POINTER(ExpertLayout),
                                     _P, _P, _P, ctypes.c_size_t, _P]),
    "bigrig_switch_glu_noalloc": (_I, [_P, _P, _I, _I, _I, _P, _P, ctypes.POINTER(ExpertLayout),
                                       _P, _P]),
    "bigrig_peer_buffer_bytes": (ctypes.c_size_t, [_I, _I, _I, _I]),
    "bigrig_peer_alloc": (_I, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), _P]),
    "bigrig_peer_free": (_I, [_P]),
    "bigrig_peer_open": (_I, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "bigrig_peer_close": (_I, [_P]),
    "bigrig_peer_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(PeerGroup), _I, _I,
                                                      ctypes.POINTER(ExpertLayout)]),
    "bigrig_peer_layer": (_I, [ctypes.POINTER(PeerGroup), _P, _P, _P, _I, _I, _I, _I, _I, _P, _P,
                               ctypes.POINTER(ExpertLayout), _P, _P, _P, ctypes.c_size_t, _P]),
    "bigrig_peer_errors": (_I, [ctypes.POINTER(PeerGroup), _P, _P]),
}


def library_path() -> str:
    return _build.LIB


def load(build_if_stale: bool = True):
    """The loaded library (ctypes.CDLL).  Raises LibraryError when it cannot be had."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if build_if_stale:
            try:
                if _build._stale(path, _build.sources() + _build.headers()):
                    _build.build()
            except Exception as e:  # noqa: BLE001 -- a prebuilt library may still be usable
                if not os.path.exists(path):
                    raise LibraryError(f"cannot build {path}: {e}") from e
        if not os.path.exists(path):
            raise LibraryError(f"{path} is missing: run `python -m bigrig_b200.build`")
        try:
            lib = ctypes.CDLL(path)
        except OSError as e:
            raise LibraryError(f"cannot load {path}: {e}") from e
        for name, (res, args) in _SIG.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    return load().bigrig_last_error().decode(errors="replace")


def check(rc: int, what: str = "") -> None:
    """Map a BIGRIG_ERR_* return code onto the reference's exception types."""
    if rc == OK:
        return
    msg = f"{what}: {last_error()}" if what else last_error()
    if rc in (ERR_INVALID, ERR_WORKSPACE):
        raise ValueError(msg)
    if rc == ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)


def launch_counts() -> dict:
    """{kernel name: launches issued by the library since it loaded}."""
    arr = (ctypes.c_int64 * len(KERNELS))()
    check(load().bigrig_launch_counts(arr), "launch_counts")
    return {name: int(arr[i]) for name, i in KERNELS.items()}


def timing_enable(kernels=()) -> None:
    """Time the named kernels' launches with CUDA events (empty: off)."""
    mask = 0
    for name in kernels:
        mask |= 1 << KERNELS[name]
    check(load().bigrig_timing_enable(mask), "timing_enable")


def timing_read(kernel: str) -> tuple:
    """(total ms, timed launches) of ``kernel`` since the last read."""
    ms = ctypes.c_double(0.0)
    n = ctypes.c_int64(0)
    check(load().bigrig_timing_read(KERNELS[kernel], ctypes.byref(ms), ctypes.byref(n)),
          "timing_read")
    return float(ms.value), int(n.value)


def get_path() -> tuple:
    """(mode, gemm_min_rows) as set_path last set them."""
    mode, rows = ctypes.c_int(0), ctypes.c_int(0)
    check(load().bigrig_get_path(ctypes.byref(mode), ctypes.byref(rows)), "get_path")
    return {v: k for k, v in PATHS.items()}[mode.value], int(rows.value)


def set_path(mode: str = "auto", gemm_min_rows: int = 8) -> str:
    """Choose the expert kernels: "auto" (GEMV for calls of at most 32 routed pairs, the
    tcgen05 grouped GEMM above that or once the mean rows per routed expert reaches
    ``gemm_min_rows``, one-token
    ``moe_layer`` calls as one persistent kernel), "gemv" or "gemm" (force one expert
    path), or "chain" ("auto" with one-token layers on the three-kernel chain).  Returns
    the previous mode."""
    rc = load().bigrig_set_path(PATHS[mode], int(gemm_min_rows))
    if rc < 0:
        check(rc, "set_path")
    return {v: k for k, v in PATHS.items()}[rc]
