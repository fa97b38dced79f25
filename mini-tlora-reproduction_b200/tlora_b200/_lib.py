"""ctypes binding of the native library ``libmlora.so`` (C ABI in include/mlora.h).

There is no fallback: if the library is missing or cannot be loaded, every
entry point raises.  Build it with ``python -c "import __graft_entry__ as g;
g.build()"`` (or ``python mini-tlora-reproduction_b200/tlora_b200/_build.py``).
"""

from __future__ import annotations

import ctypes
import os
import threading

import numpy as np

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libmlora.so")

# status codes (include/mlora.h)
OK = 0
ERR_INVALID_ARG = 1
ERR_UNSUPPORTED = 2
ERR_WORKSPACE = 3
ERR_CUDA = 4
ERR_DEVICE_FLAG = 5
ERR_TIMEOUT = 6

F32 = 0
BF16 = 1
F16 = 2
PLAN_RESIDENT = 1  # mlora_problem.flags

RANK_CHUNK = 64
TILE_ROWS = 256

STAGE_SHRINK = 1
STAGE_MAIN = 2
STAGE_NO_EXPAND = 4

BWD_DZ = 1
BWD_DX = 2
BWD_DA = 4
BWD_DB = 8
BWD_SGD_A = 16
BWD_SGD_B = 32
FUSED_SGD = 2  # mlora_problem.flags

IMPL_AUTO = 0
IMPL_SIMT = 1
IMPL_TC = 2
IMPL_TC_1SM = 3
IMPL_TC_2SM = 4
IMPL_TC_WIDE = 5

_c_int32_p = ctypes.POINTER(ctypes.c_int32)
_c_float_p = ctypes.POINTER(ctypes.c_float)


class Problem(ctypes.Structure):
    _fields_ = [
        ("rows", ctypes.c_int64),
        ("d_in", ctypes.c_int32),
        ("d_out", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("impl", ctypes.c_int32),
        ("max_ctas", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("err_word", ctypes.c_void_p),  # device int32 of this call's flags, or NULL (library-wide word)
        ("lr", ctypes.c_float),          # learning rate of the fused SGD step
    ]


class Routing(ctypes.Structure):
    _fields_ = [
        ("n_seg", ctypes.c_int32),
        ("seg_start", _c_int32_p),
        ("seg_adapter", _c_int32_p),
        ("n_adapters", ctypes.c_int32),
        ("rank", _c_int32_p),
        ("pack_off", _c_int32_p),
        ("scaling", _c_float_p),
        ("r_pack", ctypes.c_int32),
        ("out_rows", ctypes.c_void_p),  # device int32 [rows] or NULL
    ]


AR_MAX_RANKS = 8


class PeerAr(ctypes.Structure):
    """mlora_peer_ar: the peer buffers of the K-sharded forward's all-reduce."""
    _fields_ = [
        ("rank", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("n_tiles", ctypes.c_int32),
        ("d_out", ctypes.c_int32),
        ("recv", ctypes.c_void_p * AR_MAX_RANKS),
        ("arrive", ctypes.c_void_p * AR_MAX_RANKS),
        ("y", ctypes.c_void_p * AR_MAX_RANKS),
        ("done", ctypes.c_void_p * AR_MAX_RANKS),
        ("timeout_ns", ctypes.c_int64),
        ("err_word", ctypes.c_void_p),
    ]


MC_SLOTS = 64
MC_FLAG_WORDS = 4 * MC_SLOTS


class McAr(ctypes.Structure):
    """mlora_mc_ar: the multicast buffers of the K-sharded forward's all-reduce."""
    _fields_ = [
        ("rank", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("rows", ctypes.c_int64),
        ("d_out", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("y_mc", ctypes.c_void_p),
        ("flags_mc", ctypes.c_void_p),
        ("flags", ctypes.c_void_p),
        ("timeout_ns", ctypes.c_int64),
        ("err_word", ctypes.c_void_p),
    ]


class SgdItem(ctypes.Structure):
    _fields_ = [
        ("param", ctypes.c_void_p),
        ("grad", ctypes.c_void_p),
        ("rows", ctypes.c_int64),
        ("cols", ctypes.c_int64),
        ("ld_param", ctypes.c_int64),
        ("ld_grad", ctypes.c_int64),
    ]


# every symbol include/mlora.h declares, with its ctypes signature
_VP = ctypes.c_void_p
SIGNATURES = {
    "mlora_zsave_bytes": (ctypes.c_int, [ctypes.POINTER(Problem), ctypes.POINTER(Routing), ctypes.POINTER(ctypes.c_size_t)]),
    "mlora_workspace_bytes": (ctypes.c_int, [ctypes.POINTER(Problem), ctypes.POINTER(Routing), ctypes.POINTER(ctypes.c_size_t)]),
    "mlora_plan_upload": (ctypes.c_int, [ctypes.POINTER(Problem), ctypes.POINTER(Routing), _VP, ctypes.c_size_t, _VP]),
    "mlora_forward": (ctypes.c_int, [ctypes.POINTER(Problem), ctypes.POINTER(Routing), _VP, _VP, _VP, _VP, _VP,
                                     _VP, _VP, _VP, ctypes.c_size_t, _VP]),
    "mlora_forward_staged": (ctypes.c_int, [ctypes.POINTER(Problem), ctypes.POINTER(Routing), _VP, _VP, _VP, _VP,
                                            _VP, _VP, _VP, _VP, ctypes.c_size_t, ctypes.c_int32, ctypes.c_int32,
                                            ctypes.c_int32, _VP]),
    "mlora_num_tiles": (ctypes.c_int32, [ctypes.c_int64]),
    "mlora_ar_layout": (ctypes.c_int, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                       ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_size_t)]),
    "mlora_ar_reset": (ctypes.c_int, [ctypes.POINTER(PeerAr), _VP]),
    "mlora_forward_push": (ctypes.c_int, [ctypes.POINTER(Problem), ctypes.POINTER(Routing), _VP, _VP, _VP, _VP,
                                          _VP, _VP, _VP, ctypes.c_size_t, ctypes.c_int32, ctypes.c_int32,
                                          ctypes.c_int32, ctypes.POINTER(PeerAr), _VP]),
    "mlora_ar_finish": (ctypes.c_int, [ctypes.POINTER(PeerAr), ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                       ctypes.c_int32, _VP]),
    "mlora_ar_wait": (ctypes.c_int, [ctypes.POINTER(PeerAr), _VP]),
    "mlora_mc_allreduce": (ctypes.c_int, [ctypes.POINTER(McAr), ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, _VP]),
    "mlora_mc_wait": (ctypes.c_int, [ctypes.POINTER(McAr), ctypes.c_int32, _VP]),
    "mlora_peer_copy": (ctypes.c_int, [_VP, _VP, ctypes.c_size_t, _VP]),
    "mlora_peer_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]),
    "mlora_peer_free": (ctypes.c_int, [_VP]),
    "mlora_ipc_handle": (ctypes.c_int, [_VP, _VP]),
    "mlora_ipc_open": (ctypes.c_int, [_VP, ctypes.POINTER(ctypes.c_void_p)]),
    "mlora_ipc_close": (ctypes.c_int, [_VP]),
    "mlora_forward_noalloc": (ctypes.c_int, [ctypes.POINTER(Problem), ctypes.POINTER(Routing), _VP, _VP, _VP, _VP,
                                             _VP, _VP, _VP]),
    "mlora_backward": (ctypes.c_int, [ctypes.POINTER(Problem), ctypes.POINTER(Routing), _VP, _VP, _VP, _VP, _VP,
                                      _VP, _VP, _VP, _VP, _VP, ctypes.c_size_t, _VP]),
    "mlora_backward_staged": (ctypes.c_int, [ctypes.POINTER(Problem), ctypes.POINTER(Routing), _VP, _VP, _VP, _VP,
                                             _VP, _VP, _VP, _VP, _VP, _VP, _VP, ctypes.c_size_t, ctypes.c_int32,
                                             ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _VP]),
    "mlora_sgd": (ctypes.c_int, [ctypes.POINTER(SgdItem), ctypes.c_int32, ctypes.c_float, ctypes.c_int32, _VP]),
    "mlora_route_runs": (ctypes.c_int, [_VP, ctypes.c_int64, _VP, _VP, ctypes.c_int32, ctypes.c_int32, _VP, _VP]),
    "mlora_route_sort_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int32]),
    "mlora_route_sort": (ctypes.c_int, [_VP, ctypes.c_int64, _VP, _VP, ctypes.c_int32, _VP, _VP, _VP, _VP]),
    "mlora_gather_rows": (ctypes.c_int, [_VP, _VP, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, _VP, _VP]),
    "mlora_scatter_rows": (ctypes.c_int, [_VP, _VP, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, _VP, _VP]),
    "mlora_get_error": (ctypes.c_int, [_c_int32_p]),
    "mlora_clear_error": (ctypes.c_int, []),
    "mlora_launch_count": (ctypes.c_int64, []),
    "mlora_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "mlora_timing_enable": (ctypes.c_int, [ctypes.c_int32]),
    "mlora_timing_read": (ctypes.c_int, [ctypes.c_int32, ctypes.POINTER(ctypes.c_double),
                                         ctypes.POINTER(ctypes.c_int64)]),
    "mlora_timing_reset": (ctypes.c_int, []),
}

# kernel roles of mlora_timing_read
KERNEL_ROLES = {0: "fwd_main", 1: "dx_main", 2: "fwd_shrink", 3: "bwd_shrink", 4: "dadb_reduce"}

_lock = threading.Lock()
_lib = None


class MloraError(RuntimeError):
    """A native entry point returned a non-zero status."""

    def __init__(self, fn, status, text):
        super().__init__(f"{fn} failed with status {status}: {text}")
        self.status = status


def lib():
    """Load libmlora.so once; raise if it is missing (there is no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"native library {LIB_PATH} is missing; build it with __graft_entry__.build() "
                "(there is no CPU or PyTorch fallback)")
        # make sure torch's CUDA runtime/driver state is initialised in-process first
        h = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_LOCAL)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(h, name)
            f.restype = res
            f.argtypes = args
        _lib = h
        return _lib


def check(fn_name, status):
    if status == OK:
        return
    text = lib().mlora_status_string(status).decode()
    if status == ERR_INVALID_ARG:
        raise ValueError(f"{fn_name}: {text}")
    if status == ERR_UNSUPPORTED:
        raise NotImplementedError(f"{fn_name}: {text}")
    raise MloraError(fn_name, status, text)


def call(fn_name, *args):
    check(fn_name, getattr(lib(), fn_name)(*args))


def launch_count() -> int:
    return int(lib().mlora_launch_count())


def device_error() -> int:
    v = ctypes.c_int32(0)
    call("mlora_get_error", ctypes.byref(v))
    return int(v.value)


def clear_device_error() -> None:
    call("mlora_clear_error")


def timing_enable(on: bool) -> None:
    call("mlora_timing_enable", 1 if on else 0)


def timing_reset() -> None:
    call("mlora_timing_reset")


def timing_read() -> dict:
    """{role: (total device ms, launches)} of the tensor-core kernels since the
    last reset (waits for the recorded events)."""
    out = {}
    for k, name in KERNEL_ROLES.items():
        ms = ctypes.c_double(0.0)
        n = ctypes.c_int64(0)
        call("mlora_timing_read", k, ctypes.byref(ms), ctypes.byref(n))
        out[name] = (float(ms.value), int(n.value))
    return out


def i32_ptr(a: np.ndarray):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(_c_int32_p)


def f32_ptr(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_c_float_p)
