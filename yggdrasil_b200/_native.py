"""ctypes binding of libygg_b200.so (the C-ABI declared in include/ygg_b200.h).

The library is required: there is no CPU or PyTorch fallback for the step, and every entry point raises if the
library cannot be loaded.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libygg_b200.so"

EXPORTS = ("ygg_load", "ygg_info", "ygg_step", "ygg_step_debug", "ygg_score", "ygg_score_grouped_workspace",
           "ygg_score_grouped", "ygg_score_grouped_noalloc", "ygg_status", "ygg_selftest_wait", "ygg_free",
           "ygg_strerror", "ygg_version", "ygg_fload", "ygg_fstep", "ygg_fstep_stats", "ygg_fstatus", "ygg_ffree")

YGG_OK = 0
YGG_E_ARG, YGG_E_FORMAT, YGG_E_UNSUPPORTED, YGG_E_MISSING, YGG_E_CUDA, YGG_E_OOM, YGG_E_TOKEN, YGG_E_TIMEOUT, \
    YGG_E_DEVICE, YGG_E_CAPACITY = range(-1, -11, -1)


class YggInfo(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in (
        "n_layers", "d_state", "block_size", "vocab", "router_depth", "readout_rank", "layer_input_rank",
        "router_token_dim", "input_rank", "shift", "n_experts", "vocab_pad", "factored", "group_scales")] + [
        ("file_array_bytes", ctypes.c_int64), ("device_bytes", ctypes.c_int64), ("record_bytes", ctypes.c_int32),
        ("warps_per_block", ctypes.c_int32), ("slots_per_block", ctypes.c_int32)]


class YggError(RuntimeError):
    def __init__(self, code: int, what: str):
        self.code = code
        super().__init__(f"{what}: {strerror(code)} ({code})")


_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it is missing (build it with `python -m yggdrasil_b200.build`)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m yggdrasil_b200.build`")
        l = ctypes.CDLL(str(LIB_PATH))
        vp, i32, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
        l.ygg_load.argtypes = [vp, sz, i32, ctypes.POINTER(vp)]
        l.ygg_info.argtypes = [vp, ctypes.POINTER(YggInfo)]
        l.ygg_step.argtypes = [vp, i32, vp, vp, vp, vp, vp]
        l.ygg_step_debug.argtypes = [vp, i32, vp, vp, vp, vp, vp, vp, vp]
        l.ygg_score.argtypes = [vp, i32, i32, vp, vp, vp, vp]
        l.ygg_score_grouped_workspace.argtypes = [vp, i32]
        l.ygg_score_grouped_workspace.restype = sz
        l.ygg_score_grouped.argtypes = [vp, i32, i32, vp, vp, vp, i32, vp, sz, vp]
        l.ygg_score_grouped_noalloc.argtypes = [vp, i32, i32, vp, vp, vp, i32, vp]
        l.ygg_status.argtypes = [vp, vp, i32, ctypes.POINTER(ctypes.c_int)]
        l.ygg_selftest_wait.argtypes = [i32, ctypes.c_longlong, vp, ctypes.POINTER(ctypes.c_int)]
        l.ygg_free.argtypes = [vp]
        l.ygg_free.restype = None
        l.ygg_strerror.argtypes = [i32]
        l.ygg_strerror.restype = ctypes.c_char_p
        l.ygg_version.argtypes = []
        l.ygg_version.restype = ctypes.c_char_p
        for f in (l.ygg_load, l.ygg_info, l.ygg_step, l.ygg_step_debug, l.ygg_score, l.ygg_score_grouped,
                  l.ygg_score_grouped_noalloc, l.ygg_status, l.ygg_selftest_wait):
            f.restype = ctypes.c_int
        _lib = l
    return _lib


_float_bound = False


def flib() -> ctypes.CDLL:
    """The loaded library with the entry points of the fp32 float step (ygg_fload, ygg_fstep, ygg_fstatus,
    ygg_ffree) bound; raises if the library lacks them."""
    global _float_bound
    l = lib()
    if not _float_bound:
        vp, i32 = ctypes.c_void_p, ctypes.c_int
        l.ygg_fload.argtypes = [vp, ctypes.POINTER(vp), i32, ctypes.POINTER(vp)]
        l.ygg_fstep.argtypes = [vp, i32, vp, vp, vp, vp, vp, vp]
        l.ygg_fstep_stats.argtypes = [vp, i32, vp, vp, vp, vp, vp, vp, vp]
        l.ygg_fstatus.argtypes = [vp, vp, ctypes.POINTER(ctypes.c_int)]
        l.ygg_ffree.argtypes = [vp]
        l.ygg_ffree.restype = None
        for f in (l.ygg_fload, l.ygg_fstep, l.ygg_fstep_stats, l.ygg_fstatus):
            f.restype = ctypes.c_int
        _float_bound = True
    return l


def strerror(code: int) -> str:
    return lib().ygg_strerror(code).decode()


def check(code: int, what: str) -> None:
    if code != YGG_OK:
        raise YggError(code, what)
