"""ctypes binding of libbfa.so (declared in include/bfa.h).

This module only moves pointers, strides and sizes across the C ABI; all
compute happens in the library's CUDA kernels. It never falls back to a CPU
implementation: if the library is missing, every call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libbfa.so")
ABI_VERSION = 5

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
DEBUG_INJECT_STALL = 1
ERR_DEVICE_TIMEOUT = -6

EXPORTED = ("bfa_abi_version", "bfa_launch_count", "bfa_strerror", "bfa_last_error", "bfa_fwd",
            "bfa_fwd_workspace_bytes", "bfa_bwd_workspace_bytes", "bfa_bwd_delta", "bfa_bwd", "bfa_bwd_noalloc",
            "bfa_merge_partial")
ERR_SCRATCH_LIMIT = -7
NOALLOC_MAX_ROWS = 1 << 21
PHASE_DELTA, PHASE_DKDV, PHASE_DQ = 1, 2, 4

_TORCH_TO_BFA = {torch.float32: DTYPE_F32, torch.float16: DTYPE_F16,
                 torch.bfloat16: DTYPE_BF16}


class Problem(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("heads_q", ctypes.c_int32),
                ("heads_kv", ctypes.c_int32), ("seqlen_q", ctypes.c_int32),
                ("seqlen_k", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("dtype", ctypes.c_int32), ("causal", ctypes.c_int32),
                ("sliding_window", ctypes.c_int32), ("scale", ctypes.c_float),
                ("soft_cap", ctypes.c_float), ("alibi_slopes", ctypes.c_void_p),
                ("q_pos_offset", ctypes.c_int64), ("k_pos_offset", ctypes.c_int64),
                ("doc_start", ctypes.c_void_p), ("doc_end", ctypes.c_void_p),
                ("block_mask", ctypes.c_void_p), ("block_mask_stride", ctypes.c_int64 * 3)]


class Tensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("stride", ctypes.c_int64 * 4)]


class FwdArgs(ctypes.Structure):
    _fields_ = [("q", Tensor), ("k", Tensor), ("v", Tensor), ("o", Tensor),
                ("lse", ctypes.c_void_p), ("status", ctypes.c_void_p),
                ("wait_timeout_ns", ctypes.c_int64), ("debug_flags", ctypes.c_uint32),
                ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
                ("accumulate", ctypes.c_uint32)]


class BwdArgs(ctypes.Structure):
    _fields_ = [("q", Tensor), ("k", Tensor), ("v", Tensor), ("o", Tensor),
                ("dout", Tensor), ("lse", ctypes.c_void_p), ("dq", Tensor),
                ("dk", Tensor), ("dv", Tensor), ("status", ctypes.c_void_p),
                ("wait_timeout_ns", ctypes.c_int64), ("debug_flags", ctypes.c_uint32),
                ("phases", ctypes.c_uint32), ("accumulate", ctypes.c_uint32)]


_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load libbfa.so once and declare its signatures."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing; build it with `python {HERE}/build.py` "
                "(there is no CPU fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        lib.bfa_abi_version.restype = ctypes.c_int
        lib.bfa_abi_version.argtypes = []
        lib.bfa_launch_count.restype = ctypes.c_uint64
        lib.bfa_launch_count.argtypes = []
        lib.bfa_strerror.restype = ctypes.c_char_p
        lib.bfa_strerror.argtypes = [ctypes.c_int]
        lib.bfa_last_error.restype = ctypes.c_char_p
        lib.bfa_last_error.argtypes = []
        lib.bfa_fwd.restype = ctypes.c_int
        lib.bfa_fwd.argtypes = [ctypes.POINTER(Problem), ctypes.POINTER(FwdArgs), ctypes.c_void_p]
        lib.bfa_fwd_workspace_bytes.restype = ctypes.c_size_t
        lib.bfa_fwd_workspace_bytes.argtypes = [ctypes.POINTER(Problem)]
        lib.bfa_bwd_workspace_bytes.restype = ctypes.c_size_t
        lib.bfa_bwd_workspace_bytes.argtypes = [ctypes.POINTER(Problem)]
        lib.bfa_bwd_delta.restype = ctypes.c_int
        lib.bfa_bwd_delta.argtypes = [ctypes.POINTER(Problem), ctypes.POINTER(BwdArgs),
                                      ctypes.c_void_p, ctypes.c_void_p]
        lib.bfa_bwd.restype = ctypes.c_int
        lib.bfa_bwd.argtypes = [ctypes.POINTER(Problem), ctypes.POINTER(BwdArgs),
                                ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
        lib.bfa_bwd_noalloc.restype = ctypes.c_int
        lib.bfa_bwd_noalloc.argtypes = [ctypes.POINTER(Problem), ctypes.POINTER(BwdArgs),
                                        ctypes.c_void_p]
        lib.bfa_merge_partial.restype = ctypes.c_int
        lib.bfa_merge_partial.argtypes = [ctypes.c_int32] * 4 + [
            Tensor, ctypes.c_int32, ctypes.c_void_p, Tensor, ctypes.c_int32, ctypes.c_void_p,
            ctypes.c_void_p]
        ver = lib.bfa_abi_version()
        if ver != ABI_VERSION:
            raise RuntimeError(f"libbfa ABI version {ver}, expected {ABI_VERSION}")
        _lib = lib
    return _lib


ERR_CUDA = -5


def check(rc: int) -> None:
    if rc != 0:
        lib = load()
        msg = lib.bfa_strerror(rc).decode()
        if rc == ERR_CUDA:
            detail = lib.bfa_last_error().decode()
            if detail:
                msg = f"{msg} ({detail})"
        raise RuntimeError(msg)


def bfa_dtype(dt: torch.dtype) -> int:
    if dt not in _TORCH_TO_BFA:
        raise RuntimeError(f"unsupported dtype {dt} (need float32, float16 or bfloat16)")
    return _TORCH_TO_BFA[dt]


def tensor(t: torch.Tensor | None) -> Tensor:
    out = Tensor()
    if t is None:
        return out
    out.data = t.data_ptr()
    for i, s in enumerate(t.stride()):
        out.stride[i] = s
    return out


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_status = {}


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 status word that bounded device waits report into."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    if key not in _status:
        _status[key] = torch.zeros(1, dtype=torch.int32, device=device)
    return _status[key]


def read_and_clear_status(device: torch.device) -> int:
    """Synchronise the device, return its status word and reset it to 0."""
    w = status_word(device)
    val = int(w.item())
    w.zero_()
    return val
