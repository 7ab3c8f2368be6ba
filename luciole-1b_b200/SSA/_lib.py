"""ctypes binding of libssa_b200.so (declared in include/ssa_b200.h).

The library is the only compute path: if it is missing or cannot be loaded, every call
raises. There is no CPU or PyTorch fallback.
"""

from __future__ import annotations

import contextlib
import ctypes
import os
import threading
from pathlib import Path

import torch

_PKG_ROOT = Path(__file__).resolve().parent.parent
LIB_PATH = Path(os.environ.get("SSA_B200_LIB", str(_PKG_ROOT / "libssa_b200.so")))

SSA_OK = 0
SSA_ERR_BAD_SHAPE = 1
SSA_ERR_BAD_STRIDE = 2
SSA_ERR_UNSUPPORTED = 3
SSA_ERR_WORKSPACE = 4
SSA_ERR_LAUNCH = 5
SSA_ERR_DEVICE_TIMEOUT = 6
SSA_ERR_NULL = 7
SSA_ERR_CUDA = 8

DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

EXPORTED_SYMBOLS = (
    "ssa_attn_fwd", "ssa_attn_fwd_workspace_size", "ssa_attn_bwd_preprocess", "ssa_attn_bwd",
    "ssa_attn_bwd_workspace_size", "ssa_attn_kernel_family", "ssa_device_status",
    "ssa_last_error", "ssa_version", "ssa_kernel_launch_count", "ssa_attn_bwd_noalloc",
    "ssa_selftest_device_timeout",
)


class SsaTensor(ctypes.Structure):
    _fields_ = [("ptr", ctypes.c_void_p), ("sB", ctypes.c_int64), ("sH", ctypes.c_int64),
                ("sN", ctypes.c_int64)]


class SsaProblem(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("B", ctypes.c_int32), ("Hq", ctypes.c_int32),
                ("Hkv", ctypes.c_int32), ("N", ctypes.c_int32), ("D", ctypes.c_int32),
                ("causal", ctypes.c_int32), ("softmax_scale", ctypes.c_float),
                ("ssa_n", ctypes.c_void_p), ("n_per_head", ctypes.c_int32),
                ("ssa_b", ctypes.c_void_p), ("cu_seqlens", ctypes.c_void_p),
                ("max_seqlen", ctypes.c_int32), ("cu_seqlens_padded", ctypes.c_void_p),
                ("deterministic", ctypes.c_int32), ("dropout_p", ctypes.c_float),
                ("dropout_seed", ctypes.c_void_p)]


def deterministic_default() -> bool:
    """The backward's dq accumulation mode when a call does not choose: SSA_DETERMINISTIC=1 in the
    environment selects the ordered (bit-reproducible) accumulation."""
    return os.environ.get("SSA_DETERMINISTIC", "0") not in ("", "0", "false", "False")


class SSAKernelError(RuntimeError):
    """A status code other than SSA_OK returned by libssa_b200.so."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"libssa_b200 status {code}: {msg}")
        self.code = code


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load libssa_b200.so once; raise if it is absent (build it with luciole-1b_b200/build.py)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} not found: build the CUDA extension first "
                "(python luciole-1b_b200/build.py, or __graft_entry__.build())")
        lib = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.POINTER(SsaProblem)
        T = SsaTensor
        vp, sz = ctypes.c_void_p, ctypes.c_size_t
        lib.ssa_attn_fwd.argtypes = [P, T, T, T, T, vp, vp, sz, vp]
        lib.ssa_attn_fwd.restype = ctypes.c_int
        lib.ssa_attn_fwd_workspace_size.argtypes = [P]
        lib.ssa_attn_fwd_workspace_size.restype = sz
        lib.ssa_attn_bwd_preprocess.argtypes = [P, T, T, vp, vp]
        lib.ssa_attn_bwd_preprocess.restype = ctypes.c_int
        lib.ssa_attn_bwd.argtypes = [P, T, T, T, T, T, vp, T, T, T, vp, vp, vp, sz, vp]
        lib.ssa_attn_bwd.restype = ctypes.c_int
        lib.ssa_attn_bwd_noalloc.argtypes = [P, T, T, T, T, T, vp, T, T, T, vp, vp, vp]
        lib.ssa_attn_bwd_noalloc.restype = ctypes.c_int
        lib.ssa_attn_bwd_workspace_size.argtypes = [P]
        lib.ssa_attn_bwd_workspace_size.restype = sz
        lib.ssa_attn_kernel_family.argtypes = [P]
        lib.ssa_attn_kernel_family.restype = ctypes.c_int
        lib.ssa_selftest_device_timeout.argtypes = [ctypes.c_uint64, vp]
        lib.ssa_selftest_device_timeout.restype = ctypes.c_int
        lib.ssa_device_status.argtypes = [vp]
        lib.ssa_device_status.restype = ctypes.c_int
        lib.ssa_last_error.argtypes = []
        lib.ssa_last_error.restype = ctypes.c_char_p
        lib.ssa_kernel_launch_count.argtypes = []
        lib.ssa_kernel_launch_count.restype = ctypes.c_uint64
        lib.ssa_version.argtypes = []
        lib.ssa_version.restype = ctypes.c_char_p
        _lib = lib
        return lib


def check(rc: int) -> None:
    if rc != SSA_OK:
        msg = load().ssa_last_error().decode(errors="replace")
        if rc in (SSA_ERR_BAD_SHAPE, SSA_ERR_UNSUPPORTED):
            raise ValueError(f"libssa_b200 status {rc}: {msg}")
        raise SSAKernelError(rc, msg)


def tensor_bhnd(t: torch.Tensor) -> SsaTensor:
    """[B, H, N, D] view (D stride must be 1)."""
    assert t.dim() == 4 and t.stride(3) == 1
    return SsaTensor(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))


def tensor_thd(t: torch.Tensor) -> SsaTensor:
    """[T, H, D] packed view, expressed as B = 1 (sB = 0), N = T."""
    assert t.dim() == 3 and t.stride(2) == 1
    return SsaTensor(t.data_ptr(), 0, t.stride(1), t.stride(0))


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_ptr(device: torch.device) -> ctypes.c_void_p:
    """The current CUDA stream of `device` as a cudaStream_t (read without building a Stream
    object: this runs on every attention call)."""
    if _raw_stream is not None:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        return ctypes.c_void_p(_raw_stream(idx))
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def device_guard(device: torch.device):
    """Makes `device` current for the duration of a call, and restores the caller's device after
    (the C entry points make the tensors' device current). A no-op when it already is."""
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


_family_cache: dict = {}
_ws_cache: dict = {}


def kernel_family_of(prob: "SsaProblem") -> int:
    """ssa_attn_kernel_family for a validated problem; the answer depends only on the dtype, the
    head dim and the sign of the softmax scale, so it is asked once per combination."""
    key = (prob.dtype, prob.D, prob.softmax_scale > 0)
    fam = _family_cache.get(key)
    if fam is None:
        fam = load().ssa_attn_kernel_family(ctypes.byref(prob))
        if fam >= 0:
            _family_cache[key] = fam
    return fam


def bwd_workspace_size(prob: "SsaProblem") -> int:
    """ssa_attn_bwd_workspace_size, asked once per problem shape (the size depends on the shape,
    dtype, causality, head dim, per-head n, packing, the deterministic flag, whether output dropout
    is on and the q-head-slice override SSA_BWD_HSPLIT, not on pointers)."""
    key = (prob.dtype, prob.B, prob.Hq, prob.Hkv, prob.N, prob.D, prob.causal,
           prob.softmax_scale > 0, prob.n_per_head, bool(prob.cu_seqlens), prob.max_seqlen,
           prob.deterministic, prob.dropout_p > 0, os.environ.get("SSA_BWD_HSPLIT"))
    ws = _ws_cache.get(key)
    if ws is None:
        ws = int(load().ssa_attn_bwd_workspace_size(ctypes.byref(prob)))
        if len(_ws_cache) > 4096:
            _ws_cache.clear()
        _ws_cache[key] = ws
    return ws


def launch_count() -> int:
    """Kernels launched by libssa_b200.so so far in this process."""
    return int(load().ssa_kernel_launch_count())


def version() -> str:
    return load().ssa_version().decode()
