"""SSA flash-attention forward / backward wrappers over libssa_b200.so.

Drop-in for the reference module ``SSA.ssa_triton_kernel``
(training/train/train_ssa_triton/SSA/ssa_triton_kernel.py): same function names, argument
meaning and return values, computed by hand-written sm_100a CUDA (tcgen05/TMA for bf16/fp16
with D in {32, 64, 128}; fp32-arithmetic CUDA-core kernels for fp32 and D = 16). The
module name is kept so ``from SSA.ssa_triton_kernel import ...`` keeps working; nothing here
uses Triton.

Differences from the reference, all supersets:
  * ``ssa_n`` may be 0-d (reference) or a per-head ``[Hq]`` vector; ``dn`` takes its shape.
  * N need not be a multiple of 128 (reference asserts it in backward, :852-857) and D may be
    16 / 32 / 64 / 128 (reference: any power of two its Triton build handles).
  * packed documents: ``ssa_flash_attn_varlen_forward/backward`` (reference asserts packed
    sequences off, ssa_triton_attention.py:154-156).
  * ``m`` is the same base-2 normaliser M = log2(sum_j exp2(t_j log2 e)) (:248-255).
  * output dropout fused into the kernels (``dropout_p`` / ``dropout_seed``): the reference applies
    ``nn.Dropout`` to the kernel's output in its module (ssa_triton_attention.py:186-193); here the
    forward's epilogue drops and rescales, and the backward's delta pass masks dout.
"""

from __future__ import annotations

import ctypes
import math
from typing import Optional, Tuple

import torch

from . import _lib

__all__ = [
    "ssa_flash_attn_forward", "ssa_flash_attn_backward", "ssa_flash_attn_varlen_forward",
    "ssa_flash_attn_varlen_backward", "warmup_ssa_triton_kernels", "kernel_family",
    "check_device_status", "make_dropout_seed",
]


def _as_f32(x, device) -> torch.Tensor:
    if (isinstance(x, torch.Tensor) and x.dtype == torch.float32 and x.device == device
            and x.is_contiguous()):
        return x.detach()
    return torch.as_tensor(x).detach().to(device=device, dtype=torch.float32).contiguous()


def _params(ssa_n: torch.Tensor, ssa_b: torch.Tensor, hq: int, device) -> Tuple[torch.Tensor, torch.Tensor, int]:
    n = _as_f32(ssa_n, device)
    b = _as_f32(ssa_b, device)
    if b.numel() != 1:
        raise ValueError(f"ssa_b must be a scalar tensor, got shape {tuple(b.shape)}")
    if n.numel() == 1:
        per_head = 0
    elif n.numel() == hq:
        per_head = 1
    else:
        raise ValueError(f"ssa_n must be a scalar or have Hq={hq} elements, got {tuple(n.shape)}")
    return n, b, per_head


def _problem(q: torch.Tensor, hkv: int, softmax_scale: float, n: torch.Tensor, b: torch.Tensor,
             per_head: int, causal: bool, B: int, N: int,
             cu_seqlens: Optional[torch.Tensor] = None, max_seqlen: int = 0,
             cu_seqlens_padded: Optional[torch.Tensor] = None,
             deterministic: bool = False, dropout_p: float = 0.0,
             dropout_seed: Optional[torch.Tensor] = None) -> _lib.SsaProblem:
    if q.dtype not in _lib.DTYPE_CODES:
        raise ValueError(f"unsupported dtype {q.dtype}")
    hq, d = q.shape[1], q.shape[-1]
    return _lib.SsaProblem(
        _lib.DTYPE_CODES[q.dtype], B, hq, hkv, N, d, 1 if causal else 0, float(softmax_scale),
        n.data_ptr(), per_head, b.data_ptr(),
        cu_seqlens.data_ptr() if cu_seqlens is not None else None, int(max_seqlen),
        cu_seqlens_padded.data_ptr() if cu_seqlens_padded is not None else None,
        1 if deterministic else 0, float(dropout_p),
        dropout_seed.data_ptr() if dropout_seed is not None else None)


def make_dropout_seed(device) -> torch.Tensor:
    """A fresh dropout seed: two random 64-bit values (the Philox key and counter offset) drawn on
    the device from torch's CUDA generator, so the draw needs no host synchronisation, is
    replayed with fresh values under CUDA-graph capture, and follows torch.manual_seed and
    Megatron's CUDA RNG tracker (draw it inside the tracker's fork)."""
    return torch.randint(-(2 ** 63), 2 ** 63 - 1, (2,), dtype=torch.int64,
                         device=torch.device(device))


def _dropout_args(dropout_p, dropout_seed, device):
    """Validated (p, seed) for the problem block: p = 0 turns dropout off."""
    p = float(dropout_p or 0.0)
    if p == 0.0:
        return 0.0, None
    if not 0.0 < p < 1.0:
        raise ValueError(f"dropout_p must be in [0, 1), got {p}")
    if (dropout_seed is None or not isinstance(dropout_seed, torch.Tensor)
            or dropout_seed.dtype != torch.int64 or dropout_seed.numel() < 2
            or dropout_seed.device != device or not dropout_seed.is_contiguous()):
        raise ValueError("dropout_p > 0 needs dropout_seed: a contiguous int64 tensor of 2 values "
                         "on the inputs' device (make_dropout_seed)")
    return p, dropout_seed


def _tma_ok(t: torch.Tensor) -> bool:
    if t.stride(-1) != 1 or t.data_ptr() % 16:
        return False
    return all((s * t.element_size()) % 16 == 0 for s, n in zip(t.stride()[:-1], t.shape[:-1]) if n > 1)


def _prep(t: torch.Tensor, family: int) -> torch.Tensor:
    """Unit stride on D always; a 16-byte-aligned base and B/H/N strides for the TMA
    (tensor-core) family. Anything else is copied into fresh storage (``contiguous()`` would
    keep a misaligned base of an already-contiguous view)."""
    if t.stride(-1) != 1 or (family == 1 and not _tma_ok(t)):
        return t.clone(memory_format=torch.contiguous_format)
    return t


def _check_qkv(q, k, v):
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("q, k, v must be [B, H, N, D]")
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise ValueError("q, k, v must be CUDA tensors (there is no CPU path)")
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError(f"dtype mismatch q={q.dtype} k={k.dtype} v={v.dtype}")
    B, Hq, N, D = q.shape
    if k.shape != v.shape or k.shape[0] != B or k.shape[2] != N or k.shape[3] != D:
        raise ValueError(f"shape mismatch q={tuple(q.shape)} k={tuple(k.shape)} v={tuple(v.shape)}")
    Hkv = k.shape[1]
    if Hq % Hkv != 0:
        raise ValueError(f"Hq={Hq} must be divisible by Hkv={Hkv}")
    return B, Hq, Hkv, N, D


def check_device_status(device=None) -> None:
    """Raise ``SSAKernelError`` (code ``SSA_ERR_DEVICE_TIMEOUT``) if a bounded device-side wait of
    the sm_100a kernels expired on ``device`` (default: the current CUDA device) since the last
    check. Reads and clears the device status word, synchronising the current stream.

    Every wait inside the tensor-core kernels gives up after about a second instead of hanging
    the GPU. From then on, until this check clears the status, those kernels skip their work and
    write NaN into every output (out, m, dq, dk, dv, dn, db), so a training loop that never calls
    this still sees the failure as NaN (the reference's DDP ``check_for_nan_in_grad`` trips on
    it). Call it where a host synchronisation is acceptable, e.g. once per optimizer step.
    """
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    lib = _lib.load()
    rc = lib.ssa_device_status(_lib.stream_ptr(dev))
    _lib.check(rc)


def kernel_family(q: torch.Tensor, softmax_scale: float = 1.0) -> int:
    """0 = generic fp32-arithmetic kernels, 1 = sm_100a tcgen05/TMA kernels."""
    D = q.shape[-1]
    n = torch.zeros(1, device=q.device)
    prob = _lib.SsaProblem(_lib.DTYPE_CODES[q.dtype], 1, 1, 1, 1, D, 1, float(softmax_scale),
                           n.data_ptr(), 0, n.data_ptr(), None, 0)
    return _lib.load().ssa_attn_kernel_family(ctypes.byref(prob))


def ssa_flash_attn_forward(q, k, v, softmax_scale, ssa_n, ssa_b, causal=True, dropout_p=0.0,
                           dropout_seed=None):
    """Forward (reference ssa_triton_kernel.py:732-792).

    q [B, Hq, N, D], k/v [B, Hkv, N, D] (any strides with a unit D stride; other layouts
    are copied). Returns (out [B, Hq, N, D] with q's dtype and layout, m [B, Hq, N] fp32).

    dropout_p > 0 (with dropout_seed from :func:`make_dropout_seed`) returns the output with
    dropout applied (elements zeroed with probability p, survivors scaled by 1/(1-p)); m is the
    undropped normaliser. The backward needs the same p and seed.
    """
    lib = _lib.load()
    B, Hq, Hkv, N, D = _check_qkv(q, k, v)
    n, b, per_head = _params(ssa_n, ssa_b, Hq, q.device)
    dp, seed = _dropout_args(dropout_p, dropout_seed, q.device)
    prob = _problem(q, Hkv, softmax_scale, n, b, per_head, causal, B, N, dropout_p=dp,
                    dropout_seed=seed)
    fam = _lib.kernel_family_of(prob)
    q, k, v = _prep(q, fam), _prep(k, fam), _prep(v, fam)
    out = torch.empty_like(q)
    if fam == 1 and not _tma_ok(out):
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    m = torch.empty((B, Hq, N), device=q.device, dtype=torch.float32)
    with _lib.device_guard(q.device):
        rc = lib.ssa_attn_fwd(ctypes.byref(prob), _lib.tensor_bhnd(q), _lib.tensor_bhnd(k),
                              _lib.tensor_bhnd(v), _lib.tensor_bhnd(out), m.data_ptr(), None, 0,
                              _lib.stream_ptr(q.device))
    _lib.check(rc)
    return out, m


def _param_grad_pair(n, device):
    """dn (n's shape) and db (0-d), fp32, as adjacent views of one buffer: a data-parallel
    caller sums both across ranks with one in-place all-reduce and no copies."""
    k = n.numel()
    buf = torch.empty(k + 1, device=device, dtype=torch.float32)
    return buf[:k].view(n.shape), buf[k]


def ssa_flash_attn_backward(q, k, v, out, dout, m, softmax_scale, ssa_n, ssa_b, causal=True,
                            deterministic=None, dropout_p=0.0, dropout_seed=None):
    """Backward (reference ssa_triton_kernel.py:795-897).

    Returns (dq, dk, dv, dn, db): dq/dk/dv in the inputs' dtype and layout; dn fp32 with
    ssa_n's shape (0-d in the reference); db a 0-d fp32 tensor. dn/db are reduced on the
    device (fp64, deterministic); no host synchronisation happens.

    deterministic: True adds each dQ tile's contributions in a fixed order, so dq is
    bit-identical from run to run (the reference's determinism rule,
    check_ssa_triton_parity.py:507-562); dk, dv, dn and db are bit-reproducible either way.
    None (default) takes SSA_DETERMINISTIC from the environment (off unless set to 1).

    With output dropout (the forward's dropout_p and dropout_seed), ``out`` is the dropped output
    the forward returned and ``dout`` the gradient of the dropped output.
    """
    lib = _lib.load()
    B, Hq, Hkv, N, D = _check_qkv(q, k, v)
    n, b, per_head = _params(ssa_n, ssa_b, Hq, q.device)
    det = _lib.deterministic_default() if deterministic is None else bool(deterministic)
    dp, seed = _dropout_args(dropout_p, dropout_seed, q.device)
    prob = _problem(q, Hkv, softmax_scale, n, b, per_head, causal, B, N, deterministic=det,
                    dropout_p=dp, dropout_seed=seed)
    fam = _lib.kernel_family_of(prob)
    q, k, v, dout = _prep(q, fam), _prep(k, fam), _prep(v, fam), _prep(dout, fam)
    out = _prep(out, fam)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dn, db = _param_grad_pair(n, q.device)
    ws_bytes = _lib.bwd_workspace_size(prob)
    ws = torch.empty(max(ws_bytes, 1), device=q.device, dtype=torch.uint8)
    with _lib.device_guard(q.device):
        rc = lib.ssa_attn_bwd(ctypes.byref(prob), _lib.tensor_bhnd(q), _lib.tensor_bhnd(k),
                              _lib.tensor_bhnd(v), _lib.tensor_bhnd(out), _lib.tensor_bhnd(dout),
                              m.data_ptr(), _lib.tensor_bhnd(dq), _lib.tensor_bhnd(dk),
                              _lib.tensor_bhnd(dv), dn.data_ptr(), db.data_ptr(), ws.data_ptr(),
                              ws_bytes, _lib.stream_ptr(q.device))
    _lib.check(rc)
    if tuple(dn.shape) != tuple(torch.as_tensor(ssa_n).shape):
        dn = dn.reshape(torch.as_tensor(ssa_n).shape)
    return dq, dk, dv, dn, db


# ------------------------------------------------------------------------------ varlen
def _check_thd(q, k, v, cu_seqlens):
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3:
        raise ValueError("varlen q, k, v must be [T, H, D]")
    if not (q.is_cuda and k.is_cuda and v.is_cuda and cu_seqlens.is_cuda):
        raise ValueError("varlen tensors must be CUDA tensors (there is no CPU path)")
    if cu_seqlens.dtype != torch.int32 or cu_seqlens.dim() != 1 or cu_seqlens.numel() < 2:
        raise ValueError("cu_seqlens must be a 1-D int32 tensor with ndoc+1 entries")
    T, Hq, D = q.shape
    if k.shape != v.shape or k.shape[0] != T or k.shape[2] != D:
        raise ValueError(f"shape mismatch q={tuple(q.shape)} k={tuple(k.shape)}")
    if Hq % k.shape[1] != 0:
        raise ValueError(f"Hq={Hq} must be divisible by Hkv={k.shape[1]}")
    return T, Hq, k.shape[1], D, cu_seqlens.numel() - 1


def _check_padded(cu_seqlens, cu_seqlens_padded):
    if cu_seqlens_padded is None:
        return None
    if (cu_seqlens_padded.dtype != torch.int32 or cu_seqlens_padded.shape != cu_seqlens.shape
            or not cu_seqlens_padded.is_cuda):
        raise ValueError("cu_seqlens_padded must be a CUDA int32 tensor shaped like cu_seqlens")
    return cu_seqlens_padded


def ssa_flash_attn_varlen_forward(q, k, v, cu_seqlens, max_seqlen, softmax_scale, ssa_n, ssa_b,
                                  causal=True, cu_seqlens_padded=None, dropout_p=0.0,
                                  dropout_seed=None):
    """Packed documents: q [T, Hq, D], k/v [T, Hkv, D], cu_seqlens int32 [ndoc+1].

    Each document attends only within itself (causal or not). Returns (out [T, Hq, D],
    lse [Hq, T] fp32). With cu_seqlens_padded (Megatron's cu_seqlens_q_padded), document z
    starts at row cu_seqlens_padded[z] and the padding rows between documents are ignored; their
    output rows are zero. No reference counterpart: the reference asserts packed sequences off
    (ssa_triton_attention.py:154-156). dropout_p / dropout_seed as in
    :func:`ssa_flash_attn_forward`.
    """
    lib = _lib.load()
    T, Hq, Hkv, D, ndoc = _check_thd(q, k, v, cu_seqlens)
    cu_pad = _check_padded(cu_seqlens, cu_seqlens_padded)
    n, b, per_head = _params(ssa_n, ssa_b, Hq, q.device)
    dp, seed = _dropout_args(dropout_p, dropout_seed, q.device)
    prob = _problem(q, Hkv, softmax_scale, n, b, per_head, causal, ndoc, T,
                    cu_seqlens, max_seqlen, cu_pad, dropout_p=dp, dropout_seed=seed)
    fam = _lib.kernel_family_of(prob)
    q, k, v = _prep(q, fam), _prep(k, fam), _prep(v, fam)
    alloc = torch.zeros if cu_pad is not None else torch.empty
    out = alloc(q.shape, dtype=q.dtype, device=q.device)
    lse = torch.empty((Hq, T), device=q.device, dtype=torch.float32)
    with _lib.device_guard(q.device):
        rc = lib.ssa_attn_fwd(ctypes.byref(prob), _lib.tensor_thd(q), _lib.tensor_thd(k),
                              _lib.tensor_thd(v), _lib.tensor_thd(out), lse.data_ptr(), None, 0,
                              _lib.stream_ptr(q.device))
    _lib.check(rc)
    return out, lse


def ssa_flash_attn_varlen_backward(q, k, v, out, dout, lse, cu_seqlens, max_seqlen,
                                   softmax_scale, ssa_n, ssa_b, causal=True,
                                   cu_seqlens_padded=None, deterministic=None, dropout_p=0.0,
                                   dropout_seed=None):
    """Backward of :func:`ssa_flash_attn_varlen_forward`. Returns (dq, dk, dv, dn, db); with
    cu_seqlens_padded the gradient rows of padding tokens are zero. ``deterministic`` and the
    dropout arguments as in :func:`ssa_flash_attn_backward`."""
    lib = _lib.load()
    T, Hq, Hkv, D, ndoc = _check_thd(q, k, v, cu_seqlens)
    cu_pad = _check_padded(cu_seqlens, cu_seqlens_padded)
    n, b, per_head = _params(ssa_n, ssa_b, Hq, q.device)
    det = _lib.deterministic_default() if deterministic is None else bool(deterministic)
    dp, seed = _dropout_args(dropout_p, dropout_seed, q.device)
    prob = _problem(q, Hkv, softmax_scale, n, b, per_head, causal, ndoc, T,
                    cu_seqlens, max_seqlen, cu_pad, deterministic=det, dropout_p=dp,
                    dropout_seed=seed)
    fam = _lib.kernel_family_of(prob)
    q, k, v, dout = _prep(q, fam), _prep(k, fam), _prep(v, fam), _prep(dout, fam)
    out = _prep(out, fam)
    alloc = torch.zeros if cu_pad is not None else torch.empty
    dq = alloc(q.shape, dtype=q.dtype, device=q.device)
    dk = alloc(k.shape, dtype=k.dtype, device=k.device)
    dv = alloc(v.shape, dtype=v.dtype, device=v.device)
    dn, db = _param_grad_pair(n, q.device)
    ws_bytes = _lib.bwd_workspace_size(prob)
    ws = torch.empty(max(ws_bytes, 1), device=q.device, dtype=torch.uint8)
    with _lib.device_guard(q.device):
        rc = lib.ssa_attn_bwd(ctypes.byref(prob), _lib.tensor_thd(q), _lib.tensor_thd(k),
                              _lib.tensor_thd(v), _lib.tensor_thd(out), _lib.tensor_thd(dout),
                              lse.data_ptr(), _lib.tensor_thd(dq), _lib.tensor_thd(dk),
                              _lib.tensor_thd(dv), dn.data_ptr(), db.data_ptr(), ws.data_ptr(),
                              ws_bytes, _lib.stream_ptr(q.device))
    _lib.check(rc)
    if tuple(dn.shape) != tuple(torch.as_tensor(ssa_n).shape):
        dn = dn.reshape(torch.as_tensor(ssa_n).shape)
    return dq, dk, dv, dn, db


def warmup_ssa_triton_kernels(B: int = 2, Hq: int = 24, Hkv: int = 8, N: int = 128, D: int = 32,
                              dtype: torch.dtype = torch.bfloat16, device: str = "cuda"):
    """Run one tiny forward + backward (reference ssa_triton_kernel.py:904-928).

    Nothing is JIT-compiled here (the kernels are built ahead of time); this loads the
    library, creates the CUDA module and resolves the TMA encoder. The RNG state is restored.
    """
    state = torch.cuda.get_rng_state(device) if torch.cuda.is_available() else None
    try:
        q = torch.randn(B, Hq, N, D, dtype=dtype, device=device)
        k = torch.randn(B, Hkv, N, D, dtype=dtype, device=device)
        v = torch.randn(B, Hkv, N, D, dtype=dtype, device=device)
        ssa_n = torch.tensor(1.5, dtype=torch.float32, device=device)
        ssa_b = torch.tensor(0.8, dtype=torch.float32, device=device)
        scale = 1.0 / math.sqrt(D)
        out, m = ssa_flash_attn_forward(q, k, v, scale, ssa_n, ssa_b, causal=True)
        dout = torch.randn_like(out)
        ssa_flash_attn_backward(q, k, v, out, dout, m, scale, ssa_n, ssa_b, causal=True)
        torch.cuda.synchronize(device)
    finally:
        if state is not None:
            torch.cuda.set_rng_state(state, device)
