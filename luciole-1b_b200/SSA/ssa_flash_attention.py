"""Differentiable SSA flash attention over libssa_b200.so.

Drop-in for the reference ``SSA.ssa_flash_attention``
(training/train/train_ssa_triton/SSA/ssa_flash_attention.py): ``SSAFlashAttnFunc`` takes the
same 9 positional arguments and its backward returns 9 gradients in the same order
(``dq, dk, dv, None, dn, db, None, None, None``, reference :66). Saved state is q, k, v, out,
m and the fp32 parameters (reference :43); no O(N^2) tensor is kept.

``SSAVarlenFlashAttnFunc`` / ``ssa_flash_attn_varlen_func`` add packed documents
(``cu_seqlens``), which the reference does not support.

Output dropout. The reference's function accepts ``dropout_p`` and ``training`` but leaves
dropout to its caller (its module applies ``nn.Dropout`` after the kernel,
ssa_triton_attention.py:186-193), and so does this one by default. Given a ``dropout_seed``
(``make_dropout_seed``), training mode and ``dropout_p > 0``, the kernels apply it themselves:
the forward's epilogue drops and rescales the output, and the backward's delta pass masks the
incoming gradient, so no separate dropout launches run in either direction.
"""

from __future__ import annotations

import torch
from torch.autograd import Function

from .ssa_triton_kernel import (
    ssa_flash_attn_backward,
    ssa_flash_attn_forward,
    ssa_flash_attn_varlen_backward,
    ssa_flash_attn_varlen_forward,
)

__all__ = ["SSAFlashAttnFunc", "ssa_flash_attention", "SSAVarlenFlashAttnFunc",
           "ssa_flash_attn_varlen_func"]


def _grad_like(g: torch.Tensor, ref: torch.Tensor) -> torch.Tensor:
    g = g.reshape(ref.shape)
    return g if g.dtype == ref.dtype else g.to(ref.dtype)


def _fused_dropout(dropout_p, training, dropout_seed) -> float:
    """The dropout probability the kernels apply: dropout_p when a seed is given in training mode,
    else 0 (the caller applies dropout itself, as with the reference)."""
    if dropout_seed is None or not training or not dropout_p:
        return 0.0
    return float(dropout_p)


class SSAFlashAttnFunc(Function):
    """out = softmax(n * sign(s) * log1p(b |s|)) @ V with s = scale * Q K^T (causal optional)."""

    @staticmethod
    def forward(ctx, q, k, v, softmax_scale, ssa_n, ssa_b, causal, dropout_p, training,
                deterministic=None, dropout_seed=None):
        # deterministic (optional 10th argument, no reference counterpart): bit-reproducible dq
        # in the backward; None takes SSA_DETERMINISTIC from the environment.
        # dropout_seed (optional 11th): fused output dropout (module docstring).
        ssa_n_f32 = ssa_n.float().contiguous()
        ssa_b_f32 = ssa_b.float().contiguous()
        p = _fused_dropout(dropout_p, training, dropout_seed)
        seed = dropout_seed if p > 0 else None
        out, m = ssa_flash_attn_forward(q, k, v, softmax_scale, ssa_n_f32, ssa_b_f32, causal,
                                        dropout_p=p, dropout_seed=seed)
        ctx.save_for_backward(q, k, v, out, m, ssa_n_f32, ssa_b_f32, seed)
        ctx.softmax_scale = softmax_scale
        ctx.causal = causal
        ctx.deterministic = deterministic
        ctx.dropout_p = p
        ctx.n_meta = (ssa_n.shape, ssa_n.dtype)
        ctx.b_meta = (ssa_b.shape, ssa_b.dtype)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, m, ssa_n_f32, ssa_b_f32, seed = ctx.saved_tensors
        # The reference makes dout contiguous (ssa_flash_attention.py:56); the kernels take its
        # strides, so a Megatron-layout gradient ([B, H, S, D] view of [S, B, H*D]) is read in
        # place and only layouts the kernels cannot address are copied (in the kernel wrapper).
        dq, dk, dv, dn, db = ssa_flash_attn_backward(
            q, k, v, out, dout, m, ctx.softmax_scale, ssa_n_f32, ssa_b_f32, ctx.causal,
            deterministic=ctx.deterministic, dropout_p=ctx.dropout_p, dropout_seed=seed)
        dn = dn.reshape(ctx.n_meta[0]).to(ctx.n_meta[1])
        db = db.reshape(ctx.b_meta[0]).to(ctx.b_meta[1])
        grads = (dq, dk, dv, None, dn, db, None, None, None, None, None)
        return grads[:len(ctx.needs_input_grad)]  # 9 for the reference's 9 arguments


def ssa_flash_attention(q, k, v, softmax_scale, ssa_n, ssa_b, causal=True, dropout_p=0.0,
                        training=True, deterministic=None, dropout_seed=None):
    """High-level API (reference ssa_flash_attention.py:69-97): q [B, Hq, N, D],
    k/v [B, Hkv, N, D] (native GQA), ssa_n 0-d or [Hq], ssa_b 0-d. Returns [B, Hq, N, D].
    deterministic: bit-reproducible dq in the backward (default: SSA_DETERMINISTIC).
    dropout_seed: with training and dropout_p > 0, the kernels apply output dropout themselves
    (module docstring); without it dropout_p is left to the caller, as in the reference."""
    return SSAFlashAttnFunc.apply(q, k, v, softmax_scale, ssa_n, ssa_b, causal, dropout_p,
                                  training, deterministic, dropout_seed)


class SSAVarlenFlashAttnFunc(Function):
    """Packed-document SSA attention: q [T, Hq, D], k/v [T, Hkv, D], cu_seqlens int32, and
    optionally cu_seqlens_padded (start row of each document when padding separates them)."""

    @staticmethod
    def forward(ctx, q, k, v, cu_seqlens, max_seqlen, softmax_scale, ssa_n, ssa_b, causal,
                cu_seqlens_padded=None, dropout_p=0.0, dropout_seed=None):
        ssa_n_f32 = ssa_n.float().contiguous()
        ssa_b_f32 = ssa_b.float().contiguous()
        p = float(dropout_p) if dropout_seed is not None and dropout_p else 0.0
        seed = dropout_seed if p > 0 else None
        out, lse = ssa_flash_attn_varlen_forward(q, k, v, cu_seqlens, max_seqlen, softmax_scale,
                                                 ssa_n_f32, ssa_b_f32, causal, cu_seqlens_padded,
                                                 dropout_p=p, dropout_seed=seed)
        ctx.save_for_backward(q, k, v, out, lse, cu_seqlens, ssa_n_f32, ssa_b_f32,
                              cu_seqlens_padded, seed)
        ctx.max_seqlen = max_seqlen
        ctx.softmax_scale = softmax_scale
        ctx.causal = causal
        ctx.dropout_p = p
        ctx.n_meta = (ssa_n.shape, ssa_n.dtype)
        ctx.b_meta = (ssa_b.shape, ssa_b.dtype)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse, cu, n32, b32, cu_pad, seed = ctx.saved_tensors
        dq, dk, dv, dn, db = ssa_flash_attn_varlen_backward(
            q, k, v, out, dout, lse, cu, ctx.max_seqlen, ctx.softmax_scale, n32, b32,
            ctx.causal, cu_pad, dropout_p=ctx.dropout_p, dropout_seed=seed)
        dn = dn.reshape(ctx.n_meta[0]).to(ctx.n_meta[1])
        db = db.reshape(ctx.b_meta[0]).to(ctx.b_meta[1])
        return dq, dk, dv, None, None, None, dn, db, None, None, None, None


def ssa_flash_attn_varlen_func(q, k, v, cu_seqlens, max_seqlen, softmax_scale, ssa_n, ssa_b,
                               causal=True, cu_seqlens_padded=None, dropout_p=0.0,
                               dropout_seed=None):
    """Packed documents (THD + cu_seqlens); each document attends only within itself. With
    cu_seqlens_padded, document z starts at row cu_seqlens_padded[z] (Megatron's
    PackedSeqParams.cu_seqlens_q_padded) and padding rows get zero output and gradient.
    dropout_p with a dropout_seed: fused output dropout (module docstring)."""
    return SSAVarlenFlashAttnFunc.apply(q, k, v, cu_seqlens, int(max_seqlen), softmax_scale,
                                        ssa_n, ssa_b, causal, cu_seqlens_padded, dropout_p,
                                        dropout_seed)
