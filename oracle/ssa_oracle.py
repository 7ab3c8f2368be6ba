"""CPU oracle for SSA ("Softmax-Substituted Attention") forward and backward.

TEST INFRASTRUCTURE ONLY. Nothing in the product path imports this module: only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` use it,
and only as the checker (or as the timed CPU baseline), never as the thing measured
or shipped.

This is an eager restatement of the reference's own parity oracle,
``training/train/train_ssa_triton/check_ssa_triton_parity.py:169-206``
(``_ssa_reference_forward``) and ``:209-237`` (``_run_reference_grads``), which in turn
restate the original unfused module
``training/train/train_ssa_triton/SSA/archive/legacy_pre_triton/ssa_attention.py:90-157``:

    s    = softmax_scale * q @ k^T                         (fp32 or fp64)
    s    = -inf where causal-masked (triu, diagonal=1)
    w    = exp(n * sign(s) * log1p(b * |s|))  (0 where masked)
    p    = w / max(sum_j w, 1e-12)
    out  = p @ v

GQA repeats each KV head ``Hq // Hkv`` times (``repeat_interleave``, parity.py:183-185).
Gradients come from autograd of ``sum(out * dout)`` (parity.py:209-237).

Extensions that have no reference counterpart, with the semantics the reference implies:
  * ``ssa_n`` may be a 0-d tensor (reference) or an ``[Hq]`` vector (per-head n, as in
    the legacy FlexAttention variant ``SSA/archive/legacy_pre_triton/ssa_flex_attention.py:82-92``);
    ``dn`` then has shape ``[Hq]``.
  * varlen (packed documents, ``cu_seqlens``): one independent causal/non-causal attention
    per document (loop), since the reference asserts packed sequences off
    (``SSA/ssa_triton_attention.py:154-156``).
  * ``lse2`` = log2(sum_j exp2(t_j * log2 e)): the base-2 normaliser the reference's forward
    kernel stores as ``M`` (``SSA/ssa_triton_kernel.py:248-255``).

The oracle is pinned against golden vectors produced by the reference's own Triton
kernels (``tests/golden/make_golden.py``).
"""

from __future__ import annotations


import math
from typing import Optional

import torch

LOG2E = 1.4426950408889634


def _expand_n(ssa_n: torch.Tensor, hq: int, dtype) -> torch.Tensor:
    n = ssa_n.to(dtype)
    if n.dim() == 0:
        return n
    if n.numel() != hq:
        raise ValueError(f"per-head ssa_n must have Hq={hq} elements, got {tuple(n.shape)}")
    return n.reshape(1, hq, 1, 1)


def ssa_reference_forward(q, k, v, softmax_scale: float, ssa_n, ssa_b, causal: bool,
                          compute_dtype=torch.float64):
    """Forward of the eager oracle (parity.py:169-206).

    q [B,Hq,N,D], k/v [B,Hkv,N,D] (any strides). Returns (out, lse2), both in
    ``compute_dtype``; out is NOT cast back to q's dtype so callers can compare at full
    precision (the reference casts with ``out.to(q.dtype)``).
    """
    bsz, hq, n_q, _ = q.shape
    hkv = k.shape[1]
    n_k = k.shape[2]
    if hq % hkv != 0:
        raise ValueError(f"HQ={hq} must be divisible by HKV={hkv}")
    g = hq // hkv
    k_exp = k.repeat_interleave(g, dim=1).to(compute_dtype)
    v_exp = v.repeat_interleave(g, dim=1).to(compute_dtype)
    s = torch.matmul(q.to(compute_dtype), k_exp.transpose(-1, -2)) * float(softmax_scale)
    if causal:
        mask = torch.triu(torch.ones((n_q, n_k), dtype=torch.bool, device=s.device), diagonal=1)
        s = s.masked_fill(mask.view(1, 1, n_q, n_k), float("-inf"))
    valid = torch.isfinite(s)
    s_safe = torch.where(valid, s, torch.zeros_like(s))
    n_val = _expand_n(torch.as_tensor(ssa_n), hq, compute_dtype)
    b_val = torch.as_tensor(ssa_b).to(compute_dtype)
    t = n_val * torch.sign(s_safe) * torch.log1p(b_val * s_safe.abs())
    w = torch.where(valid, torch.exp(t), torch.zeros_like(s))
    l = w.sum(dim=-1)
    p = w / l.clamp_min(1e-12).unsqueeze(-1)
    out = torch.matmul(p, v_exp)
    lse2 = torch.log2(l.clamp_min(1e-300))
    return out, lse2


def ssa_reference_grads(q, k, v, softmax_scale: float, ssa_n, ssa_b, dout, causal: bool,
                        compute_dtype=torch.float64) -> dict:
    """Forward + autograd backward of the oracle (parity.py:209-237), in ``compute_dtype``.

    Returns dict(out, lse2, dq, dk, dv, dn, db); dn has ssa_n's shape, db is 0-d.
    """
    q_r = q.detach().to(compute_dtype).requires_grad_(True)
    k_r = k.detach().to(compute_dtype).requires_grad_(True)
    v_r = v.detach().to(compute_dtype).requires_grad_(True)
    n_r = torch.as_tensor(ssa_n).detach().to(compute_dtype).clone().requires_grad_(True)
    b_r = torch.as_tensor(ssa_b).detach().to(compute_dtype).clone().requires_grad_(True)
    out, lse2 = ssa_reference_forward(q_r, k_r, v_r, softmax_scale, n_r, b_r, causal,
                                      compute_dtype=compute_dtype)
    loss = torch.sum(out * dout.detach().to(compute_dtype))
    loss.backward()
    return {
        "out": out.detach(), "lse2": lse2.detach(),
        "dq": q_r.grad.detach(), "dk": k_r.grad.detach(), "dv": v_r.grad.detach(),
        "dn": n_r.grad.detach(), "db": b_r.grad.detach(),
    }


def ssa_reference_grads_varlen(q, k, v, cu_seqlens, softmax_scale: float, ssa_n, ssa_b, dout,
                               causal: bool, compute_dtype=torch.float64) -> dict:
    """Packed-document (THD) oracle: q [T,Hq,D], k/v [T,Hkv,D], cu_seqlens int [ndoc+1].

    Each document is an independent attention (loop over documents); grads of n/b are summed.
    """
    cu = [int(x) for x in torch.as_tensor(cu_seqlens).tolist()]
    T, hq, D = q.shape
    outs = torch.zeros((T, hq, D), dtype=compute_dtype)
    lse = torch.zeros((T, hq), dtype=compute_dtype)
    dq = torch.zeros((T, hq, D), dtype=compute_dtype)
    dk = torch.zeros((T, k.shape[1], D), dtype=compute_dtype)
    dv = torch.zeros((T, k.shape[1], D), dtype=compute_dtype)
    dn = torch.zeros_like(torch.as_tensor(ssa_n), dtype=compute_dtype)
    db = torch.zeros((), dtype=compute_dtype)
    for i in range(len(cu) - 1):
        a, e = cu[i], cu[i + 1]
        if e <= a:
            continue
        sl = slice(a, e)
        r = ssa_reference_grads(
            q[sl].permute(1, 0, 2).unsqueeze(0), k[sl].permute(1, 0, 2).unsqueeze(0),
            v[sl].permute(1, 0, 2).unsqueeze(0), softmax_scale, ssa_n, ssa_b,
            dout[sl].permute(1, 0, 2).unsqueeze(0), causal, compute_dtype=compute_dtype)
        outs[sl] = r["out"][0].permute(1, 0, 2)
        lse[sl] = r["lse2"][0].permute(1, 0)
        dq[sl] = r["dq"][0].permute(1, 0, 2)
        dk[sl] = r["dk"][0].permute(1, 0, 2)
        dv[sl] = r["dv"][0].permute(1, 0, 2)
        dn = dn + r["dn"]
        db = db + r["db"]
    return {"out": outs, "lse2": lse, "dq": dq, "dk": dk, "dv": dv, "dn": dn, "db": db}


def ssa_pair_backward_with_lse(q, k, v, out, dout, lse2, softmax_scale: float, ssa_n, ssa_b,
                               causal: bool, compute_dtype=torch.float64):
    """Gradients of one (query block, key block) pair given the FINAL output and base-2
    normaliser of the full rows -- the reference backward's per-block math
    (ssa_triton_kernel.py:348-397 for dK/dV/dn/db, :444-477 for dQ):
        P = exp2(t2 - M),  delta = rowsum(O dO),  ds_ssa = P (dO V^T - delta),
        ds = ds_ssa n b / (1 + b|s|),  dV = P^T dO,  dK = ds^T Q scale,  dQ = ds K scale,
        dn = sum ds_ssa sign(s) log1p(b|s|),  db = sum ds_ssa n sign(s) |s| / (1 + b|s|).
    q/out/dout [B,Hq,Nq,D], k/v [B,Hkv,Nk,D], lse2 [B,Hq,Nq]. Returns (dq, dk, dv, dn, db)."""
    cd = compute_dtype
    bsz, hq, n_q, _ = q.shape
    hkv = k.shape[1]
    g = hq // hkv
    qf, kf, vf = q.to(cd), k.repeat_interleave(g, dim=1).to(cd), v.repeat_interleave(g, dim=1).to(cd)
    of, dof = out.to(cd), dout.to(cd)
    s = torch.matmul(qf, kf.transpose(-1, -2)) * float(softmax_scale)
    n_k = k.shape[2]
    valid = torch.ones((n_q, n_k), dtype=torch.bool)
    if causal:
        valid = ~torch.triu(torch.ones((n_q, n_k), dtype=torch.bool), diagonal=1)
    n_val = _expand_n(torch.as_tensor(ssa_n), hq, cd)
    b_val = torch.as_tensor(ssa_b).to(cd)
    sign, u = torch.sign(s), b_val * s.abs()
    lg = torch.log1p(u)
    t2 = n_val * sign * lg / math.log(2.0)
    p = torch.where(valid, torch.exp2(t2 - lse2.to(cd).unsqueeze(-1)), torch.zeros_like(s))
    delta = (of * dof).sum(-1, keepdim=True)
    dp = torch.matmul(dof, vf.transpose(-1, -2))
    ds_ssa = p * (dp - delta)
    ds = ds_ssa * n_val * b_val / (1.0 + u)
    dq = torch.matmul(ds, kf) * float(softmax_scale)
    dk_full = torch.matmul(ds.transpose(-1, -2), qf) * float(softmax_scale)
    dv_full = torch.matmul(p.transpose(-1, -2), dof)
    dk = dk_full.reshape(bsz, hkv, g, n_k, -1).sum(2)
    dv = dv_full.reshape(bsz, hkv, g, n_k, -1).sum(2)
    dn_el = ds_ssa * sign * lg
    dn = dn_el.sum() if torch.as_tensor(ssa_n).dim() == 0 else dn_el.sum(dim=(0, 2, 3))
    db = (ds_ssa * n_val * s / (1.0 + u)).sum()
    return dq, dk, dv, dn, db


def ssa_reference_grads_blocked(q, k, v, softmax_scale: float, ssa_n, ssa_b, dout, causal: bool,
                                heads=None, block: int = 512,
                                compute_dtype=torch.float64) -> dict:
    """The oracle of :func:`ssa_reference_grads` for long sequences, evaluated block by block so
    that no [N, N] tensor is held (one [block, N] slab at a time).

    Pass 1, per block of query rows, the rows of the eager forward (parity.py:169-206):
    w = exp(n sign(s) log1p(b|s|)) over the visible keys, l = sum_j w, out = (w / l) V,
    lse2 = log2 l. Pass 2, per block, the reference backward's per-element gradient math given
    the final out and l (ssa_triton_kernel.py:348-397 for dK/dV/dn/db, :444-477 for dQ):
        P = w / l,  delta = rowsum(out dout),  ds_ssa = P (dout V^T - delta),
        ds = ds_ssa n b / (1 + b|s|),  dQ = ds K scale,  dK += ds^T Q scale,  dV += P^T dout,
        dn += sum ds_ssa sign(s) log1p(b|s|),  db += sum ds_ssa n s / (1 + b|s|),
    which is what autograd of the eager forward computes (pinned against it in the CPU tests).

    q/dout [B, Hq, N, D], k/v [B, Hkv, N, D]. ``heads``: the q-heads to evaluate (default all);
    rows of other heads stay zero in out/dq and contribute nothing to dk/dv/dn/db. Returns
    dict(out, lse2, dq, dk, dv, dn, db) like :func:`ssa_reference_grads` (dn has ssa_n's shape).
    """
    cd = compute_dtype
    bsz, hq, n_q, d = q.shape
    hkv, n_k = k.shape[1], k.shape[2]
    if hq % hkv != 0:
        raise ValueError(f"HQ={hq} must be divisible by HKV={hkv}")
    g = hq // hkv
    heads = list(range(hq)) if heads is None else [int(h) for h in heads]
    n_t = torch.as_tensor(ssa_n).detach().to(cd)
    per_head = n_t.dim() == 1 and n_t.numel() == hq
    b_val = float(torch.as_tensor(ssa_b))
    scale = float(softmax_scale)
    out = torch.zeros((bsz, hq, n_q, d), dtype=cd)
    lse2 = torch.zeros((bsz, hq, n_q), dtype=cd)
    dq = torch.zeros((bsz, hq, n_q, d), dtype=cd)
    dk = torch.zeros((bsz, hkv, n_k, d), dtype=cd)
    dv = torch.zeros((bsz, hkv, n_k, d), dtype=cd)
    dn = torch.zeros(n_t.shape, dtype=cd)
    db = torch.zeros((), dtype=cd)
    for z in range(bsz):
        for h in heads:
            hk = h // g
            nval = float(n_t.reshape(-1)[h if per_head else 0])
            kf, vf = k[z, hk].to(cd), v[z, hk].to(cd)
            qf, dof = q[z, h].to(cd), dout[z, h].to(cd)
            dn_h = torch.zeros((), dtype=cd)
            for m0 in range(0, n_q, block):
                m1 = min(n_q, m0 + block)
                nk = min(n_k, m1) if causal else n_k
                s = (qf[m0:m1] @ kf[:nk].T) * scale
                lg = torch.log1p(b_val * s.abs())
                w = torch.exp(nval * torch.sign(s) * lg)
                if causal:
                    rows = torch.arange(m0, m1).unsqueeze(1)
                    w = torch.where(torch.arange(nk).unsqueeze(0) <= rows, w, torch.zeros_like(w))
                l = w.sum(-1, keepdim=True)
                p = w / l.clamp_min(1e-12)
                o = p @ vf[:nk]
                out[z, h, m0:m1] = o
                lse2[z, h, m0:m1] = torch.log2(l.clamp_min(1e-300)).squeeze(-1)
                delta = (o * dof[m0:m1]).sum(-1, keepdim=True)
                ds_ssa = p * (dof[m0:m1] @ vf[:nk].T - delta)
                inv = 1.0 / (1.0 + b_val * s.abs())
                ds = ds_ssa * (nval * b_val) * inv
                dq[z, h, m0:m1] = (ds @ kf[:nk]) * scale
                dk[z, hk, :nk] += (ds.T @ qf[m0:m1]) * scale
                dv[z, hk, :nk] += p.T @ dof[m0:m1]
                dn_h += (ds_ssa * torch.sign(s) * lg).sum()
                db += (ds_ssa * (nval * s) * inv).sum()
                del s, lg, w, p, ds_ssa, inv, ds
            if per_head:
                dn.view(-1)[h] += dn_h
            else:
                dn += dn_h
    return {"out": out, "lse2": lse2, "dq": dq, "dk": dk, "dv": dv, "dn": dn, "db": db}


def causal_score_elements(B: int, Hq: int, N: int, causal: bool) -> int:
    """Number of score elements E in the FlashAttention FLOP convention (S^2/2 causal)."""
    return B * Hq * (N * N // 2 if causal else N * N)


def attn_flops_fwd_bwd(B: int, Hq: int, N: int, D: int, causal: bool) -> float:
    """Algorithmic fwd+bwd FLOPs = 14 * D * E (5 GEMMs: fwd 4*D*E, bwd 10*D*E)."""
    return 14.0 * D * causal_score_elements(B, Hq, N, causal)


def check_close(name: str, got, ref, atol: float, rtol: float) -> Optional[str]:
    """Elementwise |got-ref| <= atol + rtol*|ref| (torch.allclose semantics); returns an
    error string on failure, None on success."""
    g = torch.as_tensor(got).to(torch.float64)
    r = torch.as_tensor(ref).to(torch.float64)
    if g.shape != r.shape:
        return f"{name}: shape {tuple(g.shape)} != {tuple(r.shape)}"
    if not torch.isfinite(g).all():
        return f"{name}: non-finite values"
    d = (g - r).abs()
    lim = atol + rtol * r.abs()
    bad = d > lim
    if bool(bad.any()):
        i = int(torch.argmax((d - lim).reshape(-1)))
        return (f"{name}: {int(bad.sum())} / {d.numel()} elements out of tolerance "
                f"(atol={atol}, rtol={rtol}); worst |d|={d.reshape(-1)[i].item():.3e} "
                f"ref={r.reshape(-1)[i].item():.3e}; max|d|={d.max().item():.3e}")
    return None


def max_rel(got, ref) -> float:
    """max|got-ref| / max|ref| (check_ssa_triton_vs_original.py:54-58 convention)."""
    g = torch.as_tensor(got).to(torch.float64)
    r = torch.as_tensor(ref).to(torch.float64)
    den = r.abs().max().item()
    return (g - r).abs().max().item() / (den if den > 0 else 1.0)


__all__ = [
    "LOG2E", "ssa_reference_forward", "ssa_reference_grads", "ssa_reference_grads_varlen",
    "ssa_reference_grads_blocked",
    "causal_score_elements", "attn_flops_fwd_bwd", "check_close", "max_rel",
]

