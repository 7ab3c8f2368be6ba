"""Context-parallel (ring) SSA attention for long sequences (benchmark config 4).

No reference counterpart: the reference asserts context parallelism off for SSA
(training/train/train_ssa_triton/SSA/ssa_triton_attention.py:74-76). This module adds it with
the semantics of single-GPU attention over the full sequence.

Layout ("zig-zag"): the sequence is cut into 2*g equal chunks; rank r of g holds chunks r and
2g-1-r (concatenated, in that order) of q, k, v, out, dout. Causal work is then balanced: every
rank computes 2g+1 (q-chunk, k-chunk) pairs.

Forward: the ranks' K/V chunk pairs travel around the ring (g-1 hops, NCCL send/recv on a side
stream, overlapped with compute). For each q-chunk i and k-chunk j a rank computes the SSA
attention of the pair (non-causal if j < i, causal if j == i, skipped if j > i) with the
single-GPU kernels, and merges the partial (O, lse) results in base 2:
    lse = log2(sum_j 2^lse_j),  O = sum_j 2^(lse_j - lse) O_j
The 2g+1 visible pairs of a rank run as g launches. At step 0 (its own K/V) the three pairs are
one causal attention over the rank's two chunks in local order: local order agrees with global
order for every visible pair, and the pair the mask hides (chunk r against chunk 2g-1-r) is the
one causality removes. At every later step the two visible pairs share a key chunk (K/V from a
lower rank: both of this rank's q-chunks see its first chunk) or a query chunk (K/V from a higher
rank: the second q-chunk sees both of its chunks), and run as one non-causal launch with the two
pairs stacked in the batch dimension.
Backward: K/V travel again together with their dK/dV accumulators, which end on the owner
after g hops; every pair's gradients use the FINAL out and lse (the base-2 normaliser of the
whole row), so P = exp2(t2 - lse) and delta = rowsum(O dO) are those of full attention.
dq, dk, dv partial sums are accumulated in fp32 (or wider); dn / db are all-reduced once.

The pair computation is pluggable (`pair_fwd`, `pair_bwd`) so the ring logic can be tested on
the CPU with the oracle; by default it runs the library's CUDA kernels.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Tuple

import torch

PairFwd = Callable[..., Tuple[torch.Tensor, torch.Tensor]]
PairBwd = Callable[..., Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]]


def zigzag_chunks(world: int, rank: int) -> Tuple[int, int]:
    """The two sequence chunks (of 2*world) that `rank` owns."""
    return rank, 2 * world - 1 - rank


def zigzag_split(x: torch.Tensor, world: int, rank: int, dim: int = 2) -> torch.Tensor:
    """Rank-local part of a full-sequence tensor: chunks (r, 2g-1-r) concatenated along dim."""
    chunks = x.chunk(2 * world, dim=dim)
    a, b = zigzag_chunks(world, rank)
    return torch.cat([chunks[a], chunks[b]], dim=dim)


def zigzag_gather(parts: List[torch.Tensor], dim: int = 2) -> torch.Tensor:
    """Inverse of zigzag_split over all ranks' parts (for tests / reassembly)."""
    world = len(parts)
    out: List[Optional[torch.Tensor]] = [None] * (2 * world)
    for r, p in enumerate(parts):
        c0, c1 = p.chunk(2, dim=dim)
        a, b = zigzag_chunks(world, r)
        out[a], out[b] = c0, c1
    return torch.cat(out, dim=dim)


def _kernel_pair_fwd(q, k, v, scale, n, b, causal):
    from .ssa_triton_kernel import ssa_flash_attn_forward
    return ssa_flash_attn_forward(q, k, v, scale, n, b, causal=causal)


def _kernel_pair_bwd(q, k, v, out, dout, lse, scale, n, b, causal):
    from .ssa_triton_kernel import ssa_flash_attn_backward
    return ssa_flash_attn_backward(q, k, v, out, dout, lse, scale, n, b, causal=causal)


def _acc_dtype(t: torch.Tensor) -> torch.dtype:
    """Accumulation type: fp32, or the input's type when it is wider."""
    return torch.promote_types(t.dtype, torch.float32)


def _merge(o_acc, lse_acc, o_j, lse_j):
    """Base-2 log-sum-exp merge of normalised partial outputs (accumulated in >= fp32)."""
    dt = _acc_dtype(o_j)
    if o_acc is None:
        return o_j.to(dt), lse_j.to(torch.promote_types(lse_j.dtype, torch.float32))
    lse = torch.logaddexp2(lse_acc, lse_j.to(lse_acc.dtype))
    w_old = torch.exp2(lse_acc - lse).unsqueeze(-1).to(dt)
    w_new = torch.exp2(lse_j.to(lse.dtype) - lse).unsqueeze(-1).to(dt)
    return o_acc * w_old + o_j.to(dt) * w_new, lse


def _stack_chunks(x: torch.Tensor, c: int) -> torch.Tensor:
    """[B, H, 2c, ...] -> [2B, H, c, ...]: the first chunk's batch entries, then the second's.
    A strided view when B == 1 and x is contiguous (the kernels take B/H/N strides), else a copy."""
    if x.shape[0] == 1 and x.is_contiguous():
        return x.unflatten(2, (2, c)).movedim(2, 0).squeeze(1)
    return torch.cat([x[:, :, :c], x[:, :, c:]], dim=0)


def _twice(x: torch.Tensor) -> torch.Tensor:
    """[B, ...] -> [2B, ...]: two copies of the same batch entries."""
    return torch.cat([x, x], dim=0)


def _halves(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """[2B, ...] -> the first and second B entries."""
    b = x.shape[0] // 2
    return x[:b], x[b:]


class _Ring:
    """One send/recv hop of a list of tensors around the ring (prev -> self -> next)."""

    def __init__(self, group, world: int, rank: int, device):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world, self.rank = world, rank
        self.nxt = dist.get_global_rank(group, (rank + 1) % world) if group is not None else (rank + 1) % world
        self.prv = dist.get_global_rank(group, (rank - 1) % world) if group is not None else (rank - 1) % world
        self.stream = torch.cuda.Stream(device) if device.type == "cuda" else None

    def start(self, send: List[torch.Tensor]):
        recv = [torch.empty_like(t) for t in send]
        ops = []
        for t in send:
            ops.append(self.dist.P2POp(self.dist.isend, t.contiguous(), self.nxt, self.group))
        for t in recv:
            ops.append(self.dist.P2POp(self.dist.irecv, t, self.prv, self.group))
        if self.stream is not None:
            self.stream.wait_stream(torch.cuda.current_stream(send[0].device))
            with torch.cuda.stream(self.stream):
                reqs = self.dist.batch_isend_irecv(ops)
        else:
            reqs = self.dist.batch_isend_irecv(ops)
        return reqs, recv

    def finish(self, pending):
        reqs, recv = pending
        for r in reqs:
            r.wait()
        if self.stream is not None:
            torch.cuda.current_stream(recv[0].device).wait_stream(self.stream)
        return recv


def ring_ssa_forward(q, k, v, softmax_scale, ssa_n, ssa_b, group=None,
                     pair_fwd: PairFwd = _kernel_pair_fwd):
    """q [B, Hq, 2c, D], k/v [B, Hkv, 2c, D]: this rank's zig-zag chunks. Causal attention over
    the full sequence. Returns (out [B, Hq, 2c, D] in q's dtype, lse [B, Hq, 2c] fp32)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    c = q.shape[2] // 2
    qs = (q[:, :, :c], q[:, :, c:])
    acc_o = [None, None]
    acc_l = [None, None]
    ring = _Ring(group, world, rank, q.device)
    kv = [k, v]
    for step in range(world):
        src = (rank - step) % world
        pending = ring.start(kv) if step + 1 < world else None
        if src == rank:  # own chunks: one causal attention over the local order
            o, l = pair_fwd(q, kv[0], kv[1], softmax_scale, ssa_n, ssa_b, True)
            parts = [(0, o[:, :, :c], l[:, :, :c]), (1, o[:, :, c:], l[:, :, c:])]
        elif src < rank:  # both q-chunks against the sender's first chunk
            o, l = pair_fwd(_stack_chunks(q, c), _twice(kv[0][:, :, :c]),
                            _twice(kv[1][:, :, :c]), softmax_scale, ssa_n, ssa_b, False)
            (o0, o1), (l0, l1) = _halves(o), _halves(l)
            parts = [(0, o0, l0), (1, o1, l1)]
        else:  # the second q-chunk against both of the sender's chunks
            o, l = pair_fwd(_twice(qs[1]), _stack_chunks(kv[0], c), _stack_chunks(kv[1], c),
                            softmax_scale, ssa_n, ssa_b, False)
            (o0, o1), (l0, l1) = _halves(o), _halves(l)
            parts = [(1, o0, l0), (1, o1, l1)]
        for qi, o_p, l_p in parts:
            acc_o[qi], acc_l[qi] = _merge(acc_o[qi], acc_l[qi], o_p, l_p)
        if pending is not None:
            kv = ring.finish(pending)
    out = torch.cat([acc_o[0], acc_o[1]], dim=2).to(q.dtype)
    lse = torch.cat([acc_l[0], acc_l[1]], dim=2)
    return out, lse


def ring_ssa_backward(q, k, v, out, dout, lse, softmax_scale, ssa_n, ssa_b, group=None,
                      pair_bwd: PairBwd = _kernel_pair_bwd):
    """Gradients of ring_ssa_forward for this rank's chunks: (dq, dk, dv, dn, db); dn/db are
    summed over all ranks."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    c = q.shape[2] // 2
    qs = (q[:, :, :c], q[:, :, c:])
    os_ = (out[:, :, :c], out[:, :, c:])
    dos = (dout[:, :, :c], dout[:, :, c:])
    ls = (lse[:, :, :c].contiguous(), lse[:, :, c:].contiguous())
    acc = _acc_dtype(q)
    dq = torch.zeros(q.shape, dtype=acc, device=q.device)
    dn = torch.zeros(torch.as_tensor(ssa_n).shape, dtype=acc, device=q.device)
    db = torch.zeros((), dtype=acc, device=q.device)
    ring = _Ring(group, world, rank, q.device)
    # travelling state: this step's K/V pair and the dK/dV accumulators that belong to it
    kv = [k, v]
    dkv = [torch.zeros(k.shape, dtype=acc, device=k.device),
           torch.zeros(v.shape, dtype=acc, device=v.device)]
    for step in range(world):
        src = (rank - step) % world
        # K/V for the next step can move now; the accumulators only after this step's adds
        pending_kv = ring.start(kv) if step + 1 < world else None
        if src == rank:  # own chunks: one causal attention over the local order
            dq_p, dk_p, dv_p, dn_p, db_p = pair_bwd(q, kv[0], kv[1], out, dout, lse.contiguous(),
                                                    softmax_scale, ssa_n, ssa_b, True)
            dq += dq_p.to(acc)
            dkv[0] += dk_p.to(acc)
            dkv[1] += dv_p.to(acc)
        elif src < rank:  # both q-chunks against the sender's first chunk
            dq_p, dk_p, dv_p, dn_p, db_p = pair_bwd(
                _stack_chunks(q, c), _twice(kv[0][:, :, :c]), _twice(kv[1][:, :, :c]),
                _stack_chunks(out, c), _stack_chunks(dout, c), _stack_chunks(lse, c).contiguous(),
                softmax_scale, ssa_n, ssa_b, False)
            dq0, dq1 = _halves(dq_p)
            dq[:, :, :c] += dq0.to(acc)
            dq[:, :, c:] += dq1.to(acc)
            dk0, dk1 = _halves(dk_p)
            dv0, dv1 = _halves(dv_p)
            dkv[0][:, :, :c] += dk0.to(acc) + dk1.to(acc)
            dkv[1][:, :, :c] += dv0.to(acc) + dv1.to(acc)
        else:  # the second q-chunk against both of the sender's chunks
            dq_p, dk_p, dv_p, dn_p, db_p = pair_bwd(
                _twice(qs[1]), _stack_chunks(kv[0], c), _stack_chunks(kv[1], c), _twice(os_[1]),
                _twice(dos[1]), _twice(ls[1]), softmax_scale, ssa_n, ssa_b, False)
            dq0, dq1 = _halves(dq_p)
            dq[:, :, c:] += dq0.to(acc) + dq1.to(acc)
            dk0, dk1 = _halves(dk_p)
            dv0, dv1 = _halves(dv_p)
            dkv[0][:, :, :c] += dk0.to(acc)
            dkv[0][:, :, c:] += dk1.to(acc)
            dkv[1][:, :, :c] += dv0.to(acc)
            dkv[1][:, :, c:] += dv1.to(acc)
        dn += dn_p.to(acc).reshape(dn.shape)
        db += db_p.to(acc).reshape(())
        # dK/dV follow their K/V chunk; after `world` hops they are back on the owner
        pending_d = ring.start(dkv)
        if pending_kv is not None:
            kv = ring.finish(pending_kv)
        dkv = ring.finish(pending_d)
    buf = torch.cat([dn.reshape(-1), db.reshape(1)])
    dist.all_reduce(buf, group=group)
    dn = buf[:-1].reshape(dn.shape)
    db = buf[-1].reshape(())
    return dq.to(q.dtype), dkv[0].to(k.dtype), dkv[1].to(v.dtype), dn, db


class RingSSAAttnFunc(torch.autograd.Function):
    """Autograd wrapper: inputs are this rank's zig-zag chunks; causal attention over the whole
    sequence held by the process group."""

    @staticmethod
    def forward(ctx, q, k, v, softmax_scale, ssa_n, ssa_b, group):
        n32 = ssa_n.float().contiguous()
        b32 = ssa_b.float().contiguous()
        out, lse = ring_ssa_forward(q, k, v, softmax_scale, n32, b32, group)
        ctx.save_for_backward(q, k, v, out, lse, n32, b32)
        ctx.softmax_scale = softmax_scale
        ctx.group = group
        ctx.n_meta = (ssa_n.shape, ssa_n.dtype)
        ctx.b_meta = (ssa_b.shape, ssa_b.dtype)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse, n32, b32 = ctx.saved_tensors
        dq, dk, dv, dn, db = ring_ssa_backward(q, k, v, out, dout.contiguous(), lse,
                                               ctx.softmax_scale, n32, b32, ctx.group)
        return (dq, dk, dv, None, dn.reshape(ctx.n_meta[0]).to(ctx.n_meta[1]),
                db.reshape(ctx.b_meta[0]).to(ctx.b_meta[1]), None)


def ring_ssa_attention(q, k, v, softmax_scale, ssa_n, ssa_b, group=None):
    """Context-parallel causal SSA attention (see module docstring)."""
    return RingSSAAttnFunc.apply(q, k, v, softmax_scale, ssa_n, ssa_b, group)
