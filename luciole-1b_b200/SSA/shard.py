"""Partitioning SSA attention across GPUs by (batch, kv-head) units.

Every (sequence, kv-head group) of SSA attention is independent in forward and backward
(the reference's kernels index programs by batch x head, ssa_triton_kernel.py:176,522), so the
path shards with no data-path communication. The only cross-rank quantity is the gradient of the
SSA parameters: dn (1 or Hq floats) and db (1 float) are sums over every score element, so each
rank's partial sums are added with one all-reduce (in training, DDP's gradient all-reduce does
the same for the ``ssa_n_raw`` parameter).
"""

from __future__ import annotations

from typing import List, Optional, Tuple

import torch


def balanced_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, stop) of n items for `rank` of `world`, sizes differing by at most 1."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def unit_shard(B: int, Hkv: int, world: int, rank: int) -> List[Tuple[int, int]]:
    """(batch, kv-head) units owned by `rank`: a balanced contiguous range of the B*Hkv units in
    batch-major order, so a rank's units are whole sequences whenever world divides B."""
    a, b = balanced_range(B * Hkv, world, rank)
    return [(u // Hkv, u % Hkv) for u in range(a, b)]


def batch_shard(B: int, world: int, rank: int) -> slice:
    """Batch entries owned by `rank` (balanced contiguous slice)."""
    a, b = balanced_range(B, world, rank)
    return slice(a, b)


def allreduce_ssa_param_grads(dn: torch.Tensor, db: torch.Tensor, group=None,
                              buffer: Optional[torch.Tensor] = None, async_op: bool = False):
    """Sum dn and db over the ranks of `group` with a single all-reduce (in place).

    dn: 0-d or [Hq]; db: 0-d. When dn and db are adjacent in one buffer (as the SSA backward
    returns them), that buffer is reduced in place with no copies; otherwise they are packed into
    `buffer` (numel >= dn.numel() + 1, same device; allocated when None) and unpacked after.
    async_op=True (adjacent case only) returns the collective's Work without waiting: the caller
    waits on it before reading dn / db, and the reduction overlaps whatever runs meanwhile.
    Returns (dn, db), or the Work when async_op is True.
    """
    import torch.distributed as dist
    k = dn.numel()
    flat = _adjacent_span(dn, db)
    if flat is not None:
        work = dist.all_reduce(flat, group=group, async_op=async_op)
        return work if async_op else (dn, db)
    if async_op:
        raise ValueError("async_op needs dn and db adjacent in one buffer (as the SSA backward "
                         "returns them)")
    buf = buffer if buffer is not None else torch.empty(k + 1, dtype=torch.float32, device=dn.device)
    buf[:k].copy_(dn.reshape(-1))
    buf[k:k + 1].copy_(db.reshape(1))
    dist.all_reduce(buf[:k + 1], group=group)
    dn.copy_(buf[:k].reshape(dn.shape))
    db.copy_(buf[k].reshape(db.shape))
    return dn, db


def _adjacent_span(dn: torch.Tensor, db: torch.Tensor) -> Optional[torch.Tensor]:
    """A 1-D view covering dn followed immediately by db, when they are laid out that way in one
    storage (dn contiguous, same dtype and device); else None."""
    k = dn.numel()
    if (db.numel() != 1 or dn.dtype != db.dtype or dn.device != db.device
            or not dn.is_contiguous()
            or dn.untyped_storage().data_ptr() != db.untyped_storage().data_ptr()
            or db.data_ptr() != dn.data_ptr() + k * dn.element_size()):
        return None
    return dn.reshape(-1).as_strided((k + 1,), (1,))
