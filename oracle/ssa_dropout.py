"""CPU restatement of the attention-output dropout mask the kernels fuse into the forward epilogue
and the backward's delta pass.

TEST INFRASTRUCTURE ONLY: imported by ``tests/`` as the checker, never by the product path.

Semantics being restated. The reference applies ``nn.Dropout(p)`` to the attention output after
its kernel, in training only, under Megatron's CUDA RNG tracker
(``training/train/train_ssa_triton/SSA/ssa_triton_attention.py:110-113,186-193``): every output
element is zeroed with probability p and the survivors are scaled by 1/(1-p). The fused path draws
its keep decisions from a counter-based generator instead of torch's dropout stream (torch's mask
depends on its kernel's launch shape and cannot be reproduced element by element); the
distribution is the same.

Generator: Philox4x32-10, the counter-based generator of J. K. Salmon, M. A. Moraes, R. O. Dror and
D. E. Shaw, "Parallel random numbers: as easy as 1, 2, 3" (SC 2011). Ten rounds on a 128-bit
counter (c0, c1, c2, c3) with a 64-bit key (k0, k1); each round computes the two 32x32->64-bit
products M0*c0 and M1*c2 and permutes/xors, and the key is advanced by the Weyl increments
between rounds. The multipliers and increments are the ones the paper publishes.

Element addressing (shared with the CUDA kernels):
  * an element's index e is its position in the logical contiguous layout of the output:
    ``((z * Hq + h) * N + row) * D + d`` for dense [B, Hq, N, D], and ``(t * Hq + h) * D + d``
    for packed [T, Hq, D] (t = the row in the packed tensor);
  * elements 4c .. 4c+3 take the four 32-bit words of one Philox call with counter
    (lo32(c), hi32(c), lo32(offset), hi32(offset)) and key (lo32(seed), hi32(seed)), where
    ``seed, offset`` are the two 64-bit values of the seed tensor;
  * element e is kept iff (word >> 8) >= ceil(p * 2^24), i.e. iff the 24-bit uniform
    (word >> 8) * 2^-24 is >= p; a kept element is multiplied by 1/(1-p) computed in fp32.
"""

from __future__ import annotations

import math

import numpy as np

PHILOX_M0 = 0xD2511F53
PHILOX_M1 = 0xCD9E8D57
PHILOX_W0 = 0x9E3779B9
PHILOX_W1 = 0xBB67AE85
MASK32 = 0xFFFFFFFF


def philox4x32(ctr, key, rounds: int = 10):
    """Philox4x32-R on arrays: ctr uint32 [..., 4], key uint32 [..., 2] (broadcastable).
    Returns uint32 [..., 4]."""
    c = np.asarray(ctr, dtype=np.uint64) & MASK32
    k = np.asarray(key, dtype=np.uint64) & MASK32
    c0, c1, c2, c3 = (c[..., i] for i in range(4))
    k0, k1 = k[..., 0].copy(), k[..., 1].copy()
    for r in range(rounds):
        p0 = c0 * np.uint64(PHILOX_M0)  # exact: both factors < 2^32
        p1 = c2 * np.uint64(PHILOX_M1)
        hi0, lo0 = p0 >> np.uint64(32), p0 & np.uint64(MASK32)
        hi1, lo1 = p1 >> np.uint64(32), p1 & np.uint64(MASK32)
        c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
        if r + 1 < rounds:
            k0 = (k0 + np.uint64(PHILOX_W0)) & np.uint64(MASK32)
            k1 = (k1 + np.uint64(PHILOX_W1)) & np.uint64(MASK32)
    return np.stack([c0, c1, c2, c3], axis=-1).astype(np.uint32)


def keep_threshold(p: float) -> int:
    """Integer threshold on the 24-bit uniform: keep iff (word >> 8) >= ceil(p * 2^24)."""
    if not 0.0 <= p < 1.0:
        raise ValueError("dropout probability must be in [0, 1)")
    return int(math.ceil(float(np.float32(p)) * 16777216.0))


def keep_scale(p: float) -> float:
    """1 / (1 - p) as the kernels compute it (fp32)."""
    return float(np.float32(1.0) / (np.float32(1.0) - np.float32(p)))


def keep_mask_flat(index, seed: int, offset: int, p: float):
    """Keep decisions (bool) for flat element indices ``index`` (int64 array, any shape)."""
    idx = np.asarray(index, dtype=np.uint64)
    ctr = idx >> np.uint64(2)
    lane = (idx & np.uint64(3)).astype(np.int64)
    seed &= (1 << 64) - 1
    offset &= (1 << 64) - 1
    c = np.stack([ctr & np.uint64(MASK32), ctr >> np.uint64(32),
                  np.full_like(ctr, offset & MASK32), np.full_like(ctr, offset >> 32)], axis=-1)
    k = np.array([seed & MASK32, seed >> 32], dtype=np.uint64)
    words = philox4x32(c, k)
    w = np.take_along_axis(words, lane[..., None], axis=-1)[..., 0]
    return (w >> np.uint32(8)) >= np.uint32(keep_threshold(p))


def keep_mask_dense(B: int, Hq: int, N: int, D: int, seed: int, offset: int, p: float):
    """Keep mask [B, Hq, N, D] of a dense output."""
    idx = np.arange(B * Hq * N * D, dtype=np.int64).reshape(B, Hq, N, D)
    return keep_mask_flat(idx, seed, offset, p)


def keep_mask_packed(T: int, Hq: int, D: int, seed: int, offset: int, p: float):
    """Keep mask [T, Hq, D] of a packed output (rows are packed-tensor rows)."""
    idx = np.arange(T * Hq * D, dtype=np.int64).reshape(T, Hq, D)
    return keep_mask_flat(idx, seed, offset, p)


def seed_pair(seed_tensor) -> tuple:
    """The two 64-bit values of a seed tensor (int64 [2], device or host) as Python ints."""
    vals = [int(x) for x in seed_tensor.detach().cpu().reshape(-1).tolist()[:2]]
    return vals[0] & ((1 << 64) - 1), vals[1] & ((1 << 64) - 1)
