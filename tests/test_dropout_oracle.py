"""Output dropout on the CPU: the oracle's Philox4x32-10 against the published known-answer
vectors, the keep rule, and the host-side validation of the dropout arguments (no GPU).

Known-answer vectors: the Random123 distribution's kat_vectors for philox4x32 (counter, key ->
output, 7 and 10 rounds), the test vectors of the generator's authors (Salmon et al., SC 2011).
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle.ssa_dropout import (keep_mask_dense, keep_mask_flat, keep_mask_packed, keep_scale,
                                keep_threshold, philox4x32)

KAT = [
    # rounds, counter (4 words), key (2 words), expected output (4 words)
    (7, (0, 0, 0, 0), (0, 0), (0x5F6FB709, 0x0D893F64, 0x4F121F81, 0x4F730A48)),
    (7, (0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0x4DFCCABA, 0x190A87F0, 0xC47362BA, 0xB6B5242A)),
    (10, (0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    (10, (0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    (10, (0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


@pytest.mark.parametrize("rounds,ctr,key,want", KAT)
def test_philox_known_answers(rounds, ctr, key, want):
    got = philox4x32(np.array(ctr, dtype=np.uint64), np.array(key, dtype=np.uint64), rounds)
    assert tuple(int(x) for x in got) == want


def test_philox_vectorised_matches_scalar_calls():
    rng = np.random.default_rng(0)
    ctr = rng.integers(0, 2 ** 32, size=(64, 4), dtype=np.uint64)
    key = rng.integers(0, 2 ** 32, size=(2,), dtype=np.uint64)
    many = philox4x32(ctr, key)
    for i in range(0, 64, 9):
        assert (philox4x32(ctr[i], key) == many[i]).all()


def test_keep_rule():
    assert keep_threshold(0.0) == 0 and keep_threshold(0.5) == 1 << 23
    assert keep_threshold(0.1) == int(np.ceil(float(np.float32(0.1)) * 2 ** 24))
    assert keep_scale(0.5) == 2.0
    with pytest.raises(ValueError):
        keep_threshold(1.0)
    # each element uses word e % 4 of the call for counter e // 4
    seed, off = 0x1234_5678_9ABC_DEF0, 0x0F0E_0D0C_0B0A_0908
    idx = np.arange(64, dtype=np.int64)
    m = keep_mask_flat(idx, seed, off, 0.3)
    thr = keep_threshold(0.3)
    for e in (0, 1, 2, 3, 17, 63):
        c = e // 4
        w = philox4x32(np.array([c & 0xFFFFFFFF, c >> 32, off & 0xFFFFFFFF, off >> 32],
                                dtype=np.uint64),
                       np.array([seed & 0xFFFFFFFF, seed >> 32], dtype=np.uint64))[e % 4]
        assert bool(m[e]) == (int(w) >> 8 >= thr)
    # the dense and packed layouts index the same flat positions
    assert (keep_mask_dense(2, 3, 5, 8, seed, off, 0.3).reshape(-1)
            == keep_mask_flat(np.arange(240), seed, off, 0.3)).all()
    assert keep_mask_packed(5, 3, 8, seed, off, 0.3).shape == (5, 3, 8)


def test_keep_fraction():
    m = keep_mask_flat(np.arange(1 << 18), 7, 11, 0.25)
    assert abs(m.mean() - 0.75) < 0.005


def test_capi_validates_dropout_arguments():
    """dropout_p outside [0, 1) and dropout_p > 0 without a seed are rejected by the library's
    problem check (no device work; ssa_attn_kernel_family only validates)."""
    from SSA import _lib
    lib = _lib.load()
    n = ctypes.c_float(0.5)
    base = dict(dtype=2, B=1, Hq=2, Hkv=2, N=64, D=64, causal=1, softmax_scale=0.125,
                ssa_n=ctypes.addressof(n), n_per_head=0, ssa_b=ctypes.addressof(n))
    seed = (ctypes.c_uint64 * 2)(1, 2)
    ok = _lib.SsaProblem(**base, dropout_p=0.1, dropout_seed=ctypes.addressof(seed))
    assert lib.ssa_attn_kernel_family(ctypes.byref(ok)) == 1
    for bad in (_lib.SsaProblem(**base, dropout_p=1.0, dropout_seed=ctypes.addressof(seed)),
                _lib.SsaProblem(**base, dropout_p=-0.1, dropout_seed=ctypes.addressof(seed))):
        assert lib.ssa_attn_kernel_family(ctypes.byref(bad)) == -1
    noseed = _lib.SsaProblem(**base, dropout_p=0.2)
    assert lib.ssa_attn_kernel_family(ctypes.byref(noseed)) == -1
    assert b"dropout_seed" in lib.ssa_last_error()


def test_wrapper_rejects_bad_dropout_arguments():
    from SSA.ssa_triton_kernel import _dropout_args
    dev = torch.device("cpu")
    assert _dropout_args(0.0, None, dev) == (0.0, None)
    with pytest.raises(ValueError):
        _dropout_args(0.1, None, dev)
    with pytest.raises(ValueError):
        _dropout_args(1.0, torch.zeros(2, dtype=torch.int64), dev)
    with pytest.raises(ValueError):
        _dropout_args(0.1, torch.zeros(2, dtype=torch.int32), dev)
    s = torch.zeros(2, dtype=torch.int64)
    assert _dropout_args(0.1, s, dev)[1] is s
