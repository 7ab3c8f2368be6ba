"""ssa_attn_bwd_noalloc: the backward entry point that allocates nothing.

It exists for callers that cannot allocate device memory where they run the backward (for
example a binding from another host language with no device allocator, or a loop whose device
memory is all reserved by another allocator). It keeps its scratch in a fixed device array
inside the library. This file is collected last on purpose: if it fails, a run that stops at
the first failure has already run every other test.

Checked here, through the C ABI: its dq/dk/dv/dn/db equal those of the workspace-taking
ssa_attn_bwd within the tolerances the parity tests use, on two calls in a row (the second
call sees the first call's leftovers in the shared array), and an oversized problem is
rejected with SSA_ERR_WORKSPACE before anything runs.
"""

import ctypes
import math

import pytest
import torch

from oracle.ssa_oracle import max_rel
from parity_rules import assert_lowp_close, assert_scalar_close

pytestmark = pytest.mark.gpu


def _setup(dtype, cuda_device, causal=True, per_head=True):
    from SSA import ssa_triton_kernel as K
    B, Hq, Hkv, N, D = 2, 8, 2, 384, 64
    g = torch.Generator().manual_seed(77)
    q = (torch.randn(B, Hq, N, D, generator=g) * 0.5).to(dtype).to(cuda_device)
    k = (torch.randn(B, Hkv, N, D, generator=g) * 0.5).to(dtype).to(cuda_device)
    v = (torch.randn(B, Hkv, N, D, generator=g) * 0.5).to(dtype).to(cuda_device)
    do = torch.randn(B, Hq, N, D, generator=g).to(dtype).to(cuda_device)
    n = (0.3 + 0.3 * torch.rand(Hq, generator=g) if per_head else torch.tensor(1.5)).to(cuda_device)
    b = torch.tensor(0.8, device=cuda_device)
    scale = 1.0 / math.sqrt(D)
    out, m = K.ssa_flash_attn_forward(q, k, v, scale, n, b, causal=causal)
    ref = K.ssa_flash_attn_backward(q, k, v, out, do, m, scale, n, b, causal=causal)
    return dict(q=q, k=k, v=v, do=do, out=out, m=m, n=n, b=b, scale=scale, causal=causal,
                ref=ref)


def _call_noalloc(s):
    from SSA import _lib
    lib = _lib.load()
    q = s["q"]
    B, Hq, N, D = q.shape
    prob = _lib.SsaProblem(_lib.DTYPE_CODES[q.dtype], B, Hq, s["k"].shape[1], N, D,
                           1 if s["causal"] else 0, s["scale"], s["n"].data_ptr(),
                           1 if s["n"].numel() > 1 else 0, s["b"].data_ptr(), None, 0)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(s["k"]), torch.empty_like(s["v"])
    dn = torch.empty(s["n"].shape, device=q.device, dtype=torch.float32)
    db = torch.empty((), device=q.device, dtype=torch.float32)
    T = _lib.tensor_bhnd
    rc = lib.ssa_attn_bwd_noalloc(ctypes.byref(prob), T(q), T(s["k"]), T(s["v"]), T(s["out"]),
                                  T(s["do"]), s["m"].data_ptr(), T(dq), T(dk), T(dv),
                                  dn.data_ptr(), db.data_ptr(), _lib.stream_ptr(q.device))
    assert rc == _lib.SSA_OK, lib.ssa_last_error()
    torch.cuda.synchronize()
    return dq, dk, dv, dn, db


def _assert_match(dtype, got, ref):
    """The parity tests' rules (parity_rules.py): for bf16, 2e-2 + 5e-2|r| elementwise, max-abs
    2e-2 where |r| <= 4 and finite values; dn / db by the reference's scalar rule; fp32 within
    1e-5 relative."""
    for name, a, r in zip(("dq", "dk", "dv", "dn", "db"), got, ref):
        if dtype == torch.float32:
            a64, r64 = a.double().cpu(), r.double().cpu()
            assert torch.isfinite(a64).all(), name
            if name in ("dn", "db"):
                assert torch.allclose(a64, r64, rtol=1e-5, atol=1e-6), name
            else:
                assert max_rel(a64, r64) <= 1e-5, name
        elif name in ("dn", "db"):
            assert_scalar_close(name, a, r)
        else:
            assert_lowp_close(name, a, r)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_workspace_backward_twice(dtype, cuda_device):
    s = _setup(dtype, cuda_device)
    first = _call_noalloc(s)
    _assert_match(dtype, first, s["ref"])
    second = _call_noalloc(s)
    _assert_match(dtype, second, s["ref"])
    for a, b2 in zip(first, second):
        assert torch.equal(a, b2)


def test_noalloc_scalar_n_noncausal(cuda_device):
    s = _setup(torch.bfloat16, cuda_device, causal=False, per_head=False)
    _assert_match(torch.bfloat16, _call_noalloc(s), s["ref"])


def test_noalloc_rejects_problems_beyond_its_scratch(cuda_device):
    from SSA import _lib
    lib = _lib.load()
    n = torch.ones(1, device=cuda_device)
    # delta alone: 32 heads * 64 * 4096 rows * 4 B = 32 MiB > the 16 MiB array
    prob = _lib.SsaProblem(2, 64, 32, 8, 4096, 64, 1, 0.125, n.data_ptr(), 0, n.data_ptr(),
                           None, 0)
    t = _lib.SsaTensor(n.data_ptr(), 0, 0, 0)
    rc = lib.ssa_attn_bwd_noalloc(ctypes.byref(prob), t, t, t, t, t, n.data_ptr(), t, t, t,
                                  n.data_ptr(), n.data_ptr(), _lib.stream_ptr(cuda_device))
    assert rc == _lib.SSA_ERR_WORKSPACE
    assert b"16777216" in lib.ssa_last_error()
