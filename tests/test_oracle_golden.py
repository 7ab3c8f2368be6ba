"""Pin the CPU oracle against golden vectors produced by the reference's own Triton kernels
(tests/golden/make_golden.py runs training/train/train_ssa_triton/SSA/ssa_triton_kernel.py under
TRITON_INTERPRET=1 in fp32)."""

import math

import pytest
import torch

from conftest import golden_qkv, load_golden
from oracle.ssa_oracle import (attn_flops_fwd_bwd, causal_score_elements, max_rel,
                               ssa_reference_grads, ssa_reference_grads_blocked,
                               ssa_reference_grads_varlen)

CASES = load_golden()


def test_golden_cases_present():
    names = {m["name"] for m, _ in CASES}
    assert {"mha_causal_d64", "gqa_causal_d32", "gqa_noncausal_d64", "strided_causal_d32",
            "bf16vals_gqa_causal_d64", "mha_causal_d128"} <= names


@pytest.mark.parametrize("meta,arrays", CASES, ids=[m["name"] for m, _ in CASES])
def test_oracle_matches_reference_golden(meta, arrays):
    q, k, v, do = golden_qkv(meta, arrays)
    r = ssa_reference_grads(q, k, v, meta["softmax_scale"], torch.tensor(meta["ssa_n"]),
                            torch.tensor(meta["ssa_b"]), do, meta["causal"])
    # The reference runs in fp32; the oracle in fp64. fp32 accumulation error bounds this.
    for name in ("out", "dq", "dk", "dv"):
        assert max_rel(torch.from_numpy(arrays[name]), r[name]) < 5e-6, name
    assert (torch.from_numpy(arrays["m"]).double() - r["lse2"]).abs().max() < 5e-6
    for name in ("dn", "db"):
        ref = float(arrays[name])
        assert abs(ref - float(r[name])) <= 5e-5 + 1e-5 * abs(ref), name


def test_oracle_per_head_n_reduces_to_scalar():
    g = torch.Generator().manual_seed(3)
    q = torch.randn(1, 4, 64, 16, generator=g, dtype=torch.float64)
    k = torch.randn(1, 2, 64, 16, generator=g, dtype=torch.float64)
    v = torch.randn(1, 2, 64, 16, generator=g, dtype=torch.float64)
    do = torch.randn(1, 4, 64, 16, generator=g, dtype=torch.float64)
    rs = ssa_reference_grads(q, k, v, 0.25, torch.tensor(0.7), torch.tensor(0.8), do, True)
    rh = ssa_reference_grads(q, k, v, 0.25, torch.full((4,), 0.7), torch.tensor(0.8), do, True)
    assert torch.allclose(rs["out"], rh["out"])
    assert rh["dn"].shape == (4,)
    assert torch.allclose(rh["dn"].sum(), rs["dn"])


def test_oracle_gradients_match_finite_differences():
    g = torch.Generator().manual_seed(5)
    q = torch.randn(1, 2, 12, 8, generator=g, dtype=torch.float64)
    k = torch.randn(1, 1, 12, 8, generator=g, dtype=torch.float64)
    v = torch.randn(1, 1, 12, 8, generator=g, dtype=torch.float64)
    do = torch.randn(1, 2, 12, 8, generator=g, dtype=torch.float64)
    n0, b0, sc = 0.9, 0.8, 0.35
    r = ssa_reference_grads(q, k, v, sc, torch.tensor(n0), torch.tensor(b0), do, True)
    from oracle.ssa_oracle import ssa_reference_forward

    def loss(nv, bv):
        out, _ = ssa_reference_forward(q, k, v, sc, torch.tensor(nv, dtype=torch.float64),
                                       torch.tensor(bv, dtype=torch.float64), True)
        return float((out * do).sum())
    eps = 1e-6
    fd_n = (loss(n0 + eps, b0) - loss(n0 - eps, b0)) / (2 * eps)
    fd_b = (loss(n0, b0 + eps) - loss(n0, b0 - eps)) / (2 * eps)
    assert abs(fd_n - float(r["dn"])) < 1e-6 * max(1, abs(fd_n))
    assert abs(fd_b - float(r["db"])) < 1e-6 * max(1, abs(fd_b))


def test_oracle_varlen_is_per_document():
    g = torch.Generator().manual_seed(7)
    lens = [5, 17, 9]
    T = sum(lens)
    cu = torch.tensor([0, 5, 22, 31], dtype=torch.int32)
    q = torch.randn(T, 4, 16, generator=g, dtype=torch.float64)
    k = torch.randn(T, 2, 16, generator=g, dtype=torch.float64)
    v = torch.randn(T, 2, 16, generator=g, dtype=torch.float64)
    do = torch.randn(T, 4, 16, generator=g, dtype=torch.float64)
    r = ssa_reference_grads_varlen(q, k, v, cu, 0.25, torch.tensor(0.6), torch.tensor(0.8), do, True)
    # document 1 alone
    a, e = 5, 22
    r1 = ssa_reference_grads(q[a:e].permute(1, 0, 2)[None], k[a:e].permute(1, 0, 2)[None],
                             v[a:e].permute(1, 0, 2)[None], 0.25, torch.tensor(0.6),
                             torch.tensor(0.8), do[a:e].permute(1, 0, 2)[None], True)
    assert torch.allclose(r["out"][a:e], r1["out"][0].permute(1, 0, 2))
    assert torch.allclose(r["dk"][a:e], r1["dk"][0].permute(1, 0, 2))


def test_flop_convention():
    # benchmark config 2: E = 8*32*2048^2/2 = 5.369e8, FLOPs = 14*64*E = 4.810e11
    assert causal_score_elements(8, 32, 2048, True) == 536870912
    assert math.isclose(attn_flops_fwd_bwd(8, 32, 2048, 64, True), 4.810e11, rel_tol=1e-3)


@pytest.mark.parametrize("B,Hq,Hkv,N,D,causal,per_head,block", [
    (2, 4, 2, 200, 32, True, True, 64),     # GQA, ragged last block
    (1, 6, 3, 130, 16, False, False, 50),   # non-causal, scalar n
    (1, 2, 1, 97, 64, True, False, 512),    # one block wider than the sequence
])
def test_blocked_oracle_matches_autograd_oracle(B, Hq, Hkv, N, D, causal, per_head, block):
    """The blocked oracle used by the full-size GPU tests gives the autograd oracle's results."""
    g = torch.Generator().manual_seed(B * 100 + N)
    q = torch.randn(B, Hq, N, D, generator=g) * 0.5
    k = torch.randn(B, Hkv, N, D, generator=g) * 0.5
    v = torch.randn(B, Hkv, N, D, generator=g) * 0.5
    do = torch.randn(B, Hq, N, D, generator=g)
    n = 0.3 + 0.3 * torch.rand(Hq, generator=g) if per_head else torch.tensor(0.7)
    b = torch.tensor(0.8)
    r = ssa_reference_grads(q, k, v, D ** -0.5, n, b, do, causal)
    rb = ssa_reference_grads_blocked(q, k, v, D ** -0.5, n, b, do, causal, block=block)
    for name in r:
        assert rb[name].shape == r[name].shape, name
        assert (rb[name] - r[name]).abs().max() <= 1e-12 * (1 + r[name].abs().max()), name


def test_blocked_oracle_head_subset():
    """Evaluating a subset of q-heads gives those heads' rows and their share of dk/dv/dn/db."""
    g = torch.Generator().manual_seed(5)
    B, Hq, Hkv, N, D = 1, 4, 2, 96, 16
    q, do = torch.randn(B, Hq, N, D, generator=g), torch.randn(B, Hq, N, D, generator=g)
    k, v = torch.randn(B, Hkv, N, D, generator=g), torch.randn(B, Hkv, N, D, generator=g)
    n, b = 0.3 + 0.3 * torch.rand(Hq, generator=g), torch.tensor(0.8)
    do_sparse = torch.zeros_like(do)
    do_sparse[:, 2] = do[:, 2]
    full = ssa_reference_grads(q, k, v, 0.25, n, b, do_sparse, True)
    sub = ssa_reference_grads_blocked(q, k, v, 0.25, n, b, do_sparse, True, heads=[2], block=32)
    for name in ("out", "dq"):
        assert torch.allclose(sub[name][:, 2], full[name][:, 2], atol=1e-12), name
    for name in ("dk", "dv", "dn", "db"):
        assert torch.allclose(sub[name], full[name], atol=1e-12), name
