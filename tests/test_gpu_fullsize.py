"""GPU parity at the benchmarked sizes: the kernels run over whole benchmark workloads (configs 2,
3 and 4) and slices of their outputs are checked against the blocked fp64 oracle
(oracle.ssa_oracle.ssa_reference_grads_blocked, itself pinned to the autograd oracle on the CPU).

Long rows and long sums are where a kernel can drift while small cases stay green: the forward's
running normaliser over 32,768 keys, dK/dV accumulated over 32,768 queries, and dn / db summed over
up to 5.4e8 score elements in fp32 partials. Tolerances are the parity tests' (parity_rules.py).

To keep the oracle's CPU time bounded, dO is non-zero only on the slices that are checked. Every
gradient is a sum of dS = P (dP - delta) terms, and dP and delta vanish with dO, so the gradients
of the other slices must then be exactly zero and dn / db are sums over the checked slices alone;
the forward still runs on the full random inputs.
"""

import math

import pytest
import torch

from oracle.ssa_oracle import ssa_reference_grads_blocked
from parity_rules import assert_lowp_close, assert_scalar_close

pytestmark = pytest.mark.gpu


def _api():
    from SSA import ssa_triton_kernel as K
    return K


def _inputs(shape_q, shape_kv, seed):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(*shape_q, generator=g) * 0.5).to(torch.bfloat16)
    k = (torch.randn(*shape_kv, generator=g) * 0.5).to(torch.bfloat16)
    v = (torch.randn(*shape_kv, generator=g) * 0.5).to(torch.bfloat16)
    do = torch.randn(*shape_q, generator=g).to(torch.bfloat16)
    n = 0.3 + 0.3 * torch.rand(shape_q[-3] if len(shape_q) == 4 else shape_q[1], generator=g)
    return q, k, v, do, n


def test_config4_full_length(cuda_device):
    """Config 4 at full size: B=1, Hq=32, Hkv=8, S=32768, D=128, bf16, causal, per-head n. q-head 13
    (kv-head 3) is checked over all 32,768 rows: out, lse, dq, dk / dv of kv-head 3, dn[13], db."""
    K = _api()
    B, Hq, Hkv, N, D = 1, 32, 8, 32768, 128
    h0 = 13
    hk = h0 // (Hq // Hkv)
    q, k, v, do, n = _inputs((B, Hq, N, D), (B, Hkv, N, D), seed=4)
    do_sparse = torch.zeros_like(do)
    do_sparse[:, h0] = do[:, h0]
    b = torch.tensor(0.8)
    dev = cuda_device
    scale = 1.0 / math.sqrt(D)
    qd, kd, vd, dod, nd, bd = (t.to(dev) for t in (q, k, v, do_sparse, n, b))
    out, m = K.ssa_flash_attn_forward(qd, kd, vd, scale, nd, bd, causal=True)
    dq, dk, dv, dn, db = K.ssa_flash_attn_backward(qd, kd, vd, out, dod, m, scale, nd, bd, True)
    torch.cuda.synchronize()
    ref = ssa_reference_grads_blocked(q, k, v, scale, n, b, do_sparse, True, heads=[h0],
                                      block=1024)
    assert_lowp_close("out", out[:, h0], ref["out"][:, h0])
    assert (m[:, h0].double().cpu() - ref["lse2"][:, h0]).abs().max() < 2e-3
    assert_lowp_close("dq", dq[:, h0], ref["dq"][:, h0])
    assert_lowp_close("dk", dk[:, hk], ref["dk"][:, hk])
    assert_lowp_close("dv", dv[:, hk], ref["dv"][:, hk])
    assert_scalar_close("dn[13]", dn[h0], ref["dn"][h0])
    assert_scalar_close("db", db, ref["db"])
    # no dO elsewhere: every other gradient is exactly zero
    others = [h for h in range(Hq) if h != h0]
    assert (dq[:, others] == 0).all()
    assert (dk[:, [h for h in range(Hkv) if h != hk]] == 0).all()
    assert (dv[:, [h for h in range(Hkv) if h != hk]] == 0).all()
    assert (dn[others] == 0).all()
    assert torch.isfinite(out.float()).all() and torch.isfinite(m).all()


def test_config3_full_packing(cuda_device):
    """Config 3 at full size: the benchmark's seeded packing of 65,536 tokens (33 documents,
    lengths U[128, 4096]), Hq=32, Hkv=8, D=64, bf16, causal, per-head n. Checked for kv-head 5
    (q-heads 20..23) on four documents: the longest, the shortest, the first and the last
    (clipped) one: out, lse, dq, dk, dv, dn[20:24] and db."""
    import bench
    K = _api()
    lens = bench.c3_doc_lengths()
    T, Hq, Hkv, D = sum(lens), 32, 8, 64
    assert T == 65536
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    docs = sorted({max(range(len(lens)), key=lambda i: lens[i]),
                   min(range(len(lens)), key=lambda i: lens[i]), 0, len(lens) - 1})
    hk, heads = 5, list(range(20, 24))
    q, k, v, do, n = _inputs((T, Hq, D), (T, Hkv, D), seed=3)
    do_sparse = torch.zeros_like(do)
    for z in docs:
        a, e = int(cu[z]), int(cu[z + 1])
        do_sparse[a:e, 20:24] = do[a:e, 20:24]
    b = torch.tensor(0.8)
    dev = cuda_device
    scale = D ** -0.5
    qd, kd, vd, dod, nd, bd, cud = (t.to(dev) for t in (q, k, v, do_sparse, n, b, cu))
    out, lse = K.ssa_flash_attn_varlen_forward(qd, kd, vd, cud, max(lens), scale, nd, bd, True)
    dq, dk, dv, dn, db = K.ssa_flash_attn_varlen_backward(qd, kd, vd, out, dod, lse, cud,
                                                          max(lens), scale, nd, bd, True)
    torch.cuda.synchronize()
    out, lse, dq, dk, dv = (t.cpu() for t in (out, lse, dq, dk, dv))
    dn_ref = torch.zeros(Hq, dtype=torch.float64)
    db_ref = torch.zeros((), dtype=torch.float64)
    for z in docs:
        a, e = int(cu[z]), int(cu[z + 1])
        as_bhnd = lambda t: t[a:e].permute(1, 0, 2).unsqueeze(0)  # noqa: E731
        r = ssa_reference_grads_blocked(as_bhnd(q), as_bhnd(k), as_bhnd(v), scale, n, b,
                                        as_bhnd(do_sparse), True, heads=heads, block=1024)
        as_thd = lambda t: t[0].permute(1, 0, 2)  # noqa: E731
        tag = f"doc {z} (L={e - a})"
        assert_lowp_close(f"out {tag}", out[a:e, 20:24], as_thd(r["out"])[:, 20:24])
        assert (lse[20:24, a:e].double() - r["lse2"][0, 20:24]).abs().max() < 2e-3, tag
        assert_lowp_close(f"dq {tag}", dq[a:e, 20:24], as_thd(r["dq"])[:, 20:24])
        assert_lowp_close(f"dk {tag}", dk[a:e, hk], as_thd(r["dk"])[:, hk])
        assert_lowp_close(f"dv {tag}", dv[a:e, hk], as_thd(r["dv"])[:, hk])
        dn_ref += r["dn"]
        db_ref += r["db"]
    assert_scalar_close("dn[20:24]", dn[20:24], dn_ref[20:24])
    assert_scalar_close("db", db, db_ref)
    assert (dn[[h for h in range(Hq) if h not in heads]] == 0).all()
    rows = torch.zeros(T, dtype=torch.bool)
    for z in docs:
        rows[int(cu[z]):int(cu[z + 1])] = True
    assert (dq[~rows] == 0).all() and (dk[~rows] == 0).all() and (dv[~rows] == 0).all()
    assert (dq[:, [h for h in range(Hq) if h not in heads]] == 0).all()
    assert (dk[:, [h for h in range(Hkv) if h != hk]] == 0).all()
    assert (dv[:, [h for h in range(Hkv) if h != hk]] == 0).all()
    assert torch.isfinite(out.float()).all() and torch.isfinite(lse).all()


def test_config2_full_size_dn(cuda_device):
    """Config 2 at full size (B=8, Hq=32, Hkv=8, S=2048, D=64, bf16, causal, per-head n, dO random
    everywhere): kv-head 5 is checked across all 8 sequences, including dn[20:24], which sums
    ds_ssa sign(s) log1p(b|s|) over 6.7e7 score elements per group (the reference Kahan-compensates
    these sums, ssa_triton_kernel.py:386-397; here they are per-thread fp32 partials reduced in
    fp64)."""
    K = _api()
    B, Hq, Hkv, N, D = 8, 32, 8, 2048, 64
    q, k, v, do, n = _inputs((B, Hq, N, D), (B, Hkv, N, D), seed=0)
    b = torch.tensor(0.8)
    dev = cuda_device
    scale = D ** -0.5
    qd, kd, vd, dod, nd, bd = (t.to(dev) for t in (q, k, v, do, n, b))
    out, m = K.ssa_flash_attn_forward(qd, kd, vd, scale, nd, bd, causal=True)
    dq, dk, dv, dn, db = K.ssa_flash_attn_backward(qd, kd, vd, out, dod, m, scale, nd, bd, True)
    torch.cuda.synchronize()
    hk, hs = 5, slice(20, 24)
    ref = ssa_reference_grads_blocked(q[:, hs], k[:, hk:hk + 1], v[:, hk:hk + 1], scale, n[hs], b,
                                      do[:, hs], True, block=1024)
    assert_lowp_close("out", out[:, hs], ref["out"])
    assert_lowp_close("dq", dq[:, hs], ref["dq"])
    assert_lowp_close("dk", dk[:, hk:hk + 1], ref["dk"])
    assert_lowp_close("dv", dv[:, hk:hk + 1], ref["dv"])
    assert_scalar_close("dn[20:24]", dn[hs], ref["dn"])
    for t in (out, m, dq, dk, dv, dn, db):
        assert torch.isfinite(t.float()).all()
