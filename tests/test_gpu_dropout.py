"""GPU: output dropout fused into the kernels, against the CPU oracle.

The reference drops attention-output elements with ``nn.Dropout`` after its kernel
(ssa_triton_attention.py:110-113,186-193). With ``dropout_p`` and a seed the forward's epilogue
applies the mask and the backward's delta pass masks the incoming gradient. Checked here:
  * the keep mask the kernels used is exactly the oracle's Philox4x32-10 mask for the seed
    (oracle/ssa_dropout.py, pinned to the generator's known-answer vectors): bit-exact;
  * the dropped output equals the undropped output times keep / (1 - p), within the output
    dtype's rounding (one bf16 rounding of the scaled value against a rounding before scaling);
  * the gradients equal the fp64 oracle's gradients of sum(dropout(out) * g), i.e. the oracle
    run with dout = g * keep / (1 - p), with the parity tests' tolerances (parity_rules.py);
  * every kernel family: tcgen05 D = 32 / 64 / 128, generic fp32 and D = 16, packed documents;
  * the module in training and eval mode, and the SSA_FUSED_DROPOUT=0 fallback.
"""

import numpy as np
import pytest
import torch

from oracle.ssa_dropout import keep_mask_dense, keep_mask_packed, keep_scale, seed_pair
from oracle.ssa_oracle import max_rel, ssa_reference_grads, ssa_reference_grads_varlen
from parity_rules import assert_lowp_close, assert_scalar_close

pytestmark = pytest.mark.gpu


def _api():
    from SSA import ssa_triton_kernel as K
    return K


def _inputs(B, Hq, Hkv, N, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, Hq, N, D, generator=g) * 0.5).to(dtype)
    k = (torch.randn(B, Hkv, N, D, generator=g) * 0.5).to(dtype)
    v = (torch.randn(B, Hkv, N, D, generator=g) * 0.5).to(dtype)
    do = torch.randn(B, Hq, N, D, generator=g).to(dtype)
    return q, k, v, do


def _check_out(name, dropped, plain, keep, p, dtype):
    """dropped == plain * keep / (1 - p) up to the output rounding; zero exactly where dropped."""
    d = dropped.detach().double().cpu()
    u = plain.detach().double().cpu()
    keep_t = torch.from_numpy(keep)
    assert (d[~keep_t] == 0).all(), f"{name}: dropped elements not zero"
    nz = keep_t & (u != 0)
    assert (d[nz] != 0).all(), f"{name}: kept elements zeroed"
    want = u * keep_scale(p)
    # two roundings (the kernel's of the scaled value, the undropped output's) of half an ulp
    # each; below fp16's normal range its ulp is the fixed subnormal spacing 2^-24
    tol = 1e-6 if dtype == torch.float32 else 2.0 ** -6
    floor = 2.0 ** -22 if dtype == torch.float16 else 0.0
    excess = ((d - want).abs() - tol * want.abs() - floor)[nz].max()
    assert excess <= 0, f"{name}: kept values off by {excess:.3e} beyond the rounding bound"


CASES = [
    # B, Hq, Hkv, N, D, dtype, causal, p
    (2, 4, 2, 256, 64, torch.bfloat16, True, 0.1),
    (1, 4, 1, 200, 64, torch.bfloat16, False, 0.5),
    (1, 4, 2, 192, 128, torch.bfloat16, True, 0.25),
    (2, 6, 2, 160, 32, torch.float16, True, 0.3),
    (1, 2, 2, 96, 64, torch.float32, True, 0.2),
    (1, 2, 1, 80, 16, torch.bfloat16, True, 0.4),
]


@pytest.mark.parametrize("B,Hq,Hkv,N,D,dtype,causal,p", CASES,
                         ids=[f"D{c[4]}-{str(c[5])[6:]}-p{c[7]}" for c in CASES])
def test_dropout_forward_backward(B, Hq, Hkv, N, D, dtype, causal, p, cuda_device):
    K = _api()
    q, k, v, g = _inputs(B, Hq, Hkv, N, D, dtype, seed=D + N)
    n = torch.tensor(0.45)
    b = torch.tensor(0.8)
    scale = D ** -0.5
    dev = cuda_device
    qd, kd, vd, gd, nd, bd = (t.to(dev) for t in (q, k, v, g, n, b))
    seed = K.make_dropout_seed(dev)
    plain, m0 = K.ssa_flash_attn_forward(qd, kd, vd, scale, nd, bd, causal)
    out, m = K.ssa_flash_attn_forward(qd, kd, vd, scale, nd, bd, causal, dropout_p=p,
                                      dropout_seed=seed)
    dq, dk, dv, dn, db = K.ssa_flash_attn_backward(qd, kd, vd, out, gd, m, scale, nd, bd, causal,
                                                   dropout_p=p, dropout_seed=seed)
    torch.cuda.synchronize()
    assert torch.equal(m, m0), "lse must be the undropped normaliser"
    s0, s1 = seed_pair(seed)
    keep = keep_mask_dense(B, Hq, N, D, s0, s1, p)
    _check_out("out", out, plain, keep, p, dtype)
    # gradients of sum(dropout(out) * g) = the oracle's gradients for dout = g * keep / (1 - p)
    g_eff = g.double() * torch.from_numpy(keep).double() * keep_scale(p)
    ref = ssa_reference_grads(q, k, v, scale, n, b, g_eff, causal)
    if dtype == torch.float32:
        for name, got in (("dq", dq), ("dk", dk), ("dv", dv)):
            assert max_rel(got.cpu(), ref[name]) <= 1e-5, name
        for name, got in (("dn", dn), ("db", db)):
            r = float(ref[name])
            assert abs(float(got) - r) <= 1e-5 * abs(r) + 1e-6, (name, float(got), r)
    else:
        for name, got in (("dq", dq), ("dk", dk), ("dv", dv)):
            assert_lowp_close(name, got, ref[name])
        assert_scalar_close("dn", dn, ref["dn"])
        assert_scalar_close("db", db, ref["db"])


def test_dropout_fraction_and_fresh_seeds(cuda_device):
    """About p of the outputs are dropped, and consecutive seeds give different masks."""
    K = _api()
    q, k, v, _ = _inputs(2, 8, 2, 512, 64, torch.bfloat16, seed=5)
    qd, kd, vd = (t.to(cuda_device) for t in (q, k, v))
    n, b = torch.tensor(0.4, device=cuda_device), torch.tensor(0.8, device=cuda_device)
    s1, s2 = K.make_dropout_seed(cuda_device), K.make_dropout_seed(cuda_device)
    o1, _ = K.ssa_flash_attn_forward(qd, kd, vd, 0.125, n, b, True, dropout_p=0.3, dropout_seed=s1)
    o2, _ = K.ssa_flash_attn_forward(qd, kd, vd, 0.125, n, b, True, dropout_p=0.3, dropout_seed=s2)
    o1b, _ = K.ssa_flash_attn_forward(qd, kd, vd, 0.125, n, b, True, dropout_p=0.3,
                                      dropout_seed=s1)
    frac = float((o1 == 0).float().mean())
    assert abs(frac - 0.3) < 0.01, frac
    assert not torch.equal(o1 == 0, o2 == 0)
    assert torch.equal(o1, o1b), "the same seed must give the same output"


def test_dropout_packed_documents(cuda_device):
    """Packed documents: the mask follows the packed rows ((t * Hq + h) * D + d)."""
    K = _api()
    lens = [150, 64, 300]
    T, Hq, Hkv, D, p = sum(lens), 4, 2, 64, 0.2
    g = torch.Generator().manual_seed(3)
    q = (torch.randn(T, Hq, D, generator=g) * 0.5).bfloat16()
    k = (torch.randn(T, Hkv, D, generator=g) * 0.5).bfloat16()
    v = (torch.randn(T, Hkv, D, generator=g) * 0.5).bfloat16()
    gr = torch.randn(T, Hq, D, generator=g).bfloat16()
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
    n, b = torch.tensor(0.5), torch.tensor(0.8)
    dev = cuda_device
    qd, kd, vd, gd, cud, nd, bd = (t.to(dev) for t in (q, k, v, gr, cu, n, b))
    seed = K.make_dropout_seed(dev)
    plain, _ = K.ssa_flash_attn_varlen_forward(qd, kd, vd, cud, max(lens), D ** -0.5, nd, bd, True)
    out, lse = K.ssa_flash_attn_varlen_forward(qd, kd, vd, cud, max(lens), D ** -0.5, nd, bd, True,
                                               dropout_p=p, dropout_seed=seed)
    dq, dk, dv, dn, db = K.ssa_flash_attn_varlen_backward(
        qd, kd, vd, out, gd, lse, cud, max(lens), D ** -0.5, nd, bd, True, dropout_p=p,
        dropout_seed=seed)
    torch.cuda.synchronize()
    s0, s1 = seed_pair(seed)
    keep = keep_mask_packed(T, Hq, D, s0, s1, p)
    _check_out("out", out, plain, keep, p, torch.bfloat16)
    g_eff = gr.double() * torch.from_numpy(keep).double() * keep_scale(p)
    ref = ssa_reference_grads_varlen(q, k, v, cu, D ** -0.5, n, b, g_eff, True)
    for name, got in (("dq", dq), ("dk", dk), ("dv", dv)):
        assert_lowp_close(name, got, ref[name])
    assert_scalar_close("dn", dn, ref["dn"])
    assert_scalar_close("db", db, ref["db"])


def test_dropout_deterministic_mode(cuda_device):
    """With the deterministic backward, two runs with the same seed are bit-identical."""
    K = _api()
    q, k, v, g = _inputs(2, 4, 2, 384, 64, torch.bfloat16, seed=9)
    qd, kd, vd, gd = (t.to(cuda_device) for t in (q, k, v, g))
    n, b = torch.tensor(0.4, device=cuda_device), torch.tensor(0.8, device=cuda_device)
    seed = K.make_dropout_seed(cuda_device)
    runs = []
    for _ in range(2):
        out, m = K.ssa_flash_attn_forward(qd, kd, vd, 0.125, n, b, True, dropout_p=0.2,
                                          dropout_seed=seed)
        runs.append((out,) + K.ssa_flash_attn_backward(qd, kd, vd, out, gd, m, 0.125, n, b, True,
                                                       deterministic=True, dropout_p=0.2,
                                                       dropout_seed=seed))
    for a, c in zip(*runs):
        assert torch.equal(a, c)


def _module(dropout, n_heads=4, kv=2, D=64):
    from SSA.ssa_triton_attention import SSAAttentionConfig, SSATritonAttention
    cfg = SSAAttentionConfig(num_attention_heads=n_heads, kv_channels=D, num_query_groups=kv,
                             attention_dropout=dropout)
    with pytest.warns(UserWarning):
        return SSATritonAttention(cfg, layer_number=1)


def test_module_fused_dropout_train_and_eval(cuda_device, monkeypatch):
    """Training mode drops about p of the context (fused, no nn.Dropout launch) and the gradient
    flows through the mask; eval mode and SSA_FUSED_DROPOUT=0 behave like the reference module."""
    from SSA import _lib
    mod = _module(0.25).to(cuda_device)
    S, B, Hq, Hkv, D = 256, 2, 4, 2, 64
    g = torch.Generator().manual_seed(1)
    qm = (torch.randn(S, B, Hq, D, generator=g) * 0.5).bfloat16().to(cuda_device)
    km = (torch.randn(S, B, Hkv, D, generator=g) * 0.5).bfloat16().to(cuda_device)
    vm = (torch.randn(S, B, Hkv, D, generator=g) * 0.5).bfloat16().to(cuda_device)
    qm.requires_grad_(True)
    mod.train()
    n0 = _lib.launch_count()
    ctx = mod(qm, km, vm, None)
    assert ctx.shape == (S, B, Hq * D)
    frac = float((ctx == 0).float().mean())
    assert abs(frac - 0.25) < 0.02, frac
    ctx.float().sum().backward()
    assert torch.isfinite(qm.grad.float()).all() and qm.grad.abs().sum() > 0
    assert _lib.launch_count() - n0 >= 4  # forward + preprocess + backward + conversion
    mod.eval()
    with torch.no_grad():
        ev = mod(qm, km, vm, None)
    assert float((ev == 0).float().mean()) < 0.01
    monkeypatch.setenv("SSA_FUSED_DROPOUT", "0")
    mod.train()
    with torch.no_grad():
        eager = mod(qm, km, vm, None)
    assert abs(float((eager == 0).float().mean()) - 0.25) < 0.02
    kept = eager != 0
    assert torch.allclose(eager[kept].float(), (ev[kept].float() / 0.75), rtol=2e-2, atol=1e-3)
