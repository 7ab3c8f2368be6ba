"""GPU parity: the CUDA kernels (through libssa_b200.so's C ABI) against the CPU oracle and the
reference's golden vectors, on identical seeded inputs.

Tolerances (written here, applied below):
  * fp32 inputs (generic kernels): max|a-r| / max|r| <= 1e-5 for out/dq/dk/dv, and
    |a-r| <= 1e-5 * |r| + 1e-6 for dn/db.
  * bf16/fp16 inputs (tcgen05 kernels for D in {32,64,128}): against the fp64 oracle evaluated on
    the same 16-bit inputs, elementwise |a-r| <= 2e-2 + 5e-2 |r| (the reference's own bf16 rule,
    check_ssa_triton_parity.py:1059-1062) AND max-abs <= 2e-2 wherever |r| <= 4 (bf16 cannot
    represent values above 4 to within 2e-2 absolute: its spacing there is 2^-5);
    dn/db: |a-r| <= 2e-3 + 2e-2 |r| (check_ssa_triton_parity.py:1066-1067).
    The rules live in parity_rules.py.
"""

import math

import pytest
import torch

from conftest import golden_qkv, load_golden
from oracle.ssa_oracle import max_rel, ssa_reference_grads, ssa_reference_grads_varlen
from parity_rules import assert_lowp_close, assert_scalar_close

pytestmark = pytest.mark.gpu

GOLDEN = load_golden()


def _api():
    from SSA import ssa_triton_kernel as K
    return K


def run_fwd_bwd(q, k, v, do, scale, n, b, causal):
    K = _api()
    out, m = K.ssa_flash_attn_forward(q, k, v, scale, n, b, causal=causal)
    dq, dk, dv, dn, db = K.ssa_flash_attn_backward(q, k, v, out, do, m, scale, n, b, causal=causal)
    torch.cuda.synchronize()
    return dict(out=out, m=m, dq=dq, dk=dk, dv=dv, dn=dn, db=db)


def seeded(shape, seed, scale=1.0, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype)


# ----------------------------------------------------------------------------- golden vectors
@pytest.mark.parametrize("meta,arrays", GOLDEN, ids=[m["name"] for m, _ in GOLDEN])
def test_golden_fp32(meta, arrays, cuda_device):
    q, k, v, do = golden_qkv(meta, arrays, device=cuda_device)
    n = torch.tensor(meta["ssa_n"], device=cuda_device)
    b = torch.tensor(meta["ssa_b"], device=cuda_device)
    r = run_fwd_bwd(q, k, v, do, meta["softmax_scale"], n, b, meta["causal"])
    for name in ("out", "dq", "dk", "dv"):
        err = max_rel(r[name].cpu(), torch.from_numpy(arrays[name]))
        assert err <= 1e-5, f"{name}: max-rel {err:.3e}"
    assert (r["m"].cpu().double() - torch.from_numpy(arrays["m"]).double()).abs().max() < 1e-5
    for name in ("dn", "db"):
        ref = float(arrays[name])
        assert abs(float(r[name]) - ref) <= 1e-5 * abs(ref) + 1e-6, (name, float(r[name]), ref)


@pytest.mark.parametrize("meta,arrays", GOLDEN, ids=[m["name"] for m, _ in GOLDEN])
def test_golden_bf16(meta, arrays, cuda_device):
    """bf16 inputs against the fp64 oracle on the same bf16 values; for the case whose inputs
    are bf16-representable the reference's fp32 golden outputs are checked directly too."""
    q, k, v, do = golden_qkv(meta, arrays, device=cuda_device, dtype=torch.bfloat16)
    n = torch.tensor(meta["ssa_n"], device=cuda_device)
    b = torch.tensor(meta["ssa_b"], device=cuda_device)
    r = run_fwd_bwd(q, k, v, do, meta["softmax_scale"], n, b, meta["causal"])
    ref = ssa_reference_grads(q.cpu(), k.cpu(), v.cpu(), meta["softmax_scale"], n.cpu(), b.cpu(),
                              do.cpu(), meta["causal"])
    for name in ("out", "dq", "dk", "dv"):
        assert_lowp_close(name, r[name], ref[name])
    assert_scalar_close("dn", r["dn"], ref["dn"])
    assert_scalar_close("db", r["db"], ref["db"])
    if meta["bf16_representable"]:
        for name in ("out", "dq", "dk", "dv"):
            assert_lowp_close(name + "(golden)", r[name], torch.from_numpy(arrays[name]))
        assert_scalar_close("dn(golden)", r["dn"], float(arrays["dn"]))


# ----------------------------------------------------------------------------- tensor-core path
CASES = [
    # B, Hq, Hkv, N, D, causal, dtype, per_head_n
    (2, 8, 2, 512, 64, True, torch.bfloat16, False),
    (1, 4, 4, 512, 64, False, torch.bfloat16, False),
    (1, 8, 2, 384, 64, True, torch.bfloat16, True),
    (2, 4, 1, 200, 64, True, torch.bfloat16, False),    # ragged: N not a tile multiple
    (1, 4, 1, 333, 64, False, torch.bfloat16, True),
    (1, 4, 2, 256, 128, True, torch.bfloat16, False),
    (1, 2, 1, 300, 128, False, torch.bfloat16, False),
    (1, 8, 2, 256, 64, True, torch.float16, True),
    (1, 4, 4, 130, 128, True, torch.float16, False),
    (1, 4, 2, 64, 64, True, torch.bfloat16, False),     # shorter than one tile
    (1, 6, 2, 256, 64, True, torch.bfloat16, True),     # GQA ratio 3 (not a power of two)
    (2, 4, 2, 144, 64, True, torch.bfloat16, False),    # one tile + 16: a lone 16-query chunk
    (1, 4, 1, 47, 64, True, torch.bfloat16, True),      # ragged inside the first 16-query chunk
    (1, 6, 3, 144, 128, True, torch.bfloat16, True),    # D = 128, GQA 2, ragged
    # D = 32 runs the D = 64 kernels, whose TMA boxes zero-fill columns 32..63
    (2, 8, 2, 512, 32, True, torch.bfloat16, False),
    (1, 4, 2, 300, 32, False, torch.float16, True),     # non-causal, ragged, fp16
    (1, 24, 8, 256, 32, True, torch.bfloat16, True),    # 24 heads of 32 (GQA 3)
    (2, 4, 1, 200, 32, True, torch.bfloat16, True),     # ragged, GQA 4
]


@pytest.mark.parametrize("B,Hq,Hkv,N,D,causal,dtype,per_head", CASES)
def test_kernel_vs_oracle(B, Hq, Hkv, N, D, causal, dtype, per_head, cuda_device):
    K = _api()
    seed = B * 1000 + Hq * 100 + N + D
    q = seeded((B, Hq, N, D), seed, 0.5, dtype)
    k = seeded((B, Hkv, N, D), seed + 1, 0.5, dtype)
    v = seeded((B, Hkv, N, D), seed + 2, 0.5, dtype)
    do = seeded((B, Hq, N, D), seed + 3, 1.0, dtype)
    if per_head:
        n = 0.3 + 0.3 * torch.rand(Hq, generator=torch.Generator().manual_seed(seed + 4))
    else:
        n = torch.tensor(0.43)
    b = torch.tensor(0.8)
    scale = 1.0 / math.sqrt(D)
    assert K.kernel_family(q.to(cuda_device), scale) == 1
    r = run_fwd_bwd(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), do.to(cuda_device),
                    scale, n.to(cuda_device), b.to(cuda_device), causal)
    ref = ssa_reference_grads(q, k, v, scale, n, b, do, causal)
    for name in ("out", "dq", "dk", "dv"):
        assert_lowp_close(name, r[name], ref[name])
    assert (r["m"].cpu().double() - ref["lse2"]).abs().max() < 2e-3
    assert r["dn"].shape == n.shape
    assert_scalar_close("dn", r["dn"], ref["dn"])
    assert_scalar_close("db", r["db"], ref["db"])


@pytest.mark.parametrize("D", [32, 64, 128])
def test_qhead_slices_of_a_key_block(D, cuda_device, monkeypatch):
    """With few sequences the backward splits each key block's GQA q-heads over 2 or 4 CTAs
    (their fp32 dK / dV partials are summed in slice order by the dq conversion). Every split,
    forced here through SSA_BWD_HSPLIT, matches the oracle, and dK / dV differ between splits by
    rounding only."""
    K = _api()
    B, Hq, Hkv, N = 1, 8, 2, 700  # ragged last key block
    q = seeded((B, Hq, N, D), 301, 0.5)
    k = seeded((B, Hkv, N, D), 302, 0.5)
    v = seeded((B, Hkv, N, D), 303, 0.5)
    do = seeded((B, Hq, N, D), 304)
    n = 0.3 + 0.3 * torch.rand(Hq, generator=torch.Generator().manual_seed(305))
    b = torch.tensor(0.8)
    scale = D ** -0.5
    ref = ssa_reference_grads(q, k, v, scale, n, b, do, True)
    dev = cuda_device
    got = {}
    for s in (1, 2, 4):
        monkeypatch.setenv("SSA_BWD_HSPLIT", str(s))
        r = run_fwd_bwd(q.to(dev), k.to(dev), v.to(dev), do.to(dev), scale, n.to(dev),
                        b.to(dev), True)
        for name in ("out", "dq", "dk", "dv"):
            assert_lowp_close(f"{name} (slices {s})", r[name], ref[name])
        assert_scalar_close(f"dn (slices {s})", r["dn"], ref["dn"])
        assert_scalar_close(f"db (slices {s})", r["db"], ref["db"])
        got[s] = r
    for s in (2, 4):
        for name in ("dk", "dv"):
            d = (got[s][name].float() - got[1][name].float()).abs()
            assert (d <= got[1][name].float().abs() * 2 ** -7 + 1e-6).all(), (s, name)
        assert torch.equal(got[s]["out"], got[1]["out"])


def test_strided_megatron_layout(cuda_device):
    """[S, B, H, D]-permuted views (check_ssa_triton_parity.py:262-265) go through TMA as-is."""
    K = _api()
    S, B, Hq, Hkv, D = 256, 2, 8, 2, 64
    qs = seeded((S, B, Hq, D), 11, 0.5).to(cuda_device)
    ks = seeded((S, B, Hkv, D), 12, 0.5).to(cuda_device)
    vs = seeded((S, B, Hkv, D), 13, 0.5).to(cuda_device)
    q, k, v = (t.permute(1, 2, 0, 3) for t in (qs, ks, vs))
    do = seeded((B, Hq, S, D), 14).to(cuda_device)
    n, b = torch.tensor(1.5, device=cuda_device), torch.tensor(0.8, device=cuda_device)
    r = run_fwd_bwd(q, k, v, do, D ** -0.5, n, b, True)
    assert r["out"].stride() == q.stride()  # empty_like keeps the Megatron layout
    ref = ssa_reference_grads(q.cpu(), k.cpu(), v.cpu(), D ** -0.5, n.cpu(), b.cpu(), do.cpu(), True)
    for name in ("out", "dq", "dk", "dv"):
        assert_lowp_close(name, r[name], ref[name])
    assert_scalar_close("dn", r["dn"], ref["dn"])


def test_megatron_layout_read_and_written_in_place(cuda_device):
    """Layout fusion at the module boundary: q/k/v are read from [S, B, H, D] views, O is
    written in [S, B, H, D] order (the module's [S, B, H*D] context is a view of the kernel's
    output), and a gradient arriving as [S, B, H*D] is read in place as a strided dout."""
    from SSA.ssa_triton_attention import SSAAttentionConfig, SSATritonAttention
    K = _api()
    S, B, Hq, Hkv, D = 384, 2, 8, 2, 64
    qs = seeded((S, B, Hq, D), 61, 0.5).to(cuda_device)
    ks = seeded((S, B, Hkv, D), 62, 0.5).to(cuda_device)
    vs = seeded((S, B, Hkv, D), 63, 0.5).to(cuda_device)
    g = seeded((S, B, Hq * D), 64).to(cuda_device)
    q, k, v = (t.permute(1, 2, 0, 3) for t in (qs, ks, vs))
    do = g.view(S, B, Hq, D).permute(1, 2, 0, 3)  # strided, not copied
    n, b = torch.tensor(0.9, device=cuda_device), torch.tensor(0.8, device=cuda_device)
    r = run_fwd_bwd(q, k, v, do, D ** -0.5, n, b, True)
    assert r["out"].permute(2, 0, 1, 3).is_contiguous()
    assert r["dq"].stride() == q.stride() and r["dk"].stride() == k.stride()
    ref = ssa_reference_grads(q.cpu(), k.cpu(), v.cpu(), D ** -0.5, n.cpu(), b.cpu(), do.cpu(), True)
    for name in ("out", "dq", "dk", "dv"):
        assert_lowp_close(name, r[name], ref[name])
    assert_scalar_close("dn", r["dn"], ref["dn"])
    assert_scalar_close("db", r["db"], ref["db"])
    cfg = SSAAttentionConfig(num_attention_heads=Hq, kv_channels=D, num_query_groups=Hkv)
    mod = SSATritonAttention(cfg, layer_number=1, ssa_n=0.9, ssa_b=0.8).to(cuda_device)
    ctx = mod(qs, ks, vs, None)
    assert ctx.is_contiguous() and ctx._base is not None  # a view, no permute-back copy
    assert ctx.data_ptr() == ctx._base.data_ptr()


def test_backward_on_a_thread_without_cuda_context(cuda_device):
    """Autograd runs backward on its own device threads; a thread that has not used CUDA yet has
    no current context. The library binds the device owning the tensors itself, so the call
    works there (and launches on that device) without the caller touching CUDA first."""
    import threading
    K = _api()
    q = seeded((1, 4, 256, 64), 71, 0.5).to(cuda_device)
    k = seeded((1, 2, 256, 64), 72, 0.5).to(cuda_device)
    v = seeded((1, 2, 256, 64), 73, 0.5).to(cuda_device)
    do = seeded((1, 4, 256, 64), 74).to(cuda_device)
    n, b = torch.tensor(0.7, device=cuda_device), torch.tensor(0.8, device=cuda_device)
    r = run_fwd_bwd(q, k, v, do, 0.125, n, b, True)
    res = {}

    def work():
        try:
            res["r"] = K.ssa_flash_attn_backward(q, k, v, r["out"], do, r["m"], 0.125, n, b,
                                                 causal=True)
            torch.cuda.synchronize(cuda_device)
        except Exception as e:  # reported below
            res["e"] = e

    th = threading.Thread(target=work)
    th.start()
    th.join()
    assert "e" not in res, repr(res.get("e"))
    for name, got in zip(("dq", "dk", "dv", "dn", "db"), res["r"]):
        ref = r[name]
        assert torch.allclose(got.float(), ref.float(), rtol=2 ** -7, atol=1e-6), name


def test_fp32_generic_path(cuda_device):
    """fp32 within 1e-5 relative (benchmark config 1 shape, reduced batch*heads)."""
    q = seeded((1, 4, 512, 64), 21, 1.0, torch.float32)
    k = seeded((1, 4, 512, 64), 22, 1.0, torch.float32)
    v = seeded((1, 4, 512, 64), 23, 1.0, torch.float32)
    do = seeded((1, 4, 512, 64), 24, 1.0, torch.float32)
    n = torch.full((4,), 0.43)
    b = torch.tensor(0.8)
    r = run_fwd_bwd(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), do.to(cuda_device),
                    0.125, n.to(cuda_device), b.to(cuda_device), True)
    ref = ssa_reference_grads(q, k, v, 0.125, n, b, do, True)
    for name in ("out", "dq", "dk", "dv"):
        assert max_rel(r[name].cpu(), ref[name]) <= 1e-5, name
    assert torch.allclose(r["dn"].cpu().double(), ref["dn"], rtol=1e-5, atol=1e-6)
    assert abs(float(r["db"]) - float(ref["db"])) <= 1e-5 * abs(float(ref["db"])) + 1e-6


@pytest.mark.parametrize("D,dtype", [(64, torch.bfloat16), (128, torch.bfloat16),
                                     (32, torch.bfloat16), (64, torch.float32)])
def test_varlen_packed_documents(D, dtype, cuda_device):
    K = _api()
    lens = [100, 257, 31, 512, 128]
    T = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    Hq, Hkv = 8, 2
    q = seeded((T, Hq, D), 31, 0.5, dtype)
    k = seeded((T, Hkv, D), 32, 0.5, dtype)
    v = seeded((T, Hkv, D), 33, 0.5, dtype)
    do = seeded((T, Hq, D), 34, 1.0, dtype)
    n, b = torch.tensor(0.43), torch.tensor(0.8)
    dev = cuda_device
    out, lse = K.ssa_flash_attn_varlen_forward(q.to(dev), k.to(dev), v.to(dev), cu.to(dev),
                                               max(lens), D ** -0.5, n.to(dev), b.to(dev), True)
    dq, dk, dv, dn, db = K.ssa_flash_attn_varlen_backward(
        q.to(dev), k.to(dev), v.to(dev), out, do.to(dev), lse, cu.to(dev), max(lens), D ** -0.5,
        n.to(dev), b.to(dev), True)
    torch.cuda.synchronize()
    ref = ssa_reference_grads_varlen(q, k, v, cu, D ** -0.5, n, b, do, True)
    got = dict(out=out, dq=dq, dk=dk, dv=dv)
    for name in ("out", "dq", "dk", "dv"):
        if dtype == torch.float32:
            assert max_rel(got[name].cpu(), ref[name]) <= 1e-5, name
        else:
            assert_lowp_close(name, got[name], ref[name])
    assert (lse.cpu().double() - ref["lse2"].transpose(0, 1)).abs().max() < 2e-3
    assert_scalar_close("dn", dn, ref["dn"])
    assert_scalar_close("db", db, ref["db"])


@pytest.mark.parametrize("D,dtype", [(64, torch.bfloat16), (128, torch.bfloat16),
                                     (64, torch.float32)])
def test_varlen_padded_packing(D, dtype, cuda_device):
    """Megatron PackedSeqParams with cu_seqlens_q_padded: documents separated by padding rows
    (NeMo's packed datasets, training/finetune/nemo_patch/data/core.py:874-999). Padding rows,
    filled with large values here, must not influence any document, and their output and
    gradient rows must be zero."""
    from types import SimpleNamespace
    from SSA.ssa_triton_attention import SSAAttentionConfig, SSATritonAttention
    lens, pads = [100, 257, 31, 200], [12, 0, 33, 7]
    Hq, Hkv = 8, 2
    starts = [0]
    for ln, pd in zip(lens, pads):
        starts.append(starts[-1] + ln + pd)
    T = starts[-1]
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    cu_pad = torch.tensor(starts, dtype=torch.int32)
    valid = torch.zeros(T, dtype=torch.bool)
    for st, ln in zip(starts[:-1], lens):
        valid[st:st + ln] = True
    g = torch.Generator().manual_seed(81)

    def filled(h, scale):
        x = torch.randn(T, h, D, generator=g) * scale
        x[~valid] = 30.0  # padding garbage
        return x.to(dtype)

    q, k, v, do = filled(Hq, 0.5), filled(Hkv, 0.5), filled(Hkv, 0.5), filled(Hq, 1.0)
    n, b = torch.tensor(0.55), torch.tensor(0.8)
    dev = cuda_device
    qd, kd, vd, dod = (t.to(dev).requires_grad_(True) if i < 3 else t.to(dev)
                       for i, t in enumerate((q, k, v, do)))
    from SSA.ssa_flash_attention import ssa_flash_attn_varlen_func
    nd = n.to(dev).requires_grad_(True)
    out = ssa_flash_attn_varlen_func(qd, kd, vd, cu.to(dev), max(lens), D ** -0.5, nd, b.to(dev),
                                     True, cu_pad.to(dev))
    out.backward(dod)
    torch.cuda.synchronize()
    ref = ssa_reference_grads_varlen(q[valid], k[valid], v[valid], cu, D ** -0.5, n, b, do[valid],
                                     True)
    got = dict(out=out.detach(), dq=qd.grad, dk=kd.grad, dv=vd.grad)
    for name in ("out", "dq", "dk", "dv"):
        x = got[name].cpu()
        assert (x[~valid] == 0).all(), f"{name}: padding rows not zero"
        if dtype == torch.float32:
            assert max_rel(x[valid], ref[name]) <= 1e-5, name
        else:
            assert_lowp_close(name, x[valid], ref[name])
    assert_scalar_close("dn", nd.grad, ref["dn"])
    # the module takes the same layout through packed_seq_params
    cfg = SSAAttentionConfig(num_attention_heads=Hq, kv_channels=D, num_query_groups=Hkv)
    mod = SSATritonAttention(cfg, layer_number=1, ssa_n=0.55, ssa_b=0.8).to(dev)
    psp = SimpleNamespace(cu_seqlens_q=cu.to(dev), cu_seqlens_kv=None,
                          cu_seqlens_q_padded=cu_pad.to(dev), cu_seqlens_kv_padded=None,
                          max_seqlen_q=max(lens))
    ctx = mod(q.to(dev).unsqueeze(1), k.to(dev).unsqueeze(1), v.to(dev).unsqueeze(1), None,
              packed_seq_params=psp)
    torch.cuda.synchronize()
    assert ctx.shape == (T, 1, Hq * D)
    assert torch.equal(ctx.reshape(T, Hq, D), out.detach())


def test_backward_out_with_unaligned_strides(cuda_device):
    """`out` handed to the backward in a layout the TMA path cannot read (row stride of 65
    elements, 130 bytes) is copied like q/k/v/dout and gives the same gradients."""
    K = _api()
    B, Hq, Hkv, N, D = 1, 4, 2, 256, 64
    q = seeded((B, Hq, N, D), 71, 0.5).to(cuda_device)
    k = seeded((B, Hkv, N, D), 72, 0.5).to(cuda_device)
    v = seeded((B, Hkv, N, D), 73, 0.5).to(cuda_device)
    do = seeded((B, Hq, N, D), 74).to(cuda_device)
    n, b = torch.tensor(1.5, device=cuda_device), torch.tensor(0.8, device=cuda_device)
    out, m = K.ssa_flash_attn_forward(q, k, v, D ** -0.5, n, b, causal=True)
    padded = torch.zeros(B, Hq, N, D + 1, dtype=out.dtype, device=cuda_device)
    padded[..., :D] = out
    odd = padded[..., :D]
    assert (odd.stride(2) * odd.element_size()) % 16 != 0
    ref = K.ssa_flash_attn_backward(q, k, v, out, do, m, D ** -0.5, n, b, causal=True)
    got = K.ssa_flash_attn_backward(q, k, v, odd, do, m, D ** -0.5, n, b, causal=True)
    torch.cuda.synchronize()
    for name, g, r in zip(("dq", "dk", "dv", "dn", "db"), got, ref):
        if name == "dq":  # fp32 reduce-add order across key blocks is not fixed
            assert (g.float() - r.float()).abs().max() <= r.float().abs().max() * 2 ** -7, name
        else:
            assert torch.equal(g, r), name


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_bit_deterministic(dtype, cuda_device):
    """Two identical runs are bit-identical (check_ssa_triton_parity.py:507-562, atol 0).

    Exception, tensor-core path only: dq is accumulated across key blocks with fp32 reduce-adds
    in L2 whose order is not fixed, so it may differ by rounding between runs; it must stay
    within one 16-bit ulp of the first run. Everything else (out, lse, dk, dv, dn, db) is exact.
    """
    q = seeded((2, 8, 384, 64), 41, 0.5, dtype).to(cuda_device)
    k = seeded((2, 2, 384, 64), 42, 0.5, dtype).to(cuda_device)
    v = seeded((2, 2, 384, 64), 43, 0.5, dtype).to(cuda_device)
    do = seeded((2, 8, 384, 64), 44, 1.0, dtype).to(cuda_device)
    n, b = torch.tensor(1.5, device=cuda_device), torch.tensor(0.8, device=cuda_device)
    r1 = run_fwd_bwd(q, k, v, do, 0.125, n, b, True)
    r2 = run_fwd_bwd(q, k, v, do, 0.125, n, b, True)
    tensor_core = dtype != torch.float32
    for name in r1:
        if name == "dq" and tensor_core:
            d = (r1[name].float() - r2[name].float()).abs()
            assert (d <= r1[name].float().abs() * 2 ** -7 + 1e-6).all(), name
        else:
            assert torch.equal(r1[name], r2[name]), name


@pytest.mark.parametrize("B,Hq,Hkv,N,D,causal", [
    (2, 8, 2, 1024, 64, True),     # 8 key blocks per sequence: long chains of ordered dQ adds
    (1, 8, 2, 700, 64, False),     # non-causal: every key block adds to every tile; q-head slices
    (1, 4, 2, 640, 128, True),     # D = 128 kernel (64-query tiles)
    (2, 8, 2, 512, 32, True),      # D = 32 through the D = 64 kernel
])
def test_deterministic_dq_is_bit_identical(B, Hq, Hkv, N, D, causal, cuda_device):
    """deterministic=True: every dQ tile's contributions are added in ascending key-block order,
    so two identical runs give bit-identical dq as well as out, lse, dk, dv, dn, db
    (check_ssa_triton_parity.py:507-562, atol 0), and the result matches the oracle."""
    K = _api()
    q = seeded((B, Hq, N, D), 401, 0.5).to(cuda_device)
    k = seeded((B, Hkv, N, D), 402, 0.5).to(cuda_device)
    v = seeded((B, Hkv, N, D), 403, 0.5).to(cuda_device)
    do = seeded((B, Hq, N, D), 404).to(cuda_device)
    n = (0.3 + 0.3 * torch.rand(Hq, generator=torch.Generator().manual_seed(405))).to(cuda_device)
    b = torch.tensor(0.8, device=cuda_device)
    scale = D ** -0.5
    runs = []
    for _ in range(3):
        out, m = K.ssa_flash_attn_forward(q, k, v, scale, n, b, causal=causal)
        grads = K.ssa_flash_attn_backward(q, k, v, out, do, m, scale, n, b, causal=causal,
                                          deterministic=True)
        torch.cuda.synchronize()
        runs.append((out, m) + tuple(grads))
    for r in runs[1:]:
        for name, a, b2 in zip(("out", "m", "dq", "dk", "dv", "dn", "db"), runs[0], r):
            assert torch.equal(a, b2), f"{name} differs between deterministic runs"
    ref = ssa_reference_grads(q.cpu(), k.cpu(), v.cpu(), scale, n.cpu(), b.cpu(), do.cpu(), causal)
    for name, got in zip(("out", "dq", "dk", "dv"), (runs[0][0],) + runs[0][2:5]):
        assert_lowp_close(name, got, ref[name])
    assert_scalar_close("dn", runs[0][5], ref["dn"])
    assert_scalar_close("db", runs[0][6], ref["db"])
    # the default (unordered) mode computes the same gradients up to rounding
    dq_fast = K.ssa_flash_attn_backward(q, k, v, runs[0][0], do, runs[0][1], scale, n, b,
                                        causal=causal, deterministic=False)[0]
    d = (dq_fast.float() - runs[0][2].float()).abs()
    assert (d <= runs[0][2].float().abs() * 2 ** -7 + 1e-6).all()


def test_deterministic_dq_packed_documents(cuda_device):
    """Deterministic dq on packed documents (per-document key blocks and query tiles), through
    the environment switch SSA_DETERMINISTIC=1 and the autograd Function."""
    import os
    from SSA.ssa_flash_attention import ssa_flash_attn_varlen_func
    lens = [300, 1000, 77, 513]
    T, Hq, Hkv, D = sum(lens), 8, 2, 64
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    q = seeded((T, Hq, D), 411, 0.5)
    k = seeded((T, Hkv, D), 412, 0.5)
    v = seeded((T, Hkv, D), 413, 0.5)
    do = seeded((T, Hq, D), 414)
    n, b = torch.tensor(0.6), torch.tensor(0.8)
    dev = cuda_device
    old = os.environ.get("SSA_DETERMINISTIC")
    os.environ["SSA_DETERMINISTIC"] = "1"
    try:
        grads = []
        for _ in range(3):
            qd = q.to(dev).requires_grad_(True)
            out = ssa_flash_attn_varlen_func(qd, k.to(dev), v.to(dev), cu.to(dev), max(lens),
                                             D ** -0.5, n.to(dev), b.to(dev), True)
            out.backward(do.to(dev))
            torch.cuda.synchronize()
            grads.append(qd.grad.clone())
    finally:
        if old is None:
            os.environ.pop("SSA_DETERMINISTIC")
        else:
            os.environ["SSA_DETERMINISTIC"] = old
    assert torch.equal(grads[0], grads[1]) and torch.equal(grads[0], grads[2])
    ref = ssa_reference_grads_varlen(q, k, v, cu, D ** -0.5, n, b, do, True)
    assert_lowp_close("dq", grads[0], ref["dq"])


def test_autograd_function_and_module(cuda_device):
    from SSA.ssa_flash_attention import ssa_flash_attention
    from SSA.ssa_triton_attention import SSAAttentionConfig, SSATritonAttention
    S, B, Hq, Hkv, D = 256, 2, 8, 2, 64
    cfg = SSAAttentionConfig(num_attention_heads=Hq, kv_channels=D, num_query_groups=Hkv)
    mod = SSATritonAttention(cfg, layer_number=1, ssa_n=1.5, ssa_b=0.8).to(cuda_device)
    qs = seeded((S, B, Hq, D), 51, 0.5).to(cuda_device).requires_grad_(True)
    ks = seeded((S, B, Hkv, D), 52, 0.5).to(cuda_device).requires_grad_(True)
    vs = seeded((S, B, Hkv, D), 53, 0.5).to(cuda_device).requires_grad_(True)
    ctx = mod(qs, ks, vs, None)
    assert ctx.shape == (S, B, Hq * D)
    g = seeded((S, B, Hq * D), 54).to(cuda_device)
    ctx.backward(g)
    q, k, v = (t.detach().cpu().permute(1, 2, 0, 3) for t in (qs, ks, vs))
    do = g.cpu().reshape(S, B, Hq, D).permute(1, 2, 0, 3)
    ref = ssa_reference_grads(q, k, v, D ** -0.5, torch.tensor(1.5), torch.tensor(0.8), do, True)
    assert_lowp_close("ctx", ctx.detach().reshape(S, B, Hq, D).permute(1, 2, 0, 3), ref["out"])
    assert_lowp_close("dq", qs.grad.permute(1, 2, 0, 3), ref["dq"])
    assert_lowp_close("dk", ks.grad.permute(1, 2, 0, 3), ref["dk"])
    assert_scalar_close("dn", mod.ssa_n_raw.grad, ref["dn"])
    # autograd.Function returns 9 grads, dn shaped like ssa_n, db computed even if unused
    n = torch.full((Hq,), 0.5, device=cuda_device, requires_grad=True)
    b = torch.tensor(0.8, device=cuda_device, requires_grad=True)
    qd = q.to(cuda_device).requires_grad_(True)
    out = ssa_flash_attention(qd, k.to(cuda_device), v.to(cuda_device), D ** -0.5, n, b, True)
    out.sum().backward()
    assert n.grad.shape == (Hq,) and b.grad.shape == ()


def test_config2_full_size_slice(cuda_device):
    """benchmark config 2 shape (B=8, Hq=32, Hkv=8, S=2048, D=64, bf16, causal, per-head n). The
    (batch, kv-group) units are independent, so one unit's 4 q-heads are checked exactly against
    the fp64 oracle at full sequence length."""
    B, Hq, Hkv, N, D = 8, 32, 8, 2048, 64
    gen = torch.Generator(device="cpu").manual_seed(0)
    q = (torch.randn(B, Hq, N, D, generator=gen) * 0.5).to(torch.bfloat16)
    k = (torch.randn(B, Hkv, N, D, generator=gen) * 0.5).to(torch.bfloat16)
    v = (torch.randn(B, Hkv, N, D, generator=gen) * 0.5).to(torch.bfloat16)
    do = torch.randn(B, Hq, N, D, generator=gen).to(torch.bfloat16)
    n = 0.3 + 0.3 * torch.rand(Hq, generator=gen)
    b = torch.tensor(0.8)
    dev = cuda_device
    r = run_fwd_bwd(q.to(dev), k.to(dev), v.to(dev), do.to(dev), D ** -0.5, n.to(dev), b.to(dev), True)
    zb, g0 = 3, 5  # batch 3, kv head 5 -> q heads 20..23
    hs = slice(4 * g0, 4 * g0 + 4)
    ref = ssa_reference_grads(q[zb:zb + 1, hs], k[zb:zb + 1, g0:g0 + 1], v[zb:zb + 1, g0:g0 + 1],
                              D ** -0.5, n[hs], b, do[zb:zb + 1, hs], True)
    assert_lowp_close("out", r["out"][zb:zb + 1, hs], ref["out"])
    assert_lowp_close("dq", r["dq"][zb:zb + 1, hs], ref["dq"])
    assert_lowp_close("dk", r["dk"][zb:zb + 1, g0:g0 + 1], ref["dk"])
    assert_lowp_close("dv", r["dv"][zb:zb + 1, g0:g0 + 1], ref["dv"])
    for t in r.values():
        assert torch.isfinite(t).all()


@pytest.mark.parametrize("D", [64, 128])
def test_negative_and_large_n_large_scores(D, cuda_device):
    """Per-head n of both signs and up to 2.5 with scores of larger magnitude (q, k scaled 1.5):
    the forward's normaliser bound (|n| log2(1 + b max|s|)) and its rescaling both come into
    play, and for n < 0 the largest transformed score comes from the most negative s."""
    K = _api()
    B, Hq, Hkv, N = 1, 4, 2, 384
    seed = 900 + D
    q = seeded((B, Hq, N, D), seed, 1.5)
    k = seeded((B, Hkv, N, D), seed + 1, 1.5)
    v = seeded((B, Hkv, N, D), seed + 2, 0.5)
    do = seeded((B, Hq, N, D), seed + 3, 1.0)
    n = torch.tensor([-1.5, -0.4, 0.9, 2.5])
    b = torch.tensor(0.8)
    scale = 1.0 / math.sqrt(D)
    assert K.kernel_family(q.to(cuda_device), scale) == 1
    r = run_fwd_bwd(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), do.to(cuda_device),
                    scale, n.to(cuda_device), b.to(cuda_device), True)
    ref = ssa_reference_grads(q, k, v, scale, n, b, do, True)
    for name in ("out", "dq", "dk", "dv"):
        assert_lowp_close(name, r[name], ref[name])
    assert_scalar_close("dn", r["dn"], ref["dn"])
    assert_scalar_close("db", r["db"], ref["db"])


def test_d128_long_sequence_slice(cuda_device):
    """D = 128 at S = 4096 (the config-4 head dim, 32 key blocks per sequence), one kv group's
    two q-heads checked against the fp64 oracle over the whole sequence."""
    B, Hq, Hkv, N, D = 1, 4, 2, 4096, 128
    gen = torch.Generator(device="cpu").manual_seed(7)
    q = (torch.randn(B, Hq, N, D, generator=gen) * 0.5).to(torch.bfloat16)
    k = (torch.randn(B, Hkv, N, D, generator=gen) * 0.5).to(torch.bfloat16)
    v = (torch.randn(B, Hkv, N, D, generator=gen) * 0.5).to(torch.bfloat16)
    do = torch.randn(B, Hq, N, D, generator=gen).to(torch.bfloat16)
    n = 0.3 + 0.3 * torch.rand(Hq, generator=gen)
    b = torch.tensor(0.8)
    dev = cuda_device
    r = run_fwd_bwd(q.to(dev), k.to(dev), v.to(dev), do.to(dev), D ** -0.5, n.to(dev), b.to(dev), True)
    g0 = 1  # kv head 1 -> q heads 2, 3
    hs = slice(2 * g0, 2 * g0 + 2)
    ref = ssa_reference_grads(q[:, hs], k[:, g0:g0 + 1], v[:, g0:g0 + 1], D ** -0.5, n[hs], b,
                              do[:, hs], True)
    assert_lowp_close("out", r["out"][:, hs], ref["out"])
    assert_lowp_close("dq", r["dq"][:, hs], ref["dq"])
    assert_lowp_close("dk", r["dk"][:, g0:g0 + 1], ref["dk"])
    assert_lowp_close("dv", r["dv"][:, g0:g0 + 1], ref["dv"])


def test_device_timeout_path_reports_and_recovers(cuda_device):
    """Failure path without a GPU fault: a bounded wait that nothing completes (a 2M-cycle
    limit, about a millisecond) must record SSA_ERR_DEVICE_TIMEOUT, the status read must clear
    it, and the context must stay usable: an attention call afterwards computes normally."""
    from SSA import _lib
    lib = _lib.load()
    st = _lib.stream_ptr(cuda_device)
    assert lib.ssa_device_status(st) == _lib.SSA_OK
    assert lib.ssa_selftest_device_timeout(2_000_000, st) == _lib.SSA_OK
    assert lib.ssa_device_status(st) == _lib.SSA_ERR_DEVICE_TIMEOUT
    assert lib.ssa_device_status(st) == _lib.SSA_OK  # cleared by the read
    K = _api()
    q = seeded((1, 2, 128, 64), 91, 0.5).to(cuda_device)
    k = seeded((1, 2, 128, 64), 92, 0.5).to(cuda_device)
    v = seeded((1, 2, 128, 64), 93, 0.5).to(cuda_device)
    n, b = torch.tensor(0.7, device=cuda_device), torch.tensor(0.8, device=cuda_device)
    out, _ = K.ssa_flash_attn_forward(q, k, v, 0.125, n, b, causal=True)
    ref = ssa_reference_grads(q.cpu(), k.cpu(), v.cpu(), 0.125, n.cpu(), b.cpu(),
                              torch.zeros(1, 2, 128, 64), True)
    assert_lowp_close("out", out, ref["out"])
    assert lib.ssa_device_status(st) == _lib.SSA_OK


@pytest.mark.parametrize("D", [64, 128])
def test_outputs_are_nan_after_a_device_timeout(D, cuda_device):
    """No silent failure: once a bounded wait has expired (made to expire here by the self-test,
    without any fault) and until the status word is read, the tensor-core kernels skip their work
    and write NaN into every output (out, m, dq, dk, dv, dn, db), so a caller that never checks
    the status cannot keep training on stale memory. SSA.check_device_status() then raises
    SSAKernelError(SSA_ERR_DEVICE_TIMEOUT), clears the status, and the next call computes
    normally."""
    import SSA
    from SSA import _lib
    lib = _lib.load()
    st = _lib.stream_ptr(cuda_device)
    assert lib.ssa_device_status(st) == _lib.SSA_OK
    K = _api()
    B, Hq, Hkv, N = 1, 4, 2, 200  # ragged: the second tile is partial
    q = seeded((B, Hq, N, D), 95, 0.5).to(cuda_device)
    k = seeded((B, Hkv, N, D), 96, 0.5).to(cuda_device)
    v = seeded((B, Hkv, N, D), 97, 0.5).to(cuda_device)
    do = seeded((B, Hq, N, D), 98).to(cuda_device)
    n = torch.tensor([0.4, 0.5, 0.6, 0.7], device=cuda_device)
    b = torch.tensor(0.8, device=cuda_device)
    scale = D ** -0.5
    assert lib.ssa_selftest_device_timeout(2_000_000, st) == _lib.SSA_OK
    out, m = K.ssa_flash_attn_forward(q, k, v, scale, n, b, causal=True)
    dq, dk, dv, dn, db = K.ssa_flash_attn_backward(q, k, v, out, do, m, scale, n, b, causal=True)
    torch.cuda.synchronize()
    for name, t in zip(("out", "m", "dq", "dk", "dv", "dn", "db"), (out, m, dq, dk, dv, dn, db)):
        assert torch.isnan(t.float()).all(), f"{name}: not NaN after a device timeout"
    with pytest.raises(_lib.SSAKernelError) as ei:
        SSA.check_device_status(cuda_device)
    assert ei.value.code == _lib.SSA_ERR_DEVICE_TIMEOUT
    SSA.check_device_status(cuda_device)  # cleared by the read: no error now
    r = run_fwd_bwd(q, k, v, do, scale, n, b, True)
    ref = ssa_reference_grads(q.cpu(), k.cpu(), v.cpu(), scale, n.cpu(), b.cpu(), do.cpu(), True)
    for name in ("out", "dq", "dk", "dv"):
        assert_lowp_close(name, r[name], ref[name])
    assert_scalar_close("dn", r["dn"], ref["dn"])


def test_device_status_clean(cuda_device):
    from SSA import _lib
    rc = _lib.load().ssa_device_status(_lib.stream_ptr(cuda_device))
    assert rc == _lib.SSA_OK
