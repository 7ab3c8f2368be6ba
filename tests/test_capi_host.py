"""C-ABI library checks that need no GPU: it loads, exports every function include/ssa_b200.h
declares, sizes workspaces, rejects bad problems with the right status codes, and the Python
host layer (module shims, parameters, checkpoint keys) behaves like the reference's."""

import ctypes
import os
import sys
import re
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def lib():
    from SSA import _lib
    if not _lib.LIB_PATH.exists():
        import __graft_entry__
        __graft_entry__.build()
    return _lib.load()


def header_functions():
    text = (REPO / "include" / "ssa_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(ssa_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_expected_entry_points():
    fns = header_functions()
    for f in ("ssa_attn_fwd", "ssa_attn_bwd", "ssa_attn_bwd_preprocess",
              "ssa_attn_bwd_workspace_size", "ssa_attn_fwd_workspace_size",
              "ssa_attn_kernel_family", "ssa_device_status", "ssa_last_error", "ssa_version"):
        assert f in fns


def test_library_exports_every_declared_symbol(lib):
    for f in header_functions():
        assert hasattr(lib, f), f"libssa_b200.so does not export {f}"
    from SSA import _lib
    assert set(_lib.EXPORTED_SYMBOLS) <= set(header_functions())


def test_version(lib):
    assert b"sm_100a" in lib.ssa_version()


def _prob(**kw):
    from SSA import _lib
    base = dict(dtype=2, B=2, Hq=8, Hkv=2, N=256, D=64, causal=1, softmax_scale=0.125,
                ssa_n=1, n_per_head=0, ssa_b=1, cu_seqlens=None, max_seqlen=0)
    base.update(kw)
    return _lib.SsaProblem(**base)


def test_family_selection(lib):
    assert lib.ssa_attn_kernel_family(ctypes.byref(_prob())) == 1          # bf16 D=64
    assert lib.ssa_attn_kernel_family(ctypes.byref(_prob(dtype=1, D=128))) == 1
    assert lib.ssa_attn_kernel_family(ctypes.byref(_prob(dtype=0))) == 0   # fp32 -> generic
    assert lib.ssa_attn_kernel_family(ctypes.byref(_prob(D=32))) == 1      # D=32: the D=64 kernels
    assert lib.ssa_attn_kernel_family(ctypes.byref(_prob(D=16))) == 0      # D=16 -> generic
    assert lib.ssa_attn_kernel_family(ctypes.byref(_prob(softmax_scale=-1.0))) == 0
    assert lib.ssa_attn_kernel_family(ctypes.byref(_prob(Hq=6, Hkv=4))) == -1


def test_bad_problems_rejected_before_any_cuda_call(lib):
    from SSA import _lib
    t = _lib.SsaTensor(16, 0, 0, 0)
    cases = [(_prob(Hq=6, Hkv=4), _lib.SSA_ERR_BAD_SHAPE, b"divisible"),
             (_prob(D=48), _lib.SSA_ERR_UNSUPPORTED, b"head dim"),
             (_prob(dtype=7), _lib.SSA_ERR_UNSUPPORTED, b"dtype"),
             (_prob(N=0), _lib.SSA_ERR_BAD_SHAPE, b"non-positive"),
             (_prob(ssa_n=None), _lib.SSA_ERR_NULL, b"ssa_n"),
             (_prob(cu_seqlens=64, max_seqlen=0), _lib.SSA_ERR_BAD_SHAPE, b"max_seqlen"),
             (_prob(cu_seqlens_padded=64), _lib.SSA_ERR_BAD_SHAPE, b"cu_seqlens_padded")]
    for prob, code, msg in cases:
        rc = lib.ssa_attn_fwd(ctypes.byref(prob), t, t, t, t, 16, None, 0, None)
        assert rc == code, (rc, code)
        assert msg in lib.ssa_last_error()
    rc = lib.ssa_attn_fwd(ctypes.byref(_prob()), _lib.SsaTensor(None, 0, 0, 0), t, t, t, 16,
                          None, 0, None)
    assert rc == _lib.SSA_ERR_NULL and b"q is NULL" in lib.ssa_last_error()


def test_bwd_workspace_requirement_enforced(lib):
    from SSA import _lib
    prob = _prob()
    need = lib.ssa_attn_bwd_workspace_size(ctypes.byref(prob))
    # delta alone is Hq * B * N fp32
    assert need >= 8 * 2 * 256 * 4
    t = _lib.SsaTensor(16, 0, 0, 0)
    rc = lib.ssa_attn_bwd(ctypes.byref(prob), t, t, t, t, t, 16, t, t, t, 16, 16, 16, need - 1, None)
    assert rc == _lib.SSA_ERR_WORKSPACE
    # tensor-core path: delta + the fp32 dQ accumulator (B*Hq*N*D*4) + dn/db partials
    assert need >= 8 * 2 * 256 * 4 + 2 * 8 * 256 * 64 * 4
    # generic path: delta + dn/db partials only
    p32 = _prob(dtype=0)
    need32 = lib.ssa_attn_bwd_workspace_size(ctypes.byref(p32))
    assert 8 * 2 * 256 * 4 <= need32 < need


def test_python_layer_rejects_cpu_tensors():
    from SSA.ssa_flash_attention import ssa_flash_attention
    q = torch.randn(1, 2, 8, 16)
    with pytest.raises(ValueError, match="CUDA"):
        ssa_flash_attention(q, q, q, 0.25, torch.tensor(1.5), torch.tensor(0.8))


def test_module_matches_reference_construction():
    from SSA.ssa_triton_attention import SSAAttentionConfig, SSATritonAttention
    cfg = SSAAttentionConfig(num_attention_heads=32, kv_channels=64, num_query_groups=8,
                             apply_query_key_layer_scaling=True)
    m = SSATritonAttention(cfg, layer_number=4, ssa_n=1.5, ssa_b=0.8)
    assert m.gqa_ratio == 4
    assert abs(m.softmax_scale - 1.0 / 8.0 / 4) < 1e-12
    keys = set(m.state_dict().keys())
    assert keys == {"ssa_n_raw", "ssa_b"}          # checkpoint keys of the reference
    assert m.ssa_n_raw.requires_grad and m.ssa_n_raw.dim() == 0
    m2 = SSATritonAttention(cfg, 1, learnable_ssa=True, learnable_b=True)
    assert set(m2.state_dict().keys()) == {"ssa_n_raw", "ssa_b_raw"}
    m3 = SSATritonAttention(cfg, 1, learnable_ssa=False)
    assert set(m3.state_dict().keys()) == {"ssa_n", "ssa_b"}
    m4 = SSATritonAttention(cfg, 1, ssa_n=[0.43] * 32)
    assert m4.ssa_n_raw.shape == (32,)
    with pytest.raises(AssertionError):
        SSATritonAttention(SSAAttentionConfig(32, 64, 8, context_parallel_size=2), 1)


def test_layer_spec_requires_megatron_only_when_called():
    import SSA.ssa_triton_layer_specs as ls
    assert callable(ls.get_ssa_triton_gpt_layer_spec)
    try:
        import megatron  # noqa: F401
    except ImportError:
        with pytest.raises(ImportError):
            ls.get_ssa_triton_gpt_layer_spec()


def test_bias_dropout_add_factories():
    """The reference's bias-dropout-add factories exist with its signatures; without Megatron the
    eager function computes residual + dropout(x + bias), with dropout only in training."""
    import SSA.ssa_triton_layer_specs as ls
    g = torch.Generator().manual_seed(0)
    x, bias, res = (torch.randn(4, 8, generator=g) for _ in range(3))
    try:
        import megatron  # noqa: F401
        have_megatron = True
    except ImportError:
        have_megatron = False
    eval_fn = ls.get_bias_dropout_add(False, False)
    assert torch.allclose(eval_fn((x, bias), res, 0.5), x + bias + res)
    assert torch.allclose(eval_fn((x, None), res, 0.0), x + res)
    if not have_megatron:
        train_fn = ls.get_bias_dropout_add(True, False)
        y = train_fn((x, bias), res, 0.5) - res
        kept = y != 0
        assert kept.any() and (~kept).any()
        assert torch.allclose(y[kept], 2.0 * (x + bias)[kept])
    assert ls.get_compiled_bias_dropout_add(True, False) is ls.get_compiled_bias_dropout_add(True, True)
    assert callable(ls.get_compiled_bias_dropout_add(False, False))


def test_missing_library_fails_loudly():
    """No CPU or PyTorch fallback: without libssa_b200.so every entry point raises."""
    import subprocess
    code = ("import sys; sys.path[:0] = [%r, %r]\n"
            "from SSA import _lib\n"
            "try:\n    _lib.load()\nexcept RuntimeError as e:\n    print('raised', 'not found' in str(e))\n")
    env = dict(os.environ, SSA_B200_LIB="/nonexistent/libssa_b200.so")
    r = subprocess.run([sys.executable, "-c", code % (str(REPO), str(REPO / "luciole-1b_b200"))],
                       capture_output=True, text=True, env=env, timeout=120)
    assert r.stdout.strip() == "raised True", (r.stdout, r.stderr)


def test_packed_params_validation_before_any_kernel():
    """Megatron PackedSeqParams handling: mismatched kv boundaries and a missing cu_seqlens_q
    are rejected on the host, without a device synchronisation when q / kv share storage."""
    from types import SimpleNamespace
    from SSA.ssa_triton_attention import SSAAttentionConfig, SSATritonAttention, _same
    cfg = SSAAttentionConfig(num_attention_heads=4, kv_channels=64, num_query_groups=2)
    mod = SSATritonAttention(cfg, layer_number=1)
    q = torch.zeros(10, 1, 4, 64)
    kv = torch.zeros(10, 1, 2, 64)
    cu = torch.tensor([0, 4, 10], dtype=torch.int32)
    with pytest.raises(ValueError, match="cu_seqlens_q"):
        mod(q, kv, kv, None, packed_seq_params=SimpleNamespace(cu_seqlens_q=None))
    bad = SimpleNamespace(cu_seqlens_q=cu, cu_seqlens_kv=torch.tensor([0, 5, 10], dtype=torch.int32),
                          max_seqlen_q=6)
    with pytest.raises(ValueError, match="cu_seqlens_kv"):
        mod(q, kv, kv, None, packed_seq_params=bad)
    assert _same(None, cu) and _same(cu, cu) and _same(cu.clone(), cu)
    assert not _same(torch.tensor([0, 5, 10], dtype=torch.int32), cu)


def test_layout_rule_of_the_wrappers():
    """Which layouts the wrappers hand to the kernels as they are and which they copy: unit D
    stride always; for the TMA (tensor-core) family also a 16-byte-aligned base and B/H/N
    strides. Megatron's [S, B, H, D] permuted view passes untouched."""
    from SSA.ssa_triton_kernel import _prep, _tma_ok
    x = torch.zeros(2, 4, 64, 64, dtype=torch.bfloat16)
    megatron = torch.zeros(64, 2, 4, 64, dtype=torch.bfloat16).permute(1, 2, 0, 3)
    odd_rows = torch.zeros(2, 4, 64, 65, dtype=torch.bfloat16)[..., :64]  # 130-byte rows
    odd_base = torch.zeros(2 * 4 * 64 * 64 + 1, dtype=torch.bfloat16)[1:].view(2, 4, 64, 64)
    d_strided = torch.zeros(2, 4, 64, 128, dtype=torch.bfloat16)[..., ::2]
    assert _tma_ok(x) and _tma_ok(megatron)
    assert not _tma_ok(odd_rows) and not _tma_ok(odd_base) and not _tma_ok(d_strided)
    for t in (x, megatron):
        assert _prep(t, 1) is t and _prep(t, 0) is t
    for t in (odd_rows, odd_base):
        c = _prep(t, 1)
        assert c is not t and c.is_contiguous() and torch.equal(c, t) and _tma_ok(c)
        assert _prep(t, 0) is t  # the generic kernels only need a unit D stride
    c = _prep(d_strided, 0)
    assert c is not d_strided and c.stride(-1) == 1 and torch.equal(c, d_strided)


def test_ctypes_structs_match_the_c_header(tmp_path):
    """The ctypes mirrors of ssa_problem_t / ssa_tensor_t have the C header's field offsets and
    sizes (compiled here with gcc against include/ssa_b200.h)."""
    import ctypes
    import shutil
    import subprocess
    from SSA import _lib
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    fields = [f for f, _ in _lib.SsaProblem._fields_]
    prog = ["#include <stdio.h>", "#include <stddef.h>", '#include "ssa_b200.h"',
            "int main(void) {",
            '  printf("problem %zu\\n", sizeof(ssa_problem_t));',
            '  printf("tensor %zu\\n", sizeof(ssa_tensor_t));']
    for f in fields:
        prog.append(f'  printf("{f} %zu\\n", offsetof(ssa_problem_t, {f}));')
    prog += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(prog) + "\n")
    exe = tmp_path / "layout"
    subprocess.run([gcc, "-I", str(REPO / "include"), str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True,
                                                       text=True, check=True).stdout.splitlines())
    assert int(out["problem"]) == ctypes.sizeof(_lib.SsaProblem)
    assert int(out["tensor"]) == ctypes.sizeof(_lib.SsaTensor)
    for f in fields:
        assert int(out[f]) == getattr(_lib.SsaProblem, f).offset, f
