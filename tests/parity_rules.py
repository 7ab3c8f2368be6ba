"""Tolerance rules shared by the GPU parity tests (one definition, used by every test file).

bf16/fp16 outputs (O, dQ, dK, dV) against the fp64 oracle evaluated on the same 16-bit inputs:
  * elementwise |a - r| <= 2e-2 + 5e-2 |r|: the reference's own bf16 rule
    (check_ssa_triton_parity.py:1059-1062);
  * AND max-abs |a - r| <= 2e-2 wherever |r| <= 4: the stated 2e-2 max-abs bar. Above 4 a bf16
    value cannot be within 2e-2 of most reals (its spacing there is 2^-5 = 0.031), so the
    relative rule alone applies;
  * every element finite.
dn / db (sums over every score element): |a - r| <= 2e-3 + 2e-2 |r|, the reference's scalar
rule (check_ssa_triton_parity.py:1066-1067); the reference's own bf16 kernel misses an absolute
2e-2 bar on these (its A100 parity report).
fp32 outputs: max|a - r| / max|r| <= 1e-5 (check_ssa_triton_vs_original.py:54-58 convention).
"""

import torch

LOWP_ATOL = 2e-2
LOWP_RTOL = 5e-2
LOWP_MAXABS_CUT = 4.0
SCALAR_ATOL = 2e-3
SCALAR_RTOL = 2e-2


def assert_lowp_close(name, got, ref):
    g = got.detach().double().cpu()
    r = ref.detach().double().cpu()
    assert g.shape == r.shape, f"{name}: shape {tuple(g.shape)} != {tuple(r.shape)}"
    assert torch.isfinite(g).all(), f"{name}: non-finite"
    d = (g - r).abs()
    lim = LOWP_ATOL + LOWP_RTOL * r.abs()
    bad = int((d > lim).sum())
    assert bad == 0, f"{name}: {bad} elements outside 2e-2+5e-2|r| (max|d|={d.max():.3e})"
    small = r.abs() <= LOWP_MAXABS_CUT
    if small.any():
        worst = d[small].max()
        assert worst <= LOWP_ATOL, f"{name}: max-abs {worst:.3e} > 2e-2 on |r|<=4"


def assert_scalar_close(name, got, ref, atol=SCALAR_ATOL, rtol=SCALAR_RTOL):
    g = torch.as_tensor(got).detach().double().cpu().reshape(-1)
    r = torch.as_tensor(ref).detach().double().cpu().reshape(-1)
    assert g.shape == r.shape, name
    assert torch.isfinite(g).all(), f"{name}: non-finite {g.tolist()}"
    d = (g - r).abs()
    assert (d <= atol + rtol * r.abs()).all(), f"{name}: {g.tolist()} vs {r.tolist()}"


def max_abs_where(got, ref, cut=LOWP_MAXABS_CUT) -> float:
    """max |a - r| over the elements with |r| <= cut (a diagnostic printed beside the checks)."""
    g = got.detach().double().cpu()
    r = ref.detach().double().cpu()
    m = r.abs() <= cut
    return float((g - r).abs()[m].max()) if m.any() else 0.0
