"""GPU: the reference's own kernel parity matrix, with its own elementwise rule.

The reference's parity suite (check_ssa_triton_parity.py, kernel suite; its A100 report is
training/train/train_ssa_triton/logs/parity_reports/ssa_triton_v4_parity_76887.json) runs its
bf16 and fp16 kernels on D = 32, Hkv = 8, Hq 8 / 16 / 24, B 1 / 2, N 128 / 512, causal and not,
contiguous and Megatron-strided layouts, with q, k, v, dO ~ N(0, 1), n = 1.5, b = 0.8, and
checks O / dQ / dK / dV with allclose(atol=2e-2, rtol=5e-2) against an fp32 eager reference
(check_ssa_triton_parity.py:1059-1062). This test runs our kernels on the same matrix and
distribution (seeded draws of our own) against the fp64 oracle on the same 16-bit inputs, and
requires, per case and output:
  * every element finite;
  * rel_rmse (rms error / rms of the reference) at most the reference kernel's own worst level in
    its report: bf16 0.0037, fp16 0.0008 (bounds 0.004 and 0.001);
  * at most 1e-5 of the elements outside 2e-2 + 5e-2|r|. With N(0, 1) inputs the bf16 error tail
    reaches the rule's 2e-2 floor near r = 0 for both implementations (the reference's own worst
    dQ error on this matrix is 0.0215); the count outside is printed.
dn / db are recorded, not asserted: with unit-variance inputs these sums cancel heavily, and the
reference's own kernels exceed its scalar rule on this matrix (the report marks the run failed).
Run with -s to see the per-group worst rel_rmse / max_abs, the figures quoted beside the
reference's report.
"""

import itertools
import math

import pytest
import torch

from oracle.ssa_oracle import ssa_reference_grads

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 5e-2
REL_RMSE_MAX = {"bf16": 4e-3, "fp16": 1e-3}
TAIL_FRACTION_MAX = 1e-5
CASES = list(itertools.product(("bf16", "fp16"), (1, 2), (8, 16, 24), (128, 512), (True, False),
                               ("contig", "strided")))
_RESULTS = {}


def _stats(a, r):
    d = a.double().cpu() - r
    return float(d.abs().max()), float(torch.sqrt((d * d).mean()) / (torch.sqrt((r * r).mean())
                                                                      + 1e-12))


@pytest.mark.parametrize("dt,B,Hq,N,causal,layout", CASES,
                         ids=[f"{c[0]}-B{c[1]}-Hq{c[2]}-N{c[3]}-{'c' if c[4] else 'nc'}-{c[5]}"
                              for c in CASES])
def test_reference_matrix_case(dt, B, Hq, N, causal, layout, cuda_device):
    from SSA import ssa_triton_kernel as K
    dtype = torch.bfloat16 if dt == "bf16" else torch.float16
    Hkv, D = 8, 32
    g = torch.Generator().manual_seed(B * 100003 + Hq * 1009 + N * 7 + int(causal) * 3 +
                                      int(layout == "strided"))
    if layout == "contig":
        q, k, v = (torch.randn(B, h, N, D, generator=g).to(dtype) for h in (Hq, Hkv, Hkv))
    else:  # [S, B, H, D] storage seen as [B, H, S, D], as Megatron hands it over
        q, k, v = (torch.randn(N, B, h, D, generator=g).to(dtype).permute(1, 2, 0, 3)
                   for h in (Hq, Hkv, Hkv))
    do = torch.randn(B, Hq, N, D, generator=g).to(dtype)
    n, b, scale = torch.tensor(1.5), torch.tensor(0.8), 1.0 / math.sqrt(D)
    qd, kd, vd, dod = (t.to(cuda_device) for t in (q, k, v, do))
    nd, bd = n.to(cuda_device), b.to(cuda_device)
    out, m = K.ssa_flash_attn_forward(qd, kd, vd, scale, nd, bd, causal)
    dq, dk, dv, dn, db = K.ssa_flash_attn_backward(qd, kd, vd, out, dod, m, scale, nd, bd, causal)
    torch.cuda.synchronize()
    ref = ssa_reference_grads(q, k, v, scale, n, b, do, causal)
    row = {"outside": 0}
    for name, got in (("out", out), ("dq", dq), ("dk", dk), ("dv", dv)):
        g64, r64 = got.double().cpu(), ref[name]
        assert torch.isfinite(g64).all(), name
        bad = int(((g64 - r64).abs() > ATOL + RTOL * r64.abs()).sum())
        row[name] = _stats(got, r64)
        row["outside"] += bad
        assert row[name][1] <= REL_RMSE_MAX[dt], f"{name}: rel_rmse {row[name][1]:.4g}"
        assert bad <= TAIL_FRACTION_MAX * g64.numel(), \
            f"{name}: {bad} of {g64.numel()} elements outside {ATOL} + {RTOL}|r|"
    for name, got in (("dn", dn), ("db", db)):
        r = float(ref[name])
        row[name] = abs(float(got) - r) / (2e-3 + 2e-2 * abs(r))  # fraction of the scalar rule
    _RESULTS[(dt, causal, B, Hq, N, layout)] = row


def test_reference_matrix_summary():
    """Prints the per-group worst rel_rmse / max_abs (runs after the cases in file order)."""
    if not _RESULTS:
        pytest.skip("no case ran")
    for dt in ("bf16", "fp16"):
        for causal in (True, False):
            rows = [v for k, v in _RESULTS.items() if k[0] == dt and k[1] == causal]
            if not rows:
                continue
            cells = [f"{x}: {max(r[x][1] for r in rows):.4f} / {max(r[x][0] for r in rows):.4f}"
                     for x in ("out", "dq", "dk", "dv")]
            scal = max(max(r["dn"], r["db"]) for r in rows)
            outside = sum(r["outside"] for r in rows)
            print(f"[reference matrix] {dt} {'causal' if causal else 'non-causal'}: "
                  + " | ".join(cells) + f" | dn/db worst {scal:.2f} of the scalar rule"
                  + f" | {outside} elements outside 2e-2 + 5e-2|r| in {len(rows)} cases")
