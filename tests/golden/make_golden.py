#!/usr/bin/env python3
"""Generate the golden SSA attention vectors from the reference implementation itself.

This script is test infrastructure. It imports the reference's own Triton kernels
(``training/train/train_ssa_triton/SSA/ssa_triton_kernel.py``) from a read-only checkout
and runs them on the CPU under ``TRITON_INTERPRET=1``. The interpreter evaluates
``tl.dot`` in exact fp32 (no TF32), so these vectors are the reference algorithm's
fp32 results: forward ``ssa_flash_attn_forward`` (ssa_triton_kernel.py:732-792) and
backward ``ssa_flash_attn_backward`` (ssa_triton_kernel.py:795-897).

The autotuner needs a GPU to benchmark, so the forward config list is replaced by one
config at runtime (BLOCK_M=64, BLOCK_N=32); this changes the tiling, not the math.
bf16 is not generated: the interpreter's bf16 path returns garbage (checked by hand),
so bf16 parity is anchored on fp32 vectors computed on bf16-representable inputs.

Usage (in a container that has the reference checkout; never needed on a GPU box):
    python tests/golden/make_golden.py --reference <path-to-luciole-1B-checkout>
Writes ``tests/golden/ssa_golden_<case>.npz``.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

HERE = Path(__file__).resolve().parent

# (name, B, Hq, Hkv, N, D, causal, layout, n, b, scale_inputs, bf16_round)
CASES = [
    ("mha_causal_d64", 1, 2, 2, 128, 64, True, "contig", 1.5, 0.8, 1.0, False),
    ("gqa_causal_d32", 1, 4, 2, 256, 32, True, "contig", 1.5, 0.8, 1.0, False),
    ("gqa_noncausal_d64", 1, 4, 1, 128, 64, False, "contig", 0.43, 0.8, 1.0, False),
    ("strided_causal_d32", 2, 2, 1, 128, 32, True, "strided", 1.5, 0.8, 1.0, False),
    ("bf16vals_gqa_causal_d64", 1, 4, 1, 128, 64, True, "contig", 0.43, 0.8, 0.5, True),
    ("mha_causal_d128", 1, 1, 1, 128, 128, True, "contig", 1.5, 0.8, 0.5, False),
]


def _make(B, Hq, Hkv, N, D, layout, scale_inputs, bf16_round, gen):
    import torch

    def rnd(*shape):
        t = torch.randn(*shape, generator=gen, dtype=torch.float32) * scale_inputs
        if bf16_round:
            t = t.to(torch.bfloat16).to(torch.float32)
        return t

    # Always generate in [S, B, H, D] order so "strided" is the Megatron permuted view
    q_sbhd = rnd(N, B, Hq, D)
    k_sbhd = rnd(N, B, Hkv, D)
    v_sbhd = rnd(N, B, Hkv, D)
    do_sbhd = rnd(N, B, Hq, D)
    q, k, v, do = (t.permute(1, 2, 0, 3) for t in (q_sbhd, k_sbhd, v_sbhd, do_sbhd))
    if layout == "contig":
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    return q, k, v, do.contiguous()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="path to the luciole-1B checkout (the directory holding training/)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "training/train/train_ssa_triton"))

    import torch
    import triton
    import SSA.ssa_triton_kernel as K  # the reference's module

    K._ssa_attn_fwd.configs = [triton.Config({"BLOCK_M": 64, "BLOCK_N": 32}, num_stages=2, num_warps=4)]

    for i, (name, B, Hq, Hkv, N, D, causal, layout, n, b, sc, r16) in enumerate(CASES):
        gen = torch.Generator().manual_seed(1000 + i)
        q, k, v, do = _make(B, Hq, Hkv, N, D, layout, sc, r16, gen)
        scale = 1.0 / math.sqrt(D)
        ssa_n = torch.tensor(n, dtype=torch.float32)
        ssa_b = torch.tensor(b, dtype=torch.float32)
        out, m = K.ssa_flash_attn_forward(q, k, v, scale, ssa_n, ssa_b, causal=causal)
        dq, dk, dv, dn, db = K.ssa_flash_attn_backward(q, k, v, out, do, m, scale, ssa_n, ssa_b,
                                                       causal=causal)
        meta = dict(name=name, B=B, Hq=Hq, Hkv=Hkv, N=N, D=D, causal=causal, layout=layout,
                    ssa_n=n, ssa_b=b, softmax_scale=scale, bf16_representable=r16,
                    generator="reference ssa_triton_kernel.py under TRITON_INTERPRET=1, fp32")
        path = HERE / f"ssa_golden_{name}.npz"
        import numpy as np
        np.savez_compressed(
            path,
            meta=json.dumps(meta),
            q=q.contiguous().numpy(), k=k.contiguous().numpy(), v=v.contiguous().numpy(),
            dout=do.numpy(), out=out.contiguous().numpy(), m=m.numpy(),
            dq=dq.contiguous().numpy(), dk=dk.contiguous().numpy(), dv=dv.contiguous().numpy(),
            dn=np.float64(dn.item()), db=np.float64(db.item()),
        )
        print(f"{name}: dn={dn.item():.6f} db={db.item():.6f} |out|max={out.abs().max().item():.4f} -> {path.name}")


if __name__ == "__main__":
    main()
