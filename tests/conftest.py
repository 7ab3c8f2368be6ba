"""Test configuration: markers, import paths and shared fixtures.

``-m gpu`` tests need a B200 and call the CUDA kernels through the C ABI; everything else
runs on the CPU (oracle vs golden vectors, host logic, library loading and symbol export).
"""

import json
import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "luciole-1b_b200"
for p in (str(REPO), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


def load_golden():
    """All committed golden cases: list of (meta dict, arrays dict)."""
    import numpy as np
    cases = []
    for f in sorted(GOLDEN.glob("ssa_golden_*.npz")):
        z = np.load(f)
        meta = json.loads(str(z["meta"]))
        arrays = {k: z[k] for k in z.files if k != "meta"}
        cases.append((meta, arrays))
    return cases


def golden_qkv(meta, arrays, device="cpu", dtype=None):
    """Rebuild q, k, v, dout exactly as the generator laid them out ('strided' is the
    Megatron [S,B,H,D]-permuted view)."""
    import torch
    dtype = dtype or torch.float32
    q, k, v, do = (torch.from_numpy(arrays[x]) for x in ("q", "k", "v", "dout"))
    if meta["layout"] == "strided":
        q, k, v = (t.permute(2, 0, 1, 3).contiguous().to(device=device, dtype=dtype).permute(1, 2, 0, 3)
                   for t in (q, k, v))
    else:
        q, k, v = (t.to(device=device, dtype=dtype) for t in (q, k, v))
    return q, k, v, do.to(device=device, dtype=dtype)


def to_queue(obj) -> bytes:
    """Serialise a worker's result (tensors of any dtype included) for a multiprocessing queue.
    Tensors put on a queue directly travel as shared-memory handles that the parent can no longer
    open once the worker has exited; these bytes travel by value."""
    import io
    import torch
    buf = io.BytesIO()
    torch.save(obj, buf)
    return buf.getvalue()


def from_queue(data: bytes):
    import io
    import torch
    return torch.load(io.BytesIO(data), weights_only=False)


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
