"""Multi-rank host logic on CPU with gloo (world size 2): the (batch, kv-head) shard plan covers
every unit exactly once, the dn/db all-reduce sums partial gradients exactly as the full-batch
oracle does, and a rank that fails before the collective makes the other rank's collective end
with an error (short process-group timeout) instead of hanging."""

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

from conftest import from_queue, to_queue

REPO = Path(__file__).resolve().parent.parent


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_unit_shard_covers_all_units_once():
    from SSA.shard import balanced_range, batch_shard, unit_shard
    for B, Hkv in ((8, 8), (3, 5), (1, 8), (16, 1)):
        for world in (1, 2, 3, 4, 8):
            seen = []
            sizes = []
            for r in range(world):
                u = unit_shard(B, Hkv, world, r)
                seen += u
                sizes.append(len(u))
            assert sorted(seen) == [(b, h) for b in range(B) for h in range(Hkv)]
            assert max(sizes) - min(sizes) <= 1
    assert batch_shard(8, 4, 3) == slice(6, 8)
    assert balanced_range(5, 2, 0) == (0, 3) and balanced_range(5, 2, 1) == (3, 5)
    with pytest.raises(ValueError):
        balanced_range(4, 2, 2)


def _worker(rank, world, port, q, k, v, do, n, b, out_q):
    sys.path[:0] = [str(REPO), str(REPO / "luciole-1b_b200")]
    import datetime
    import torch.distributed as dist
    from SSA.shard import allreduce_ssa_param_grads, batch_shard
    from oracle.ssa_oracle import ssa_reference_grads
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    sl = batch_shard(q.shape[0], world, rank)
    r = ssa_reference_grads(q[sl], k[sl], v[sl], 0.25, n, b, do[sl], True,
                            compute_dtype=torch.float64)
    dn, db = r["dn"].clone(), r["db"].clone()
    allreduce_ssa_param_grads(dn, db, buffer=torch.empty(dn.numel() + 1, dtype=torch.float64))
    # the layout the SSA backward returns (dn, db adjacent in one buffer): in place, async
    pair = torch.cat([r["dn"].reshape(-1), r["db"].reshape(1)])
    dn2, db2 = pair[:dn.numel()].view(dn.shape), pair[dn.numel()]
    allreduce_ssa_param_grads(dn2, db2, async_op=True).wait()
    assert torch.equal(dn2, dn) and torch.equal(db2, db)
    out_q.put(to_queue((rank, dn, db)))
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_dn_db_allreduce_matches_full_batch():
    from oracle.ssa_oracle import ssa_reference_grads
    g = torch.Generator().manual_seed(11)
    B, Hq, Hkv, N, D = 4, 4, 2, 32, 8
    q = torch.randn(B, Hq, N, D, generator=g, dtype=torch.float64)
    k = torch.randn(B, Hkv, N, D, generator=g, dtype=torch.float64)
    v = torch.randn(B, Hkv, N, D, generator=g, dtype=torch.float64)
    do = torch.randn(B, Hq, N, D, generator=g, dtype=torch.float64)
    n = torch.full((Hq,), 0.5, dtype=torch.float64)
    b = torch.tensor(0.8, dtype=torch.float64)
    full = ssa_reference_grads(q, k, v, 0.25, n, b, do, True)
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, k, v, do, n, b, out_q))
             for r in range(2)]
    for p in procs:
        p.start()
    results = [from_queue(out_q.get(timeout=120)) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, dn, db in results:
        assert torch.allclose(dn, full["dn"], rtol=1e-12, atol=1e-12), rank
        assert torch.allclose(db, full["db"], rtol=1e-12, atol=1e-12), rank


def test_adjacent_param_grads_reduce_in_place():
    from SSA.shard import _adjacent_span, allreduce_ssa_param_grads
    buf = torch.arange(5, dtype=torch.float32)
    dn, db = buf[:4].view(4), buf[4]
    span = _adjacent_span(dn, db)
    assert span is not None and span.data_ptr() == buf.data_ptr() and span.numel() == 5
    assert _adjacent_span(buf[:1].view(()), buf[1]) is not None  # scalar n
    assert _adjacent_span(torch.zeros(4), torch.zeros(())) is None  # separate storages
    assert _adjacent_span(buf[:3], buf[4]) is None  # gap
    assert _adjacent_span(buf[:4].double(), buf[4]) is None  # dtype
    with pytest.raises(ValueError, match="adjacent"):
        allreduce_ssa_param_grads(torch.zeros(4), torch.zeros(()), async_op=True)


def _failing_worker(rank, world, port, out_q):
    sys.path[:0] = [str(REPO), str(REPO / "luciole-1b_b200")]
    import datetime
    import torch.distributed as dist
    from SSA.shard import allreduce_ssa_param_grads
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        out_q.put((rank, "left before the collective"))
        out_q.close()
        out_q.join_thread()
        os._exit(0)  # a rank that dies between steps
    try:
        allreduce_ssa_param_grads(torch.ones(4, dtype=torch.float64),
                                  torch.ones((), dtype=torch.float64))
        out_q.put((rank, "no error"))
    except Exception as e:  # the collective must fail, not hang
        out_q.put((rank, f"error: {type(e).__name__}"))
    out_q.close()
    out_q.join_thread()
    os._exit(0)


def test_missing_rank_fails_collective_instead_of_hanging():
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, out_q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(out_q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "left before the collective"
    assert res[0].startswith("error"), res[0]
