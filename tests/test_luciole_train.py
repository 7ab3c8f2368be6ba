"""The config-5 training step (Luciole-1B-shaped decoder over the SSA path).

CPU tests run the decoder with the oracle's eager SSA attention injected (the product path has
no CPU attention): parameter count of the real config, a loss that falls when one batch is
fitted, fp32 master weights, and DDP over two gloo ranks keeping the replicas identical.
GPU tests run the real kernels: a small decoder's logits and gradients against the same
weights with the oracle attention (bf16 tolerance), and the full-size config's step running.
"""

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parent.parent

TINY = dict(layers=2, hidden=128, heads=4, kv_heads=2, ffn=256, vocab=512)


def _oracle_attention(q, k, v, scale, n, b):
    from oracle.ssa_oracle import ssa_reference_forward
    out, _ = ssa_reference_forward(q, k, v, scale, n, b, True, compute_dtype=torch.float32)
    return out.to(q.dtype)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_param_count_is_luciole_1b():
    import luciole_train as LT
    cfg = LT.LucioleConfig()
    assert 0.95e9 < LT.param_count(cfg) < 1.10e9
    tiny = LT.LucioleConfig(**TINY)
    model = LT.build(tiny, "cpu", torch.float32, attn_fn=_oracle_attention)
    assert LT.param_count(tiny) == sum(p.numel() for p in model.parameters())


def test_fitting_one_batch_lowers_the_loss_fp32_masters():
    import luciole_train as LT
    cfg = LT.LucioleConfig(**TINY)
    model = LT.build(cfg, "cpu", torch.bfloat16, seed=1, attn_fn=_oracle_attention)
    opt = LT.MasterWeightAdamW(list(model.parameters()), lr=3e-3, weight_decay=0.0)
    assert all(m.dtype == torch.float32 for m in opt.master)
    g = torch.Generator().manual_seed(2)
    tok = torch.randint(0, cfg.vocab, (2, 64), generator=g)
    losses = [float(LT.train_step(model, opt, tok[:, :-1], tok[:, 1:])) for _ in range(12)]
    assert losses[-1] < losses[0] - 0.5, losses
    # the bf16 weights are the rounded fp32 masters
    for p, m in zip(opt.params, opt.master):
        assert torch.equal(p, m.to(p.dtype))


def _ddp_worker(rank, world, port, out_q):
    sys.path[:0] = [str(REPO), str(REPO / "luciole-1b_b200")]
    import datetime
    import torch.distributed as dist
    from torch.nn.parallel import DistributedDataParallel as DDP
    import luciole_train as LT
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    cfg = LT.LucioleConfig(**TINY)
    model = LT.build(cfg, "cpu", torch.float32, seed=5, attn_fn=_oracle_attention)
    ddp = DDP(model)
    opt = LT.MasterWeightAdamW(list(model.parameters()), lr=1e-3)
    g = torch.Generator().manual_seed(100 + rank)  # different data per rank
    for _ in range(2):
        tok = torch.randint(0, cfg.vocab, (2, 33), generator=g)
        LT.train_step(ddp, opt, tok[:, :-1], tok[:, 1:])
    flat = torch.cat([p.detach().reshape(-1) for p in model.parameters()])
    # a numpy copy travels by value (a tensor would travel as a shared-memory handle, which the
    # parent cannot open once this process has exited)
    out_q.put((rank, flat.numpy().copy()))
    dist.barrier()
    dist.destroy_process_group()


def test_ddp_two_gloo_ranks_keep_replicas_identical():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ddp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert (res[0] == res[1]).all()


@pytest.mark.gpu
def test_decoder_with_kernels_matches_oracle_attention(cuda_device):
    import luciole_train as LT
    cfg = LT.LucioleConfig(layers=2, hidden=512, heads=8, kv_heads=2, ffn=1024, vocab=1024)
    dev = cuda_device
    model = LT.build(cfg, dev, torch.bfloat16, seed=3)
    ref = LT.build(cfg, dev, torch.bfloat16, seed=3, attn_fn=_oracle_attention)
    g = torch.Generator().manual_seed(4)
    tok = torch.randint(0, cfg.vocab, (2, 257), generator=g).to(dev)
    la = model.loss(tok[:, :-1], tok[:, 1:])
    lb = ref.loss(tok[:, :-1], tok[:, 1:])
    la.backward()
    lb.backward()
    torch.cuda.synchronize()
    assert abs(float(la.detach()) - float(lb.detach())) < 2e-2 * abs(float(lb.detach()))
    for (name, pa), pb in zip(model.named_parameters(), ref.parameters()):
        ga, gb = pa.grad.float(), pb.grad.float()
        rel = (ga - gb).norm() / gb.norm().clamp_min(1e-12)
        assert rel < 5e-2, (name, float(rel))


@pytest.mark.gpu
def test_full_config_step_runs_and_learns(cuda_device):
    import luciole_train as LT
    cfg = LT.LucioleConfig()
    dev = cuda_device
    model = LT.build(cfg, dev, torch.bfloat16, seed=0)
    opt = LT.MasterWeightAdamW(list(model.parameters()), lr=1e-3, weight_decay=0.0)
    g = torch.Generator().manual_seed(9)
    tok = torch.randint(0, cfg.vocab, (1, 2049), generator=g).to(dev)
    losses = [float(LT.train_step(model, opt, tok[:, :-1], tok[:, 1:])) for _ in range(4)]
    assert all(torch.isfinite(torch.tensor(losses)))
    assert abs(losses[0] - torch.log(torch.tensor(float(cfg.vocab)))) < 1.0  # near uniform
    assert losses[-1] < losses[0]
    del model, opt
    torch.cuda.empty_cache()
