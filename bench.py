#!/usr/bin/env python3
"""SSA attention fwd+bwd benchmark (benchmark config 2) on B200, one process per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    (N > 1: python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...)

One step = forward + backward of SSA attention over one batch: B=8, Hq=32, Hkv=8, S=2048,
D=64, bf16, causal, per-head n ~ U(0.3, 0.6), b = 0.8 (seeded synthetic data with the config's
shapes and value distributions: q, k, v ~ N(0,1)*0.5, dO ~ N(0,1)). FLOPs follow the
FlashAttention convention, 14*D*E with E = B*Hq*S^2/2 causal score elements (SSA transform
work is not counted).

Multi-GPU: the (batch, kv-head) units are independent, so each rank owns its own batch of 8
sequences (weak scaling, global batch 8*N) and the only exchange is one all-reduce of the
33 floats of dn/db per step. ``value`` = total FLOPs of all ranks / max-over-ranks device time.

Lines printed (rank 0, one JSON line):
  value     device-resident inputs, timed with CUDA events on the launching stream;
  e2e       the same metric through the public API with pinned HOST buffers: H2D of
            q, k, v, dO and D2H of out, dq, dk, dv, dn, db inside the timed region;
  roofline  the backward call (the dominant launch) against the measured dense bf16 peak;
  cpu_baseline  the CPU oracle (fp32 eager restatement of the reference's SSA math) timed on
            this host's cores on a bounded sample (one q-head of one sequence).
``--impl reference`` times that CPU restatement alone (the reference's own Triton code is not
present on the GPU box and may not be copied into this repository) and prints its line with
"impl": "reference".
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
for _p in (str(REPO), str(REPO / "luciole-1b_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

# Workloads (the benchmark configs). c2 is the headline and the default; c3 / c4 are measured with
# --config for the record. c3: packed documents, lengths seeded uniform in [128, 4096] until
# 65,536 tokens (last one clipped); c4: one 32,768-token sequence at D = 128.
CONFIGS = {
    "c2": dict(B=8, HQ=32, HKV=8, S=2048, D=64, varlen=False,
               workload="config2: SSA causal GQA fwd+bwd, B=8 Hq=32 Hkv=8 S=2048 D=64 bf16, per-head n",
               metric="SSA attn fwd+bwd TFLOP/s (bf16, B=8 Hq=32 Hkv=8 S=2048 D=64 causal)"),
    "c3": dict(B=1, HQ=32, HKV=8, S=65536, D=64, varlen=True,
               workload="config3: SSA causal GQA fwd+bwd, packed documents 65536 tokens, lengths U[128,4096], Hq=32 Hkv=8 D=64 bf16",
               metric="SSA attn fwd+bwd TFLOP/s (bf16, varlen 65536 tokens, Hq=32 Hkv=8 D=64 causal)"),
    "c4": dict(B=1, HQ=32, HKV=8, S=32768, D=128, varlen=False,
               workload="config4: SSA causal GQA fwd+bwd, B=1 Hq=32 Hkv=8 S=32768 D=128 bf16, per-head n",
               metric="SSA attn fwd+bwd TFLOP/s (bf16, B=1 Hq=32 Hkv=8 S=32768 D=128 causal)"),
}
CFG = CONFIGS["c2"]
B, HQ, HKV, S, D = 8, 32, 8, 2048, 64
CAUSAL = True
SSA_B = 0.8
WORKLOAD = CFG["workload"]
METRIC = CFG["metric"]
UNIT = "TFLOP/s"
DOC_LENS = None  # varlen document lengths (c3)


def c3_doc_lengths(total: int = 65536, seed: int = 3) -> list:
    """Config 3's packing: document lengths drawn seeded and uniform in [128, 4096] until they
    sum to `total` tokens (the last one clipped). The GPU parity tests check the same packing."""
    g = torch.Generator().manual_seed(seed)
    lens, tot = [], 0
    while tot < total:
        L = min(int(torch.randint(128, 4097, (1,), generator=g)), total - tot)
        lens.append(L)
        tot += L
    return lens


def select_config(name: str) -> None:
    global CFG, B, HQ, HKV, S, D, WORKLOAD, METRIC, DOC_LENS
    CFG = CONFIGS[name]
    B, HQ, HKV, S, D = CFG["B"], CFG["HQ"], CFG["HKV"], CFG["S"], CFG["D"]
    WORKLOAD, METRIC = CFG["workload"], CFG["metric"]
    DOC_LENS = c3_doc_lengths(S) if CFG["varlen"] else None


def score_elements() -> float:
    if DOC_LENS is not None:
        return float(HQ * sum(L * L // 2 for L in DOC_LENS))
    return float(B * HQ * (S * S // 2 if CAUSAL else S * S))

def shard_score_elements(n_seq: int, n_qheads: int) -> float:
    """Score elements of a shard holding n_seq sequences (all documents when packed) x n_qheads."""
    if DOC_LENS is not None:
        return float(n_qheads * sum(L * L // 2 for L in DOC_LENS))
    return float(n_seq * n_qheads * (S * S // 2 if CAUSAL else S * S))


def strong_shard(world: int, rank: int):
    """This rank's part of the config's fixed batch for strong scaling: the balanced contiguous
    range of (batch, kv-head) units that SSA.shard.unit_shard assigns, as (batch slice, kv-head
    slice). Needs the range to be a rectangle: world divides B (whole sequences) or world is a
    multiple of B whose share of each sequence divides Hkv (a kv-head range of one sequence)."""
    from SSA.shard import unit_shard
    units = unit_shard(B, HKV, world, rank)
    bs = sorted({u[0] for u in units})
    hs = sorted({u[1] for u in units})
    rect = (len(units) == len(bs) * len(hs) and bs == list(range(bs[0], bs[-1] + 1))
            and hs == list(range(hs[0], hs[-1] + 1)))
    if not units or not rect:
        raise SystemExit(f"--scaling strong: {world} ranks do not split B={B} x Hkv={HKV} into "
                         f"rectangles of (batch, kv-head) units; use --scaling weak")
    return slice(bs[0], bs[-1] + 1), slice(hs[0], hs[-1] + 1)


# DRAM traffic per launch of the dominant kernel (bwd_sm100_kernel) comes from the committed ncu
# summary of this workload, and only while the kernel source is the one that capture measured:
# the summary's "bench-traffic:" line carries the source file's sha256 prefix and the bytes.
TRAFFIC_PROFILE = REPO / "profiles" / "ssa_bwd_sm100_config2.md"
TRAFFIC_SOURCE = REPO / "luciole-1b_b200" / "csrc" / "ssa_sm100_bwd.cu"


def ncu_traffic():
    """(dram bytes per launch or None, note)."""
    import hashlib
    import re
    if not TRAFFIC_PROFILE.exists():
        return None, "no ncu summary committed"
    m = re.search(r"^bench-traffic:.*sha256_16=([0-9a-f]{16}).*dram_bytes=([0-9.e+]+)",
                  TRAFFIC_PROFILE.read_text(), re.M)
    if not m:
        return None, "ncu summary has no bench-traffic line"
    sha = hashlib.sha256(TRAFFIC_SOURCE.read_bytes()).hexdigest()[:16]
    if sha != m.group(1):
        return None, "stale: the ncu capture measured an earlier ssa_sm100_bwd.cu"
    return float(m.group(2)), f"ncu capture of ssa_sm100_bwd.cu sha256 {sha}"


REFERENCE_TRITON = {
    "unavailable": "the reference's Triton SSA kernels cannot be timed on the B200 box: the "
                   "reference is not an installable package (pip: 'Neither setup.py nor "
                   "pyproject.toml found', so baseline/_ref stays empty) and its Python "
                   "sources may not travel to the box or be copied into this repository"}


def flops_per_rank() -> float:
    return 14.0 * D * score_elements()


def flops_bwd_per_rank() -> float:
    return 10.0 * D * score_elements()


# The SSA transform's special-function work (not counted in the FLOPs): lg2 and ex2 per score
# element in the forward and again in the backward (the reciprocal runs on the FMA pipe). B200
# issues 16 such operations per clock per SM.
SFU_OPS_PER_ELEMENT = 4
SFU_OPS_PER_CLK_SM = 16


def sfu_floor(ms_per_step: float, elements: float) -> dict:
    """The special-function floor of one step over `elements` score elements on one GPU
    (algorithmic elements, max SM clock) and the fraction of it the measured step reaches."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count if torch.cuda.is_available() else 148
    mhz = 1965.0
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        mhz = float(json.loads(p.read_text()).get("sm_max_mhz", mhz))
    ops = SFU_OPS_PER_ELEMENT * elements
    peak = SFU_OPS_PER_CLK_SM * sms * mhz * 1e6
    floor_ms = ops / peak * 1e3
    return {"ops_per_step": ops, "peak_ops_per_s": peak, "floor_ms": floor_ms,
            "frac": floor_ms / ms_per_step}


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while the timed region runs (reads
    only; no GPU setting is changed).

    deferred=True samples only after arm(), which the caller invokes once the host has queued
    the whole timed region and is about to block in a synchronize: the samples then fall while
    the device runs the queued work, and the sampling thread never competes for the interpreter
    lock with the thread that launches the kernels (a sampler running during the launches
    delayed them by up to 15 ms, long enough to show in a timed region of 20 steps of ~1 ms)."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, index: int, deferred: bool = False):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop, self._armed = threading.Event(), threading.Event()
        self._interval = 0.002 if deferred else 0.02
        if not deferred:
            self._armed.set()
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            # first calls resolve the library entry points: done here, outside the timed region
            pynvml.nvmlDeviceGetClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            pynvml.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        except Exception:
            self._nv = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def arm(self):
        self._armed.set()

    def _run(self):
        self._armed.wait()
        while not self._stop.is_set():
            self._sample()
            self._stop.wait(self._interval)

    def _sample(self):
        try:
            self.samples.append(self._nv.nvmlDeviceGetClockInfo(self._h, self._nv.NVML_CLOCK_SM))
            r = self._nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            for bit, name in self.REASONS.items():
                if r & bit and name != "gpu_idle":
                    self.reasons.add(name)
        except Exception:
            pass

    def __enter__(self):
        if self._nv is not None:
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._armed.set()
        if self._nv is not None:
            self._t.join(timeout=1)
            self._sample()  # the timed region's end

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


def make_inputs(device, seed):
    """Seeded synthetic tensors: [B, H, S, D], or packed [T, H, D] for varlen."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    if DOC_LENS is not None:
        q = (torch.randn(S, HQ, D, generator=g) * 0.5).to(torch.bfloat16)
        k = (torch.randn(S, HKV, D, generator=g) * 0.5).to(torch.bfloat16)
        v = (torch.randn(S, HKV, D, generator=g) * 0.5).to(torch.bfloat16)
        do = torch.randn(S, HQ, D, generator=g).to(torch.bfloat16)
    else:
        q = (torch.randn(B, HQ, S, D, generator=g) * 0.5).to(torch.bfloat16)
        k = (torch.randn(B, HKV, S, D, generator=g) * 0.5).to(torch.bfloat16)
        v = (torch.randn(B, HKV, S, D, generator=g) * 0.5).to(torch.bfloat16)
        do = torch.randn(B, HQ, S, D, generator=g).to(torch.bfloat16)
    n = 0.3 + 0.3 * torch.rand(HQ, generator=g)
    return q, k, v, do, n


def cpu_oracle_sample(threads: int):
    """Time the CPU restatement of the reference's eager SSA path (fp32, autograd) on one q-head
    of one sequence at S=2048; returns (TFLOP/s, seconds, flops)."""
    from oracle.ssa_oracle import ssa_reference_grads
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(123)
    Sc = min(S, 2048)  # a bounded sample: one q-head of one sequence of at most 2048 tokens
    q = torch.randn(1, 1, Sc, D, generator=g) * 0.5
    k = torch.randn(1, 1, Sc, D, generator=g) * 0.5
    v = torch.randn(1, 1, Sc, D, generator=g) * 0.5
    do = torch.randn(1, 1, Sc, D, generator=g)
    n, b = torch.tensor(0.43), torch.tensor(SSA_B)
    flops = 14.0 * D * (Sc * Sc // 2)
    ssa_reference_grads(q, k, v, D ** -0.5, n, b, do, CAUSAL, compute_dtype=torch.float32)  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        ssa_reference_grads(q, k, v, D ** -0.5, n, b, do, CAUSAL, compute_dtype=torch.float32)
        reps += 1
        el = time.perf_counter() - t0
        if el > 12.0 or reps >= 1000:
            break
    return flops * reps / el / 1e12, el, flops * reps, reps


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    vals, secs = [], []
    fl = 0.0
    for i in range(args.warmup + args.steps):
        v, el, fl, _ = _one_ref_step(threads)
        if i >= args.warmup:
            vals.append(v)
            secs.append(el)
    val = statistics.median(vals)
    step_s = statistics.median(secs)
    sample = (f"one q-head of one sequence (S={min(S, 2048)}, D={D}, causal) per step: "
              f"{fl:.4g} FLOPs in a median {step_s * 1e3:.1f} ms; fp32 eager restatement of the "
              f"reference's SSA path with autograd, {threads} threads")
    line = {"impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "ms_per_step": step_s * 1e3, "sample_flops_per_step": fl,
            # the whole config's work at this rate (the sample is a bounded slice of it)
            "config_ms_equivalent": flops_per_rank() / (val * 1e12) * 1e3,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "global_batch": B, "seq_len": S},
            "cpu_baseline": {"value": val, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _one_ref_step(threads):
    from oracle.ssa_oracle import ssa_reference_grads
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(7)
    Sc = min(S, 2048)
    q = torch.randn(1, 1, Sc, D, generator=g) * 0.5
    k = torch.randn(1, 1, Sc, D, generator=g) * 0.5
    v = torch.randn(1, 1, Sc, D, generator=g) * 0.5
    do = torch.randn(1, 1, Sc, D, generator=g)
    t0 = time.perf_counter()
    ssa_reference_grads(q, k, v, D ** -0.5, torch.tensor(0.43), torch.tensor(SSA_B), do, CAUSAL,
                        compute_dtype=torch.float32)
    el = time.perf_counter() - t0
    fl = 14.0 * D * (Sc * Sc // 2)
    return fl / el / 1e12, el, fl, 1


def run_train(args):
    """Benchmark config 5: one Luciole-1B-shaped training step per timed step (forward, loss,
    backward with DDP's gradient all-reduce, AdamW on fp32 masters) on random token ids,
    sequence 2048, micro-batch 4 per GPU. value = tokens/s of the whole job."""
    import luciole_train as LT
    from SSA import _lib
    world, rank, local = dist_setup(args)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = LT.LucioleConfig()
    mbs, seq = 4, 2048
    model = LT.build(cfg, dev, torch.bfloat16, seed=0)
    net = model
    if world > 1:
        from torch.nn.parallel import DistributedDataParallel as DDP
        net = DDP(model, device_ids=[local], gradient_as_bucket_view=True)
    opt = LT.MasterWeightAdamW(list(model.parameters()))
    g = torch.Generator().manual_seed(1000 + rank)
    tok_h = torch.randint(0, cfg.vocab, (mbs, seq + 1), generator=g).pin_memory()
    tok = tok_h.to(dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        LT.train_step(net, opt, tok[:, :-1], tok[:, 1:])
    barrier()
    steps = min(args.steps, 30)
    st = torch.cuda.current_stream(dev)
    launches0 = _lib.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        e0.record(st)
        for _ in range(steps):
            LT.train_step(net, opt, tok[:, :-1], tok[:, 1:])
        e1.record(st)
        barrier()
    launches = _lib.launch_count() - launches0
    ms = e0.elapsed_time(e1) / steps
    # e2e: token ids copied from pinned host memory and the loss read back, every step
    buf = torch.empty_like(tok)
    loss_h = torch.empty((), dtype=torch.float32).pin_memory()
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(3, min(steps, 10))
    e2.record(st)
    for _ in range(e2e_steps):
        buf.copy_(tok_h, non_blocking=True)
        loss = LT.train_step(net, opt, buf[:, :-1], buf[:, 1:])
        loss_h.copy_(loss, non_blocking=True)
    e3.record(st)
    barrier()
    e2e_ms = e2.elapsed_time(e3) / e2e_steps
    if world > 1:
        t = torch.tensor([ms, e2e_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, e2e_ms = (float(x) for x in t.tolist())
    tokens = world * mbs * seq
    value = tokens / (ms * 1e-3)
    flops_tok = LT.train_flops_per_token(cfg, seq)
    peak_tf, _, peak_kind = measured_peaks()
    sustained = peak_tf
    pk = REPO / "MEASURED_PEAKS.json"
    if pk.exists():
        sustained = json.loads(pk.read_text()).get("bf16_tflops_sustained", peak_tf)
    achieved = flops_tok * tokens / world / (ms * 1e-3) / 1e12
    if rank == 0:
        line = {
            "metric": "Luciole-1B train tokens/s (bf16 weights, fp32 master AdamW, seq 2048, "
                      "mbs 4 per GPU)",
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "config5: Llama-style decoder 16 x 2048, 32/8 heads (D=64), "
                                   "SwiGLU 5632, RMSNorm, RoPE 1e4, vocab 65536, SSA attention "
                                   "kernels; random-init weights, uniform random token ids",
                       "global_batch": mbs * world, "seq_len": seq,
                       "params": LT.param_count(cfg),
                       "parallelism": f"DDP x{world} (NCCL all-reduce of bf16 grads)"},
            "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": tok_h.numel() * tok_h.element_size(),
                    "d2h_bytes_per_step": 4, "ms_per_step": e2e_ms},
            "roofline": {"bound": "tensor", "kernel": "whole training step (model FLOPs)",
                         "achieved": achieved, "peak": sustained, "unit": "TFLOP/s",
                         "frac": achieved / sustained,
                         "peak_kind": f"{peak_kind} bf16 sustained", "traffic": None},
            "cpu_baseline": None,
            "clocks": clk.summary(),
            "gpu_launches": launches,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS) + ["c5"],
                    help="c2 (headline), c3, c4: attention workloads; c5: the Luciole-1B "
                         "training step (tokens/s)")
    ap.add_argument("--cp", action="store_true",
                    help="context-parallel ring over the ranks (strong scaling of one sequence; "
                         "use with --config c4 under torchrun)")
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="strong (default): the config's fixed batch is split across the ranks "
                         "by (batch, kv-head) units; weak: every rank runs the whole config on "
                         "its own data (global batch = N x the config's)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.config == "c5":
        if args.impl == "reference":
            if int(os.environ.get("RANK", "0")) == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference's training "
                                  "step needs NeMo / Megatron and its Triton kernels on a GPU, "
                                  "none of which is in this image"}), flush=True)
            return
        run_train(args)
        return
    select_config(args.config)
    if args.impl == "reference":
        run_reference(args)
        return

    world, rank, local = dist_setup(args)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    from SSA import _lib
    from SSA.shard import allreduce_ssa_param_grads
    from SSA.ssa_triton_kernel import ssa_flash_attn_backward, ssa_flash_attn_forward
    import torch.distributed as dist

    from SSA.ssa_triton_kernel import (ssa_flash_attn_varlen_backward,
                                       ssa_flash_attn_varlen_forward)
    strong = args.scaling == "strong" and not args.cp
    if strong:
        # The config's fixed batch, split by (batch, kv-head) units: every rank builds the same
        # seeded inputs and keeps its own units (a rectangle of sequences x kv-heads).
        bsl, hsl = strong_shard(world, rank)
        g = HQ // HKV
        qsl = slice(hsl.start * g, hsl.stop * g)
        q_h, k_h, v_h, do_h, n_h = make_inputs(dev, seed=0)
        if DOC_LENS is not None:
            q_h, do_h = (t[:, qsl].contiguous() for t in (q_h, do_h))
            k_h, v_h = (t[:, hsl].contiguous() for t in (k_h, v_h))
        else:
            q_h, do_h = (t[bsl, qsl].contiguous() for t in (q_h, do_h))
            k_h, v_h = (t[bsl, hsl].contiguous() for t in (k_h, v_h))
        n_h = n_h[qsl].contiguous()
        shard_elems = shard_score_elements(bsl.stop - bsl.start, qsl.stop - qsl.start)
    else:
        q_h, k_h, v_h, do_h, n_h = make_inputs(dev, seed=rank)
        qsl = slice(0, HQ)
        shard_elems = score_elements()
    all_heads = qsl.stop - qsl.start == HQ
    q, k, v, do = (t.to(dev) for t in (q_h, k_h, v_h, do_h))
    n = n_h.to(dev)
    bb = torch.tensor(SSA_B, device=dev)
    scale = D ** -0.5
    if DOC_LENS is not None:
        cu = torch.tensor([0] + list(torch.tensor(DOC_LENS).cumsum(0)), dtype=torch.int32,
                          device=dev)
        maxl = max(DOC_LENS)

        def attn_fwd(q_, k_, v_):
            return ssa_flash_attn_varlen_forward(q_, k_, v_, cu, maxl, scale, n, bb, CAUSAL)

        def attn_bwd(q_, k_, v_, o_, do_, m_):
            return ssa_flash_attn_varlen_backward(q_, k_, v_, o_, do_, m_, cu, maxl, scale, n, bb,
                                                  CAUSAL)
    else:
        def attn_fwd(q_, k_, v_):
            return ssa_flash_attn_forward(q_, k_, v_, scale, n, bb, causal=CAUSAL)

        def attn_bwd(q_, k_, v_, o_, do_, m_):
            return ssa_flash_attn_backward(q_, k_, v_, o_, do_, m_, scale, n, bb, causal=CAUSAL)

    reduce_params = world > 1
    if args.cp:
        # Context parallel: every rank builds the same full sequence and keeps its zig-zag part;
        # K/V travel around the ring, dn/db are reduced inside the ring backward.
        from SSA.context_parallel import ring_ssa_backward, ring_ssa_forward, zigzag_split
        if DOC_LENS is not None or world < 2:
            raise SystemExit("--cp needs a dense config and at least 2 ranks")
        full = make_inputs(dev, seed=0)
        q_h, k_h, v_h, do_h = (zigzag_split(t, world, rank) for t in full[:4])
        n_h = full[4]
        q, k, v, do = (t.to(dev) for t in (q_h, k_h, v_h, do_h))
        n = n_h.to(dev)
        reduce_params = False

        def attn_fwd(q_, k_, v_):
            return ring_ssa_forward(q_, k_, v_, scale, n, bb)

        def attn_bwd(q_, k_, v_, o_, do_, m_):
            return ring_ssa_backward(q_, k_, v_, o_, do_, m_, scale, n, bb)

    dnb_full = torch.zeros(HQ + 1, device=dev, dtype=torch.float32)

    def reduce_dn_db(dn_, db_, async_op=False):
        """Sum dn / db over the ranks: in place when this rank holds every q-head (dn and db are
        adjacent in one buffer), else through a full-width [Hq + 1] buffer."""
        if all_heads:
            return allreduce_ssa_param_grads(dn_, db_, async_op=async_op)
        dnb_full.zero_()
        dnb_full[qsl].copy_(dn_)
        dnb_full[HQ:].copy_(db_.reshape(1))
        return dist.all_reduce(dnb_full, async_op=async_op)

    st = torch.cuda.current_stream(dev)

    def step(pending, evs=None):
        """One step as the timed loop runs it: the dn/db all-reduce is issued asynchronously and
        overlaps the next step's forward (the warm-up runs the same steps, so the first
        asynchronous collective is not inside the timed region). evs: events recorded before
        the forward, between forward and backward, and after the backward."""
        if evs:
            evs[0].record(st)
        out, m = attn_fwd(q, k, v)
        if evs:
            evs[1].record(st)
        dq, dk, dv, dn, db = attn_bwd(q, k, v, out, do, m)
        if evs:
            evs[2].record(st)
        if reduce_params:
            # in place on the (adjacent) dn/db
            pending.append(reduce_dn_db(dn, db, async_op=True))

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    pending = []
    for _ in range(args.warmup):
        step(pending)
    for w in pending:
        w.wait()
    barrier()

    # ---- value: device-resident inputs; per-call events for the roofline
    launches0 = _lib.launch_count()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pending = []
    with ClockSampler(local, deferred=True) as clk:
        barrier()
        # A device-side wait of ~2 ms ahead of the start event lets the host queue the first
        # steps before the device reaches them, as in a training loop's steady state; without it
        # the first timed step also carries the host's launch latency (~0.1 ms, 4% of a 20-step
        # region at 8 GPUs), and a host thread delayed early in the region (by the OS, on a host
        # running one process per GPU) idles every rank through the collective. The timed region
        # still holds exactly the K steps.
        torch.cuda._sleep(4_000_000)
        start.record(st)
        for i in range(args.steps):
            step(pending, ev[i])
        for w in pending:  # every reduction finishes inside the timed region
            w.wait()
        stop.record(st)
        clk.arm()
        barrier()
    launches = _lib.launch_count() - launches0
    ms = start.elapsed_time(stop) / args.steps
    t_fwd = statistics.median(a.elapsed_time(b) for a, b, _ in ev)
    t_bwd = statistics.median(b.elapsed_time(c) for _, b, c in ev)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    # strong / cp: the config's fixed work split over the ranks; weak: every rank runs it all
    job_flops = flops_per_rank() * (world if (not strong and not args.cp) else 1)
    value = job_flops / (ms * 1e-3) / 1e12

    # ---- e2e: through the public API with pinned host buffers, copies inside the timed region.
    # Every step copies its inputs host->device and its results device->host; the copies run on
    # their own streams (two per direction: each tensor is copied as two halves, one per stream,
    # which a single copy engine per direction cannot saturate PCIe without) and overlap the
    # neighbouring steps' compute, the way a training input pipeline would. Device input buffers
    # and host result buffers are double-buffered; the timed region spans the first input copy to
    # the last result copy.
    q_p, k_p, v_p, do_p = (t.pin_memory() for t in (q_h, k_h, v_h, do_h))
    outs_p = [[torch.empty(q_h.shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)] +
              [torch.empty(k_h.shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)] +
              [torch.empty(n_h.numel() + 1, dtype=torch.float32).pin_memory()]
              for _ in range(2)]
    dev_in = [[torch.empty_like(t, device=dev) for t in (q_p, k_p, v_p, do_p)] for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in (q_p, k_p, v_p, do_p))
    d2h = sum(t.numel() * t.element_size() for t in outs_p[0])
    e2e_steps = max(3, min(args.steps, 20))
    NCOPY = 2
    s_in = [torch.cuda.Stream(dev) for _ in range(NCOPY)]
    s_out = [torch.cuda.Stream(dev) for _ in range(NCOPY)]
    ev_free = [None, None]  # compute finished with dev_in[slot]

    def half(t, k):  # k-th of NCOPY contiguous pieces of a contiguous tensor
        assert t.is_contiguous()
        flat = t.view(-1)
        n = flat.numel()
        return flat[k * n // NCOPY:(k + 1) * n // NCOPY]

    def e2e_step(i):
        slot = i & 1
        for k, s in enumerate(s_in):
            with torch.cuda.stream(s):
                if ev_free[slot] is not None:
                    s.wait_event(ev_free[slot])
                for dst, src in zip(dev_in[slot], (q_p, k_p, v_p, do_p)):
                    half(dst, k).copy_(half(src, k), non_blocking=True)
            st.wait_stream(s)
        qd, kd, vd, dod = dev_in[slot]
        out_, m_ = attn_fwd(qd, kd, vd)
        dq_, dk_, dv_, dn_, db_ = attn_bwd(qd, kd, vd, out_, dod, m_)
        if reduce_params:
            reduce_dn_db(dn_, db_)
        res = torch.cat([dn_.reshape(-1), db_.reshape(1)])
        ev = torch.cuda.Event()
        ev.record(st)
        ev_free[slot] = ev
        for k, s in enumerate(s_out):
            with torch.cuda.stream(s):
                s.wait_event(ev)
                for dst, src in zip(outs_p[slot], (out_, dq_, dk_, dv_, res)):
                    half(dst, k).copy_(half(src, k), non_blocking=True)
                    src.record_stream(s)

    e2e_step(0)
    e2e_step(1)
    torch.cuda.synchronize(dev)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for s in s_in:
        s.wait_stream(st)
    for i in range(e2e_steps):
        e2e_step(i)
    for s in s_out:
        st.wait_stream(s)
    e1.record(st)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    e2e_per_rank = [e2e_ms]
    if world > 1:
        t = torch.zeros(world, device=dev)
        t[rank] = e2e_ms
        dist.all_reduce(t)  # every rank's time (each slot written by one rank)
        e2e_per_rank = [float(x) for x in t.tolist()]
        e2e_ms = max(e2e_per_rank)
    e2e_val = job_flops / (e2e_ms * 1e-3) / 1e12

    status = _lib.load().ssa_device_status(_lib.stream_ptr(dev))
    peak_tf, _, peak_kind = measured_peaks()
    # this rank's own backward work over its own backward time
    rank_elems = score_elements() / world if args.cp else shard_elems
    traffic, traffic_note = ncu_traffic()
    achieved = 10.0 * D * rank_elems / (t_bwd * 1e-3) / 1e12
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v_cpu, el, _, reps = cpu_oracle_sample(threads)
        cpu = {"value": v_cpu, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{reps} x fwd+bwd of one q-head of one sequence (S={min(S, 2048)}, "
                         f"D={D}, causal), fp32 eager oracle with autograd, {el:.1f} s"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak" if not (strong or args.cp) else "strong", "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": WORKLOAD,
                       "global_batch": B * (world if not (strong or args.cp) else 1),
                       "seq_len": S,
                       "heads_q": HQ, "heads_kv": HKV, "head_dim": D, "causal": CAUSAL,
                       "parallelism": (f"context-parallel ring x{world} (zig-zag, NCCL P2P)"
                                       if args.cp else
                                       (f"(batch, kv-head) unit shard x{world} of the fixed "
                                        f"batch (strong), dn/db all-reduce" if strong else
                                        f"batch-shard x{world} (weak), dn/db all-reduce")),
                       "l2": "inputs larger than L2 (~300 MB resident per rank)"},
            "fwd_ms": t_fwd, "bwd_ms": t_bwd,
            "frac_of_peak": value / world / peak_tf,
            "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                    "ms_per_step_per_rank": e2e_per_rank},
            "roofline": {"bound": "tensor", "kernel": "ssa_attn_bwd call (dominant)",
                         "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": achieved / peak_tf, "peak_kind": f"{peak_kind} bf16 burst",
                         "traffic": traffic if args.config == "c2" else None,
                         "traffic_note": traffic_note if args.config == "c2" else None,
                         # what bounds SSA at D = 64: the special-function unit (lg2 / ex2)
                         # per rank: its own score elements over the max-over-ranks step time
                         "sfu": sfu_floor(ms, rank_elems)},
            "reference_triton": REFERENCE_TRITON,
            "cpu_baseline": cpu,
            "clocks": clk.summary(),
            "gpu_launches": launches,
            "device_status": status,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
