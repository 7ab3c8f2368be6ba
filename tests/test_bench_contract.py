"""bench.py on the CPU: the FLOP accounting of each workload (the FlashAttention convention,
14 * D per causal score element) and the reference arm's JSON line, which runs the CPU oracle
and needs no GPU."""

import json
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


@pytest.fixture
def bench():
    sys.path.insert(0, str(REPO))
    import bench as b
    yield b
    b.select_config("c2")


def test_flop_counts_match_the_workloads(bench):
    bench.select_config("c2")  # B=8, Hq=32, S=2048, D=64, causal: E = 8*32*2048^2/2
    assert bench.score_elements() == 8 * 32 * 2048 * 2048 // 2 == 536870912
    assert bench.flops_per_rank() == pytest.approx(4.810e11, rel=1e-3)
    assert bench.flops_bwd_per_rank() == pytest.approx(10 * 64 * 536870912)
    bench.select_config("c4")  # B=1, Hq=32, S=32768, D=128
    assert bench.flops_per_rank() == pytest.approx(3.079e13, rel=1e-3)
    # special-function floor: lg2 + ex2 per element in each direction at 16 per clock per SM
    sf = bench.sfu_floor(1.0, bench.score_elements())
    assert sf["ops_per_step"] == 4 * bench.score_elements()
    assert sf["floor_ms"] == pytest.approx(sf["ops_per_step"] / sf["peak_ops_per_s"] * 1e3)
    assert sf["frac"] == pytest.approx(sf["floor_ms"])
    bench.select_config("c3")  # packed documents: E = Hq * sum(L^2 / 2)
    lens = bench.DOC_LENS
    assert sum(lens) == 65536 and all(1 <= L <= 4096 for L in lens)
    assert bench.score_elements() == 32 * sum(L * L // 2 for L in lens)


def test_strong_scaling_shards_are_unit_rectangles(bench):
    """Strong scaling splits the config's fixed batch by (batch, kv-head) units (SSA.shard's
    balanced contiguous ranges): whole sequences when the ranks divide B, else kv-head ranges of
    one sequence; every unit is owned exactly once."""
    bench.select_config("c2")  # B = 8, Hkv = 8
    for world in (1, 2, 4, 8, 16, 32, 64):
        seen = set()
        for rank in range(world):
            bs, hs = bench.strong_shard(world, rank)
            units = {(b, h) for b in range(bs.start, bs.stop) for h in range(hs.start, hs.stop)}
            assert not units & seen
            seen |= units
            if world <= 8:
                assert hs == slice(0, 8) and bs.stop - bs.start == 8 // world
        assert seen == {(b, h) for b in range(8) for h in range(8)}
    with pytest.raises(SystemExit):
        bench.strong_shard(3, 0)
    bench.select_config("c3")  # one packed sequence: kv-head ranges
    assert [bench.strong_shard(2, r) for r in range(2)] == [(slice(0, 1), slice(0, 4)),
                                                          (slice(0, 1), slice(4, 8))]
    assert bench.shard_score_elements(1, 16) * 2 == bench.score_elements()


def test_roofline_traffic_only_for_the_captured_source(bench, tmp_path, monkeypatch):
    """roofline.traffic comes from the committed ncu summary only while the kernel source still
    has the sha256 that capture recorded; otherwise it is null with a note."""
    import hashlib
    src = tmp_path / "k.cu"
    src.write_text("kernel v1")
    sha = hashlib.sha256(b"kernel v1").hexdigest()[:16]
    prof = tmp_path / "p.md"
    prof.write_text(f"bench-traffic: kernel=bwd sha256_16={sha} dram_bytes=1.5e9 workload=c2\n")
    monkeypatch.setattr(bench, "TRAFFIC_PROFILE", prof)
    monkeypatch.setattr(bench, "TRAFFIC_SOURCE", src)
    assert bench.ncu_traffic()[0] == 1.5e9
    src.write_text("kernel v2")
    t, note = bench.ncu_traffic()
    assert t is None and "stale" in note


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "3",
                        "--warmup", "3"], cwd=REPO, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["unit"] == "TFLOP/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["steps"] == 3 and d["warmup"] >= 3 and d["n_gpus"] == 1
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["ms_per_step"] > 0 and d["sample_flops_per_step"] > 0


def test_clock_sampler_defers_until_armed(bench, monkeypatch):
    """A deferred sampler takes no sample while the timed region is being queued (its thread
    would compete with the launching thread for the interpreter lock), samples after arm(), and
    reports throttle reasons other than gpu_idle. NVML is a fake here: nothing is queried."""
    import threading
    import time
    import types

    calls = []
    armed_at = []
    fake = types.SimpleNamespace(
        NVML_CLOCK_SM=0,
        nvmlInit=lambda: None,
        nvmlDeviceGetHandleByIndex=lambda i: i,
        nvmlDeviceGetMaxClockInfo=lambda h, c: 1965,
        nvmlDeviceGetClockInfo=lambda h, c: calls.append(time.monotonic()) or 1900,
        nvmlDeviceGetCurrentClocksEventReasons=lambda h: 0x1 | 0x4,
    )
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    with bench.ClockSampler(0, deferred=True) as clk:
        warm = len(calls)  # the constructor's warm-up query, discarded
        time.sleep(0.05)
        assert len(calls) == warm, "sampled before arm()"
        armed_at.append(time.monotonic())
        clk.arm()
        time.sleep(0.05)
    s = clk.summary()
    assert clk.samples and all(t >= armed_at[0] for t in calls[warm:])
    assert s["samples"] >= 2 and s["sm_mhz"] == 1900 and s["sm_max_mhz"] == 1965
    assert s["reasons"] == ["sw_power_cap"]
    assert not any(t.name == clk._t.name and t.is_alive() for t in threading.enumerate())
