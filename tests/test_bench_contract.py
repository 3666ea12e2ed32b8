"""bench.py's launch count (its gpu_launches claim) against the kernels one learner step
launches, as the ncu launch lists show them: c0 (256 rows: one launch) and c3 (1,048,576
rows: 28 kernels)."""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402
from spo_mojo_b200.workloads import WORKLOADS  # noqa: E402


def test_launch_count_matches_launch_lists():
    # c0 (256 rows) and c1 (4,096 rows): the one-launch small-batch step; under data
    # parallelism its backward, then Adam after the all-reduce
    assert bench.count_launches(WORKLOADS["c0"], clip=False) == 1
    assert bench.count_launches(WORKLOADS["c1"], clip=True) == 1
    assert bench.count_launches(WORKLOADS["c0"], clip=False, world=2) == 2
    # c2 above the small-step rows: per network the W1/W2 splits, the input layer's W0^T and
    # input splits (65,536 rows: tensor cores), three forward GEMMs, head, two hidden dW,
    # two dX, input-layer dW; then reduction and Adam
    assert bench.count_launches(WORKLOADS["c2"], clip=False) == 28
    # c3, actor and critic: the same sequence
    assert bench.count_launches(WORKLOADS["c3"], clip=False) == 28
    # the same network below the input layer's tensor-core threshold: two launches fewer each
    assert bench.count_launches(WORKLOADS["c3"], clip=False, rows=bench.TC0_MIN_ROWS - 1) == 24
    # the CUDA-core engine has no splits
    assert bench.count_launches(WORKLOADS["c3"], clip=False, engine="cuda") == 20
    # a clipped step adds the grouped sum of squares
    assert bench.count_launches(WORKLOADS["c3"], clip=True) == 29


def test_reference_arm_prints_the_contract_line():
    """bench.py --impl reference (the reference's algorithm on the host cores; no GPU)
    prints one JSON line with the keys the driver reads, on the ours arm's metric."""
    import json
    import subprocess
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload", "c0",
                        "--steps", "2", "--warmup", "1"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    d = json.loads(r.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config"):
        assert key in d, key
    assert d["impl"] == "reference" and d["steps"] == 2 and d["warmup"] == 1
    assert d["metric"] == "learner samples/sec (fwd+bwd+loss+Adam)" and d["unit"] == "samples/s"
    assert d["higher_is_better"] is True and d["value"] > 0
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "samples/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_print_nothing():
    """Under torchrun only rank 0 runs the reference arm; the other ranks exit 0 silently."""
    import subprocess
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2",
                        "--steps", "1", "--warmup", "0"], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == ""


def test_small_step_eligibility_follows_the_shared_memory_layout():
    from spo_mojo_b200.workloads import NetSpec, Workload
    assert bench.small_step_fits(WORKLOADS["c0"], 256)
    assert bench.small_step_fits(WORKLOADS["c1"], 4096)
    assert not bench.small_step_fits(WORKLOADS["c1"], 8193)
    assert bench.small_step_fits(Workload("ac3", actor=NetSpec((27, 96, 160, 64, 9)),
                                          critic=NetSpec((27, 96, 160, 64, 1)), batch=1000), 1000)
    # 27-256-256-9: 82 k weights do not fit beside the activations of a 32-row block
    assert not bench.small_step_fits(Workload("w", actor=NetSpec((27, 256, 256, 9)), batch=64), 64)
    assert not bench.small_step_fits(WORKLOADS["c2"], 4096)


def test_clock_sampler_reports_the_timed_region():
    """The sampler's parsing and window: samples taken during the timed region are the ones
    reported (with any active throttle reason); when the region was shorter than the
    sampling interval, the samples since start() stand in, and the window says so."""
    import time

    class FakeProc:
        def terminate(self):
            pass

        def wait(self, timeout=None):
            return 0

        def kill(self):
            pass

    idle = "0, 1965, 1965, 500, 0x0, Not Active, Not Active, Not Active, Not Active\n"
    capped = "0, 1700, 1965, 990, 0x4, Not Active, Not Active, Not Active, Active\n"
    c = bench.ClockSampler([0])
    c.proc = FakeProc()
    now = time.perf_counter()
    c.lines = [(now - 1.0, idle), (now + 0.01, capped)]
    c.t_mark = now
    clk = c.stop()
    assert clk["sm_mhz"] == 1700.0 and clk["sm_max_mhz"] == 1965.0 and clk["reasons"] == ["sw_power_cap"]
    assert clk["samples"] == 1 and clk["window"] == "timed region"
    c = bench.ClockSampler([0])
    c.proc = FakeProc()
    c.lines = [(now - 1.0, idle)]
    c.t_mark = time.perf_counter()
    clk = c.stop()
    assert clk["sm_mhz"] == 1965.0 and clk["samples"] == 1 and clk["window"].startswith("warm-up")
