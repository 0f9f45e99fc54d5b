"""CPU: bench.py's reference arm prints the one JSON line of the benchmark contract
(runs the oracle port on the host cores; a few seconds)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run(*args):
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                         timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


def test_reference_arm_line():
    d = run("--impl", "reference", "--steps", "1", "--warmup", "3")
    assert d["impl"] == "reference" and d["metric"] == "memory-layer fwd+bwd tokens/sec" and d["unit"] == "tokens/s"
    assert d["value"] > 0 and d["higher_is_better"] is True and d["steps"] == 1 and d["warmup"] == 3
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"] == "omega_rnn_c1"
    assert d["slice"]["reps_per_step"] >= 5 and d["ms_per_step"] == d["slice"]["ms_per_rep_median"]
    # the same config dict as our arm prints (bench.config_dict), so the driver can match the two
    sys.path.insert(0, ROOT)
    import bench
    from atlas_rnn_b200.workloads import CONFIGS
    assert d["config"] == json.loads(json.dumps(bench.config_dict(CONFIGS[1], 1)))
    # no CUDA device here: the reference kernels' block says so
    assert "unavailable" in d["reference_kernel_shapes"]


def test_reference_cuda_arm_refuses_other_shapes():
    d = run("--impl", "reference-cuda", "--config", "1", "--steps", "1", "--warmup", "3")
    assert d["impl"] == "reference-cuda" and "unavailable" in d


def test_shard_workload_partitions_the_configuration():
    """bench.py --gpus N: the long-context configuration splits its tokens over the ranks,
    the others their batch (heads when the batch does not divide); the shards cover the job."""
    sys.path.insert(0, ROOT)
    import bench
    from atlas_rnn_b200.workloads import CONFIGS
    for ws in (1, 2, 4, 8):
        w1 = bench.shard_workload(CONFIGS[1], ws)
        assert w1.N * w1.T * ws == CONFIGS[1].N * CONFIGS[1].T and w1.T == CONFIGS[1].T
        w2 = bench.shard_workload(CONFIGS[2], ws)
        assert w2.T * ws == CONFIGS[2].T and w2.N == CONFIGS[2].N
        w4 = bench.shard_workload(CONFIGS[4], ws)
        assert w4.N * ws == CONFIGS[4].N
    assert bench.config_dict(CONFIGS[2], 8)["parallelism"].startswith("sequence-parallel x8")
    assert bench.config_dict(CONFIGS[1], 1)["parallelism"] == "single GPU"
