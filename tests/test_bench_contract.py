"""bench.py's reference arm on the CPU under torchrun: rank 0 alone prints one JSON line of the contract.

The reference arm times the NumPy restatement of the config-2 attention on the
host cores (the reference is JAX, which is not installed). Two ranks over gloo:
rank 1 exits 0 without work, rank 0 prints the line. Each step is the whole
8-row config-2 batch, the GPU arm's step (about 30 s on 8 cores).
"""

import json
import os
import socket
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_reference_arm_prints_one_contract_line_from_rank_zero():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), "bench.py", "--impl", "reference",
           "--gpus", "2", "--steps", "1", "--warmup", "0"]
    env = dict(os.environ, OMP_NUM_THREADS="2")
    run = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert run.returncode == 0, run.stderr[-2000:]
    lines = [ln for ln in run.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, run.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["n_gpus"] == 2 and line["steps"] == 1
    for key in ("metric", "value", "unit", "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["value"] > 0 and line["unit"] == line["e2e"]["unit"] == line["cpu_baseline"]["unit"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["cpu_baseline"]["kind"] == "port"
    assert line["config"]["batch"] == 8 and "whole batch" in line["cpu_baseline"]["sample"]


def test_cpu_baseline_legs_return_positive_rates():
    """The per-config CPU legs bench.py attaches at N=1 (bounded samples of configs 1, 3, 4, 5)."""
    sys.path.insert(0, ROOT)
    import bench
    from minifield_training_b200 import workloads

    tf, dt, sample = bench.cpu_attention_sample(workloads.CONFIG1)
    assert tf > 0 and dt > 0 and "cfg1" in sample
    tps, gbs, dt, sample = bench.cpu_decode_sample(layers=1)
    assert tps > 0 and gbs > 0 and "1 of 6 layers" in sample
    for kind in ("int8-channel-absmax-v1", "int4-g128-absmax-v1"):
        tf, tps, dt, sample = bench.cpu_qat_sample(kind, tokens=64)
        assert tf > 0 and tps > 0 and kind in sample
    tps, tf, dt, sample = bench.cpu_encoder_sample(rows=1)
    assert tps > 0 and tf > 0
