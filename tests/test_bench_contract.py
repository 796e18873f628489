"""CPU checks of bench.py: argument rules and the reference arm's JSON line (which runs the
CPU oracle port and needs no GPU)."""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def test_warmup_below_three_is_rejected():
    with pytest.raises(SystemExit):
        bench.parse_args(["--warmup", "2"])


def test_defaults_are_the_headline_workload():
    args = bench.parse_args([])
    assert (args.gpus, args.workload, args.impl, args.decode_kernel) == (1, "decode", "ours", "auto")
    assert args.warmup >= 3


def test_reference_arm_prints_one_contract_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    result = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "3",
                             "--cpu-seconds", "2",
                             "--warmup", "3"], capture_output=True, text=True, timeout=600, env=env, check=True)
    lines = [line for line in result.stdout.splitlines() if line.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["unit"] == "tokens/s" and line["value"] > 0
    assert line["metric"] == bench.METRIC
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    torch_path = line["reference_torch"]
    if "unavailable" not in torch_path:
        assert torch_path["kind"] == "reference" and torch_path["value"] > 0 and torch_path["cores"] >= 1
        configs = line["reference_torch_configs"]
        assert configs["cores"] >= 1 and configs["torch"]
        for name in ("config1", "config2", "config3"):
            assert configs[name]["runs"] >= 5 and configs[name]["tokens_per_s"] > 0
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["config"]["workload"] == "config2_decode"


@pytest.mark.parametrize("workload", ["decode_bf16", "commit"])
def test_reference_arm_without_a_cpu_path_says_so(workload):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    result = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", workload,
                             "--steps", "3", "--warmup", "3"], capture_output=True, text=True, timeout=600, env=env,
                            check=True)
    line = json.loads(result.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and "unavailable" in line


def test_reference_arm_times_config4_copies_on_the_host():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    result = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", "copy",
                             "--steps", "3", "--warmup", "3"], capture_output=True, text=True, timeout=600, env=env,
                            check=True)
    line = json.loads(result.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "slots/s" and line["value"] > 0
    assert line["config"]["workload"] == "config4_copy"
    assert line["cpu_baseline"]["kind"] == "reference" and line["e2e"]["value"] == line["value"]


def test_reference_arm_under_torchrun_prints_one_line_from_rank_zero():
    """The launch the driver uses for N > 1: rank 0 alone runs and prints the reference line, the
    other ranks exit 0 without work."""
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    result = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                             "--master-addr", "127.0.0.1", "--master-port", str(port), str(ROOT / "bench.py"),
                             "--impl", "reference", "--gpus", "2", "--steps", "3", "--warmup", "3",
                             "--cpu-seconds", "1"], capture_output=True, text=True, timeout=600, env=env, check=True)
    lines = [line for line in result.stdout.splitlines() if line.strip().startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["value"] > 0 and line["n_gpus"] == 2
