"""Runs the REFERENCE's compiled operators (oracle/_ref/_C.so) in a process of their own.

Invoked by tests/test_reference_kernel_gpu.py as
    python tests/ref_kernel_worker.py parity <case-name> <out.npz>
    python tests/ref_kernel_worker.py timing <json-shapes> <out.json>
The reference library registers the same `lightdelta` torch.library namespace as
lightdelta_b200, so the two can never share a process.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

REF_LIB = ROOT / "oracle" / "_ref" / "_C.so"


def reference_case(batch: int, width: int, seed: int, device):
    """The reference benchmark's input recipe (benchmarks/gdn.py:13-37) at H=16, HV=48."""
    torch.manual_seed(seed)
    n = batch * width
    qkvz = torch.randn(n, 16384, device=device, dtype=torch.bfloat16) * 0.2
    ba = torch.randn(n, 96, device=device, dtype=torch.bfloat16)
    return dict(
        qkv=qkvz[:, :10240], a=ba[:, 48:], b=ba[:, :48], a_log=torch.randn(48, device=device),
        dt_bias=torch.randn(48, device=device, dtype=torch.bfloat16),
        slots=torch.arange(1, n + 1, device=device, dtype=torch.int32).view(batch, width),
        cu=torch.arange(0, n + 1, width, device=device, dtype=torch.int32),
        accepted=torch.ones(batch, device=device, dtype=torch.int32),
        pool=torch.randn(n + 1, 48, 128, 128, device=device) * 0.1,
        gate=qkvz[:, 10240:].view(n, 48, 128), weight=torch.randn(128, device=device, dtype=torch.bfloat16),
        out=torch.empty(n, 48, 128, device=device, dtype=torch.bfloat16),
    )


def op_args(t: dict) -> tuple:
    return (t["qkv"], t["a"], t["b"], t["a_log"], t["dt_bias"], t["slots"], t["cu"], t["accepted"], t["pool"],
            t["gate"], t["weight"], t["out"], 1e-6)


def time_decode(t: dict, iterations: int = 50) -> float:
    """Median CUDA-event time (us) of one decode launch, state restored outside the timed region."""
    args = op_args(t)
    saved = t["pool"].clone()
    for _ in range(5):
        torch.ops.lightdelta.decode(*args)
    torch.cuda.synchronize()
    samples = []
    for _ in range(iterations):
        t["pool"].copy_(saved)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        torch.ops.lightdelta.decode(*args)
        end.record()
        end.synchronize()
        samples.append(start.elapsed_time(end) * 1000)
    return float(np.median(samples))


def main() -> int:
    mode, arg, out = sys.argv[1:4]
    torch.ops.load_library(str(REF_LIB))
    device = torch.device("cuda", 0)
    if mode == "parity":
        from golden import cases
        from helpers import backend_torch

        t = backend_torch(cases.spec_by_name(arg), device)
        torch.ops.lightdelta.decode(*op_args(t))
        torch.cuda.synchronize()
        np.savez(out, out=t["out"].cpu().view(torch.int16).numpy(), pool=t["pool"].cpu().numpy())
    elif mode == "timing":
        results = {}
        for batch, width, seed in json.loads(arg):
            results[f"{batch}x{width}"] = time_decode(reference_case(batch, width, seed, device))
        Path(out).write_text(json.dumps(results))
    else:
        raise SystemExit(f"unknown mode {mode}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
