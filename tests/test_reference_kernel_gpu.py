"""The reference's own CUDA kernel (built from its sources for sm_100a into oracle/_ref/) as a
second oracle and as the kernel to compare against:
  * at its native H=16 / HV=48 geometry through its own operator library, which registers the
    same torch.library namespace and therefore runs in a subprocess (tests/ref_kernel_worker.py);
  * at the BASELINE geometry H=16 / HV=32 through oracle/ref_kernel.py, which launches the same
    kernel template at value-head ratio 2 in this process (the stock launcher runs ratio 3 only).
Speed comparisons assert that ours is faster and print both times."""

import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from oracle import ref_kernel

from golden import cases
from helpers import assert_out_close, assert_state_close, backend_torch, bits, to_numpy_case
from lightdelta_b200 import capi, workloads

ROOT = Path(__file__).resolve().parent.parent
WORKER = ROOT / "tests" / "ref_kernel_worker.py"
REF_LIB = ROOT / "oracle" / "_ref" / "_C.so"

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not REF_LIB.exists(), reason="reference library not built (python oracle/build_ref.py)"),
]


def run_worker(*args, timeout=600):
    subprocess.run([sys.executable, str(WORKER), *map(str, args)], check=True, timeout=timeout)


@pytest.mark.parametrize("name", [c["name"] for c in cases.BACKEND_CASES])
def test_reference_kernel_agrees_with_ours(device, name, tmp_path):
    result = tmp_path / "ref.npz"
    run_worker("parity", name, result)
    ref = np.load(result)
    t = backend_torch(cases.spec_by_name(name), device)
    torch.ops.lightdelta.decode(t["qkv"], t["a"], t["b"], t["a_log"], t["dt_bias"], t["slots"], t["cu"],
                                t["accepted"], t["pool"], t["gate"], t["weight"], t["out"], 1e-6)
    torch.cuda.synchronize()
    assert_out_close(bits(t["out"]), ref["out"].view(np.uint16), name + " vs reference kernel out")
    assert_state_close(t["pool"].cpu().numpy(), ref["pool"], name + " vs reference kernel pool")


def test_speed_against_the_reference_kernel(device, tmp_path):
    """Same shapes and inputs as the reference's operator benchmark (benchmarks/gdn.py:76-80) plus a
    batch-256 decode at HV=48; prints both kernels' median times (state restored outside timing)."""
    sys.path.insert(0, str(WORKER.parent))
    import ref_kernel_worker as w

    shapes = [(b, t, 42) for b in (1, 4, 8) for t in (1, 2, 3, 4)] + [(64, 4, 42), (256, 1, 42)]
    out = tmp_path / "ref.json"
    run_worker("timing", json.dumps(shapes), out)
    ref = json.loads(out.read_text())
    capi.set_decode_kernel("auto")
    rows = []
    for batch, width, seed in shapes:
        ours = w.time_decode(w.reference_case(batch, width, seed, device))
        rows.append((batch, width, ref[f"{batch}x{width}"], ours))
    state = {f"{b}x{t}": {"reference_us": r, "ours_us": o} for b, t, r, o in rows}
    print("\nHV=48 decode, median us (reference kernel vs lightdelta_b200):")
    for b, t, r, o in rows:
        print(f"  B={b:3d} T={t}: reference {r:8.2f}  ours {o:8.2f}  speed-up {r / o:5.2f}x")
    print("JSON " + json.dumps(state))
    speedups = np.array([r / o for _, _, r, o in rows])
    # Small launches are a few microseconds either way (one wave of CTAs); the large ones and the
    # geometric mean over all shapes must favour ours.
    assert float(np.exp(np.log(speedups).mean())) > 1.0, speedups
    assert all(r / o > 1.0 for b, t, r, o in rows if b * t >= 256), speedups


def _event_us(fn, steps=200, warmup=10):
    """Average device time of one launch over `steps` back-to-back launches (one event pair)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) * 1000 / steps


def _baseline_case(config, device):
    return workloads.config2(device) if config == "config2" else workloads.config3(device)


@pytest.mark.skipif(not ref_kernel.available(), reason="reference harness not built (python oracle/build_ref.py)")
@pytest.mark.parametrize("config", ["config2", "config3"])
def test_reference_kernel_at_the_baseline_geometry_matches_the_oracle(device, config):
    """BASELINE config 2 / 3 at HV=32: the reference kernel (ratio-2 instantiation) and ours, each
    on its own copy of the pool, against the oracle on every touched slot and every output."""
    case = _baseline_case(config, device)
    twin_pool = case.pool.clone()
    twin_out = torch.empty_like(case.out)
    host = to_numpy_case(case.kwargs())
    args = case.op_args()
    ref_kernel.decode(*args[:8], twin_pool, args[9], args[10], twin_out, case.eps)
    torch.ops.lightdelta.decode(*args)
    torch.cuda.synchronize()
    oracle.decode(host["qkv"], host["a"], host["b"], host["a_log"], host["dt_bias"], host["slots"], host["cu"],
                  host["accepted"], host["pool"], host["gate"], host["weight"], host["out"],
                  num_k_heads=case.num_k_heads, eps=case.eps)
    touched = sorted(set(case.slots.flatten().tolist()) - {0})
    idx = torch.as_tensor(touched, device=device, dtype=torch.long)
    ref_stats = assert_out_close(bits(twin_out), host["out"], f"{config} reference kernel vs oracle out")
    assert_state_close(twin_pool[idx].cpu().numpy(), host["pool"][touched], f"{config} reference kernel pool")
    our_stats = assert_out_close(bits(case.out), host["out"], f"{config} ours vs oracle out")
    assert_state_close(case.pool[idx].cpu().numpy(), host["pool"][touched], f"{config} ours pool")
    print(config, "reference kernel", ref_stats, "ours", our_stats)


@pytest.mark.skipif(not ref_kernel.available(), reason="reference harness not built (python oracle/build_ref.py)")
@pytest.mark.parametrize("config", ["config2", "config3"])
def test_faster_than_the_reference_kernel_at_the_baseline_geometry(device, config):
    """Device time per launch, in place on a pool larger than L2, back-to-back launches: the
    reference kernel at HV=32 against ours on identical inputs (separate pools)."""
    case = _baseline_case(config, device)
    twin_pool = case.pool.clone()
    twin_out = torch.empty_like(case.out)
    args = case.op_args()
    capi.set_decode_kernel("auto")

    def reference():
        ref_kernel.decode(*args[:8], twin_pool, args[9], args[10], twin_out, case.eps)

    def ours():
        torch.ops.lightdelta.decode(*args)

    ref_us = min(_event_us(reference), _event_us(reference))
    our_us = min(_event_us(ours), _event_us(ours))
    print(f"\n{config} HV=32: reference kernel {ref_us:.1f} us, ours {our_us:.1f} us, speed-up {ref_us / our_us:.2f}x")
    assert our_us < ref_us
