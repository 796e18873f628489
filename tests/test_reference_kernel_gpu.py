"""The reference's own CUDA kernel (built from its sources for sm_100a into oracle/_ref/) as a
second oracle at its native H=16 / HV=48 geometry, and as the kernel to compare against.

The reference library registers the same torch.library namespace, so it runs in a
subprocess (tests/ref_kernel_worker.py)."""

import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from golden import cases
from helpers import assert_out_close, assert_state_close, backend_torch, bits
from lightdelta_b200 import capi

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
    assert all(r > 0 and o > 0 for _, _, r, o in rows)
