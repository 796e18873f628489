"""The reference's own torch CPU path (oracle/ref_torch.py: its post_conv_gdn compiled unmodified,
run with GDNBackend's packed gather and commit) -- the second CPU figure bench.py reports beside the
C port.  Pinned here two ways: against the golden fixtures that the reference's GDNBackend itself
produced (H=16, HV=48; tests/golden/make_golden.py), and against the C oracle at the BASELINE
geometry (H=16, HV=32) on a config-2-shaped and a config-3-shaped case."""

import numpy as np
import pytest
import torch

import oracle
from golden import cases
from helpers import assert_out_close, assert_state_close, backend_torch, bits, to_numpy_case
from lightdelta_b200 import workloads
from oracle import ref_torch

pytestmark = pytest.mark.skipif(
    not ref_torch.available(),
    reason="oracle/_ref/torch_path not built (python oracle/build_ref.py, needs the reference)")


def _golden(name):
    from pathlib import Path

    with np.load(Path(__file__).parent / "golden" / f"{name}.npz") as data:
        return {k: data[k] for k in data.files}


@pytest.mark.parametrize("name", [c["name"] for c in cases.BACKEND_CASES])
def test_reference_torch_path_reproduces_the_reference_backend(name):
    x = backend_torch(cases.spec_by_name(name), "cpu")
    before = x["pool"][0].clone()
    ref_torch.packed_decode(**x, num_k_heads=16)
    golden = _golden(name)
    np.testing.assert_array_equal(bits(x["out"]), golden["out_bits"])
    np.testing.assert_array_equal(x["pool"].numpy().reshape(-1)[golden["pool_positions"]], golden["pool_values"])
    assert torch.equal(x["pool"][0], before)


@pytest.mark.parametrize("requests,width", [(8, 1), (4, 4)])
def test_reference_torch_path_matches_the_c_oracle_at_hv32(requests, width):
    case = workloads.make_decode_case(requests, width, 4 * requests * width, device="cpu", seed=21 + width,
                                      accepted="uniform")
    kwargs = case.kwargs()
    host = to_numpy_case(kwargs)
    host["pool"] = host["pool"].copy()  # on the CPU the numpy view shares the tensor's memory
    oracle.decode(host["qkv"], host["a"], host["b"], host["a_log"], host["dt_bias"], host["slots"], host["cu"],
                  host["accepted"], host["pool"], host["gate"], host["weight"], host["out"],
                  num_k_heads=case.num_k_heads, eps=case.eps)
    ref_torch.packed_decode(**kwargs, num_k_heads=case.num_k_heads)
    assert_out_close(bits(case.out), host["out"], f"torch path B={requests} T={width} out")
    assert_state_close(case.pool.numpy(), host["pool"], f"torch path B={requests} T={width} pool")
