"""GPU parity tests of lightdelta::decode (decode + MTP verify) against the oracle and the
reference's golden results.  Patterns follow the reference's tests/test_gdn.py:58-122."""

import numpy as np
import pytest
import torch

import oracle
from golden import cases
from helpers import (
    assert_out_close,
    assert_state_close,
    backend_numpy,
    backend_torch,
    bits,
    to_numpy_case,
)
from lightdelta_b200 import capi, workloads
from lightdelta_b200.backend import GDNBackend
from lightdelta_b200.config import BackendConfig

pytestmark = pytest.mark.gpu

VARIANTS = ["auto", "stream", "rowreg"]


@pytest.fixture(params=VARIANTS)
def kernel(request, device):
    """Runs the test once per decode kernel variant (all must match the oracle)."""
    previous = capi.set_decode_kernel(request.param)
    yield request.param
    capi.set_decode_kernel(previous)


def _golden(name):
    return np.load(cases.__file__.replace("cases.py", f"{name}.npz"))


def run_decode(path, t):
    args = (t["qkv"], t["a"], t["b"], t["a_log"], t["dt_bias"], t["slots"], t["cu"], t["accepted"], t["pool"],
            t["gate"], t["weight"], t["out"], t.get("eps", 1e-6))
    if path == "torch_op":
        torch.ops.lightdelta.decode(*args)
    else:
        capi.decode(*args)


def run_oracle(host, num_k_heads, eps=1e-6):
    oracle.decode(host["qkv"], host["a"], host["b"], host["a_log"], host["dt_bias"], host["slots"], host["cu"],
                  host["accepted"], host["pool"], host["gate"], host["weight"], host["out"],
                  num_k_heads=num_k_heads, eps=eps)


def check_against_oracle(t, host, num_k_heads, touched=None, what="decode"):
    """Run the oracle on `host` (a pre-call copy) and compare out and the pool with the device results."""
    run_oracle(host, num_k_heads, t.get("eps", 1e-6))
    stats = assert_out_close(bits(t["out"]), host["out"], what + " out")
    pool = t["pool"]
    if touched is None:
        assert_state_close(pool.cpu().numpy(), host["pool"], what + " pool")
    else:
        idx = torch.as_tensor(touched, device=pool.device, dtype=torch.long)
        assert_state_close(pool[idx].cpu().numpy(), host["pool"][touched], what + " touched slots")
    return stats


@pytest.mark.parametrize("path", ["torch_op", "capi"])
@pytest.mark.parametrize("name", [c["name"] for c in cases.BACKEND_CASES])
def test_decode_matches_reference_golden(device, kernel, name, path):
    """Indexed decode on the reference geometry (H=16, HV=48) against the reference backend's own
    results and against the oracle on the whole pool."""
    spec = cases.spec_by_name(name)
    t = backend_torch(spec, device)
    host = backend_numpy(spec)
    pool0 = t["pool"][0].clone()
    run_decode(path, t)
    torch.cuda.synchronize()
    golden = _golden(name)
    assert_out_close(bits(t["out"]), golden["out_bits"], name + " vs reference out")
    flat = t["pool"].reshape(-1)[torch.as_tensor(golden["pool_positions"], device=device)]
    assert_state_close(flat.cpu().numpy(), golden["pool_values"], name + " vs reference pool")
    assert torch.equal(t["pool"][0], pool0)
    oracle.decode(host["qkv"], host["a"], host["b"], host["a_log"], host["dt_bias"], host["slots"], host["cu"],
                  host["accepted"], host["pool"], host["gate"], host["weight"], host["out"], num_k_heads=16)
    assert_out_close(bits(t["out"]), host["out"], name + " vs oracle out")
    assert_state_close(t["pool"].cpu().numpy(), host["pool"], name + " vs oracle pool")
    assert capi.fault_flags() == 0


@pytest.mark.parametrize("width", [1, 2, 3, 4])
@pytest.mark.parametrize("state_io", ["packed", "indexed"])
def test_backend_matches_oracle(device, kernel, width, state_io):
    """Reference tests/test_gdn.py:58-75 at HV=32: mixed accepted counts and a padding request."""
    case = workloads.make_decode_case(4, width, 24, device=device, seed=100 + width, accepted="ones")
    case.accepted.copy_(torch.arange(4, device=device, dtype=torch.int32) % width + 1)
    case.slots[-1] = 0
    t = case.kwargs()
    host = to_numpy_case(t)
    pool0 = case.pool[0].clone()
    GDNBackend(BackendConfig(compute="cuda_fused", state_io=state_io))(**t)
    torch.cuda.synchronize()
    check_against_oracle(t, host, case.num_k_heads, what=f"{state_io} w{width}")
    assert torch.equal(case.pool[0], pool0)


@pytest.mark.parametrize("state_io", ["packed", "indexed"])
def test_graph_replay_changed_state_indices(device, kernel, state_io):
    """Reference tests/test_gdn.py:78-102: capture once, then change slots and accepted counts."""
    case = workloads.make_decode_case(2, 3, 16, device=device, seed=7)
    t = case.kwargs()
    backend = GDNBackend(BackendConfig(compute="cuda_fused", state_io=state_io, cuda_graph=True))
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(3):
            backend(**t)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        backend(**t)
    case.slots.copy_(case.slots.flip(0))
    case.accepted.fill_(2)
    host = to_numpy_case(t)
    graph.replay()
    torch.cuda.synchronize()
    check_against_oracle(t, host, case.num_k_heads, what=f"graph {state_io}")


def test_packed_and_indexed_are_bit_identical(device):
    case = workloads.make_decode_case(8, 4, 40, device=device, seed=9, accepted="uniform")
    case.slots[3, 1] = 0
    packed_pool = case.pool.clone()
    out_packed = torch.empty_like(case.out)
    args = case.kwargs()
    GDNBackend(BackendConfig(compute="cuda_fused", state_io="indexed"))(**args)
    GDNBackend(BackendConfig(compute="cuda_fused", state_io="packed"))(**{**args, "pool": packed_pool,
                                                                          "out": out_packed})
    torch.cuda.synchronize()
    assert torch.equal(case.out.view(torch.int16), out_packed.view(torch.int16))
    assert torch.equal(case.pool, packed_pool)


@pytest.mark.parametrize("config", ["config2", "config3"])
def test_baseline_config_full_size_matches_oracle(device, kernel, config):
    """BASELINE config 2 (B=256, T=1, pool 1024 x [32,128,128]) and config 3 (B=64, T=4 verify,
    accepted ~ U{1..4}) at full size: every touched slot and every output against the oracle."""
    case = workloads.config2(device) if config == "config2" else workloads.config3(device)
    t = case.kwargs()
    host = to_numpy_case(t)
    untouched = sorted(set(range(1, case.pool.shape[0])) - set(case.slots.flatten().tolist()))[:8]
    before_untouched = case.pool[untouched].clone()
    pool0 = case.pool[0].clone()
    torch.ops.lightdelta.decode(*case.op_args())
    torch.cuda.synchronize()
    touched = sorted(set(case.slots.flatten().tolist()) - {0})
    stats = check_against_oracle(t, host, case.num_k_heads, touched=touched, what=config)
    assert torch.equal(case.pool[untouched], before_untouched)
    assert torch.equal(case.pool[0], pool0)
    print(config, stats)


@pytest.mark.parametrize("heads", [(16, 16), (8, 32), (16, 48), (4, 12)])
def test_head_geometries(device, kernel, heads):
    h, hv = heads
    case = workloads.make_decode_case(3, 2, 12, device=device, seed=h * 100 + hv, num_k_heads=h, num_v_heads=hv,
                                      accepted="uniform", state_scale=0.1)
    t = case.kwargs()
    host = to_numpy_case(t)
    capi.decode(*case.op_args())
    torch.cuda.synchronize()
    check_against_oracle(t, host, h, what=f"H={h} HV={hv}")


def test_unaligned_activations_use_the_scalar_path(device):
    """qkv / gate rows starting at an odd element (no 8-byte alignment) must give the same results."""
    base = workloads.make_decode_case(4, 2, 16, device=device, seed=31, accepted="uniform")
    n, width = base.qkv.shape
    wide = torch.zeros(n, width + 1 + base.gate[0].numel(), device=device, dtype=torch.bfloat16)
    wide[:, 1:width + 1] = base.qkv
    wide[:, width + 1:] = base.gate.reshape(n, -1)
    t = base.kwargs()
    t["qkv"] = wide[:, 1:width + 1]
    t["gate"] = wide[:, width + 1:].view(n, base.num_v_heads, 128)
    host = to_numpy_case(t)
    run_decode("capi", t)
    torch.cuda.synchronize()
    check_against_oracle(t, host, base.num_k_heads, what="unaligned")


def test_invalid_requests_and_fault_word(device, kernel):
    """Zero outputs and no writes for a bad accepted count, a request longer than the window and an
    out-of-range source slot; nothing for a request with no tokens; out-of-range destinations are
    skipped.  Each raises its bit in the device fault word."""
    case = workloads.make_decode_case(5, 2, 16, device=device, seed=5)
    capi.fault_flags(clear=True)
    case.accepted.copy_(torch.tensor([0, 3, 1, 1, 1], device=device, dtype=torch.int32))
    case.slots[2, 0] = case.pool.shape[0] + 3       # source out of range
    case.slots[4, 1] = case.pool.shape[0]           # destination out of range: skipped
    case.cu.copy_(torch.tensor([0, 2, 4, 6, 6, 8], device=device, dtype=torch.int32))
    case.out.fill_(1.0)
    t = case.kwargs()
    host = to_numpy_case(t)
    before = case.pool.clone()
    capi.decode(*case.op_args())
    torch.cuda.synchronize()
    assert case.out[:6].count_nonzero() == 0
    live = case.slots[:2].flatten().long()  # requests 0 and 1 have in-range slots and must be untouched
    assert torch.equal(case.pool[live], before[live])
    flags = capi.fault_flags(clear=True)
    assert flags == capi.LD_FAULT_DECODE_SLOT_RANGE
    run_oracle(host, case.num_k_heads)
    assert_out_close(bits(case.out), host["out"], "invalid requests out")
    assert_state_close(case.pool.cpu().numpy(), host["pool"], "invalid requests pool")


def test_one_token_launch_with_padding_requests(device, kernel):
    """One-token decode with padding requests (no tokens: cu repeats, as in a batch padded to a
    captured size) at a size where `auto` picks the streaming kernel (320 x 32 items)."""
    batch = 320
    case = workloads.make_decode_case(batch, 1, batch + 8, device=device, seed=31)
    live = torch.ones(batch, dtype=torch.int32)
    live[3::4] = 0
    cu = torch.zeros(batch + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(live, 0)
    case.cu.copy_(cu.to(device))
    case.out.fill_(1.0)
    capi.fault_flags(clear=True)
    host = to_numpy_case(case.kwargs())
    capi.decode(*case.op_args())
    torch.cuda.synchronize()
    assert capi.fault_flags(clear=True) == 0
    run_oracle(host, case.num_k_heads)
    assert_out_close(bits(case.out), host["out"], "padding requests out")
    assert_state_close(case.pool.cpu().numpy(), host["pool"], "padding requests pool")


def test_too_many_tokens_sets_the_token_fault(device, kernel):
    case = workloads.make_decode_case(2, 2, 8, device=device, seed=6)
    capi.fault_flags(clear=True)
    case.cu.copy_(torch.tensor([0, 3, 4], device=device, dtype=torch.int32))  # request 0 has 3 tokens > width 2
    before = case.pool.clone()
    case.out.fill_(1.0)
    capi.decode(*case.op_args())
    torch.cuda.synchronize()
    assert case.out[:3].count_nonzero() == 0
    assert capi.fault_flags(clear=True) == capi.LD_FAULT_DECODE_TOKENS
    slot_r0 = case.slots[0].long()
    assert torch.equal(case.pool[slot_r0], before[slot_r0])


def test_repeated_in_place_decode(device, kernel):
    """Three consecutive in-place decode steps (source slot == destination slot) track the oracle."""
    case = workloads.make_decode_case(16, 1, 40, device=device, seed=12)
    t = case.kwargs()
    host = to_numpy_case(t)
    for _ in range(3):
        torch.ops.lightdelta.decode(*case.op_args())
        run_oracle(host, case.num_k_heads)
    torch.cuda.synchronize()
    assert_out_close(bits(case.out), host["out"], "step 3 out")
    assert_state_close(case.pool.cpu().numpy(), host["pool"], "step 3 pool")


@pytest.mark.parametrize("variant", ["stream", "rowreg"])
def test_programmatic_launch_does_not_change_results(device, variant):
    """Chained in-place decode steps (each reads the states the previous launch wrote), a
    gather / scatter round trip and a copy, with programmatic dependent launch on and off:
    bit-identical pools and outputs."""
    results = []
    previous_kernel = capi.set_decode_kernel(variant)
    try:
        for enable in (True, False):
            previous = capi.set_programmatic_launch(enable)
            try:
                case = workloads.make_decode_case(64, 1, 200, device=device, seed=31)
                slots = case.slots.flatten()
                packed = torch.empty(slots.numel(), *case.pool.shape[1:], device=device)
                for _ in range(5):
                    torch.ops.lightdelta.decode(*case.op_args())
                    torch.ops.lightdelta.gather_state(case.pool, slots, torch.ones_like(slots, dtype=torch.bool),
                                                      packed)
                    torch.ops.lightdelta.scatter_state(packed, slots.flip(0), case.pool)
                    torch.ops.lightdelta.copy_state(case.pool, slots[:8], slots[8:16])
                torch.cuda.synchronize()
                results.append((case.pool.cpu(), case.out.cpu()))
            finally:
                capi.set_programmatic_launch(previous)
    finally:
        capi.set_decode_kernel(previous_kernel)
    assert torch.equal(results[0][0], results[1][0])
    assert torch.equal(results[0][1].view(torch.int16), results[1][1].view(torch.int16))
