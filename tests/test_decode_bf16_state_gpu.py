"""GPU parity of torch.ops.lightdelta.decode_bf16_state / ld_decode_bf16_state (decode and MTP
verify on a bf16 state pool).

Two expectations: (1) the oracle's bf16-pool mode (fp32 recurrence, each stored step rounded):
outputs within the reference test's tolerance with at most 1e-3 outside 2e-3, stored states within
one bf16 ulp or the fp32 state tolerance; (2) the fp32 decode kernel run on the same pool widened
to fp32, to the same tolerances against its states rounded to bf16.  The bf16 tiles assign
columns to lanes differently from the fp32 tiles (eight consecutive bf16 columns per lane), so
the two kernels' dot products add in different orders and agree to rounding, not bit for bit."""

import dataclasses

import pytest
import torch

import oracle
from helpers import assert_bf16_state_close, assert_out_close_tail, bits, to_numpy_case
from lightdelta_b200 import capi, workloads

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["auto", "stream", "rowreg"])
def kernel(request, device):
    previous = capi.set_decode_kernel(request.param)
    yield request.param
    capi.set_decode_kernel(previous)


def bf16_case(batch, width, pool_slots, *, device, seed, **kw):
    case = workloads.make_decode_case(batch, width, pool_slots, device=device, seed=seed, **kw)
    case.pool = case.pool.to(torch.bfloat16)
    return case


def run(case, path="torch_op"):
    args = case.op_args()
    if path == "torch_op":
        torch.ops.lightdelta.decode_bf16_state(*args)
    else:
        capi.decode(*args)


def check(case, host, what, touched=None):
    oracle.decode(host["qkv"], host["a"], host["b"], host["a_log"], host["dt_bias"], host["slots"], host["cu"],
                  host["accepted"], host["pool"], host["gate"], host["weight"], host["out"],
                  num_k_heads=case.num_k_heads, eps=case.eps)
    out_stats = assert_out_close_tail(bits(case.out), host["out"], what + " out")
    if touched is None:
        state_stats = assert_bf16_state_close(bits(case.pool), host["pool"], what + " pool")
    else:
        idx = torch.as_tensor(touched, device=case.pool.device, dtype=torch.long)
        state_stats = assert_bf16_state_close(bits(case.pool[idx]), host["pool"][touched], what + " touched slots")
    return out_stats, state_stats


@pytest.mark.parametrize("path", ["torch_op", "capi"])
@pytest.mark.parametrize("shape", [(8, 1, "ones"), (3, 2, "uniform"), (6, 4, "uniform"), (1, 3, "uniform")])
def test_small_cases_match_oracle(device, kernel, shape, path):
    batch, width, accepted = shape
    case = bf16_case(batch, width, 1 + batch * width + 3, device=device, seed=40 + batch * width,
                     accepted=accepted, state_scale=0.1)
    host = to_numpy_case(case.kwargs())
    pool0 = case.pool[0].clone()
    run(case, path)
    torch.cuda.synchronize()
    check(case, host, f"B={batch} T={width}")
    assert torch.equal(case.pool[0], pool0)


@pytest.mark.parametrize("config", ["config2", "config3"])
def test_baseline_configs_match_oracle(device, kernel, config):
    """BASELINE configs 2 (B=256, T=1) and 3 (B=64, T=4 verify) on a bf16 pool, every touched slot."""
    if config == "config2":
        case = bf16_case(256, 1, 1024, device=device, seed=2)
    else:
        case = bf16_case(64, 4, 257, device=device, seed=3, accepted="uniform")
    host = to_numpy_case(case.kwargs())
    untouched = sorted(set(range(1, case.pool.shape[0])) - set(case.slots.flatten().tolist()))[:8]
    before = case.pool[untouched].clone()
    run(case)
    torch.cuda.synchronize()
    touched = sorted(set(case.slots.flatten().tolist()) - {0})
    stats = check(case, host, config, touched=touched)
    assert torch.equal(case.pool[untouched], before)
    print(config, stats)


@pytest.mark.parametrize("heads", [(16, 48), (4, 12)])
def test_head_geometries(device, heads):
    h, hv = heads
    case = bf16_case(3, 2, 12, device=device, seed=h * 10 + hv, num_k_heads=h, num_v_heads=hv, accepted="uniform",
                     state_scale=0.1)
    host = to_numpy_case(case.kwargs())
    run(case, "capi")
    torch.cuda.synchronize()
    check(case, host, f"H={h} HV={hv}")


@pytest.mark.parametrize("shape", [(256, 1, "ones"), (64, 4, "uniform"), (5, 3, "uniform")])
def test_matches_the_fp32_kernel_on_the_widened_pool(device, kernel, shape):
    """The bf16 pool changes the state's load and store: outputs match the fp32 decode on the
    widened pool and every stored state is that kernel's fp32 state rounded, to rounding."""
    batch, width, accepted = shape
    case = bf16_case(batch, width, 1 + batch * width + 7, device=device, seed=80 + width, accepted=accepted)
    fp32 = dataclasses.replace(case, pool=case.pool.float(), out=torch.empty_like(case.out))
    run(case)
    torch.ops.lightdelta.decode(*fp32.op_args())
    torch.cuda.synchronize()
    assert_out_close_tail(bits(case.out), bits(fp32.out), "out vs fp32 kernel")
    assert_bf16_state_close(bits(case.pool), bits(fp32.pool.to(torch.bfloat16)), "pool vs fp32 kernel")
    untouched = torch.ones(case.pool.shape[0], dtype=torch.bool, device=device)
    untouched[case.slots.flatten().long()] = False
    assert torch.equal(case.pool[untouched], fp32.pool[untouched].to(torch.bfloat16))


def test_chained_launches_track_the_fp32_kernel_rounded_between_steps(device, kernel):
    """Three in-place launches back to back (each reads what the previous one stored; with
    programmatic dependent launch they overlap their prologues) against the fp32 kernel whose
    pool is rounded to bf16 after every launch: outputs at every step and the final pool agree to
    rounding (k ulps after k launches)."""
    case = bf16_case(16, 1, 40, device=device, seed=12)
    fp32 = dataclasses.replace(case, pool=case.pool.float(), out=torch.empty_like(case.out))
    outs = []
    for _ in range(3):
        run(case)
        outs.append(case.out.clone())
    for step in range(3):
        torch.ops.lightdelta.decode(*fp32.op_args())
        fp32.pool.copy_(fp32.pool.to(torch.bfloat16).float())
        torch.cuda.synchronize()
        assert_out_close_tail(bits(outs[step]), bits(fp32.out), f"step {step + 1} out")
    assert_bf16_state_close(bits(case.pool), bits(fp32.pool.to(torch.bfloat16)), "pool after 3 steps", max_ulps=3)


def test_invalid_requests_and_fault_word(device, kernel):
    case = bf16_case(5, 2, 16, device=device, seed=5)
    capi.fault_flags(clear=True)
    case.accepted.copy_(torch.tensor([0, 3, 1, 1, 1], device=device, dtype=torch.int32))
    case.slots[2, 0] = case.pool.shape[0] + 3
    case.slots[4, 1] = case.pool.shape[0]
    case.cu.copy_(torch.tensor([0, 2, 4, 6, 6, 8], device=device, dtype=torch.int32))
    case.out.fill_(1.0)
    host = to_numpy_case(case.kwargs())
    before = case.pool.clone()
    run(case, "capi")
    torch.cuda.synchronize()
    assert case.out[:6].count_nonzero() == 0
    live = case.slots[:2].flatten().long()
    assert torch.equal(case.pool[live], before[live])
    assert capi.fault_flags(clear=True) == capi.LD_FAULT_DECODE_SLOT_RANGE
    check(case, host, "invalid requests")


def test_invalid_requests_in_the_prefetched_wave(device):
    """Multi-token launches on a bf16 pool warm L2 with the reads of the block one wave later
    (blockIdx + 2 x SMs).  Invalid requests placed in that wave prefetch nothing out of range and
    still decode as the oracle says."""
    batch, width = 24, 4
    case = bf16_case(batch, width, 1 + batch * width + 8, device=device, seed=81, accepted="uniform")
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    assert batch * case.num_v_heads > 2 * sms  # the first blocks prefetch the last requests' reads
    slots = case.pool.shape[0]
    case.accepted[batch - 4] = 0                                               # no accepted step
    case.slots[batch - 3, int(case.accepted[batch - 3]) - 1] = slots + 7       # source slot out of range
    case.slots[batch - 2, 2] = slots                                           # destination out of range
    capi.fault_flags(clear=True)
    host = to_numpy_case(case.kwargs())
    run(case)
    torch.cuda.synchronize()
    assert capi.fault_flags(clear=True) == capi.LD_FAULT_DECODE_SLOT_RANGE
    check(case, host, "invalid requests in the prefetched wave")


def test_one_token_launch_with_padding_requests(device, kernel):
    """Padding requests (no tokens: cu repeats) in a one-token launch large enough for `auto` to pick
    the two-group streaming kernel (320 x 32 items)."""
    batch = 320
    case = bf16_case(batch, 1, batch + 8, device=device, seed=32)
    live = torch.ones(batch, dtype=torch.int32)
    live[3::4] = 0
    cu = torch.zeros(batch + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(live, 0)
    case.cu.copy_(cu.to(device))
    case.out.fill_(1.0)
    capi.fault_flags(clear=True)
    host = to_numpy_case(case.kwargs())
    run(case)
    torch.cuda.synchronize()
    assert capi.fault_flags(clear=True) == 0
    check(case, host, "padding requests")


def test_repeated_in_place_decode(device, kernel):
    """Three in-place steps: each re-reads the bf16 state the previous one stored."""
    case = bf16_case(16, 1, 40, device=device, seed=12)
    host = to_numpy_case(case.kwargs())
    for _ in range(3):
        run(case)
        oracle.decode(host["qkv"], host["a"], host["b"], host["a_log"], host["dt_bias"], host["slots"], host["cu"],
                      host["accepted"], host["pool"], host["gate"], host["weight"], host["out"],
                      num_k_heads=case.num_k_heads)
    torch.cuda.synchronize()
    assert_out_close_tail(bits(case.out), host["out"], "step 3 out")
    assert_bf16_state_close(bits(case.pool), host["pool"], "step 3 pool", max_ulps=3)


def test_rejects_an_fp32_pool_and_a_misaligned_stride(device):
    case = workloads.make_decode_case(2, 1, 8, device=device, seed=1)
    with pytest.raises(RuntimeError, match="BF16"):
        torch.ops.lightdelta.decode_bf16_state(*case.op_args())
    wide = torch.zeros(8, 32 * 128 * 128 + 4, device=device, dtype=torch.bfloat16)
    pool = wide[:, :32 * 128 * 128].view(8, 32, 128, 128)  # slot stride not a multiple of 8
    case.pool = pool
    with pytest.raises(RuntimeError, match="slot stride"):
        torch.ops.lightdelta.decode_bf16_state(*case.op_args())


def test_indexed_backend_runs_a_bf16_pool(device):
    from lightdelta_b200.backend import GDNBackend
    from lightdelta_b200.config import BackendConfig

    case = bf16_case(4, 2, 16, device=device, seed=21, accepted="uniform")
    direct = dataclasses.replace(case, pool=case.pool.clone(), out=torch.empty_like(case.out))
    backend = GDNBackend(BackendConfig(compute="cuda_fused", state_io="indexed"))
    backend(*case.op_args())
    torch.ops.lightdelta.decode_bf16_state(*direct.op_args())
    torch.cuda.synchronize()
    assert torch.equal(case.out, direct.out) and torch.equal(case.pool, direct.pool)
    packed = GDNBackend(BackendConfig(compute="cuda_fused", state_io="packed"))
    with pytest.raises(ValueError, match="fp32 pool"):
        packed(*case.op_args())
