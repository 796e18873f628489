"""The persistent decode kernel's bounded waits, made to run out on purpose (no GPU fault).

ld_decode_wait_test shortens every in-kernel wait to a few hundred microseconds and makes each
state load announce more bytes than it copies, so the mbarrier phase a consumer waits for never
completes although every copy lands.  The kernel must raise LD_FAULT_WAIT_TIMEOUT, store nothing,
and return; the same context must then run the launch correctly with the default settings."""

import pytest
import torch

import oracle
from helpers import (
    assert_bf16_state_close,
    assert_out_close,
    assert_out_close_tail,
    assert_state_close,
    bits,
    to_numpy_case,
)
from lightdelta_b200 import capi, workloads

pytestmark = pytest.mark.gpu


@pytest.fixture
def streaming(device):
    previous = capi.set_decode_kernel("stream")
    yield
    capi.set_decode_kernel(previous)
    capi.set_decode_wait_test(0, 0)


@pytest.mark.parametrize("width, state_dtype", [(1, "fp32"), (4, "fp32"), (1, "bf16")])
def test_waits_run_out_store_nothing_and_return(streaming, device, width, state_dtype):
    """Both persistent kernels: the fp32 one (one-token and verify launches) and the bf16 pool's
    one-token kernel (bf16 verify launches run the one-CTA-per-item kernel, which has no waits)."""
    case = workloads.make_decode_case(40, width, 1 + 40 * width + 5, device=device, seed=70 + width,
                                      accepted="uniform", state_scale=0.1)
    if state_dtype == "bf16":
        case.pool = case.pool.to(torch.bfloat16)
    case.out.fill_(3.0)
    pool_before = case.pool.clone()
    out_before = case.out.clone()
    capi.fault_flags(clear=True)

    capi.set_decode_wait_test(200_000, 64)  # 200 us bound; every state load expects 64 bytes too many
    try:
        capi.decode(*case.op_args())
        torch.cuda.synchronize()
    finally:
        capi.set_decode_wait_test(0, 0)
    assert capi.fault_flags(clear=True) == capi.LD_FAULT_WAIT_TIMEOUT
    assert torch.equal(case.pool.view(torch.int16) if state_dtype == "bf16" else case.pool,
                       pool_before.view(torch.int16) if state_dtype == "bf16" else pool_before)
    assert torch.equal(case.out.view(torch.int16), out_before.view(torch.int16))

    # The context is intact: the same launch with the default bound matches the oracle.
    host = to_numpy_case(case.kwargs())
    capi.decode(*case.op_args())
    torch.cuda.synchronize()
    assert capi.fault_flags(clear=True) == 0
    oracle.decode(host["qkv"], host["a"], host["b"], host["a_log"], host["dt_bias"], host["slots"], host["cu"],
                  host["accepted"], host["pool"], host["gate"], host["weight"], host["out"],
                  num_k_heads=case.num_k_heads, eps=case.eps)
    if state_dtype == "bf16":
        assert_out_close_tail(bits(case.out), host["out"], "after timeout: out")
        assert_bf16_state_close(bits(case.pool), host["pool"], "after timeout: pool")
    else:
        assert_out_close(bits(case.out), host["out"], "after timeout: out")
        assert_state_close(case.pool.cpu().numpy(), host["pool"], "after timeout: pool")

