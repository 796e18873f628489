"""The packed state path without allocation (ld_decode_packed_noalloc).

Callers that cannot allocate device memory while they decode (a host binding the C ABI from a
runtime with no device allocator, an engine that reserves the whole GPU for its pools at start-up,
a loop that cannot take cudaMalloc's device-wide synchronisation) call this entry point; its
scratch slots live in one static device array of the library.  The GPU test checks it through the
C ABI against the existing packed path (GDNBackend in packed mode, whose scratch the framework
allocates) on two calls in a row, the second one reading the states the first one committed.

This file sorts last so that a run stopping at its first failure has run every other test first.
"""

import ctypes

import pytest
import torch

from helpers import assert_out_close, assert_state_close, bits
from lightdelta_b200 import capi, workloads
from lightdelta_b200.backend import GDNBackend
from lightdelta_b200.config import BackendConfig

SCRATCH_BYTES = 64 * 1024 * 1024


def _mixed(case, device):
    """Mixed accepted counts, a request with an invalid accepted count, a padding request (all slots
    null), a null destination and a request with fewer tokens than its window."""
    batch, width = case.slots.shape
    case.accepted.copy_(torch.arange(batch, device=device, dtype=torch.int32) % width + 1)
    case.accepted[1] = 0
    case.slots[batch - 1] = 0
    case.slots[2, width - 1] = 0
    if width > 1:
        cu = torch.arange(0, batch * width + 1, width, device=device, dtype=torch.int32)
        cu[4:] -= 1  # request 3 has width - 1 tokens
        case.cu.copy_(cu)
    return case


@pytest.mark.gpu
@pytest.mark.parametrize("width", [1, 4])
def test_noalloc_matches_the_packed_path_on_two_calls(device, width):
    batch = 7
    expected_pool = None
    actual_pool = None
    first_slots = None
    for call in range(2):
        case = workloads.make_decode_case(batch, width, 64, device=device, seed=40 + 10 * width + call,
                                          accepted="uniform", pool=expected_pool)
        if first_slots is None:
            first_slots = case.slots.clone()
        else:
            case.slots.copy_(first_slots.roll(1, 1))  # the slots the first call committed, other steps
        _mixed(case, device)
        if actual_pool is None:
            actual_pool = case.pool.clone()
        expected_pool = case.pool
        actual_out = torch.full_like(case.out, 3.0)
        case.out.fill_(3.0)
        GDNBackend(BackendConfig(compute="cuda_fused", state_io="packed"))(**case.kwargs())
        args = case.op_args()
        capi.decode_packed_noalloc(*args[:8], actual_pool, args[9], args[10], actual_out, case.eps)
        torch.cuda.synchronize()
        stats = assert_out_close(bits(actual_out), bits(case.out), f"call {call + 1} out")
        assert_state_close(actual_pool.cpu().numpy(), expected_pool.cpu().numpy(), f"call {call + 1} pool")
        print(f"width {width} call {call + 1}: {stats}")
    assert capi.fault_flags() == 0


def test_noalloc_rejects_more_scratch_than_it_holds(native):
    """Host-side check, no launch: 16 requests x 4 steps at HV=32 need 65 scratch slots of 2 MiB."""
    fake = 1 << 20  # 16-byte aligned, never dereferenced: the call fails validation first
    slot = 32 * 128 * 128
    lib = native.lib()
    entry = lib.ld_decode_packed_noalloc
    entry.argtypes = lib.ld_decode.argtypes
    entry.restype = ctypes.c_int
    rc = entry(fake, 8192, fake, 32, fake, 32, fake, fake, 0, fake, 16, 4, fake, fake, fake, 100, slot, fake, 4096,
               fake, 0, fake, 64, 16, 32, 1e-6, None)
    assert rc == native.LD_ERR_INVALID
    message = native.last_error()
    assert "static scratch holds" in message and str(SCRATCH_BYTES - 32 * 1024) in message
