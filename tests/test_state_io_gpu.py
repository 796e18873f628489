"""GPU tests of gather_state / scatter_state / copy_state: bit-exact against the oracle and
torch indexing (reference tests/test_gdn.py:125-143 and BASELINE config 4)."""

import numpy as np
import pytest
import torch

import oracle
from lightdelta_b200 import capi, workloads

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("index_stride", [1, 4])
@pytest.mark.parametrize("path", ["torch_op", "capi"])
def test_prefill_state_initialization_and_reuse(device, index_stride, path):
    """Reference tests/test_gdn.py:125-143: strided slot vector, zero fill, slot 0 untouched."""
    gen = torch.Generator(device=device)
    gen.manual_seed(42)
    pool = torch.randn(6, 48, 128, 128, device=device, generator=gen) * 0.1
    before = pool.clone()
    slots = torch.full((3, index_stride), -1, device=device, dtype=torch.int32)[:, 0]
    slots.copy_(torch.tensor([2, 1, 0], device=device, dtype=torch.int32))
    valid = torch.tensor([True, False, False], device=device)
    packed = torch.empty(3, *pool.shape[1:], device=device)
    gather = torch.ops.lightdelta.gather_state if path == "torch_op" else capi.gather_state
    scatter = torch.ops.lightdelta.scatter_state if path == "torch_op" else capi.scatter_state
    gather(pool, slots, valid, packed)
    torch.cuda.synchronize()
    assert torch.equal(packed[0], pool[2])
    assert packed[1:].count_nonzero() == 0
    packed.add_(1)
    scatter(packed, slots, pool)
    torch.cuda.synchronize()
    assert torch.equal(pool[0], before[0])
    assert torch.equal(pool[1], torch.ones_like(pool[1]))
    assert torch.equal(pool[2], before[2] + 1)
    assert torch.equal(pool[3:], before[3:])


@pytest.mark.parametrize("inner", [(32, 128, 128), (3, 5, 7), (2, 3, 128)])
def test_gather_scatter_match_oracle(device, inner):
    """Random slots with nulls, invalid rows and a strided slot vector; vector and scalar paths."""
    gen = torch.Generator(device=device)
    gen.manual_seed(sum(inner))
    n_slots, n = 20, 9
    pool = torch.randn(n_slots, *inner, device=device, generator=gen)
    slots_storage = torch.zeros(n, 3, device=device, dtype=torch.int32)
    slots = slots_storage[:, 1]
    chosen = torch.randperm(n_slots - 1, device=device, generator=gen)[:n] + 1
    slots.copy_(chosen.to(torch.int32))
    slots[2] = 0
    slots[5] = -3
    valid = torch.rand(n, device=device, generator=gen) > 0.25
    packed = torch.full((n, *inner), 7.0, device=device)
    host_pool = pool.cpu().numpy()
    host_packed = packed.cpu().numpy()
    torch.ops.lightdelta.gather_state(pool, slots, valid, packed)
    oracle.gather_state(host_pool, slots.cpu().numpy(), valid.cpu().numpy(), host_packed)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(packed.cpu().numpy(), host_packed)

    packed.mul_(-1)
    host_packed = packed.cpu().numpy()
    dest = torch.randperm(n_slots - 1, device=device, generator=gen)[:n].to(torch.int32) + 1
    dest[4] = 0
    torch.ops.lightdelta.scatter_state(packed, dest, pool)
    oracle.scatter_state(host_packed, dest.cpu().numpy(), host_pool)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(pool.cpu().numpy(), host_pool)


def test_copy_state_matches_oracle(device):
    gen = torch.Generator(device=device)
    gen.manual_seed(3)
    pool = torch.randn(12, 32, 128, 128, device=device, generator=gen)
    src = torch.tensor([1, 2, 0, 5, 7], device=device, dtype=torch.int32)
    dst = torch.tensor([3, 2, 4, 0, 9], device=device, dtype=torch.int32)
    host = pool.cpu().numpy()
    torch.ops.lightdelta.copy_state(pool, src, dst)
    oracle.copy_slots(host, src.cpu().numpy(), dst.cpu().numpy())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(pool.cpu().numpy(), host)


def test_out_of_range_slots_are_skipped_and_reported(device):
    pool = torch.randn(4, 2, 128, 128, device=device)
    before = pool.clone()
    capi.fault_flags(clear=True)
    slots = torch.tensor([1, 9], device=device, dtype=torch.int32)
    packed = torch.full((2, 2, 128, 128), 5.0, device=device)
    torch.ops.lightdelta.gather_state(pool, slots, torch.ones(2, device=device, dtype=torch.bool), packed)
    torch.cuda.synchronize()
    assert torch.equal(packed[0], pool[1]) and packed[1].count_nonzero() == 0
    assert capi.fault_flags(clear=True) == capi.LD_FAULT_GATHER_SLOT_RANGE
    torch.ops.lightdelta.scatter_state(packed, torch.tensor([7, 2], device=device, dtype=torch.int32), pool)
    torch.cuda.synchronize()
    assert torch.equal(pool[2], torch.zeros_like(pool[2])) and torch.equal(pool[[0, 1, 3]], before[[0, 1, 3]])
    assert capi.fault_flags(clear=True) == capi.LD_FAULT_SCATTER_SLOT_RANGE


def test_config4_layer_round_trip_bit_exact(device):
    """BASELINE config 4 on one physical layer pool (2048 x [32,128,128] fp32, 4 GiB): gather 512
    distinct slots, scatter them to a permuted distinct set; bit-exact against torch indexing."""
    gen = torch.Generator(device=device)
    gen.manual_seed(44)
    pool = torch.empty(2048, 32, 128, 128, device=device)
    pool.normal_(0.0, 0.02, generator=gen)
    gather_idx, scatter_idx = workloads.config4_indices(device)
    packed = torch.empty(512, 32, 128, 128, device=device)
    torch.ops.lightdelta.gather_state(pool, gather_idx, torch.ones(512, device=device, dtype=torch.bool), packed)
    assert torch.equal(packed, pool[gather_idx.long()])
    expected = pool.clone()
    expected[scatter_idx.long()] = packed
    torch.ops.lightdelta.scatter_state(packed, scatter_idx, pool)
    torch.cuda.synchronize()
    assert torch.equal(pool, expected)
