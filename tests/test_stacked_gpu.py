"""GPU parity of BASELINE config 5's shape: the stacked 48-layer MTP verify step (T=4) captured in
one CUDA graph, with per-layer seeds and layers cycling over fewer physical state pools than
layers, replayed twice with every layer's slots and accepted counts changed in place between
replays (the pattern of the reference's graph test, tests/test_gdn.py:78-102).  Every layer's
outputs, every slot a replay touches and a sample of untouched slots are compared with the oracle
applied layer by layer in launch order.

Layers that share a physical pool use disjoint slot ranges of it, as the separate per-layer pools
of a real model would be, so each layer starts from states the previous replay left (snapshotted
for the oracle) and the comparison is per layer at the usual tolerances rather than a chain of
layers feeding each other's rounding.  The sequence count per layer is reduced from 2048 so the
CPU oracle finishes in seconds."""

import pytest
import torch

import oracle
from helpers import assert_out_close, assert_state_close, bits, to_numpy_case
from lightdelta_b200 import capi, workloads

pytestmark = pytest.mark.gpu

LAYERS = 48
SEQUENCES = 8
WIDTH = 4
PHYSICAL_POOLS = 5
LAYERS_PER_POOL = -(-LAYERS // PHYSICAL_POOLS)
SLOTS_PER_LAYER = SEQUENCES * WIDTH
POOL_SLOTS = 1 + LAYERS_PER_POOL * SLOTS_PER_LAYER
# Outputs outside 2e-3 of the oracle over 48 layers: runs measured 4 of 12.6 M (3.2e-7) and 2 of
# 6.3 M; the bound is about three times that rate.
OUTLIER_FRACTION = 1e-6


def _slot_range(layer: int) -> range:
    first = 1 + (layer // PHYSICAL_POOLS) * SLOTS_PER_LAYER
    return range(first, first + SLOTS_PER_LAYER)


def _reseat(wl, seed: int) -> None:
    """New slots (a permutation of the layer's own range of its pool) and accepted counts for every
    layer, written into the tensors the graph captured."""
    gen = torch.Generator().manual_seed(seed)
    for layer, c in enumerate(wl.layers):
        perm = torch.randperm(SLOTS_PER_LAYER, generator=gen) + _slot_range(layer).start
        c.slots.copy_(perm.to(torch.int32).view(SEQUENCES, WIDTH))
        c.accepted.copy_(torch.randint(1, WIDTH + 1, (SEQUENCES,), generator=gen, dtype=torch.int32))


def _oracle_step(wl, host_pools):
    """The oracle over the 48 layers in launch order; layer l reads and writes host pool l % P."""
    outs = []
    for index, c in enumerate(wl.layers):
        host = to_numpy_case(c.kwargs())
        pool = host_pools[index % len(host_pools)]
        oracle.decode(host["qkv"], host["a"], host["b"], host["a_log"], host["dt_bias"], host["slots"], host["cu"],
                      host["accepted"], pool, host["gate"], host["weight"], host["out"],
                      num_k_heads=c.num_k_heads, eps=c.eps)
        outs.append(host["out"])
    return outs


def test_stacked_graph_replays_match_the_oracle(device):
    pool_bytes = POOL_SLOTS * 32 * workloads.SLOT_HEAD_BYTES
    wl = workloads.stacked_workload(device, SEQUENCES, layers=LAYERS, width=WIDTH, seed=5,
                                    max_pool_bytes=PHYSICAL_POOLS * pool_bytes, pool_slots=POOL_SLOTS)
    assert len(wl.pools) == PHYSICAL_POOLS
    assert len({int(c.qkv.data_ptr()) for c in wl.layers}) == LAYERS  # per-layer inputs
    _reseat(wl, 7)

    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for c in wl.layers:
            torch.ops.lightdelta.decode(*c.op_args())
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for c in wl.layers:
            torch.ops.lightdelta.decode(*c.op_args())
    torch.cuda.synchronize()
    capi.fault_flags(clear=True)

    for replay, seed in enumerate((101, 202)):
        _reseat(wl, seed)
        torch.cuda.synchronize()
        host_pools = [p.cpu().numpy() for p in wl.pools]
        for c in wl.layers:
            c.out.fill_(7.0)
        graph.replay()
        torch.cuda.synchronize()
        expected = _oracle_step(wl, host_pools)
        flips, worst = 0, 0
        for index, c in enumerate(wl.layers):
            # 48 layers hold 6x the outputs of a BASELINE config: at this count the rare recurrence
            # output that lands on a bf16 rounding boundary before the gated RMSNorm (which scales
            # the flip) can end two ulps from the oracle.
            stats = assert_out_close(bits(c.out), expected[index], f"replay {replay} layer {index} out",
                                     max_outlier_ulps=2, max_fraction=2e-5)
            flips += stats["outside_2e3"]
            worst = max(worst, stats["outlier_ulps"])
        total = LAYERS * SEQUENCES * WIDTH * 32 * 128
        print(f"replay {replay}: {flips} of {total} outputs outside 2e-3, at most {worst} bf16 ulps")
        assert flips <= max(2, OUTLIER_FRACTION * total)
        for p, (pool, host) in enumerate(zip(wl.pools, host_pools)):
            touched = sorted({int(s) for layer in range(p, LAYERS, PHYSICAL_POOLS)
                              for s in wl.layers[layer].slots.flatten().tolist()})
            idx = torch.as_tensor(touched, device=device, dtype=torch.long)
            assert_state_close(pool[idx].cpu().numpy(), host[touched], f"replay {replay} pool {p}")
            spare = [s for s in range(POOL_SLOTS) if s not in set(touched)][:4]  # null slot + unused slots
            assert torch.equal(pool[spare].cpu(), torch.from_numpy(host[spare]))
    assert capi.fault_flags() == 0
    del graph
