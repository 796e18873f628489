"""Multi-rank host logic on CPU (gloo, world size 2): sequence-slot sharding and the bench's
max-over-ranks aggregation.  The data path has no collective, so sharded decoding must equal
the single-process result exactly."""

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

from lightdelta_b200 import sharding

ROOT = Path(__file__).resolve().parent.parent


@pytest.mark.parametrize("total,world", [(2048, 1), (2048, 2), (2048, 8), (13, 4), (3, 8)])
def test_shards_partition_the_sequences(total, world):
    seen = []
    for rank in range(world):
        block = sharding.shard_range(total, rank, world)
        assert all(sharding.owner(s, total, world) == rank for s in block)
        seen.extend(block)
    assert seen == list(range(total))


def test_local_slots_skip_the_null_slot():
    slots = {sharding.local_slot(s, 16, 2, slots_per_sequence=4, candidate=c) for s in range(8) for c in range(4)}
    assert slots == set(range(1, 33))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    import bench
    import oracle
    from golden import detrand

    dist = bench.Dist(world)
    try:
        total, hv, h = 6, 4, 2
        block = sharding.shard_range(total, rank, world)
        n = len(block)
        # Per-sequence inputs are functions of the global sequence index, so every rank can build
        # exactly the rows it owns; the rank's pool holds only its own slots.
        width = (2 * h + hv) * 128
        qkv = np.stack([detrand.bf16_bits(detrand.normal(100 + s, (width,))) for s in block])
        ba = np.stack([detrand.bf16_bits(detrand.normal(200 + s, (2 * hv,))) for s in block])
        gate = np.stack([detrand.bf16_bits(detrand.normal(300 + s, (hv, 128), 0.2)) for s in block])
        pool = np.concatenate([np.zeros((1, hv, 128, 128), np.float32)] +
                              [detrand.normal(400 + s, (1, hv, 128, 128), 0.02) for s in block])
        out = np.zeros((n, hv, 128), np.uint16)
        oracle.decode(qkv, ba[:, hv:], ba[:, :hv], np.zeros(hv, np.float32), np.zeros(hv, np.float32),
                      np.arange(1, n + 1, dtype=np.int32).reshape(n, 1), np.arange(n + 1, dtype=np.int32),
                      np.ones(n, np.int32), pool, gate, detrand.bf16_bits(detrand.normal(7, (128,))), out,
                      num_k_heads=h)
        np.savez(Path(out_dir) / f"rank{rank}.npz", out=out, pool=pool[1:], seqs=np.array(list(block)))
        dist.barrier()
        assert dist.max(float(rank + 1)) == float(world)
        assert dist.sum(1.0) == float(world)
    finally:
        dist.close()


def test_two_rank_sharded_decode_equals_single_process(tmp_path):
    world = 2
    for name, ranks in (("w2", world), ("w1", 1)):
        (tmp_path / name).mkdir()
        mp.start_processes(_rank_main, args=(ranks, _free_port(), str(tmp_path / name)), nprocs=ranks,
                           start_method="spawn", join=True)
    single = np.load(tmp_path / "w1" / "rank0.npz")
    parts = [np.load(tmp_path / "w2" / f"rank{r}.npz") for r in range(world)]
    assert np.concatenate([p["seqs"] for p in parts]).tolist() == single["seqs"].tolist()
    np.testing.assert_array_equal(np.concatenate([p["out"] for p in parts]), single["out"])
    np.testing.assert_array_equal(np.concatenate([p["pool"] for p in parts]), single["pool"])
