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


def _gpu_rank_main(rank, world, port, out_dir, width):
    """One rank of a sharded decode on the GPU: the rank builds the rows of the sequences it owns
    (inputs are functions of the global sequence index), keeps their slots in a pool of its own and
    runs lightdelta::decode on them."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    import torch

    import bench
    from golden import detrand
    from lightdelta_b200 import ops  # noqa: F401

    dist = bench.Dist(world)
    try:
        device = torch.device("cuda", rank % torch.cuda.device_count())
        torch.cuda.set_device(device)
        total, hv, h = 24, 32, 16
        block = sharding.shard_range(total, rank, world)
        n = len(block)

        def bf16(array):
            return torch.from_numpy(detrand.bf16_bits(array).view(np.int16)).view(torch.bfloat16).to(device)

        rows = n * width
        qkvz = torch.cat([bf16(detrand.normal(100 + s, (width, (2 * h + 2 * hv) * 128))) for s in block])
        ba = torch.cat([bf16(detrand.normal(200 + s, (width, 2 * hv))) for s in block])
        pool = torch.zeros(1 + rows, hv, 128, 128, device=device)
        for i, s in enumerate(block):
            state = torch.from_numpy(detrand.normal(400 + s, (hv, 128, 128), 0.02)).to(device)
            pool[1 + i * width:1 + (i + 1) * width] = state  # every candidate slot starts from the same state
        slots = torch.tensor([[sharding.local_slot(s, total, world, width, c) for c in range(width)] for s in block],
                             dtype=torch.int32, device=device)
        accepted = torch.tensor([1 + s % width for s in block], dtype=torch.int32, device=device)
        cu = torch.arange(0, rows + 1, width, dtype=torch.int32, device=device)
        qkv_width = (2 * h + hv) * 128
        out = torch.zeros(rows, hv, 128, dtype=torch.bfloat16, device=device)
        torch.ops.lightdelta.decode(qkvz[:, :qkv_width], ba[:, hv:], ba[:, :hv], torch.zeros(hv, device=device),
                                    torch.zeros(hv, device=device), slots, cu, accepted, pool,
                                    qkvz[:, qkv_width:qkv_width + hv * 128].view(rows, hv, 128),
                                    bf16(detrand.normal(7, (128,))), out, 1e-6)
        torch.cuda.synchronize()
        np.savez(Path(out_dir) / f"rank{rank}.npz", out=out.view(torch.int16).cpu().numpy(),
                 pool=pool[1:].cpu().numpy(), seqs=np.array(list(block)))
        dist.barrier()
    finally:
        dist.close()


@pytest.mark.gpu
@pytest.mark.parametrize("width", [1, 4])
def test_two_rank_sharded_gpu_decode_equals_single_process(device, tmp_path, width):
    """The sharded data path on the GPU kernels: two ranks (processes; on one GPU they share it, with
    no kernel of one waiting on the other) each decode their block of sequences from a pool of their
    own; together they must reproduce one process decoding all of them bit for bit."""
    world = 2
    for name, ranks in (("w2", world), ("w1", 1)):
        (tmp_path / name).mkdir()
        mp.start_processes(_gpu_rank_main, args=(ranks, _free_port(), str(tmp_path / name), width), nprocs=ranks,
                           start_method="spawn", join=True)
    single = np.load(tmp_path / "w1" / "rank0.npz")
    parts = [np.load(tmp_path / "w2" / f"rank{r}.npz") for r in range(world)]
    assert np.concatenate([p["seqs"] for p in parts]).tolist() == single["seqs"].tolist()
    np.testing.assert_array_equal(np.concatenate([p["out"] for p in parts]), single["out"])
    np.testing.assert_array_equal(np.concatenate([p["pool"] for p in parts]), single["pool"])
