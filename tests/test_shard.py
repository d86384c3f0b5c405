"""Row-sharded GEMM -> LayerNorm host logic, on CPU.

The sharded path has no exchange: rank g of G computes rows [r0, r1) of
Y = LayerNorm(X W) from its slice of the seeded input stream. Here two gloo ranks
(world_size 2, spawned processes) each compute their shard with the oracle,
gather the shards over gloo and compare with the unsharded computation bit for bit;
the row partition and the per-shard stream offsets are checked directly.
"""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from paralyn_b200 import shard, synthetic

ROWS, K, N = 67, 48, 40


def test_row_ranges_partition_the_rows():
    for rows in (0, 1, 7, 64, 65536, 65537):
        for world in (1, 2, 3, 4, 8):
            ranges = [shard.row_range(rows, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == rows
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [r1 - r0 for r0, r1 in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard.row_range(10, 2, 2)


def test_shard_streams_are_slices_of_the_full_stream():
    full = synthetic.normal(4, 0, ROWS * K)
    for world in (2, 3, 8):
        for rank in range(world):
            r0, r1 = shard.row_range(ROWS, world, rank)
            part = synthetic.normal(4, 2 * r0 * K, (r1 - r0) * K)
            assert part.tobytes() == full[r0 * K:r1 * K].tobytes()
    u = synthetic.uniform(3, 0, 1000)
    assert synthetic.uniform(3, 400, 600).tobytes() == u[400:].tobytes()


def chain_rows(x, w, rows):
    z = oracle.matmul(x, w, rows, N, K)
    return oracle.layer_norm(z, np.ones(N, np.float32), np.zeros(N, np.float32), np.float32(1e-5))


def _rank(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import torch
        topology = shard.Topology.from_environment()
        assert (topology.rank, topology.world, topology.selector) == (rank, world, f"cuda:{rank}")
        r0, r1 = shard.row_range(ROWS, world, rank)
        x = synthetic.normal(4, 2 * r0 * K, (r1 - r0) * K)
        w = synthetic.normal(4, 2 * ROWS * K, K * N, 0.0, 1.0 / 8)
        mine = torch.from_numpy(chain_rows(x, w, r1 - r0))
        sizes = [shard.row_range(ROWS, world, r) for r in range(world)]
        parts = [torch.empty((b - a, N), dtype=torch.float32) for a, b in sizes]
        dist.all_gather(parts, mine) if all(p.shape == mine.shape for p in parts) else \
            [dist.broadcast(parts[r] if r != rank else mine, src=r) for r in range(world)]
        if rank == 0:
            gathered = torch.cat([mine if r == 0 else parts[r] for r in range(world)]).numpy()
            results.put(gathered.tobytes())
        dist.barrier()
    finally:
        dist.destroy_process_group()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", (2,))
def test_two_rank_gloo_chain_matches_unsharded(world):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, results)) for r in range(world)]
    for proc in procs:
        proc.start()
    gathered = results.get(timeout=120)
    for proc in procs:
        proc.join(timeout=120)
        assert proc.exitcode == 0
    x = synthetic.normal(4, 0, ROWS * K)
    w = synthetic.normal(4, 2 * ROWS * K, K * N, 0.0, 1.0 / 8)
    assert gathered == chain_rows(x, w, ROWS).tobytes()
