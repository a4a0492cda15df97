"""CPU tier, world size 2 (gloo on 127.0.0.1): the token-row sharding used by
``bench.py --gpus N``.  Each rank runs the oracle on its contiguous row shard;
the gathered shards must equal the unsharded result byte for byte (rows are
independent in quant, GEMM and epilogue), and the timing reduction must take the
max over ranks.  No GPU and no data-path collective are involved."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench
from oracle import oracle


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, M, K, N, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(5)
        x = (torch.randn(M, K, generator=g) * 0.5).to(torch.bfloat16)
        w = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int8)
        ws = torch.rand(N, generator=g) * 0.01 + 1e-3
        b = torch.randn(N, generator=g).to(torch.bfloat16)
        start, rows = bench._split_rows(M, world, rank)
        part = oracle.int8_linear(x[start:start + rows], w, ws, b)
        parts = [None] * world
        dist.all_gather_object(parts, (start, rows, part))
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            full = oracle.int8_linear(x, w, ws, b)
            parts.sort(key=lambda p: p[0])
            covered = [r for s, n, _ in parts for r in range(s, s + n)]
            got = torch.cat([p for _, _, p in parts], dim=0)
            q.put((covered == list(range(M)), torch.equal(got, full), float(t.item())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M", [37, 64])
def test_row_shards_reassemble_exactly(M):
    world, K, N = 2, 96, 40
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, K, N, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    covered, equal, tmax = q.get(timeout=10)
    assert covered and equal and tmax == 2.0


def test_split_rows_is_balanced():
    for M, world in ((65520, 8), (65520, 3), (7, 4), (9216, 2)):
        shards = [bench._split_rows(M, world, r) for r in range(world)]
        assert sum(n for _, n in shards) == M
        assert max(n for _, n in shards) - min(n for _, n in shards) <= 1
        assert all(shards[i][0] + shards[i][1] == shards[i + 1][0] for i in range(world - 1))
