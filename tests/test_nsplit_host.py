"""CPU tier for the column-parallel (N-split) FP8 linear (``b200q.nsplit``).

* The column plan covers every output column exactly once with 16-byte
  aligned starts, at the Wan block's widths and 1/2/4/8 ranks.
* World size 2 under gloo on 127.0.0.1: the IPC-handle exchange of
  ``PeerOutput`` hands every rank the other ranks' handles and offsets (a fake
  native layer stands in for CUDA IPC, which needs GPUs), and the pointers the
  fused GEMM writes to land at each rank's own first column.
* World size 2 under gloo: column blocks computed per rank with the CPU oracle
  and gathered equal the unsplit FP8 linear bit for bit (per-tensor scales make
  every column's math independent of the split).
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import conftest  # noqa: F401  (loads the pack as b200q, also in spawned ranks)
from b200q import nsplit


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("N", [5120, 13824, 15360, 3072, 100, 8])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_column_shards_cover_once_aligned(N, world):
    shards = nsplit.column_shards(N, world)
    assert len(shards) == world
    cols = [c for c0, n in shards for c in range(c0, c0 + n)]
    assert cols == list(range(N))
    assert all(c0 % nsplit.COLUMN_ALIGN == 0 for c0, n in shards if n)
    if N % (world * nsplit.COLUMN_ALIGN) == 0:
        assert len({n for _, n in shards}) == 1          # even split at the Wan widths


def test_column_shards_reject_bad_sizes():
    with pytest.raises(ValueError):
        nsplit.column_shards(0, 2)
    with pytest.raises(ValueError):
        nsplit.column_shards(8, 0)


class _FakeIPC:
    """Stands in for the CUDA IPC calls: a rank's handle is 64 bytes of its rank
    number, its offset 256 * (rank + 1); importing rank r's handle 'maps' it at
    0x1000000 * (r + 1)."""

    def __init__(self, rank):
        self.rank = rank
        self.closed = []

    def ipc_export(self, t):
        return bytes([self.rank]) * 64, 256 * (self.rank + 1)

    def ipc_import(self, handle, offset):
        src = handle[0]
        assert handle == bytes([src]) * 64 and offset == 256 * (src + 1)
        base = 0x1000000 * (src + 1)
        return base + offset, base

    def ipc_close(self, base):
        self.closed.append(base)


def _init(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)


def _exchange_worker(rank, world, port, q):
    _init(rank, world, port)
    try:
        from b200q import nsplit as ns
        fake = _FakeIPC(rank)
        out = ns.PeerOutput(4, 96, torch.bfloat16, "cpu", native=fake)
        c0, _ = ns.column_shards(96, world)[rank]
        ptrs = out.peer_ptrs(c0)
        out.close()
        q.put((rank, ptrs, fake.closed))
    finally:
        dist.destroy_process_group()


def _run(target, world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(res, key=lambda r: r[0])


def test_peer_output_exchange_gloo():
    (r0, p0, c0), (r1, p1, c1) = _run(_exchange_worker, 2)
    # rank 0 writes into rank 1's copy at its own first column (0), rank 1 into
    # rank 0's copy at column 48 (2 bytes per bf16 element)
    assert p0 == [0x2000000 + 512 + 0]
    assert p1 == [0x1000000 + 256 + 48 * 2]
    assert c0 == [0x2000000] and c1 == [0x1000000]


def _gather_worker(rank, world, port, M, K, N, q):
    _init(rank, world, port)
    try:
        from b200q import nsplit as ns
        from oracle import oracle
        g = torch.Generator().manual_seed(11)
        x = torch.randn(M, K, generator=g).to(torch.bfloat16)
        w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
        b = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16)
        xq, xs = oracle.quantize_fp8_tensorwise(x)
        wq, ws = oracle.quantize_fp8_tensorwise(w)
        c0, n = ns.column_shards(N, world)[rank]
        part = oracle.scaled_mm_fp8(xq, wq[c0:c0 + n], xs, ws, None, b[c0:c0 + n],
                                    torch.bfloat16, "gelu_tanh")
        parts = [None] * world
        dist.all_gather_object(parts, (c0, part))
        if rank == 0:
            full = oracle.scaled_mm_fp8(xq, wq, xs, ws, None, b, torch.bfloat16, "gelu_tanh")
            got = torch.cat([p for _, p in sorted(parts, key=lambda t: t[0])], dim=1)
            q.put((rank, torch.equal(got, full)))
        else:
            q.put((rank, True))
    finally:
        dist.destroy_process_group()


def test_column_blocks_gather_to_unsplit_result_gloo():
    res = _run(_gather_worker, 2, 40, 64, 200)
    assert all(ok for _, ok in res)
