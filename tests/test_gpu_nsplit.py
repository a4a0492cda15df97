"""GPU tier, two B200s: the column-parallel FP8 linear with the all-gather fused
into the GEMM epilogue (``b200q.nsplit``, ``b200q_fp8_scaled_mm_allgather``).

Two ranks (one process per GPU, NCCL on 127.0.0.1) each compute their column
block of the same layer and write it into both ranks' full-width outputs.
After the stream barrier every rank's output must equal, bit for bit, the
single-GPU ``fp8_scaled_mm`` of the full weight on that rank (each column's
arithmetic does not depend on the split), and be within 1 bf16 ULP of the
CPU oracle's fp32 value on sampled rows.  Shapes cover the fused CTA-pair route (M >=
256), a column count whose blocks end inside a tile (TMA stores clipped at
the block edge, next to the other rank's columns), two calls in a row into the
same buffers, and the copy route of small M.  The same kernel path also runs
on one GPU with local buffers standing in for the peers' copies; the two-rank
test is skipped with fewer than two GPUs.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import conftest  # noqa: F401  (loads the pack as b200q, also in spawned ranks)

pytestmark = pytest.mark.gpu

CASES = [(1024, 1024, 3072, "gelu_tanh"), (512, 640, 600, None), (100, 512, 1024, "gelu_tanh")]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    results = []
    try:
        from b200q import nsplit
        from b200q._patches import _native
        from oracle import oracle
        for M, K, N, act in CASES:
            g = torch.Generator().manual_seed(M + N)
            x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(dev)
            w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16).to(dev)
            b = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16).to(dev)
            xq, xs = _native.fp8_quant_tensorwise(x)
            wq, ws = _native.fp8_quant_tensorwise(w)
            layer = nsplit.ColumnParallelFP8Linear(wq, ws, b, act)
            out = nsplit.PeerOutput(M, N, torch.bfloat16, dev)
            ref = _native.fp8_scaled_mm(xq, wq, xs.reshape(1), ws.reshape(1), None, b,
                                        torch.bfloat16, act)
            ok = True
            for _ in range(2):  # two calls in a row into the same buffers
                out.buf.fill_(float("nan"))
                nsplit.stream_barrier(device=dev)  # every rank's buffer is reset first
                layer(xq, xs, out)
                nsplit.stream_barrier(device=dev)
                torch.cuda.synchronize()
                ok = ok and torch.equal(out.buf, ref)
            rows = torch.arange(0, M, max(1, M // 48))
            ref32 = oracle.scaled_mm_fp8(xq[rows].cpu(), wq.cpu(), xs.cpu(), ws.cpu(), None,
                                         b.cpu(), None, act)
            # bf16 output against the fp32 oracle: within 1 bf16 ULP, as for
            # the single-GPU FP8 tests
            err = oracle.elementwise_ulp_ratio(out.buf[rows].cpu(), ref32)
            nsplit.stream_barrier(device=dev)   # nobody writes into `out` while it closes
            torch.cuda.synchronize()
            out.close()
            results.append((M, K, N, bool(ok), float(err), _native.device_status()))
        q.put((rank, results, None))
    except Exception as exc:  # reported to the parent, which fails the test
        q.put((rank, results, repr(exc)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M,K,N,act", CASES)
def test_allgather_copies_on_one_gpu(native, M, K, N, act):
    """One GPU, the same kernel path: this 'rank' owns columns [c0, c0 + n) of
    a full-width output and also writes them into 3 further local buffers
    standing in for the peers' copies.  Every copy's block equals the plain
    GEMM of that weight block, and no column outside the block is touched."""
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(7 * M + N)
    xq, xs = native.fp8_quant_tensorwise(torch.randn(M, K, generator=g).to(torch.bfloat16).to(dev))
    wq, ws = native.fp8_quant_tensorwise(
        (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16).to(dev))
    b = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16).to(dev)
    c0, n = 8 * ((N // 3) // 8), N // 2          # a block in the middle of the row
    blk = wq[c0:c0 + n].contiguous()
    ref = native.fp8_scaled_mm(xq, blk, xs.reshape(1), ws.reshape(1), None, b[c0:c0 + n],
                               torch.bfloat16, act)
    copies = [torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev) for _ in range(4)]
    es = 2
    peer_ptrs = [c.data_ptr() + c0 * es for c in copies[1:]]
    for _ in range(2):
        native.fp8_scaled_mm_allgather(xq, blk, xs.reshape(1), ws.reshape(1), None, b[c0:c0 + n],
                                       copies[0], c0, peer_ptrs, act)
    torch.cuda.synchronize()
    for c in copies:
        assert torch.equal(c[:, c0:c0 + n], ref)
        assert torch.isnan(c[:, :c0].float()).all() and torch.isnan(c[:, c0 + n:].float()).all()
    assert native.device_status() == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nsplit_allgather_two_ranks_matches_single_gpu():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for rank, results, err in res:
        assert err is None, f"rank {rank}: {err}"
        assert len(results) == len(CASES)
        for M, K, N, ok, ulp_ratio, status in results:
            assert ok, f"rank {rank} M={M} K={K} N={N}: gathered output differs from one GPU"
            assert ulp_ratio <= 1.0, (rank, M, K, N, ulp_ratio)
            assert status == 0
    assert all(p.exitcode == 0 for p in procs)
