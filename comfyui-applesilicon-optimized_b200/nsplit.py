"""Column-parallel (N-split) FP8 linears over NVLink, for the Wan-shaped block.

The default multi-GPU split of this path is by token rows (the reference
chunks rows itself, _patches/int8_linear_kernel_mps.py:75-94): every rank holds
all weights and no data moves between GPUs.  The N-split is the optional other
layout: rank r of g holds only the weight rows of its output columns
[c0_r, c0_r + n_r), computes them for every token, and each layer's output is
all-gathered so that every rank holds the full [M, N] result for the next
layer.  It trades NVLink traffic ((g-1)/g of each output per rank) for 1/g of
the weight memory.

The all-gather is fused into the GEMM (b200q_fp8_scaled_mm_allgather): each
rank's output buffer is mapped into every other rank's process once (CUDA IPC
handles exchanged through torch.distributed), and the GEMM epilogue writes
every output block to all g copies, so the transfer of one tile overlaps the
MMAs of the next.  A one-element all-reduce on the stream after a layer is the
barrier after which the gathered columns may be read.

One process per GPU; `group` is the torch.distributed process group (NCCL on
GPUs).  Host logic that needs no GPU (column plan, handle exchange) also runs
under gloo.
"""
import torch
import torch.distributed as dist

from ._patches import _native

# Column offsets are multiples of 8 so that every rank's first column is 16-byte
# aligned in a 16-bit output row (the TMA store's requirement).
COLUMN_ALIGN = 8


def column_shards(N, world, align=COLUMN_ALIGN):
    """[(c0, n)] per rank: near-equal column blocks, each start a multiple of
    `align`; the last rank takes the remainder (possibly a short block)."""
    if N <= 0 or world <= 0:
        raise ValueError("N and world must be positive")
    step = -(-N // world)
    step = -(-step // align) * align
    out = []
    for r in range(world):
        c0 = min(r * step, N)
        out.append((c0, max(0, min(step, N - c0))))
    return out


class PeerOutput:
    """A full-width [M, N] output buffer on every rank, each mapped into every
    other rank's process.  ``peer_ptrs(c0)`` gives the device pointers of the
    other ranks' copies at column c0 (what the fused GEMM writes to)."""

    def __init__(self, M, N, dtype, device, group=None, native=_native):
        self.M, self.N, self.dtype = M, N, dtype
        self.group = group
        self.native = native
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.buf = torch.empty((M, N), dtype=dtype, device=device)
        mine = native.ipc_export(self.buf)
        table = [None] * self.world
        dist.all_gather_object(table, mine, group=group)
        self._peers = []  # (rank, pointer to the peer copy's element [0, 0], mapping base)
        for r, (handle, offset) in enumerate(table):
            if r != self.rank:
                ptr, base = native.ipc_import(handle, offset)
                self._peers.append((r, ptr, base))

    def peer_ptrs(self, c0):
        es = torch.empty((), dtype=self.dtype).element_size()
        return [ptr + c0 * es for _, ptr, _ in self._peers]

    def close(self):
        for _, _, base in self._peers:
            self.native.ipc_close(base)
        self._peers = []


def stream_barrier(group=None, device=None):
    """One-element all-reduce ordered on the current stream: once it completes
    on a rank, every rank's earlier launches on its stream have completed, so
    the columns they wrote into this rank's buffers are in place."""
    t = torch.zeros((1,), dtype=torch.int32, device=device)
    dist.all_reduce(t, group=group)


class ColumnParallelFP8Linear:
    """This rank's column block of an FP8 W8A8 linear (per-tensor e4m3 weight
    and activation scales, bias, optional GELU), with the output all-gathered in
    the GEMM epilogue."""

    def __init__(self, w_q, w_scale, bias, act=None, group=None):
        """w_q: the FULL [N, K] e4m3 weight (this rank keeps its block only),
        w_scale: per-tensor fp32 scale, bias: [N] or None."""
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.N, self.K = w_q.shape
        self.c0, self.n = column_shards(self.N, self.world)[self.rank]
        self.w = w_q[self.c0:self.c0 + self.n].contiguous()
        self.w_scale = w_scale.reshape(1).float().contiguous()
        self.bias = None if bias is None else bias[self.c0:self.c0 + self.n].contiguous()
        self.act = act

    def __call__(self, xq, x_scale, out: PeerOutput):
        """xq [M, K] e4m3 and its per-tensor scale (the full activation, the same
        on every rank) -> this rank's columns written into every rank's ``out``."""
        if out.N != self.N or out.M != xq.shape[0]:
            raise RuntimeError("[b200q] output buffer shape does not match the layer")
        if self.n == 0:
            return out.buf
        return _native.fp8_scaled_mm_allgather(xq, self.w, x_scale.reshape(1), self.w_scale, None,
                                               self.bias, out.buf, self.c0,
                                               out.peer_ptrs(self.c0), self.act)
