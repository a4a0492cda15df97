"""torch._int_mm on B200: exact int8 x int8 -> int32 on the tensor cores.

Mirrors the reference's _patches/int_mm_mps.py: the same seam
(``torch._int_mm = _int_mm_cuda``), the same one-time adversarial parity canary
against an exact int64 product (corner codes -128/127, ragged K, non-tile
shapes; int_mm_mps.py:67-81) before the route is trusted, and pass-through of
everything the route does not own.  Differences: the device is CUDA/sm_100;
the b200q kernel consumes ``b`` ([K,N]) as the stored [N,K] weight without the
reference's ``b.t().contiguous()`` copy; and a failing canary leaves the stock
torch._int_mm in place (the route is simply not installed) rather than an fp32
emulation tier.  Opt-in with ASFP8_INT8_EXT=1 (or the ASFP8_NATIVE master switch).
"""
import os

import torch

from . import _common

TAG = "[b200q/int_mm]"

_orig = None
_installed = False


def _canary():
    """True if the native kernel matches the exact product on the corner cases."""
    g = torch.Generator().manual_seed(0)
    for M, K, N in ((3, 129, 5), (16, 4096, 32), (130, 512, 256)):
        a = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int8)
        b = torch.randint(-128, 128, (K, N), generator=g, dtype=torch.int8)
        a[:, 0] = -128
        b[0, :] = 127
        ref = (a.long() @ b.long()).to(torch.int32)
        out = torch.ops.b200q.int_mm(a.cuda(), b.cuda())
        if not torch.equal(out.cpu(), ref):
            print(f"{TAG} parity canary FAILED at ({M},{K},{N}); torch._int_mm left stock.")
            return False
    return True


def _int_mm_cuda(a, b):
    if (a.device.type == "cuda" and b.device.type == "cuda" and a.dtype == torch.int8
            and b.dtype == torch.int8 and a.dim() == 2 and b.dim() == 2):
        return torch.ops.b200q.int_mm(a, b)
    return _orig(a, b)


def install():
    global _orig, _installed
    if _installed:
        return
    if os.environ.get("ASFP8_INT8_EXT") != "1":
        return
    if not hasattr(torch, "_int_mm") or not _common.is_b200() or not _common.native_ready():
        return
    if not _canary():
        return
    _orig = torch._int_mm
    torch._int_mm = _int_mm_cuda
    _installed = True
    print(f"{TAG} torch._int_mm on CUDA routed to the exact tcgen05 int8 kernel (canary passed).")
