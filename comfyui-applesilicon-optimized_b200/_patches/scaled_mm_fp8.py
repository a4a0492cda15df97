"""torch._scaled_mm with FP8 operands on B200: the b200q tcgen05 kind::f8f6f4 GEMM.

Mirrors the reference's _patches/scaled_mm_fp8.py: the same seam
(``torch._scaled_mm = _cuda_scaled_mm``, keyword signature of :149-159), the same
eligibility shape (e4m3 x e4m3, 2-D; :66-81) and the same epilogue arithmetic as
its native route (_fast_route :123-146: fp32 product, * scale_a, * scale_b,
* scale_result, + bias in fp32, cast to out_dtype).  Differences, B200-first:
``other`` ([K,N], column-major = the [N,K] weight) is consumed in place instead
of the reference's per-call ``other.t().contiguous()`` weight copy (a row-major
``other`` is copied to K-major once per weight and reused); the scales,
bias and cast are fused into the GEMM's epilogue instead of 3-4 elementwise
passes over an fp32 [M,N] intermediate; and there is no weight-size gate
(ASFP8_FP8_EXT_MIN_DIM defaults to 0), the kernel wins at every shape.

Calls the route does not own (non-CUDA, non-FP8, e5m2, >2-D) go to the
untouched original.  Opt-in with ASFP8_FP8_EXT=1 (or the master switch).
"""
import collections
import os
import weakref

import torch

from . import _common
from ._common import FP8_DTYPES

TAG = "[b200q/scaled_mm]"

_original = None
_installed = False


def _min_dim():
    try:
        return int(os.environ.get("ASFP8_FP8_EXT_MIN_DIM", "0"))
    except ValueError:
        return 0


def _fast_eligible(input, other):
    """Pure shape/dtype/env predicate (no device work)."""
    if os.environ.get("ASFP8_FP8_EXT") != "1":
        return False
    if input.dtype != torch.float8_e4m3fn or other.dtype != torch.float8_e4m3fn:
        return False
    if input.device.type != "cuda" or other.device.type != "cuda":
        return False
    if input.dim() != 2 or other.dim() != 2 or input.shape[1] != other.shape[0]:
        return False
    return max(int(other.shape[1]), int(input.shape[1])) >= _min_dim()


# K-major copies of row-major `other` operands, one per weight: a [K,N] tensor
# with unit stride along N cannot be the GEMM's [N,K] operand in place, and the
# reference copies it on every call (scaled_mm_fp8.py:134).  Here the copy is
# made once and reused while the same tensor (or the tensor it is a view of) is
# passed unchanged: the entry is keyed by that owner's identity and checked
# against its data pointer, shape, strides and version counter, and dies with it.
_KMAJOR_MAX = 8
_kmajor = collections.OrderedDict()  # id(owner) -> (weakref(owner), key, w_nk)


def _k_major_weight(other):
    w = other.t()
    if w.stride(1) == 1:
        return w  # column-major `other`: the stored [N,K] weight, read in place
    owner = other._base if other._base is not None else other
    key = (other.data_ptr(), tuple(other.shape), tuple(other.stride()), other._version)
    oid = id(owner)
    ent = _kmajor.get(oid)
    if ent is not None and ent[0]() is owner and ent[1] == key:
        _kmajor.move_to_end(oid)
        return ent[2]
    w_nk = w.contiguous()
    _kmajor[oid] = (weakref.ref(owner, lambda _r, oid=oid: _kmajor.pop(oid, None)), key, w_nk)
    _kmajor.move_to_end(oid)
    while len(_kmajor) > _KMAJOR_MAX:
        _kmajor.popitem(last=False)
    return w_nk


def _fast_route(input, other, scale_a, scale_b, scale_result, bias, out_dtype):
    """e4m3 x e4m3 -> out_dtype in one kernel; `other` [K,N] read as W [N,K]."""
    return torch.ops.b200q.fp8_scaled_mm(
        input, _k_major_weight(other), scale_a, scale_b, scale_result, bias,
        out_dtype if out_dtype is not None else torch.float32, "none")


def _cuda_scaled_mm(input, other, *, out_dtype=None, scale_a=None, scale_b=None, bias=None,
                    scale_result=None, use_fast_accum=False):
    if input.dtype in FP8_DTYPES and _fast_eligible(input, other):
        return _fast_route(input, other, scale_a, scale_b, scale_result, bias, out_dtype)
    return _original(input, other, out_dtype=out_dtype, scale_a=scale_a, scale_b=scale_b,
                     bias=bias, scale_result=scale_result, use_fast_accum=use_fast_accum)


def install():
    global _original, _installed
    if _installed:
        return
    if not hasattr(torch, "_scaled_mm"):
        return
    if os.environ.get("ASFP8_FP8_EXT") != "1":
        return
    if not (_common.is_b200() and _common.native_ready()):
        return
    _original = torch._scaled_mm
    torch._scaled_mm = _cuda_scaled_mm
    _installed = True
    print(f"{TAG} torch._scaled_mm e4m3 x e4m3 on CUDA routed to the b200q tcgen05 FP8 GEMM "
          f"(fused scale/bias epilogue, weight consumed in place).")
