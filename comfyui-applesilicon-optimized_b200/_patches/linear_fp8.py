"""torch.nn.functional.linear with FP8 operands on CUDA.

Mirrors the reference's _patches/linear_fp8.py (:53-73): FP8 operands reaching
``F.linear`` are decoded to the compute dtype and the original ``F.linear`` runs
on the decoded tensors; calls with no FP8 operand take the untouched original.
B200-first: the common case — 16-bit input, e4m3 weight — skips the weight
decode entirely and runs the b200q W8A16 kernel; other FP8 combinations decode
with the b200q exact decode kernel.  Opt-in with ASFP8_FP8_EXT=1.
"""
import os

import torch
import torch.nn.functional as F

from . import _common
from ._common import FP8_DTYPES, decode_fp8

TAG = "[b200q/linear_fp8]"

_original = F.linear
_installed = False


def _decode_operand(t, compute_dtype):
    if t.dtype in FP8_DTYPES:
        return decode_fp8(t, compute_dtype)
    if t.dtype != compute_dtype:
        return t.to(compute_dtype)
    return t


def _patched_linear(input, weight, bias=None):
    if (input.dtype not in FP8_DTYPES and weight.dtype not in FP8_DTYPES
            and (bias is None or bias.dtype not in FP8_DTYPES)):
        return _original(input, weight, bias)
    if input.device.type != "cuda":
        return _original(input, weight, bias)
    if (weight.dtype == torch.float8_e4m3fn and weight.dim() == 2
            and input.dtype in (torch.bfloat16, torch.float16)
            and (bias is None or bias.dtype not in FP8_DTYPES)):
        return torch.ops.b200q.w8a16_linear(input, weight, None, bias, "none", input.dtype)
    compute_dtype = torch.bfloat16 if input.dtype in FP8_DTYPES else input.dtype
    return _original(_decode_operand(input, compute_dtype), _decode_operand(weight, compute_dtype),
                     _decode_operand(bias, compute_dtype) if bias is not None else None)


def install():
    global _installed
    if _installed:
        return
    if os.environ.get("ASFP8_FP8_EXT") != "1":
        return
    if not (_common.is_b200() and _common.native_ready()):
        return
    F.linear = _patched_linear
    torch.nn.functional.linear = _patched_linear
    _installed = True
    print(f"{TAG} F.linear FP8 operands on CUDA: e4m3 weights via the W8A16 kernel, "
          f"other FP8 operands decoded on device.")
