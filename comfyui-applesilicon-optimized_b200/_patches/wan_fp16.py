"""FP16-output INT8 epilogue for Wan 14B's native INT8 projections.

Mirrors the reference's _patches/wan_fp16.py (:17-45): for the three Wan 14B
projection shapes, ``_int8_linear_prequant`` with an fp16 output first offers the
pre-quantized activation to ``maybe_prequant``, which runs the INT8 GEMM with the
fp16 two-rounding epilogue

    out = half( half(float(C) * (col_scale[n] * row_scale[m])) + bias[n] )

(``i8_matmul2d_nt_fused_cs_half``, int8_gemm.mm:1159-1243, 1965-2024) -- on B200
the channelwise tcgen05 epilogue with an fp16 output.  Same switches as the
reference (ASFP8_DIT_EXT=1 to opt in; ASFP8_WAN_FAST, ASFP8_WAN_EXACT,
ASFP8_WAN_FP16_GEMM default on), same argument guards, and the same latch: a
failure disables the route for the process and the caller keeps its own path.
"""
import os

import torch

_calls = 0
_dead = False
_shapes = {(5120, 5120), (13824, 5120), (5120, 13824)}


def maybe_prequant(kernel, x, row_scale, weight, col_scale, bias, shape):
    """FP16 output of the pre-quantized Wan projection, or None."""
    global _calls, _dead
    if (_dead or torch.is_grad_enabled()
            or os.environ.get("ASFP8_DIT_EXT") != "1"
            or os.environ.get("ASFP8_WAN_FAST", "1") != "1"
            or os.environ.get("ASFP8_WAN_EXACT", "1") != "1"
            or os.environ.get("ASFP8_WAN_FP16_GEMM", "1") != "1"
            or kernel is None or not hasattr(kernel, "i8_matmul2d_nt_fused_cs_half")
            or tuple(weight.shape) not in _shapes
            or any(type(t) is not torch.Tensor or t.device.type != "cuda"
                   for t in (x, row_scale, weight, col_scale))
            or x.dtype != torch.int8 or weight.dtype != torch.int8
            or row_scale.dtype != torch.float32 or col_scale.dtype != torch.float32
            or x.ndim != 2 or x.shape[1] != weight.shape[1]
            or row_scale.numel() != x.shape[0] or col_scale.numel() != weight.shape[0]
            or (bias is not None and (type(bias) not in (torch.Tensor, torch.nn.Parameter)
                                      or bias.device.type != "cuda"
                                      or bias.dtype != torch.float16
                                      or bias.shape != (weight.shape[0],)))):
        return None
    try:
        out = kernel.i8_matmul2d_nt_fused_cs_half(
            x.contiguous(), weight.contiguous(), row_scale.reshape(-1).contiguous(),
            col_scale.reshape(-1).contiguous(), bias)
    except Exception as exc:
        _dead = True
        print(f"[b200q/wan_fp16] keeping the general fp16 route ({exc!r}).")
        return None
    _calls += 1
    return out.reshape(*shape[:-1], weight.shape[0])
