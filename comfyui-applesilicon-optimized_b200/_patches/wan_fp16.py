"""FP16-output INT8 epilogue for Wan 14B's native INT8 projections.

Seam (reference _patches/wan_fp16.py): for the three Wan 14B projection
shapes, ``_int8_linear_prequant`` with an fp16 output first offers the
pre-quantized activation to ``maybe_prequant``; a non-None answer is the layer's
output, None means "take the general route".  Its fp16 epilogue rounds twice,

    out = half( half(float(C) * (col_scale[n] * row_scale[m])) + bias[n] )

(the reference's ``i8_matmul2d_nt_fused_cs_half``, int8_gemm.mm:1159-1243,
1965-2024), which on B200 is the channelwise tcgen05 epilogue with an fp16
output.  The switches are the reference's (ASFP8_DIT_EXT=1 opts in;
ASFP8_WAN_FAST, ASFP8_WAN_EXACT and ASFP8_WAN_FP16_GEMM default on).

Which calls are taken is decided by the binding's own argument validation
(``int8_linear_kernel.half_epilogue_problem``), run on the contiguous operands
the hook would pass, plus this hook's extra conditions: inference only, exact
``torch.Tensor`` operands (no tensor subclasses), a Wan weight shape and an
fp16 bias.  A kernel error switches the hook off for the process and the
caller keeps its general route.
"""
import os

import torch

# (N, K) of Wan 14B's projections that take this epilogue.
WAN_WEIGHT_SHAPES = frozenset({(5120, 5120), (13824, 5120), (5120, 13824)})
# Environment switches and their defaults; all must read "1".
SWITCHES = (("ASFP8_DIT_EXT", "0"), ("ASFP8_WAN_FAST", "1"), ("ASFP8_WAN_EXACT", "1"),
            ("ASFP8_WAN_FP16_GEMM", "1"))


class _HookState:
    calls = 0        # successful fp16 epilogue calls
    disabled = None  # the exception that switched the hook off, if any


state = _HookState()


def _enabled():
    return state.disabled is None and all(os.environ.get(k, d) == "1" for k, d in SWITCHES)


def _hook_problem(x, row_scale, weight, col_scale, bias):
    """Conditions of this hook on top of the binding's argument checks."""
    if torch.is_grad_enabled():
        return "autograd is on"
    if tuple(weight.shape) not in WAN_WEIGHT_SHAPES:
        return "not a Wan 14B projection"
    if any(type(t) is not torch.Tensor for t in (x, row_scale, weight, col_scale)):
        return "tensor subclass operand"
    if row_scale.dtype != torch.float32 or col_scale.dtype != torch.float32:
        return "scales are not float32"
    if bias is not None and (type(bias) not in (torch.Tensor, torch.nn.Parameter)
                             or bias.dtype != torch.float16
                             or tuple(bias.shape) != (weight.shape[0],)):
        return "bias is not an fp16 [N] tensor"
    return None


def maybe_prequant(kernel, x, row_scale, weight, col_scale, bias, shape):
    """FP16 output of the pre-quantized Wan projection, or None."""
    fn = getattr(kernel, "i8_matmul2d_nt_fused_cs_half", None)
    if fn is None or not _enabled():
        return None
    if _hook_problem(x, row_scale, weight, col_scale, bias) is not None:
        return None
    from .int8_linear_kernel import half_epilogue_problem
    args = (x.contiguous(), weight.contiguous(), row_scale.reshape(-1).contiguous(),
            col_scale.reshape(-1).contiguous(), bias)
    if half_epilogue_problem(*args) is not None:
        return None
    try:
        out = fn(*args)
    except Exception as exc:
        state.disabled = exc
        print(f"[b200q/wan_fp16] fp16 epilogue off for this process, general route kept ({exc!r}).")
        return None
    state.calls += 1
    return out.reshape(*shape[:-1], weight.shape[0])
