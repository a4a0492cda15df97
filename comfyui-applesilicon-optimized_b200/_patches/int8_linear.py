"""int8-fast node hook: its wide-batch W8A8 matmuls on the b200q INT8 kernels.

The seam is the same as the reference's _patches/int8_linear_mps.py: the
``int8-fast`` custom node's ``int8_quant`` module exposes
``int8_forward_dynamic`` and ``int8_forward_dynamic_per_row``
(x, weight, weight_scale, bias, compute_dtype), and both are replaced once that
module exists — at install time if int8-fast loaded first, otherwise right after
its import (``_common.after_import``; custom nodes load in directory order).

The route differs on purpose.  The reference sends these calls to a dequantize
+ bf16 GEMM because Apple GPUs had no fast integer GEMM; on B200 the integer
path is the fast one, so a CUDA call runs per-token quant + the tcgen05 int8
GEMM + the fused dequant epilogue (torch.ops.b200q.i8_linear) and keeps the
node's W8A8 numerics.  Calls the route does not own (CPU tensors, other dtypes)
go to the node's own functions.  Opt-in with ASFP8_INT8_EXT=1.
"""
import os

import torch

from . import _common

TAG = "[b200q/int8_linear]"

# The two entry points of int8-fast's int8_quant module that this hook replaces.
TARGETS = ("int8_forward_dynamic", "int8_forward_dynamic_per_row")

_installed = False
_patched = False


def _owns(x, weight, weight_scale):
    """CUDA activations, a 2-D int8 weight, a scalar or per-row weight scale."""
    return (isinstance(x, torch.Tensor) and x.device.type == "cuda"
            and weight.dtype == torch.int8 and weight.dim() == 2
            and weight_scale.numel() in (1, weight.shape[0]))


def _tcgen05_linear(x, weight, weight_scale, bias, compute_dtype):
    """y = dequant(quant(x) . weight^T) + bias in compute_dtype (16-bit outputs
    come straight from the epilogue; other dtypes are cast from bf16)."""
    out_dtype = compute_dtype if compute_dtype in (torch.bfloat16, torch.float16) else torch.bfloat16
    lead = x.shape[:-1]
    y = torch.ops.b200q.i8_linear(x.reshape(-1, x.shape[-1]).to(out_dtype), weight,
                                  weight_scale.float(), bias, out_dtype, "none")
    y = y.reshape(*lead, weight.shape[0])
    return y if out_dtype == compute_dtype else y.to(compute_dtype)


def _route(node_fn):
    """The replacement for one of int8-fast's functions: the native route for
    calls it owns, ``node_fn`` for the rest (kept as ``__wrapped__``)."""

    def forward(x, weight, weight_scale, bias, compute_dtype):
        if _owns(x, weight, weight_scale):
            return _tcgen05_linear(x, weight, weight_scale, bias, compute_dtype)
        return node_fn(x, weight, weight_scale, bias, compute_dtype)

    forward.__wrapped__ = node_fn
    forward.__name__ = getattr(node_fn, "__name__", "forward")
    return forward


def patch_module(mod):
    """Replace TARGETS on int8-fast's int8_quant module (once per process)."""
    global _patched
    if _patched or not all(callable(getattr(mod, name, None)) for name in TARGETS):
        return False
    for name in TARGETS:
        setattr(mod, name, _route(getattr(mod, name)))
    _patched = True
    print(f"{TAG} int8-fast W8A8 matmuls routed to the b200q tcgen05 INT8 kernels.")
    return True


def install():
    global _installed
    if _installed or os.environ.get("ASFP8_INT8_EXT") != "1":
        return
    if not (_common.is_b200() and _common.native_ready()):
        return
    _installed = True
    _common.after_import("int8_quant", patch_module, required=TARGETS)
