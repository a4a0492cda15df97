"""int8-fast node hook: its wide-batch W8A8 path on the b200q INT8 kernels.

Mirrors the reference's _patches/int8_linear_mps.py: the ``int8-fast`` custom
node's ``int8_quant`` module is patched in place, either immediately (already
imported) or by a one-shot post-import hook on ``sys.meta_path`` (:66-142), and
``int8_forward_dynamic`` / ``int8_forward_dynamic_per_row`` are replaced.  The
reference routes them to a dequantize + bf16 GEMM because Apple GPUs had no
fast integer GEMM; on B200 the native INT8 route is the fast one, so CUDA calls
run per-token quant + tcgen05 int8 GEMM + the fused dequant epilogue
(torch.ops.b200q.i8_linear).  Non-CUDA calls keep the node's own functions.
Opt-in with ASFP8_INT8_EXT=1.
"""
import os
import sys

import torch

from . import _common

TAG = "[b200q/int8_linear]"

_installed = False
_patched = False
_orig_dyn = None
_orig_dyn_pr = None


def _native_linear(x, weight, weight_scale, bias, compute_dtype):
    out_dtype = compute_dtype if compute_dtype in (torch.bfloat16, torch.float16) else torch.bfloat16
    shp = x.shape
    y = torch.ops.b200q.i8_linear(x.reshape(-1, shp[-1]).to(out_dtype), weight,
                                  weight_scale.float(), bias, out_dtype, "none")
    y = y.reshape(*shp[:-1], weight.shape[0])
    return y if compute_dtype == out_dtype else y.to(compute_dtype)


def _eligible(x, weight, weight_scale):
    return (x.device.type == "cuda" and weight.dtype == torch.int8 and weight.dim() == 2
            and weight_scale.numel() in (1, weight.shape[0]))


def _dyn(x, weight, weight_scale, bias, compute_dtype):
    if _eligible(x, weight, weight_scale):
        return _native_linear(x, weight, weight_scale, bias, compute_dtype)
    return _orig_dyn(x, weight, weight_scale, bias, compute_dtype)


def _dyn_pr(x, weight, weight_scale, bias, compute_dtype):
    if _eligible(x, weight, weight_scale):
        return _native_linear(x, weight, weight_scale, bias, compute_dtype)
    return _orig_dyn_pr(x, weight, weight_scale, bias, compute_dtype)


def _apply(mod):
    """Patch int8-fast's int8_quant module in place (idempotent)."""
    global _patched, _orig_dyn, _orig_dyn_pr
    if _patched:
        return
    if not (hasattr(mod, "int8_forward_dynamic") and hasattr(mod, "int8_forward_dynamic_per_row")):
        return
    _orig_dyn = mod.int8_forward_dynamic
    _orig_dyn_pr = mod.int8_forward_dynamic_per_row
    mod.int8_forward_dynamic = _dyn
    mod.int8_forward_dynamic_per_row = _dyn_pr
    _patched = True
    print(f"{TAG} int8-fast W8A8 matmuls routed to the b200q tcgen05 INT8 kernels.")


def _scan_loaded():
    for mod in list(sys.modules.values()):
        try:
            name = getattr(mod, "__name__", "")
            if mod is not None and name.rsplit(".", 1)[-1] == "int8_quant" \
                    and hasattr(mod, "int8_forward_dynamic"):
                _apply(mod)
                return _patched
        except Exception:
            continue
    return False


class _Finder:
    """Wraps int8_quant's loader so it is patched right after it executes."""

    def find_spec(self, fullname, path, target=None):
        if fullname.rsplit(".", 1)[-1] != "int8_quant":
            return None
        spec = None
        for finder in sys.meta_path:
            if finder is self:
                continue
            try:
                spec = finder.find_spec(fullname, path, target)
            except Exception:
                spec = None
            if spec is not None:
                break
        if spec is None or spec.loader is None or not hasattr(spec.loader, "exec_module"):
            return None
        orig_exec = spec.loader.exec_module

        def exec_module(module, _orig_exec=orig_exec):
            _orig_exec(module)
            try:
                _apply(module)
            except Exception as e:
                print(f"{TAG} post-import patch failed: {e}")

        try:
            spec.loader.exec_module = exec_module
        except Exception:
            return None
        return spec


def install():
    global _installed
    if _installed:
        return
    if os.environ.get("ASFP8_INT8_EXT") != "1":
        return
    if not (_common.is_b200() and _common.native_ready()):
        return
    _installed = True
    if not _scan_loaded():
        sys.meta_path.insert(0, _Finder())
