"""Standard-fp8 comfy Linear via the b200q W8A16 kernel (FP8 weights, 16-bit activations).

Mirrors the reference's _patches/linear_fp8_w8a16.py: replaces
``comfy.ops.disable_weight_init.Linear.forward_comfy_cast_weights`` (:199-213,
:250-251) so eligible layers (e4m3 plain-tensor weight, bf16/fp16 input, no
LoRA weight/bias functions, no offload machinery; :89-117) compute
``bf16(x . decode(W)^T + bias)`` without materialising a decoded weight, after a
one-time parity self-check against the decode path on the first eligible layer
(:120-148, rel < 5e-2).  B200-first differences: activations stay bf16 (the
reference casts them to fp16, :166-171; tcgen05 kind::f16 takes bf16 directly),
bias / per-tensor weight scale (comfy's ``scale_weight``) / cast are fused into
the epilogue, and there is no M cap (ASFP8_FP8_W8A16_M_MAX defaults to
unlimited) because the kernel wins at every M on B200.

Opt-in: ASFP8_FP8_SGEMM=1 or ASFP8_FP8_EXT=1; kill switch ASFP8_FP8_W8A16=0.
A failing self-check leaves the layer on comfy's original forward.
"""
import os

import torch

from . import _common
from ._common import FP8_DTYPES, decode_fp8

TAG = "[b200q/w8a16]"

_installed = False
_orig_forward = None
_kernel = None          # True once the native path is usable, False when latched off
_self_checked = False

_ELIGIBLE_INPUT_DTYPES = (torch.bfloat16, torch.float16)


def _min_dim():
    try:
        return int(os.environ.get("ASFP8_FP8_SGEMM_MIN_DIM", "0"))
    except ValueError:
        return 0


def _m_max():
    try:
        return int(os.environ.get("ASFP8_FP8_W8A16_M_MAX", "0")) or None
    except ValueError:
        return None


def _eligible(module, input):
    """Cheap per-call predicate; no device work."""
    w = getattr(module, "weight", None)
    if w is None or getattr(w, "dtype", None) != torch.float8_e4m3fn:
        return False
    if type(w) not in (torch.Tensor, torch.nn.Parameter):
        return False
    if w.dim() != 2 or w.device.type != "cuda" or not w.is_contiguous():
        return False
    if input.dtype not in _ELIGIBLE_INPUT_DTYPES or input.device.type != "cuda":
        return False
    if input.shape[-1] != w.shape[1]:
        return False
    if len(getattr(module, "weight_function", [])) > 0 or len(getattr(module, "bias_function", [])) > 0:
        return False
    if hasattr(module, "_v") or hasattr(module, "_prefetch"):
        return False
    N, K = int(w.shape[0]), int(w.shape[1])
    M = input.numel() // input.shape[-1]
    m_max = _m_max()
    if m_max is not None and M > m_max:
        return False
    return max(N, K) >= _min_dim()


def _weight_scale(module):
    s = getattr(module, "scale_weight", None)
    if isinstance(s, torch.Tensor) and s.numel() == 1:
        return s.to(device=module.weight.device, dtype=torch.float32).reshape(1)
    return None


def _bias(module):
    b = getattr(module, "bias", None)
    if b is None:
        return None
    if b.dtype in FP8_DTYPES:
        return decode_fp8(b, torch.float32)
    return b


def _self_check(module, x2d):
    """One-time parity check vs the decode path on the first eligible layer's
    real weight (<= 32 rows, max|d| / max|ref| < 5e-2)."""
    global _kernel
    try:
        rows = x2d[: min(int(x2d.shape[0]), 32)].contiguous()
        w = module.weight
        ref = rows.float() @ decode_fp8(w, torch.float32).t()
        s = _weight_scale(module)
        if s is not None:
            ref = ref * s
        out = torch.ops.b200q.w8a16_linear(rows, w, s, None, "none", torch.float32)
        rel = ((out - ref).abs().max() / (ref.abs().max() + 1e-9)).item()
        if rel >= 5e-2:
            print(f"{TAG} self-check failed (rel={rel:.4f}); w8a16 disabled.")
            _kernel = False
            return False
        print(f"{TAG} self-check ok (rel={rel:.2e}); w8a16 tcgen05 path live.")
        return True
    except Exception as e:
        print(f"{TAG} self-check raised; w8a16 disabled: {e!r}")
        _kernel = False
        return False


def _w8a16_forward(module, input):
    orig_shape = input.shape
    x2d = input.reshape(-1, orig_shape[-1])
    global _self_checked
    if not _self_checked:
        _self_checked = True
        if not _self_check(module, x2d):
            return _orig_forward(module, input)
    out = torch.ops.b200q.w8a16_linear(x2d, module.weight, _weight_scale(module), _bias(module),
                                       "none", input.dtype)
    return out.reshape(*orig_shape[:-1], module.weight.shape[0])


def _patched_forward(self, input):
    if _kernel and _eligible(self, input):
        return _w8a16_forward(self, input)
    return _orig_forward(self, input)


def install():
    global _installed, _orig_forward, _kernel
    if _installed:
        return
    if not (os.environ.get("ASFP8_FP8_EXT") == "1" or os.environ.get("ASFP8_FP8_SGEMM") == "1"):
        return
    if os.environ.get("ASFP8_FP8_W8A16", "1") == "0":
        return
    if not (_common.is_b200() and _common.native_ready()):
        return
    try:
        import comfy.ops as ops
    except Exception as e:
        print(f"{TAG} comfy.ops unavailable ({e!r}); not installed.")
        return
    _kernel = True
    _orig_forward = ops.disable_weight_init.Linear.forward_comfy_cast_weights
    ops.disable_weight_init.Linear.forward_comfy_cast_weights = _patched_forward
    _installed = True
    print(f"{TAG} standard-fp8 Linear routed via the b200q tcgen05 W8A16 kernel "
          f"(in-smem e4m3 dequant, fused bias/scale epilogue).")
