"""Shared helpers of the seam patches: FP8 dtypes, on-device exact FP8 decode,
the ASFP8_* environment switches and the B200 device gate.

Mirrors the reference's _patches/_common.py (FP8_DTYPES :22, NATIVE_IMPLIES
:26-33, apply_native_master_switch :77-97, decode_fp8 :249-273) with CUDA/B200
in place of MPS/M5.
"""
import os

import torch

FP8_DTYPES = (torch.float8_e4m3fn, torch.float8_e5m2)

# Routes implied by the master switch ASFP8_NATIVE=1 (explicit values win).
NATIVE_IMPLIES = (
    "ASFP8_FP8_EXT",    # FP8 W8A8 torch._scaled_mm route + F.linear FP8 route
    "ASFP8_FP8_SGEMM",  # FP8 W8A16 forward_comfy_cast_weights route
    "ASFP8_INT8_EXT",   # INT8 W8A8 routes (torch._int_mm, comfy int8 Linear, int8-fast hook)
)


def is_b200(device=None):
    """True on a CUDA device with compute capability 10.0 (B200)."""
    if not torch.cuda.is_available():
        return False
    try:
        return torch.cuda.get_device_capability(device) == (10, 0)
    except Exception:
        return False


def native_ready():
    """Library built and the current device can run it."""
    from . import _native
    return _native.available()


def apply_native_master_switch(environ=None):
    """Default to the native routes on a B200; explicit per-route values win.

    Returns the list of variables the switch set (for the startup log)."""
    if environ is None:
        environ = os.environ
    if "ASFP8_NATIVE" not in environ:
        if not is_b200():
            return []
        environ["ASFP8_NATIVE"] = "1"
    if environ.get("ASFP8_NATIVE") != "1":
        return []
    implied = []
    for var in NATIVE_IMPLIES:
        if var not in environ:
            environ[var] = "1"
            implied.append(var)
    return implied


def flag(name, default="0"):
    return os.environ.get(name, default) == "1"


def decode_fp8(t, out_dtype=torch.float32):
    """Exact FP8 -> `out_dtype` decode on the tensor's own device.

    CUDA tensors decode with the b200q kernel (every code, NaNs kept NaN);
    other devices keep torch's own cast, as the reference leaves non-MPS
    tensors to stock torch."""
    if t.device.type == "cuda":
        return torch.ops.b200q.fp8_decode(t, out_dtype)
    return t.to(out_dtype)


def decode_fp8_as(t, out_dtype):
    return decode_fp8(t, out_dtype)
