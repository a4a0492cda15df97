"""Shared helpers of the seam patches: FP8 dtypes, on-device exact FP8 decode,
the ASFP8_* environment switches, the B200 device gate, and ``after_import``
(patch a third-party module as soon as it exists).

Mirrors the reference's _patches/_common.py (FP8_DTYPES :22, NATIVE_IMPLIES
:26-33, apply_native_master_switch :77-97, decode_fp8 :249-273) with CUDA/B200
in place of MPS/M5.
"""
import importlib.abc
import os
import sys
import threading

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


# ----------------------------------------------------------------------------- after_import
class _PatchingLoader(importlib.abc.Loader):
    """Runs the real loader, then the callbacks registered for the module.
    Everything else (resources, source lookups, reload) is the real loader's."""

    def __init__(self, inner, callbacks):
        self._inner, self._callbacks = inner, callbacks

    def create_module(self, spec):
        return self._inner.create_module(spec)

    def exec_module(self, module):
        self._inner.exec_module(module)
        module.__loader__ = self._inner
        if module.__spec__ is not None:
            module.__spec__.loader = self._inner
        for cb in list(self._callbacks):
            try:
                cb(module)
            except Exception as e:  # a failed patch must not break the host's import
                print(f"[b200q] post-import patch of {module.__name__} failed: {e!r}")

    def __getattr__(self, name):
        return getattr(self._inner, name)


class _AfterImportHook(importlib.abc.MetaPathFinder):
    """One meta-path entry for every deferred patch of the pack, keyed by the
    module's last dotted component (a ComfyUI custom node's package name is its
    directory, so only the leaf is stable).  It resolves the spec through the
    finders behind it and swaps in a loader that patches after execution."""

    def __init__(self):
        self.pending = {}  # leaf name -> [callback]
        self._busy = threading.local()

    def find_spec(self, fullname, path, target=None):
        callbacks = self.pending.get(fullname.rpartition(".")[2])
        if not callbacks or getattr(self._busy, "on", False):
            return None
        self._busy.on = True
        try:
            spec = None
            for finder in sys.meta_path:
                if finder is self or not hasattr(finder, "find_spec"):
                    continue
                try:
                    spec = finder.find_spec(fullname, path, target)
                except Exception:
                    spec = None
                if spec is not None:
                    break
        finally:
            self._busy.on = False
        if spec is None or spec.loader is None or not hasattr(spec.loader, "exec_module"):
            return None
        spec.loader = _PatchingLoader(spec.loader, callbacks)
        return spec


_HOOK = _AfterImportHook()


def after_import(leaf, callback, required=()):
    """Call ``callback(module)`` for the module whose dotted name ends in
    ``leaf`` and which defines every attribute in ``required``: right away if it
    is already imported, otherwise right after its import runs.  Returns True
    when the callback ran now."""
    for mod in list(sys.modules.values()):
        name = getattr(mod, "__name__", None)
        if (isinstance(name, str) and name.rpartition(".")[2] == leaf
                and all(hasattr(mod, a) for a in required)):
            callback(mod)
            return True
    _HOOK.pending.setdefault(leaf, []).append(callback)
    if _HOOK not in sys.meta_path:
        sys.meta_path.insert(0, _HOOK)
    return False
