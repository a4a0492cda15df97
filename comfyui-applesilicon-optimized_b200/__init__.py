"""b200q — B200-native quantized DiT linears as a ComfyUI custom-node pack.

Importing the pack (ComfyUI does so by directory path) registers the
``torch.ops.b200q`` kernels and installs the seam patches, in the order of the
reference's bootstrap (__init__.py:89-122 of ComfyUI-AppleSilicon-Optimized):
the ASFP8_NATIVE master switch implies the per-route flags, explicit values win,
and ASFP8_ENABLE_ONLY / ASFP8_DISABLE bisect by patch module name.
Set B200Q_NO_BOOTSTRAP=1 to import without installing anything.
"""
import os

NODE_CLASS_MAPPINGS = {}
NODE_DISPLAY_NAME_MAPPINGS = {}

from ._patches import _native  # noqa: E402,F401  (registers torch.ops.b200q)


def bootstrap():
    """Apply the master switch and install every seam patch; returns the names
    of the patches that were attempted."""
    from . import _patches
    from ._patches import _common
    implied = _common.apply_native_master_switch()
    if implied:
        print(f"[b200q] ASFP8_NATIVE=1 -> {', '.join(v + '=1' for v in implied)}")
    only = {n.strip() for n in os.environ.get("ASFP8_ENABLE_ONLY", "").split(",") if n.strip()}
    disabled = {n.strip() for n in os.environ.get("ASFP8_DISABLE", "").split(",") if n.strip()}
    attempted = []
    for patch in _patches.ordered_patches():
        short = patch.__name__.rsplit(".", 1)[-1]
        if (only and short not in only) or short in disabled:
            print(f"[b200q] skipping {short} (ASFP8_ENABLE_ONLY/ASFP8_DISABLE)")
            continue
        attempted.append(short)
        try:
            patch.install()
        except Exception as e:  # never take the host application down
            print(f"[b200q] patch {patch.__name__} failed: {e}")
    return attempted


if os.environ.get("B200Q_NO_BOOTSTRAP") != "1":
    bootstrap()
