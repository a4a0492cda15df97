"""Seam patches of the b200q pack (one module per reference seam, each with an
idempotent ``install()``), plus ``_native`` (the C-ABI binding / torch ops)."""


def ordered_patches():
    """Install order, following the reference's bootstrap (__init__.py:116-122):
    _scaled_mm before the Linear routes, int_mm before the int8 Linear routes."""
    from . import int8_linear, int8_linear_kernel, int_mm, linear_fp8, linear_fp8_w8a16, scaled_mm_fp8
    return (scaled_mm_fp8, linear_fp8, linear_fp8_w8a16, int_mm, int8_linear, int8_linear_kernel)
