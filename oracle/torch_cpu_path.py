"""The reference's CPU fallback route, restated with torch CPU kernels — TEST AND
BASELINE INFRASTRUCTURE ONLY.

``bench.py`` times these functions as the CPU baseline (its ``cpu_baseline``
object and its ``--impl reference`` arm) on the box's host cores; ``tests/``
checks them against the numpy oracle in ``oracle.py``.  The product path never
imports this module.

What each function restates (paths inside luix93/ComfyUI-AppleSilicon-Optimized):

* ``int8_linear`` — comfy_kitchen's eager ``int8_linear`` as the reference
  drives it when its native kernel is absent: the per-token quant
  (``quantize_int8_rowwise``, stochastic rounding off, restated step by step at
  _patches/int8_ext/int8_gemm.mm:1337-1381), ``torch._int_mm`` (the reference's
  ``_int_mm`` seam falls through to it off-MPS, _patches/int_mm_mps.py:90-110)
  and the chunked fp32 rescale + bias of ``_int8_linear_prequant``
  (_patches/int8_linear_kernel_mps.py:203-215).  Bit-identical to
  ``oracle.int8_linear``.
* ``scaled_mm_fp8`` — the decode route of ``_mps_scaled_mm``
  (_patches/scaled_mm_fp8.py:178-207): both e4m3 operands decoded to bf16, one
  bf16 matmul (fp32 accumulation inside torch's CPU GEMM, bf16 result), the
  scales applied in fp32 and rounded back to bf16, the bias added in fp32, one
  cast to the output dtype.  The per-tensor e4m3 activation quant in front of
  it (BASELINE configs 3 and 5) is ``quantize_fp8_tensorwise``.
* ``w8a16_linear`` — the decode route of the W8A16 seam: the e4m3 weight
  decoded to the compute dtype, then ``F.linear`` (_patches/linear_fp8_w8a16.py:
  1-11, _patches/_common.py:249), with BASELINE config 2's per-tensor weight
  scale, bias and tanh-GELU applied to the result.

The tanh-GELU of the "up" layers is torch's ``F.gelu(approximate="tanh")`` on
the rounded linear output (the reference has no fused GELU epilogue; ComfyUI
applies the activation as its own op).
"""
import torch
import torch.nn.functional as F

_E4M3_MAX = 448.0


def quantize_int8_rowwise(x):
    """x [M,K] bf16/f16 -> (q int8 [M,K], scale f32 [M,1]):
    scale = max(absmax/127, 1e-30) in fp32, s = x.dtype(scale) (0 -> the dtype's
    tiny), q = clamp(rint(x.dtype(x / s)), -128, 127)."""
    absmax = x.abs().amax(dim=-1, keepdim=True).float()
    scale = torch.clamp(absmax / 127.0, min=1e-30)
    s = scale.to(x.dtype)
    s = torch.where(s == 0, torch.full_like(s, torch.finfo(x.dtype).tiny), s)
    q = torch.clamp(torch.round(x / s), -128, 127).to(torch.int8)
    return q, scale


def int8_dequant(c, x_scale, w_scale, bias=None, out_dtype=torch.bfloat16):
    """The chunked rescale of _int8_linear_prequant's int32 branch: per chunk of
    rows (<= 256 MB of fp32), C.float() * (w_scale * x_scale) -> out_dtype, then
    + bias (in out_dtype)."""
    m, n = c.shape
    ws = w_scale.reshape(-1).float()
    chunk = max(1, min(m, 256 * 1024 * 1024 // (n * 4)))
    parts = []
    for i in range(0, m, chunk):
        e = min(i + chunk, m)
        parts.append((c[i:e].float() * (ws * x_scale[i:e])).to(out_dtype))
    out = torch.cat(parts, dim=0)
    if bias is not None:
        out = out + bias.to(out_dtype)
    return out


def int8_linear(x, w_q, w_scale, bias=None, out_dtype=torch.bfloat16, act=None):
    """Per-token quant -> torch._int_mm(x8, W.t()) -> chunked rescale (+ GELU)."""
    q, xs = quantize_int8_rowwise(x)
    out = int8_dequant(torch._int_mm(q, w_q.t()), xs, w_scale, bias, out_dtype)
    return F.gelu(out, approximate="tanh") if act == "gelu_tanh" else out


def quantize_fp8_tensorwise(x):
    """Per-tensor e4m3 quant: s = max(amax/448, 1e-30) (fp32), q = e4m3(x / s),
    round-to-nearest-even, saturated to +-448."""
    s = torch.clamp(x.abs().amax().float() / _E4M3_MAX, min=1e-30)
    v = torch.clamp(x.float() / s, -_E4M3_MAX, _E4M3_MAX)
    return v.to(torch.float8_e4m3fn), s.reshape(1)


def scaled_mm_fp8(a, w, scale_a=None, scale_b=None, bias=None, out_dtype=torch.bfloat16,
                  act=None):
    """_mps_scaled_mm's decode route on CPU; `w` is the [N,K] weight (``other``
    of torch._scaled_mm is w.t())."""
    out = a.to(torch.bfloat16) @ w.to(torch.bfloat16).t()
    if scale_a is not None or scale_b is not None:
        acc = out.float()
        if scale_a is not None:
            acc = acc * scale_a.float()
        if scale_b is not None:
            acc = acc * scale_b.float()
        out = acc.to(out.dtype)
    if bias is not None:
        out = out.float() + bias.float()
    out = out.to(out_dtype)
    return F.gelu(out, approximate="tanh") if act == "gelu_tanh" else out


def fp8_linear(x, w, w_scale, bias=None, out_dtype=torch.bfloat16, act=None):
    """Per-tensor activation quant, then the decode route of scaled_mm."""
    q, s = quantize_fp8_tensorwise(x)
    return scaled_mm_fp8(q, w, s, w_scale, bias, out_dtype, act)


def w8a16_linear(x, w, w_scale=None, bias=None, act=None):
    """Decode the e4m3 weight to x's dtype, F.linear, then scale/bias/GELU."""
    out = F.linear(x, w.to(x.dtype))
    if w_scale is not None:
        out = (out.float() * w_scale.float()).to(x.dtype)
    if bias is not None:
        out = out + bias.to(x.dtype)
    return F.gelu(out, approximate="tanh") if act == "gelu_tanh" else out
