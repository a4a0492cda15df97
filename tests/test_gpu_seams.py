"""GPU tests through the reference's own entry points (the seams): each route's
``install()`` runs on the B200 and the caller's own call — ``torch._scaled_mm``,
comfy's ``Linear.forward_comfy_cast_weights``, ``F.linear`` with FP8 operands,
``torch._int_mm`` — is checked against the CPU oracle.

Patterns follow the reference's tests: tests/test_scaled_mm_fp8.py:57-80 (per-row
and per-column scales, bias, bf16/f32 out, ``other = b.t()`` column-major),
tests/test_linear_fp8_w8a16.py:159-211 (a fake comfy Linear with e4m3 weights,
the one-time self-check and the fall-back chain), _patches/int_mm_mps.py:54-110
(the corner-case canary, then exact int32 products).  Every test puts the
patched torch/comfy attributes back when it ends.

Tolerances: FP8 outputs within 1 bf16 ULP of the oracle's fp32 value (plus 0.1%
RMS slack near zero) and within 2% of its RMS for fp32 outputs; int32 exact.
"""
import sys
from types import ModuleType, SimpleNamespace

import pytest
import torch
import torch.nn.functional as F

from b200q._patches import int_mm, linear_fp8, linear_fp8_w8a16, scaled_mm_fp8
from oracle import oracle

pytestmark = pytest.mark.gpu

FP8_RMS_TOL = 0.02
DEV = "cuda"


def _gen(seed):
    return torch.Generator().manual_seed(seed)


def _e4m3(g, *shape, scale=0.3):
    return (torch.randn(*shape, generator=g) * scale).to(torch.float8_e4m3fn)


# ----------------------------------------------------------------------------- torch._scaled_mm
@pytest.fixture
def scaled_mm_installed(native, monkeypatch):
    monkeypatch.setenv("ASFP8_FP8_EXT", "1")
    stock = torch._scaled_mm
    monkeypatch.setattr(scaled_mm_fp8, "_installed", False)
    scaled_mm_fp8.install()
    assert scaled_mm_fp8._installed and torch._scaled_mm is scaled_mm_fp8._cuda_scaled_mm
    yield stock
    torch._scaled_mm = stock


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("M,K,N", [(64, 128, 32), (300, 1024, 384), (1024, 3072, 3072)])
def test_scaled_mm_rowcol_scales_bias(scaled_mm_installed, M, K, N, out_dtype):
    g = _gen(57)
    a, b = _e4m3(g, M, K), _e4m3(g, N, K)          # b [N,K]: other = b.t() is column-major
    sa = torch.rand(M, 1, generator=g) + 0.5
    sb = torch.rand(1, N, generator=g) + 0.5
    bias = (torch.randn(N, generator=g)).to(torch.bfloat16)
    out = torch._scaled_mm(a.to(DEV), b.to(DEV).t(), out_dtype=out_dtype, scale_a=sa.to(DEV),
                           scale_b=sb.to(DEV), bias=bias.to(DEV))
    assert out.dtype == out_dtype and tuple(out.shape) == (M, N)
    ref = oracle.scaled_mm_fp8(a, b, sa, sb, None, bias, None)
    if out_dtype == torch.float32:
        assert oracle.fp8_errors(out, ref)[0] <= FP8_RMS_TOL
    else:
        assert oracle.elementwise_ulp_ratio(out, ref) <= 1.0


def test_scaled_mm_tensorwise_scales_scale_result(scaled_mm_installed):
    g = _gen(58)
    M, K, N = 257, 2048, 640
    a, b = _e4m3(g, M, K), _e4m3(g, N, K)
    sa, sb, sr = torch.tensor(0.02), torch.tensor(0.05), torch.tensor(2.0)
    bias = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16)
    out = torch._scaled_mm(a.to(DEV), b.to(DEV).t(), scale_a=sa.to(DEV), scale_b=sb.to(DEV),
                           bias=bias.to(DEV), scale_result=sr.to(DEV), out_dtype=torch.bfloat16)
    ref = oracle.scaled_mm_fp8(a, b, sa.reshape(1), sb.reshape(1), sr.reshape(1), bias, None)
    assert oracle.elementwise_ulp_ratio(out, ref) <= 1.0


def test_scaled_mm_row_major_other(scaled_mm_installed):
    """``other`` given as a row-major [K,N] tensor (not the transpose view of a
    stored weight): same values as the column-major call."""
    g = _gen(59)
    M, K, N = 200, 512, 256
    a, b = _e4m3(g, M, K), _e4m3(g, N, K)
    sa, sb = torch.tensor(0.5), torch.tensor(0.25)
    other_rm = b.t().contiguous().to(DEV)          # [K,N], stride (N, 1)
    assert other_rm.stride() == (N, 1)
    out = torch._scaled_mm(a.to(DEV), other_rm, scale_a=sa.to(DEV), scale_b=sb.to(DEV),
                           out_dtype=torch.bfloat16)
    out_cm = torch._scaled_mm(a.to(DEV), b.to(DEV).t(), scale_a=sa.to(DEV), scale_b=sb.to(DEV),
                              out_dtype=torch.bfloat16)
    assert torch.equal(out, out_cm)
    ref = oracle.scaled_mm_fp8(a, b, sa.reshape(1), sb.reshape(1), None, None, None)
    assert oracle.elementwise_ulp_ratio(out, ref) <= 1.0
    # the K-major copy is made once per weight: a second call reuses it, an
    # in-place update of the weight makes a fresh one
    from b200q._patches import scaled_mm_fp8 as seam
    copy1 = seam._k_major_weight(other_rm)
    again = torch._scaled_mm(a.to(DEV), other_rm, scale_a=sa.to(DEV), scale_b=sb.to(DEV),
                             out_dtype=torch.bfloat16)
    assert torch.equal(again, out) and seam._k_major_weight(other_rm) is copy1
    other_rm.view(torch.uint8).add_(0)  # bumps the (shared) version counter
    assert seam._k_major_weight(other_rm) is not copy1


def test_scaled_mm_passes_through_what_it_does_not_own(scaled_mm_installed):
    """e5m2 operands and bf16 operands go to the stock torch._scaled_mm."""
    stock = scaled_mm_installed
    g = _gen(60)
    a = (torch.randn(64, 128, generator=g) * 0.3).to(torch.float8_e5m2).to(DEV)
    b = _e4m3(g, 32, 128).to(DEV)
    one = torch.tensor(1.0, device=DEV)
    try:
        want = stock(a, b.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
    except RuntimeError:
        pytest.skip("stock torch._scaled_mm has no e5m2 x e4m3 kernel here")
    got = torch._scaled_mm(a, b.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
    assert torch.equal(got, want)


# ----------------------------------------------------------------------------- torch._int_mm
@pytest.fixture
def int_mm_installed(native, monkeypatch):
    monkeypatch.setenv("ASFP8_INT8_EXT", "1")
    stock = torch._int_mm
    monkeypatch.setattr(int_mm, "_installed", False)
    int_mm.install()  # runs the corner-case canary on the GPU first
    assert int_mm._installed and torch._int_mm is int_mm._int_mm_cuda
    yield stock
    torch._int_mm = stock


@pytest.mark.parametrize("M,K,N", [(3, 129, 5), (17, 4096, 32), (130, 512, 256),
                                   (4096, 3072, 3072)])
@pytest.mark.parametrize("b_layout", ["weight_t", "row_major"])
def test_int_mm_after_install_exact(int_mm_installed, M, K, N, b_layout):
    g = _gen(61)
    a = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int8)
    w = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int8)
    a[:, 0], w[:, 0] = -128, -128
    b = w.to(DEV).t() if b_layout == "weight_t" else w.t().contiguous().to(DEV)
    out = torch._int_mm(a.to(DEV), b)
    assert out.dtype == torch.int32
    assert torch.equal(out.cpu(), oracle.int_mm(a, w.t()))


def test_int_mm_cpu_calls_keep_the_stock_function(int_mm_installed):
    a = torch.randint(-128, 128, (32, 64), dtype=torch.int8)
    b = torch.randint(-128, 128, (64, 16), dtype=torch.int8)
    assert torch.equal(torch._int_mm(a, b), int_mm_installed(a, b))


# ----------------------------------------------------------------------------- F.linear
@pytest.fixture
def linear_installed(native, monkeypatch):
    monkeypatch.setenv("ASFP8_FP8_EXT", "1")
    stock = F.linear
    monkeypatch.setattr(linear_fp8, "_installed", False)
    linear_fp8.install()
    assert linear_fp8._installed and F.linear is linear_fp8._patched_linear
    yield stock
    F.linear = stock
    torch.nn.functional.linear = stock


@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(7, 512), (3, 33, 1024)])
def test_f_linear_e4m3_weight(linear_installed, xdt, shape):
    g = _gen(62)
    K = shape[-1]
    x = torch.randn(*shape, generator=g).to(xdt)
    w = _e4m3(g, 384, K)
    b = (torch.randn(384, generator=g) * 0.1).to(xdt)
    out = F.linear(x.to(DEV), w.to(DEV), b.to(DEV))
    assert out.dtype == xdt and tuple(out.shape) == (*shape[:-1], 384)
    ref = oracle.w8a16_linear(x.reshape(-1, K), w, None, b, None, "fp32")
    assert oracle.elementwise_ulp_ratio(out.reshape(-1, 384), ref) <= 1.0


def test_f_linear_fp8_input_and_weight_decoded(linear_installed):
    """Both operands FP8: decoded (exactly) to bf16 and run by the stock F.linear."""
    stock = linear_installed
    g = _gen(63)
    x, w = _e4m3(g, 40, 256), _e4m3(g, 96, 256)
    out = F.linear(x.to(DEV), w.to(DEV))
    want = stock(x.to(torch.bfloat16).to(DEV), w.to(torch.bfloat16).to(DEV))
    assert out.dtype == torch.bfloat16 and torch.equal(out, want)


def test_f_linear_fp32_input_e4m3_weight(linear_installed):
    stock = linear_installed
    g = _gen(64)
    x, w = torch.randn(16, 128, generator=g), _e4m3(g, 64, 128)
    out = F.linear(x.to(DEV), w.to(DEV))
    want = stock(x.to(DEV), w.to(torch.float32).to(DEV))
    assert out.dtype == torch.float32 and torch.equal(out, want)


def test_f_linear_plain_calls_untouched(linear_installed):
    stock = linear_installed
    x, w = torch.randn(4, 64, device=DEV), torch.randn(8, 64, device=DEV)
    assert torch.equal(F.linear(x, w), stock(x, w))


# ----------------------------------------------------------------------------- comfy Linear
def _decode_forward(module, input):
    """comfy's own forward for an e4m3 layer: decode the weight, F.linear in
    float32, + bias (the reference tests' decode_forward)."""
    wb = module.weight.to(torch.float32)
    out = input.float() @ wb.t()
    if getattr(module, "scale_weight", None) is not None:
        out = out * module.scale_weight.float()
    if module.bias is not None:
        out = out + module.bias.float()
    return out.to(input.dtype)


@pytest.fixture
def comfy_linear(native, monkeypatch):
    comfy = ModuleType("comfy")
    ops = ModuleType("comfy.ops")
    comfy.ops = ops
    calls = []

    class Linear:
        def forward_comfy_cast_weights(self, input):
            calls.append(tuple(input.shape))
            return _decode_forward(self, input)

    ops.disable_weight_init = SimpleNamespace(Linear=Linear)
    monkeypatch.setitem(sys.modules, "comfy", comfy)
    monkeypatch.setitem(sys.modules, "comfy.ops", ops)
    monkeypatch.setenv("ASFP8_FP8_SGEMM", "1")
    monkeypatch.setattr(linear_fp8_w8a16, "_installed", False)
    monkeypatch.setattr(linear_fp8_w8a16, "_self_checked", False)
    monkeypatch.setattr(linear_fp8_w8a16, "_kernel", None)
    monkeypatch.setattr(linear_fp8_w8a16, "_orig_forward", None)
    linear_fp8_w8a16.install()
    assert linear_fp8_w8a16._installed
    assert Linear.forward_comfy_cast_weights is linear_fp8_w8a16._patched_forward
    yield Linear, calls


def _layer(Linear, g, N, K, scale=None, bias=True):
    m = Linear()
    m.weight = _e4m3(g, N, K, scale=60.0).to(DEV)
    m.bias = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16).to(DEV) if bias else None
    m.scale_weight = torch.tensor(scale).to(DEV) if scale is not None else None
    m.weight_function, m.bias_function = [], []
    return m


@pytest.mark.parametrize("M,K,N", [(64, 512, 384), (257, 384, 512), (1, 512, 512),
                                   (3000, 512, 384)])
def test_comfy_linear_w8a16_parity(comfy_linear, M, K, N):
    Linear, calls = comfy_linear
    g = _gen(65)
    m = _layer(Linear, g, N, K, scale=0.004)
    x = (torch.randn(M, K, generator=g) * 0.3).to(torch.bfloat16)
    out = Linear.forward_comfy_cast_weights(m, x.to(DEV))
    assert linear_fp8_w8a16._kernel is True and calls == []   # the kernel answered
    ref = oracle.w8a16_linear(x, m.weight.cpu(), m.scale_weight.reshape(1).cpu(), m.bias.cpu(),
                              None, "fp32")
    assert out.dtype == torch.bfloat16
    assert oracle.elementwise_ulp_ratio(out, ref) <= 1.0


def test_comfy_linear_3d_fp16_and_ragged_k(comfy_linear):
    Linear, calls = comfy_linear
    g = _gen(66)
    m = _layer(Linear, g, 384, 512)
    x3 = (torch.randn(2, 33, 512, generator=g) * 0.3).to(torch.float16)
    out = Linear.forward_comfy_cast_weights(m, x3.to(DEV))
    assert out.dtype == torch.float16 and tuple(out.shape) == (2, 33, 384)
    ref = oracle.w8a16_linear(x3.reshape(-1, 512), m.weight.cpu(), None, m.bias.cpu(), None, "fp32")
    assert oracle.elementwise_ulp_ratio(out.reshape(-1, 384), ref) <= 1.0
    m2 = _layer(Linear, g, 160, 264, bias=False)   # K = 264: not a multiple of 16
    x = (torch.randn(40, 264, generator=g) * 0.3).to(torch.bfloat16)
    out = Linear.forward_comfy_cast_weights(m2, x.to(DEV))
    ref = oracle.w8a16_linear(x, m2.weight.cpu(), None, None, None, "fp32")
    assert oracle.elementwise_ulp_ratio(out, ref) <= 1.0
    assert calls == []


def test_comfy_linear_ineligible_layers_use_comfy(comfy_linear):
    Linear, calls = comfy_linear
    g = _gen(67)
    m = _layer(Linear, g, 128, 256)
    m.weight_function = [lambda w: w]            # a LoRA-patched layer
    x = torch.randn(8, 256, generator=g).to(torch.bfloat16).to(DEV)
    Linear.forward_comfy_cast_weights(m, x)
    m2 = _layer(Linear, g, 128, 256)
    Linear.forward_comfy_cast_weights(m2, x.float())   # fp32 activations
    assert calls == [(8, 256), (8, 256)]


def test_comfy_linear_failed_self_check_falls_back(comfy_linear, monkeypatch):
    """A self-check that disagrees with the decode path latches the route off:
    this call and every later one run comfy's own forward."""
    Linear, calls = comfy_linear
    g = _gen(68)
    m = _layer(Linear, g, 256, 512)
    real = linear_fp8_w8a16.decode_fp8
    monkeypatch.setattr(linear_fp8_w8a16, "decode_fp8",
                        lambda t, dt=torch.float32: real(t, dt) * 2.0)  # a wrong reference
    x = torch.randn(16, 512, generator=g).to(torch.bfloat16).to(DEV)
    out = Linear.forward_comfy_cast_weights(m, x)
    assert linear_fp8_w8a16._kernel is False and calls == [(16, 512)]
    assert torch.equal(out, _decode_forward(m, x))
    Linear.forward_comfy_cast_weights(m, x)
    assert calls == [(16, 512), (16, 512)]


def test_comfy_linear_self_check_error_falls_back(comfy_linear, monkeypatch):
    Linear, calls = comfy_linear
    g = _gen(69)
    m = _layer(Linear, g, 256, 512)

    def boom(*a, **k):
        raise RuntimeError("decode unavailable")

    monkeypatch.setattr(linear_fp8_w8a16, "decode_fp8", boom)
    x = torch.randn(4, 512, generator=g).to(torch.bfloat16).to(DEV)
    Linear.forward_comfy_cast_weights(m, x)
    assert linear_fp8_w8a16._kernel is False and calls == [(4, 512)]
