"""GPU parity of the small-token W8A16 planes route (csrc/w8a16_planes.cuh):
activations split exactly into e4m3 planes, raw e4m3 weight tiles on
tcgen05 kind::f8f6f4, split-K across a CTA cluster with a fixed-order
distributed-shared-memory reduction.

Against the oracle's decode-the-weight linear (linear_fp8_w8a16.py:151-196 with
the per-tensor scale and tanh-GELU): bf16/fp16 outputs within 1 ULP of the fp32
result, fp32 outputs within the FP8 RMS bound, bit-reproducible across calls
and across cluster sizes' own reruns.  Shapes cover every plane-tile width
(bt = 16/32/64/128 tokens), several token tiles (M up to 256), K tails (K % 128 != 0), N tails (N % 128 != 0),
Wan/Flux projection shapes and strided activations.
"""
import os

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"
FP8_RMS_TOL = 0.02


def _case(M, K, N, dtype, seed, outliers=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    if outliers:
        x[:, torch.randperm(K, generator=g)[:8]] *= 20.0
    x = x.to(dtype)
    w = (torch.randn(N, K, generator=g) * 0.02 / (0.08 / 448)).clamp(-448, 448).to(torch.float8_e4m3fn)
    ws = torch.tensor([0.08 / 448])
    b = (torch.randn(N, generator=g) * 0.01).to(dtype)
    return x, w, ws, b


@pytest.fixture(autouse=True)
def _planes_route(monkeypatch):
    """Every eligible call takes the planes route here (by default it runs only
    for the token counts where it measured fastest); the planes GEMV, which takes
    calls of up to 16 plane rows before it, is switched off
    (test_gpu_w8a16_pgemv covers it)."""
    monkeypatch.setenv("B200Q_W8A16_PLANES", "1")
    monkeypatch.setenv("B200Q_W8A16_PGEMV", "0")


def _launches(native, fn):
    c0 = native.launch_count()
    out = fn()
    torch.cuda.synchronize()
    return out, native.launch_count() - c0


@pytest.mark.parametrize("M", [1, 2, 15, 16, 17, 31, 32, 33, 63, 64, 65, 100, 128, 129, 200, 256])
@pytest.mark.parametrize("K,N", [(3072, 12288), (1040, 1000), (5120, 5120)])
def test_planes_bf16(native, M, K, N):
    x, w, ws, b = _case(M, K, N, torch.bfloat16, M * 31 + K)
    ref = oracle.w8a16_linear(x, w, ws, b, "gelu_tanh", out_dtype="fp32")
    xd, wd, wsd, bd = x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV)
    out, launches = _launches(native, lambda: native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh"))
    assert launches == 2  # planes pass + GEMM
    assert oracle.elementwise_ulp_ratio(out, ref) <= 1.0
    out32 = native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh", torch.float32)
    assert oracle.fp8_errors(out32, ref)[0] <= FP8_RMS_TOL
    assert torch.equal(out, out32.to(torch.bfloat16))
    assert torch.equal(out, native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh"))
    assert native.device_status() == 0


@pytest.mark.parametrize("M", [1, 16, 17, 33, 64, 65, 130, 256])
@pytest.mark.parametrize("K,N", [(3072, 4096), (1040, 1000)])
def test_planes_fp16(native, M, K, N):
    x, w, ws, b = _case(M, K, N, torch.float16, M * 17 + K)
    ref = oracle.w8a16_linear(x, w, ws, b, "gelu_tanh", out_dtype="fp32")
    xd, wd, wsd, bd = x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV)
    out, launches = _launches(native, lambda: native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh"))
    assert launches == 2
    assert out.dtype == torch.float16
    assert oracle.elementwise_ulp_ratio(out, ref) <= 1.0
    out32 = native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh", torch.float32)
    assert oracle.fp8_errors(out32, ref)[0] <= FP8_RMS_TOL


@pytest.mark.parametrize("splits", ["1", "2", "3", "5", "8"])
def test_planes_cluster_sizes(native, monkeypatch, splits):
    """Every cluster size gives the same bf16 result within 1 ULP of the oracle;
    each is bit-reproducible run to run (fixed rank order)."""
    M, K, N = 20, 3072, 3072
    x, w, ws, b = _case(M, K, N, torch.bfloat16, 7)
    ref = oracle.w8a16_linear(x, w, ws, None, None, out_dtype="fp32")
    monkeypatch.setenv("B200Q_W8A16_PLANES_SPLITS", splits)
    xd, wd, wsd = x.to(DEV), w.to(DEV), ws.to(DEV)
    out, launches = _launches(native, lambda: native.w8a16_linear(xd, wd, wsd, None, None))
    assert launches == 2
    assert oracle.elementwise_ulp_ratio(out, ref) <= 1.0
    assert torch.equal(out, native.w8a16_linear(xd, wd, wsd, None, None))


def test_planes_edge_rows(native):
    """Zero rows, rows far below the weight scale, a row with a huge outlier
    (planes keep the small elements through their own exponents), and
    subnormal-range rows."""
    M, K, N = 6, 2048, 640
    x, w, ws, b = _case(M, K, N, torch.bfloat16, 3, outliers=False)
    x[0] = 0
    x[1] *= 1e-30
    x[2, 5] = 3.0e4
    x[3] *= 1e20
    x[4, :1000] = 0
    x[5] = (torch.randn(K) * 1e-38).to(torch.bfloat16)
    ref = oracle.w8a16_linear(x, w, None, None, None, out_dtype="fp32")
    out32 = native.w8a16_linear(x.to(DEV), w.to(DEV), None, None, None, torch.float32).cpu()
    for r in range(5):  # 2^-12 of the row's largest output: 16x under a bf16 ULP
        d = (out32[r].double() - ref[r].double()).abs().max().item()
        scale = max(ref[r].double().abs().max().item(), 1e-300)
        assert d <= scale * 2 ** -12, (r, d, scale)
    assert torch.equal(out32[0], torch.zeros(N))
    # Row 5 lives in bf16's subnormal range; its products fall below fp32's normal
    # range inside the accumulators, so only finiteness is asserted.
    assert torch.isfinite(out32[5]).all()


def test_planes_nonfinite_row(native):
    """A row holding inf/NaN gives a NaN output row; other rows are unaffected."""
    M, K, N = 3, 1024, 256
    x, w, ws, b = _case(M, K, N, torch.bfloat16, 4, outliers=False)
    x[1, 7] = float("inf")
    out = native.w8a16_linear(x.to(DEV), w.to(DEV), None, None, None, torch.float32).cpu()
    assert torch.isnan(out[1]).all()
    ref = oracle.w8a16_linear(x[[0, 2]], w, None, None, None, out_dtype="fp32")
    assert oracle.fp8_errors(out[[0, 2]], ref)[0] <= 1e-5


def test_planes_wide_dynamic_range_rows(native):
    """Rows spanning 2^20 (exponents uniform in [-10, 10]): elements more than
    ~2^13 below their row maximum lose bits under e4m3's subnormal spacing (below
    2^-21 of the maximum each); the fp32 output stays within 2% of each row's
    RMS, the FP8 routes' bound."""
    M, K, N = 20, 2048, 1024
    x, w, ws, b = _case(M, K, N, torch.bfloat16, 21, outliers=False)
    g = torch.Generator().manual_seed(22)
    for r in range(M):
        e = torch.rand(K, generator=g) * 20 - 10
        x[r] = (torch.randn(K, generator=g) * torch.exp2(e)).to(torch.bfloat16)
    ref = oracle.w8a16_linear(x, w, ws, b, None, out_dtype="fp32")
    out32 = native.w8a16_linear(x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV), None,
                                torch.float32).cpu()
    for r in range(M):
        assert oracle.fp8_errors(out32[r], ref[r])[0] <= FP8_RMS_TOL


def test_planes_strided_activation(native):
    M, K, N = 8, 2048, 640
    g = torch.Generator().manual_seed(5)
    xf = torch.randn(M, K + 64, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 30).clamp(-448, 448).to(torch.float8_e4m3fn)
    ref = oracle.w8a16_linear(xf[:, 32:32 + K].contiguous(), w, None, None, out_dtype="fp32")
    out32 = native.w8a16_linear(xf.to(DEV)[:, 32:32 + K], w.to(DEV), None, None, None, torch.float32)
    assert oracle.fp8_errors(out32, ref)[0] <= 1e-5


def test_planes_matches_previous_routes(native, monkeypatch):
    """The planes route and the decode-in-kernel routes agree within 1 bf16 ULP."""
    M, K, N = 24, 3072, 2048
    x, w, ws, b = _case(M, K, N, torch.bfloat16, 9)
    xd, wd, wsd, bd = x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV)
    a = native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh", torch.float32)
    monkeypatch.setenv("B200Q_W8A16_PLANES", "0")
    c, launches = _launches(native, lambda: native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh", torch.float32))
    assert launches == 1  # the GEMV
    ref = oracle.w8a16_linear(x, w, ws, b, "gelu_tanh", out_dtype="fp32")
    assert oracle.fp8_errors(a, ref)[0] <= 1e-5
    assert oracle.fp8_errors(c, ref)[0] <= 1e-3


def test_planes_without_pdl(native, monkeypatch):
    """Launched without the programmatic dependency the GEMM gives the same bits."""
    M, K, N = 40, 3072, 3072
    x, w, ws, b = _case(M, K, N, torch.bfloat16, 11)
    xd, wd, wsd, bd = x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV)
    a = native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh")
    monkeypatch.setenv("B200Q_PDL", "0")
    c = native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh")
    assert torch.equal(a, c)


def test_planes_in_cuda_graph(native):
    """Captured in a CUDA graph (the PDL edge is captured too) the replay gives
    the eager result."""
    M, K, N = 16, 3072, 12288
    x, w, ws, b = _case(M, K, N, torch.bfloat16, 12)
    xd, wd, wsd, bd = x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV)
    eager = native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh")
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        outs = [native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh") for _ in range(3)]
    g.replay()
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, eager)
    assert native.device_status() == 0
