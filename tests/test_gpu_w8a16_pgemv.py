"""GPU parity of the planes GEMV (csrc/w8a16_planes.cuh, ``w8a16_pgemv_kernel``):
calls of up to 8 activation plane rows (M <= 4 bf16 tokens, M <= 2 fp16)
split the activations exactly into e4m3 planes (the planes pass) and multiply
the raw e4m3 weight stream with them on warp-level m16n8k32 e4m3 MMAs.

Against the oracle's decode-the-weight linear (linear_fp8_w8a16.py:151-196 with
the per-tensor scale and tanh-GELU): bf16/fp16 outputs within 1 ULP of the fp32
result, fp32 outputs within the FP8 RMS bound, bit-reproducible across calls,
with and without the programmatic launch dependency, and inside a CUDA graph.
Shapes cover every routed token count, K tails (K % 512 != 0, K % 64 !=
0), N tails (N % 32 != 0), the C2 projection shape, strided activations, edge
rows (zeros, huge and tiny magnitudes) and a non-finite row (NaN output row,
as in the planes route).
"""
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
def _pgemv_route(monkeypatch):
    monkeypatch.setenv("B200Q_W8A16_PGEMV", "1")


def _launches(native, fn):
    c0 = native.launch_count()
    out = fn()
    torch.cuda.synchronize()
    return out, native.launch_count() - c0


@pytest.mark.parametrize("M", [1, 2, 3, 4])
@pytest.mark.parametrize("K,N", [(3072, 12288), (1040, 1000), (5120, 5120), (4096, 3104)])
def test_pgemv_bf16(native, M, K, N):
    x, w, ws, b = _case(M, K, N, torch.bfloat16, M * 37 + K)
    ref = oracle.w8a16_linear(x, w, ws, b, "gelu_tanh", out_dtype="fp32")
    xd, wd, wsd, bd = x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV)
    out, launches = _launches(native, lambda: native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh"))
    assert launches == 2  # planes pass + planes GEMV
    assert out.dtype == torch.bfloat16
    assert oracle.elementwise_ulp_ratio(out, ref) <= 1.0
    out32 = native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh", torch.float32)
    assert oracle.fp8_errors(out32, ref)[0] <= FP8_RMS_TOL
    assert torch.equal(out, out32.to(torch.bfloat16))
    assert torch.equal(out, native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh"))


@pytest.mark.parametrize("M", [1, 2])
@pytest.mark.parametrize("K,N", [(3072, 4096), (1040, 1000)])
def test_pgemv_fp16(native, M, K, N):
    x, w, ws, b = _case(M, K, N, torch.float16, M * 41 + K)
    ref = oracle.w8a16_linear(x, w, ws, b, "gelu_tanh", out_dtype="fp32")
    xd, wd, wsd, bd = x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV)
    out, launches = _launches(native, lambda: native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh"))
    assert launches == 2
    assert out.dtype == torch.float16
    assert oracle.elementwise_ulp_ratio(out, ref) <= 1.0


def test_pgemv_boundary_takes_other_routes(native):
    """5 bf16 tokens (10 plane rows) and 3 fp16 tokens (9) leave the planes GEMV."""
    for M, dtype in ((5, torch.bfloat16), (3, torch.float16)):
        x, w, ws, b = _case(M, 1024, 512, dtype, 50 + M)
        ref = oracle.w8a16_linear(x, w, ws, b, None, out_dtype="fp32")
        out, launches = _launches(native, lambda: native.w8a16_linear(
            x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV), None))
        assert launches == 1  # the GEMV
        assert oracle.elementwise_ulp_ratio(out, ref) <= 1.0


def test_pgemv_matches_gemv(native, monkeypatch):
    """The planes GEMV and the decode-in-kernel GEMV agree within the oracle's bounds."""
    M, K, N = 4, 3072, 2048
    x, w, ws, b = _case(M, K, N, torch.bfloat16, 9)
    xd, wd, wsd, bd = x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV)
    a = native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh", torch.float32)
    monkeypatch.setenv("B200Q_W8A16_PGEMV", "0")
    c, launches = _launches(native, lambda: native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh", torch.float32))
    assert launches == 1
    ref = oracle.w8a16_linear(x, w, ws, b, "gelu_tanh", out_dtype="fp32")
    assert oracle.fp8_errors(a, ref)[0] <= 1e-5
    assert oracle.fp8_errors(c, ref)[0] <= 1e-5


def test_pgemv_edge_rows(native):
    """Zero rows, rows far below the weight scale, a huge outlier, a row 1e20
    up, a half-zero row and a subnormal-range row (two calls of 4 and 2 tokens)."""
    K, N = 2048, 640
    x, w, ws, b = _case(6, K, N, torch.bfloat16, 3, outliers=False)
    x[0] = 0
    x[1] *= 1e-30
    x[2, 5] = 3.0e4
    x[3] *= 1e20
    x[4, :1000] = 0
    x[5] = (torch.randn(K) * 1e-38).to(torch.bfloat16)
    ref = oracle.w8a16_linear(x, w, None, None, None, out_dtype="fp32")
    wd = w.to(DEV)
    out32 = torch.cat([native.w8a16_linear(x[r0:r1].to(DEV), wd, None, None, None,
                                           torch.float32).cpu() for r0, r1 in ((0, 4), (4, 6))])
    for r in range(5):  # 2^-12 of the row's largest output: 16x under a bf16 ULP
        d = (out32[r].double() - ref[r].double()).abs().max().item()
        scale = max(ref[r].double().abs().max().item(), 1e-300)
        assert d <= scale * 2 ** -12, (r, d, scale)
    assert torch.equal(out32[0], torch.zeros(N))
    assert torch.isfinite(out32[5]).all()


def test_pgemv_nonfinite_row(native):
    """A row holding inf/NaN gives a NaN output row; other rows are unaffected."""
    M, K, N = 3, 1024, 256
    x, w, ws, b = _case(M, K, N, torch.bfloat16, 4, outliers=False)
    x[1, 7] = float("inf")
    out = native.w8a16_linear(x.to(DEV), w.to(DEV), None, None, None, torch.float32).cpu()
    assert torch.isnan(out[1]).all()
    ref = oracle.w8a16_linear(x[[0, 2]], w, None, None, None, out_dtype="fp32")
    assert oracle.fp8_errors(out[[0, 2]], ref)[0] <= 1e-5


def _wide_row(K, g):
    """A bf16 row whose magnitudes span 2^20 (exponents uniform in [-10, 10])."""
    e = torch.rand(K, generator=g) * 20 - 10
    return (torch.randn(K, generator=g) * torch.exp2(e)).to(torch.bfloat16)


def test_pgemv_wide_dynamic_range_rows(native):
    """Rows spanning 2^20: elements more than ~2^13 below their row maximum lose
    bits under e4m3's subnormal spacing (below 2^-21 of the maximum each); the
    fp32 output stays within 2% of the row's RMS, the FP8 routes' bound."""
    M, K, N = 3, 2048, 1024
    x, w, ws, b = _case(M, K, N, torch.bfloat16, 21, outliers=False)
    g = torch.Generator().manual_seed(22)
    for r in range(M):
        x[r] = _wide_row(K, g)
    ref = oracle.w8a16_linear(x, w, ws, b, None, out_dtype="fp32")
    out32 = native.w8a16_linear(x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV), None,
                                torch.float32).cpu()
    for r in range(M):
        assert oracle.fp8_errors(out32[r], ref[r])[0] <= FP8_RMS_TOL


def test_nonfinite_row_planes_vs_decode_route(native, monkeypatch):
    """With an inf in a row the planes GEMV returns a NaN row, while the
    decode-in-kernel GEMV (the reference's decode-then-matmul arithmetic)
    propagates the infinity: every output of the row is +-inf with the sign of
    the weight at that K (all nonzero here).  Other rows match the oracle."""
    M, K, N = 3, 1024, 256
    x, w, ws, b = _case(M, K, N, torch.bfloat16, 23, outliers=False)
    x[1, 7] = float("inf")
    xd, wd = x.to(DEV), w.to(DEV)
    planes = native.w8a16_linear(xd, wd, None, None, None, torch.float32).cpu()
    monkeypatch.setenv("B200Q_W8A16_PGEMV", "0")
    monkeypatch.setenv("B200Q_W8A16_PLANES", "0")
    dec = native.w8a16_linear(xd, wd, None, None, None, torch.float32).cpu()
    assert torch.isnan(planes[1]).all()
    col = w[:, 7].float()
    assert (col != 0).all()
    inf = torch.full_like(col, float("inf"))
    assert torch.equal(dec[1], torch.where(col > 0, inf, -inf))
    ref = oracle.w8a16_linear(x[[0, 2]], w, None, None, None, out_dtype="fp32")
    assert oracle.fp8_errors(planes[[0, 2]], ref)[0] <= 1e-5
    assert oracle.fp8_errors(dec[[0, 2]], ref)[0] <= 1e-4


def test_pgemv_strided_activation(native):
    M, K, N = 4, 2048, 640
    g = torch.Generator().manual_seed(5)
    xf = torch.randn(M, K + 64, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 30).clamp(-448, 448).to(torch.float8_e4m3fn)
    ref = oracle.w8a16_linear(xf[:, 32:32 + K].contiguous(), w, None, None, out_dtype="fp32")
    out32 = native.w8a16_linear(xf.to(DEV)[:, 32:32 + K], w.to(DEV), None, None, None, torch.float32)
    assert oracle.fp8_errors(out32, ref)[0] <= 1e-5


def test_pgemv_without_pdl(native, monkeypatch):
    """Launched without the programmatic dependency the GEMV gives the same bits."""
    M, K, N = 2, 3072, 3072
    x, w, ws, b = _case(M, K, N, torch.bfloat16, 11)
    xd, wd, wsd, bd = x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV)
    a = native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh")
    monkeypatch.setenv("B200Q_PDL", "0")
    c = native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh")
    assert torch.equal(a, c)


def test_pgemv_in_cuda_graph(native):
    """Captured in a CUDA graph (the PDL edges are captured too) the replays give
    the eager result; every call's planes pass waits for the GEMV before it."""
    M, K, N = 1, 3072, 12288
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
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, eager)
    assert native.device_status() == 0
