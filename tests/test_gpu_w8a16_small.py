"""GPU parity of the small-token W8A16 paths against the oracle
(decode W -> fp32 dot products, linear_fp8_w8a16.py:151-196 with the BASELINE
per-tensor scale and tanh-GELU; FP8 tolerances as in test_gpu_parity.py):

* M <= 32: the weight-streaming GEMV (TMA-fed shared-memory ring, warp
  m16n8k16 MMAs with the per-lane K permutation; 16- and 32-token fragments);
* 33 <= M <= 64: the tcgen05 streaming kernel (control case at the boundary).

Shapes exercise K tails (K % 64 != 0, K % 512 != 0), N not a multiple of the
32-row unit, fp16 activations and repeatability (fixed reduction orders).
"""
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"
FP8_RMS_TOL = 0.02


@pytest.fixture(autouse=True)
def _decode_in_kernel_routes(monkeypatch):
    """These kernels are the fallback of the planes route (test_gpu_w8a16_planes):
    they run when no workspace is given or no planes plan fits the shape, so the
    planes route and the planes GEMV are switched off here to keep them covered."""
    monkeypatch.setenv("B200Q_W8A16_PLANES", "0")
    monkeypatch.setenv("B200Q_W8A16_PGEMV", "0")


def _gen(seed):
    return torch.Generator().manual_seed(seed)


@pytest.mark.parametrize("M", [1, 2, 3, 16, 17, 32, 33])
@pytest.mark.parametrize("K,N", [(3072, 4096), (1040, 1000)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_w8a16_small_m(native, M, K, N, dtype):
    g = _gen(M * 7 + K)
    x = torch.randn(M, K, generator=g).to(dtype)
    w = (torch.randn(N, K, generator=g) * 0.02 / (0.08 / 448)).clamp(-448, 448).to(torch.float8_e4m3fn)
    ws = torch.tensor([0.08 / 448])
    b = (torch.randn(N, generator=g) * 0.01).to(dtype)
    ref = oracle.w8a16_linear(x, w, ws, b, "gelu_tanh", out_dtype="fp32")
    xd, wd, wsd, bd = x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV)
    out = native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh")
    assert out.dtype == dtype
    assert oracle.elementwise_ulp_ratio(out, ref) <= 1.0
    out32 = native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh", torch.float32)
    assert oracle.fp8_errors(out32, ref)[0] <= FP8_RMS_TOL
    assert torch.equal(out, out32.to(dtype))
    again = native.w8a16_linear(xd, wd, wsd, bd, "gelu_tanh")
    assert torch.equal(out, again)


def test_w8a16_small_m_strided_activation(native):
    g = _gen(5)
    M, K, N = 8, 2048, 640
    xf = torch.randn(M, K + 64, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 30).clamp(-448, 448).to(torch.float8_e4m3fn)
    ref = oracle.w8a16_linear(xf[:, 32:32 + K].contiguous(), w, None, None, out_dtype="fp32")
    out32 = native.w8a16_linear(xf.to(DEV)[:, 32:32 + K], w.to(DEV), None, None, None, torch.float32)
    assert oracle.fp8_errors(out32, ref)[0] <= FP8_RMS_TOL
