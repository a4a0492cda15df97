"""FP16-output INT8 epilogue (the Wan 14B projections' format adapter) on the GPU.

Mirrors the reference's tests/test_wan_fp16.py:30-59 and
tests/test_minimax_vae_int8.py:55-75: inputs are views with nonzero storage
offsets, row scales include 0, 1e-10, 1e-7, 0.01 and 1, and the fp16 result of
the Wan hook must equal both the general fp16 route and the oracle's two-rounding
epilogue bit for bit; the reference's argument checks raise before any launch.
"""
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture
def seam(monkeypatch, native):
    from b200q._patches import int8_linear_kernel as k
    for flag in ("ASFP8_DIT_EXT", "ASFP8_WAN_FAST", "ASFP8_WAN_EXACT", "ASFP8_WAN_FP16_GEMM"):
        monkeypatch.setenv(flag, "1")
    monkeypatch.setattr(k, "_kernel", k._NativeInt8Kernel())
    return k


@pytest.mark.parametrize("rows,width,inner", [(1, 5120, 5120), (65, 5120, 5120),
                                              (257, 13824, 5120), (257, 5120, 13824)])
@pytest.mark.parametrize("with_bias", [False, True])
def test_wan_fp16_scaled_integer_output(seam, monkeypatch, rows, width, inner, with_bias):
    from b200q._patches import wan_fp16
    g = torch.Generator().manual_seed(rows)
    x = torch.randint(-127, 128, (rows + 1, inner), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (width + 1, inner), generator=g, dtype=torch.int8)
    rs = torch.rand(rows + 1, 1, generator=g) * 0.02
    cs = torch.rand(width + 1, generator=g) * 0.03
    rs[1] = 0
    if rows >= 65:
        rs[2:6, 0] = torch.tensor([1e-10, 1e-7, 0.01, 1.0])
    bias = torch.randn(width, generator=g).to(torch.float16) if with_bias else None
    xd, wd, rsd, csd = x.to(DEV)[1:], w.to(DEV)[1:], rs.to(DEV)[1:], cs.to(DEV)[1:]
    bd = torch.nn.Parameter(bias.to(DEV), requires_grad=False) if with_bias else None
    shape = (1, rows, inner)
    with torch.inference_mode():
        monkeypatch.setenv("ASFP8_WAN_EXACT", "0")
        general = seam._int8_linear_prequant(xd, rsd, wd, csd, bd, torch.float16, shape)
        monkeypatch.setenv("ASFP8_WAN_EXACT", "1")
        before = wan_fp16.state.calls
        got = seam._int8_linear_prequant(xd, rsd, wd, csd, bd, torch.float16, shape)
        assert wan_fp16.state.calls == before + 1 and wan_fp16.state.disabled is None
        assert got.shape == (1, rows, width) and got.dtype == torch.float16
        assert torch.equal(got.view(torch.int16), general.view(torch.int16))
        ref = oracle.int8_dequant_epilogue(oracle.int_mm(x[1:], w[1:].t()), rs[1:], cs[1:], bias,
                                           torch.float16)
        assert torch.equal(got.reshape(rows, width).cpu().view(torch.int16), ref.view(torch.int16))
        monkeypatch.setenv("ASFP8_WAN_FP16_GEMM", "0")
        assert wan_fp16.maybe_prequant(seam._kernel, xd, rsd, wd, csd, bd, shape) is None


def test_half_epilogue_invalid_arguments_raise(seam):
    k = seam._kernel
    a = torch.zeros(3, 256, device=DEV, dtype=torch.int8)
    b = torch.zeros(8, 256, device=DEV, dtype=torch.int8)
    r, c = torch.ones(3, device=DEV), torch.ones(8, device=DEV)
    assert k.i8_matmul2d_nt_fused_cs_half(a, b, r, c).dtype == torch.float16
    for args in ((a, b, r.cpu(), c), (a, b, r, c[:1]), (a[:, ::2], b, r, c), (a[:0], b, r[:0], c)):
        with pytest.raises(RuntimeError):
            k.i8_matmul2d_nt_fused_cs_half(*args)
