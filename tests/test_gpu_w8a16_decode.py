"""W8A16 at large M: the decoded-weight route (FP8 weight decoded once to the
activation's 16-bit type, then the tcgen05 tile kernels as kind::f16) against
the fp32 oracle and against the weight-stationary in-kernel-conversion route on
the same inputs.  Tolerances are the other W8A16 tests': 16-bit outputs within
1 ULP of the fp32 oracle value, fp32 outputs within 2% of the reference RMS.
The in-kernel route is selected by passing a workspace just below the decode
route's requirement (b200q_w8a16_linear then plans without it).
"""
import ctypes

import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"
FP8_RMS_TOL = 0.02


def _run(native, x, w, ws, b, act, out_dtype, decode):
    M, K = x.shape
    N = w.shape[0]
    L = native.lib()
    need = int(L.b200q_w8a16_workspace_size(M, N, K))
    dec = (N * K * 2 + 255) // 256 * 256
    assert need >= dec, "shape should select the decoded-weight route"
    work = torch.empty(need, dtype=torch.uint8, device=DEV)
    nbytes = need if decode else dec - 256
    out = torch.empty(M, N, dtype=out_dtype, device=DEV)
    bias_dt = {torch.bfloat16: 1, torch.float16: 2, torch.float32: 3}[b.dtype] if b is not None else 0
    st = L.b200q_w8a16_linear(native._p(x), native._DT[x.dtype], x.stride(0), native._p(w.view(torch.uint8)),
                              w.stride(0), native._p(ws), native._p(b), bias_dt,
                              native.ACTS[act], native._p(out), native._DT[out_dtype], N, M, N, K,
                              native._p(work), nbytes, native._stream(x))
    native._check(st)
    return out


@pytest.mark.parametrize("M,K,N,xdt,act,bias_dt", [
    (512, 3072, 12288, torch.bfloat16, "gelu_tanh", torch.bfloat16),
    (1000, 1024, 1000, torch.float16, None, torch.float32),
    (4096, 3072, 3072, torch.bfloat16, "gelu_tanh", torch.bfloat16),
    (777, 2048, 128, torch.bfloat16, None, None),
])
def test_w8a16_decoded_route(native, M, K, N, xdt, act, bias_dt):
    g = torch.Generator().manual_seed(M + N)
    x = torch.randn(M, K, generator=g).to(xdt)
    w = (torch.randn(N, K, generator=g) * 0.02 / (0.08 / 448)).clamp(-448, 448).to(torch.float8_e4m3fn)
    ws = torch.tensor([0.08 / 448])
    b = (torch.randn(N, generator=g) * 0.01).to(bias_dt) if bias_dt is not None else None
    ref = oracle.w8a16_linear(x, w, ws, b, act, out_dtype="fp32")
    xd, wd, wsd = x.to(DEV), w.to(DEV), ws.to(DEV)
    bd = b.to(DEV) if b is not None else None
    out = _run(native, xd, wd, wsd, bd, act, xdt, True)
    assert oracle.elementwise_ulp_ratio(out, ref) <= 1.0
    out32 = _run(native, xd, wd, wsd, bd, act, torch.float32, True)
    assert oracle.fp8_errors(out32, ref)[0] <= FP8_RMS_TOL
    assert torch.equal(out, out32.to(xdt))
    # the in-kernel-conversion route on the same inputs meets the same bounds
    alt = _run(native, xd, wd, wsd, bd, act, xdt, False)
    assert oracle.elementwise_ulp_ratio(alt, ref) <= 1.0
    # and the op (which sizes its workspace itself) takes the decoded route
    op = native.w8a16_linear(xd, wd, wsd, bd, act)
    assert torch.equal(op, out)


def test_w8a16_decode_of_every_code(native):
    """Every finite e4m3 code as one weight row passes the decode exactly: x = e_k
    picks the k-th weight back (x one-hot, no scale, fp32 out)."""
    K = 256
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8)
    codes[(codes & 0x7F) == 0x7F] = 0  # the two NaN codes (NaN * 0 would reach every output)
    w = codes.view(torch.float8_e4m3fn).reshape(1, K).repeat(8, 1)
    M = 512
    x = torch.zeros(M, K, dtype=torch.bfloat16)
    x[torch.arange(M), torch.arange(M) % K] = 1.0
    out = _run(native, x.to(DEV), w.to(DEV), None, None, None, torch.float32, True).cpu()
    dec = oracle.decode_fp8(w[0:1]).reshape(-1)
    exp = dec[torch.arange(M) % K].reshape(M, 1).expand(M, 8)
    assert torch.equal(out, exp)
