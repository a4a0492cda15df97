"""GPU parity of every b200q kernel against the CPU oracle (same seeded inputs).

INT8 route: activation codes, per-token scales and int32 accumulators must be
bit-exact; the dequantized bf16/fp16 outputs must be bit-exact as well (the
north-star bound is 1 bf16 ULP; the kernels reproduce the reference's
two-rounding epilogue exactly, so the tests assert equality and report the ULP
distance on failure).

FP8 routes (tolerance written here: FP8_RMS_TOL = 2% of the reference RMS):
  * the kernel's fp32-output variant satisfies max|out - ref| <= 2% rms(ref),
    ref = the oracle's fp32 value before the final cast (the value the
    reference's FP8 route rounds once, scaled_mm_fp8.py:136-146);
  * the bf16/fp16 output is exactly the RNE rounding of that fp32 output, and
    every element lies within 1 ULP of ref (plus 0.1% rms slack near zero).
The 2%-of-RMS bound is not applied to the rounded bf16 tensor itself: a bf16
rounding of a 4-8 sigma element is up to 1.6% of sigma on its own, and GELU
outputs have an RMS well below sigma, so that comparison would measure bf16.

Shapes follow the reference's own tests: tests/test_int8_linear_kernel.py
(seeds 3/7/11/19/23, ragged M/N/K, zero and 1e-30 rows) and the _int_mm canary
(_patches/int_mm_mps.py:67-81).
"""
import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

FP8_RMS_TOL = 0.02
DEV = "cuda"


def _gen(seed):
    return torch.Generator().manual_seed(seed)


# ----------------------------------------------------------------------------- INT8 quant
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,K", [(33, 6144), (7, 100), (1, 256), (128, 300), (64, 16384),
                                 (4096, 3072), (9, 20000)])
def test_quant_rowwise_bit_exact(native, dtype, M, K):
    g = _gen(3)
    x = (torch.randn((M, K), generator=g) * 3).to(dtype)
    q_ref, s_ref = oracle.quantize_int8_rowwise(x)
    q, s = native.quant_rowwise_i8(x.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(q.cpu(), q_ref), f"codes differ {dtype} {M}x{K}"
    assert torch.equal(s.cpu(), s_ref), f"scales differ {dtype} {M}x{K}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_quant_rowwise_edge_rows(native, dtype):
    for edge in (torch.zeros(4, 512), torch.full((4, 512), 1e-30), torch.full((3, 40), -7.5)):
        x = edge.to(dtype)
        q_ref, s_ref = oracle.quantize_int8_rowwise(x)
        q, s = native.quant_rowwise_i8(x.to(DEV))
        assert torch.equal(q.cpu(), q_ref) and torch.equal(s.cpu(), s_ref)


def test_quant_rowwise_strided_rows(native):
    g = _gen(5)
    base = torch.randn((64, 1000), generator=g).to(torch.bfloat16)
    x = base[:, :768]  # row stride 1000 elements, not contiguous
    q_ref, s_ref = oracle.quantize_int8_rowwise(x.contiguous())
    xd = base.to(DEV)[:, :768]
    assert xd.stride(0) == 1000
    q, s = native.quant_rowwise_i8(xd)
    assert torch.equal(q.cpu(), q_ref) and torch.equal(s.cpu(), s_ref)


# ----------------------------------------------------------------------------- INT8 GEMM
@pytest.mark.parametrize("M,K,N", [(3, 129, 5), (16, 4096, 32), (256, 2560, 1024), (65, 768, 129),
                                   (130, 512, 256), (8209, 96, 129), (1, 6144, 640),
                                   (1000, 3072, 3000), (4096, 3072, 3072)])
def test_int_mm_exact(native, M, K, N):
    g = _gen(0)
    a = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int8)
    b = torch.randint(-128, 128, (K, N), generator=g, dtype=torch.int8)
    a[:, 0] = -128
    b[0, :] = 127
    ref = oracle.int_mm(a, b)
    out = native.int_mm(a.to(DEV), b.to(DEV))
    torch.cuda.synchronize()
    assert out.dtype == torch.int32
    assert torch.equal(out.cpu(), ref)


def test_int_mm_extreme_accumulators(native):
    """All -128 x -128 over K=12288: the largest int32 magnitude the path sees."""
    M, K, N = 128, 12288, 256
    a = torch.full((M, K), -128, dtype=torch.int8)
    w = torch.full((N, K), -128, dtype=torch.int8)
    out = native.i8_matmul_nt(a.to(DEV), w.to(DEV)).cpu()
    assert int(out.min()) == int(out.max()) == 128 * 128 * K


@pytest.mark.parametrize("M,K,N,bias,out_dtype", [
    (256, 2560, 1024, True, torch.bfloat16), (65, 768, 129, True, torch.bfloat16),
    (96, 704, 385, False, torch.bfloat16), (33, 512, 256, True, torch.bfloat16),
    (1, 2560, 512, False, torch.bfloat16), (130, 512, 256, True, torch.bfloat16),
    (8209, 96, 129, False, torch.bfloat16), (512, 3072, 3072, True, torch.float16)])
def test_dequant_epilogue_channelwise_bit_exact(native, M, K, N, bias, out_dtype):
    g = _gen(11)
    a = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int8)
    w = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int8)
    rs = torch.rand(M, generator=g) * 0.01
    cs = torch.rand(N, generator=g) * 0.01 + 0.001
    b = torch.randn(N, generator=g).to(out_dtype) if bias else None
    c = oracle.int_mm(a, w.t())
    ref = oracle.int8_dequant_epilogue(c, rs.reshape(-1, 1), cs, b, out_dtype)
    out = native.i8_matmul_nt_fused_cs(a.to(DEV), w.to(DEV), rs.to(DEV), cs.to(DEV),
                                       b.to(DEV) if b is not None else None, out_dtype).cpu()
    if out_dtype == torch.bfloat16:
        assert oracle.bf16_ulp_diff(out, ref) <= 1
    assert torch.equal(out, ref), f"mismatch M={M} K={K} N={N}"


@pytest.mark.parametrize("N", [300, 1001, 129])
def test_ragged_width_outputs_stay_in_their_columns(native, N):
    """CTA-pair route (M >= 256) with a row of N 16-bit outputs that is not a
    multiple of 16 bytes, written into a wider buffer (row stride N + 40): the
    N columns equal the contiguous call's and no column past N is touched, for
    the FP8-scaled and the INT8-dequant epilogues."""
    import ctypes
    M, K, ldo = 512, 640, N + 40
    g = _gen(N)
    L = native.lib()
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # FP8 scaled, bias + GELU
    a = (torch.randn(M, K, generator=g) * 8).to(torch.float8_e4m3fn).to(DEV)
    w = (torch.randn(N, K, generator=g) * 8).to(torch.float8_e4m3fn).to(DEV)
    sa, sb = torch.tensor([0.01], device=DEV), torch.tensor([0.02], device=DEV)
    b = torch.randn(N, generator=g).to(torch.bfloat16).to(DEV)
    ref = native.fp8_scaled_mm(a, w, sa, sb, None, b, torch.bfloat16, "gelu_tanh")
    out = torch.full((M, ldo), float("nan"), dtype=torch.bfloat16, device=DEV)
    assert L.b200q_fp8_scaled_mm(a.data_ptr(), K, w.data_ptr(), K, sa.data_ptr(), 1, sb.data_ptr(),
                                 1, None, b.data_ptr(), 1, 1, out.data_ptr(), 0, ldo, M, N, K,
                                 st) == 0
    torch.cuda.synchronize()
    assert torch.equal(out[:, :N], ref)
    assert torch.isnan(out[:, N:].float()).all()
    # INT8 dequant (two roundings), bf16 bias
    a8 = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int8).to(DEV)
    w8 = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int8).to(DEV)
    rs = (torch.rand(M, generator=g) * 0.01).to(DEV)
    cs = (torch.rand(N, generator=g) * 0.01 + 0.001).to(DEV)
    ref8 = native.i8_matmul_nt_fused_cs(a8, w8, rs, cs, b, torch.bfloat16)
    out8 = torch.full((M, ldo), float("nan"), dtype=torch.bfloat16, device=DEV)
    assert L.b200q_i8_matmul_nt_dequant(a8.data_ptr(), K, w8.data_ptr(), K, rs.data_ptr(),
                                        cs.data_ptr(), N, b.data_ptr(), 0, out8.data_ptr(), 0,
                                        ldo, M, N, K, st) == 0
    torch.cuda.synchronize()
    assert torch.equal(out8[:, :N], ref8)
    assert torch.isnan(out8[:, N:].float()).all()


@pytest.mark.parametrize("M,K,N,act", [(512, 640, 1024, "gelu_tanh"), (512, 640, 600, None),
                                      (300, 1024, 3072, "gelu_tanh"), (100, 512, 384, None),
                                      (2048, 3072, 12288, "gelu_tanh")])
def test_fp8_scaled_mm_amax_and_quant_from_amax(native, M, K, N, act):
    """fp8_scaled_mm_amax gives fp8_scaled_mm's output bit for bit plus the max
    |out| of that bf16 output (taken in the CTA-pair epilogue for M >= 256 and
    N > 128, by the absmax pass otherwise, with both store paths of the
    epilogue: 16-byte row widths and ragged N = 600); fp8_quant_from_amax with it
    gives fp8_quant_tensorwise's codes and scale bit for bit."""
    g = _gen(M + N)
    a = (torch.randn(M, K, generator=g) * 8).to(torch.float8_e4m3fn).to(DEV)
    w = (torch.randn(N, K, generator=g) * 8).to(torch.float8_e4m3fn).to(DEV)
    sa, sb = torch.tensor([0.01], device=DEV), torch.tensor([0.02], device=DEV)
    b = torch.randn(N, generator=g).to(torch.bfloat16).to(DEV)
    ref = native.fp8_scaled_mm(a, w, sa, sb, None, b, torch.bfloat16, act)
    for _ in range(2):  # the amax word is rewritten on every call
        out, amax = native.fp8_scaled_mm_amax(a, w, sa, sb, None, b, torch.bfloat16, act)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        want = ref.float().abs().max().reshape(1).view(torch.int32)
        assert torch.equal(amax, want)
    q, s = native.fp8_quant_from_amax(out, amax)
    q_ref, s_ref = native.fp8_quant_tensorwise(out)
    assert torch.equal(q.view(torch.uint8), q_ref.view(torch.uint8)) and torch.equal(s, s_ref)
    assert native.device_status() == 0


def test_dequant_epilogue_tensorwise_bit_exact(native):
    g = _gen(7)
    M, K, N = 256, 2560, 1024
    a = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int8)
    w = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int8)
    xs = torch.rand(M, generator=g) * 0.02
    ws = torch.rand(1, generator=g) * 0.01 + 0.001
    b = torch.randn(N, generator=g).to(torch.bfloat16)
    row_scale = (ws * xs).float()
    c = oracle.int_mm(a, w.t())
    ref = oracle.int8_dequant_epilogue(c, xs.reshape(-1, 1), ws, b)
    out = native.i8_matmul_nt_fused(a.to(DEV), w.to(DEV), row_scale.to(DEV), b.to(DEV)).cpu()
    assert torch.equal(out, ref)


@pytest.mark.parametrize("shape,K,N,ws_kind,bias", [
    ((256,), 2560, 1024, "scalar", False), ((256,), 2560, 1024, "scalar", True),
    ((2, 188), 4096, 2560, "channel", True), ((1,), 6144, 6144, "channel", False),
    ((4096,), 3072, 3072, "channel", True)])
def test_int8_linear_end_to_end_bit_exact(native, shape, K, N, ws_kind, bias):
    g = _gen(7)
    x = torch.randn((*shape, K), generator=g).to(torch.bfloat16) * 0.5
    w = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int8)
    ws = (torch.rand(1 if ws_kind == "scalar" else N, generator=g) * 0.01 + 0.001)
    b = torch.randn(N, generator=g).to(torch.bfloat16) if bias else None
    ref = oracle.int8_linear(x, w, ws, b)
    out = native.i8_linear(x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV) if b is not None else None)
    assert out.shape == ref.shape
    assert torch.equal(out.cpu(), ref)


# ----------------------------------------------------------------------------- FP8 W8A8
def _fp8_pair(g, M, K, N, a_scale=0.3, w_scale=0.3):
    a = (torch.randn(M, K, generator=g) * a_scale).to(torch.float8_e4m3fn)
    w = (torch.randn(N, K, generator=g) * w_scale).to(torch.float8_e4m3fn)
    return a, w


@pytest.mark.parametrize("M,K,N", [(64, 2048, 2048), (100, 512, 384), (33, 4096, 160),
                                   (1024, 3072, 3072), (512, 12288, 3072)])
@pytest.mark.parametrize("epi", ["plain", "scaled_bias", "gelu"])
def test_fp8_scaled_mm(native, M, K, N, epi):
    g = _gen(2)
    a, w = _fp8_pair(g, M, K, N)
    sa = torch.tensor([0.02]) if epi != "plain" else None
    sb = torch.tensor([0.05]) if epi != "plain" else None
    b = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16) if epi != "plain" else None
    act = "gelu_tanh" if epi == "gelu" else None
    ref = oracle.scaled_mm_fp8(a, w, sa, sb, None, b, None, act)
    dev = lambda t: t.to(DEV) if t is not None else None
    out = native.fp8_scaled_mm(dev(a), dev(w), dev(sa), dev(sb), None, dev(b), torch.bfloat16, act)
    assert oracle.elementwise_ulp_ratio(out, ref) <= 1.0
    out32 = native.fp8_scaled_mm(dev(a), dev(w), dev(sa), dev(sb), None, dev(b), torch.float32, act)
    rms_err, rel = oracle.fp8_errors(out32, ref)
    assert rms_err <= FP8_RMS_TOL, (rms_err, rel)
    assert torch.equal(out, out32.to(torch.bfloat16))  # bf16 output = RNE of the fp32 result


def test_fp8_scaled_mm_rowwise_scales_and_f32_out(native):
    g = _gen(21)
    M, K, N = 200, 1024, 320
    a, w = _fp8_pair(g, M, K, N)
    sa = torch.rand(M, 1, generator=g) * 0.1 + 0.01
    sb = torch.rand(1, N, generator=g) * 0.1 + 0.01
    ref = oracle.scaled_mm_fp8(a, w, sa, sb, None, None, None)
    out = native.fp8_scaled_mm(a.to(DEV), w.to(DEV), sa.to(DEV), sb.to(DEV), None, None,
                               torch.float32)
    assert out.dtype == torch.float32
    assert oracle.fp8_errors(out, ref)[0] <= FP8_RMS_TOL


def test_fp8_scaled_mm_vs_reference_decode_path(native):
    """Against the reference's triple-rounding decode fallback the difference is
    bounded by bf16 itself: within 2 bf16 ULPs of that path's output."""
    g = _gen(23)
    M, K, N = 256, 2048, 1024
    a, w = _fp8_pair(g, M, K, N)
    sa, sb = torch.tensor([0.02]), torch.tensor([0.05])
    b = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16)
    ref = oracle.scaled_mm_fp8_decode_path(a, w, sa, sb, None, b)
    out = native.fp8_scaled_mm(a.to(DEV), w.to(DEV), sa.to(DEV), sb.to(DEV), None, b.to(DEV)).cpu()
    rms_err, rel = oracle.fp8_errors(out, ref)
    assert rms_err <= 0.03 and rel <= 0.01  # rel: the reference's own rel_err metric


def test_fp8_ragged_k_simt_path(native):
    g = _gen(22)
    M, K, N = 50, 100, 70  # K % 16 != 0 -> SIMT kernel
    a, w = _fp8_pair(g, M, K, N)
    ref = oracle.scaled_mm_fp8(a, w, out_dtype=None)
    out = native.fp8_scaled_mm(a.to(DEV), w.to(DEV))
    assert oracle.fp8_errors(out, ref)[0] <= FP8_RMS_TOL
    assert oracle.elementwise_ulp_ratio(out, ref) <= 1.0


@pytest.mark.parametrize("M,K", [(4096, 3072), (33, 100), (1, 16), (2048, 12288)])
def test_fp8_quant_tensorwise_bit_exact(native, M, K):
    g = _gen(4)
    x = (torch.randn(M, K, generator=g) * 2).to(torch.bfloat16)
    q_ref, s_ref = oracle.quantize_fp8_tensorwise(x)
    q, s = native.fp8_quant_tensorwise(x.to(DEV))
    assert torch.equal(s.cpu().reshape(()), s_ref)
    assert torch.equal(q.cpu().view(torch.uint8), q_ref.view(torch.uint8))


def test_fp8_decode_all_codes(native):
    for kind in (torch.float8_e4m3fn, torch.float8_e5m2):
        codes = torch.arange(256, dtype=torch.uint8).view(kind)
        for od in (torch.float32, torch.bfloat16, torch.float16):
            ref = codes.to(od).float()
            out = native.fp8_decode(codes.to(DEV), od).cpu().float()
            nan = torch.isnan(ref)
            assert torch.equal(torch.isnan(out), nan)
            assert torch.equal(out[~nan], ref[~nan])


# ----------------------------------------------------------------------------- W8A16
@pytest.mark.parametrize("M", [1, 16, 100, 256, 1000, 4096])
@pytest.mark.parametrize("epi", ["bias", "scale_bias_gelu"])
def test_w8a16_linear(native, M, epi):
    g = _gen(1)
    K, N = 3072, 12288 if M <= 256 else 3072
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02 / (0.08 / 448)).clamp(-448, 448).to(torch.float8_e4m3fn)
    ws = torch.tensor([0.08 / 448]) if epi != "bias" else None
    b = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16)
    act = "gelu_tanh" if epi != "bias" else None
    ref = oracle.w8a16_linear(x, w, ws, b, act, out_dtype="fp32")
    out = native.w8a16_linear(x.to(DEV), w.to(DEV), ws.to(DEV) if ws is not None else None,
                              b.to(DEV), act)
    assert out.dtype == torch.bfloat16
    assert oracle.elementwise_ulp_ratio(out, ref) <= 1.0
    out32 = native.w8a16_linear(x.to(DEV), w.to(DEV), ws.to(DEV) if ws is not None else None,
                                b.to(DEV), act, torch.float32)
    assert oracle.fp8_errors(out32, ref)[0] <= FP8_RMS_TOL
    assert torch.equal(out, out32.to(torch.bfloat16))


def test_w8a16_fp16_activations_and_ragged(native):
    g = _gen(9)
    for M, K, N in ((37, 1024, 300), (5, 100, 64)):  # second: K % 16 != 0 (SIMT)
        x = torch.randn(M, K, generator=g).to(torch.float16)
        w = (torch.randn(N, K, generator=g) * 2).to(torch.float8_e4m3fn)
        b = torch.randn(N, generator=g).float()
        ref = oracle.w8a16_linear(x, w, None, b, out_dtype="fp32")
        out = native.w8a16_linear(x.to(DEV), w.to(DEV), None, b.to(DEV))
        assert out.dtype == torch.float16
        assert oracle.elementwise_ulp_ratio(out, ref) <= 1.0
        out32 = native.w8a16_linear(x.to(DEV), w.to(DEV), None, b.to(DEV), None, torch.float32)
        assert oracle.fp8_errors(out32, ref)[0] <= FP8_RMS_TOL


def test_w8a16_split_k_is_deterministic(native):
    """The weight-stationary kernel's split-K (fixed-order fix-up) is deterministic.
    It runs when the workspace is below the decoded-weight route's requirement."""
    g = _gen(12)
    M, K, N = 300, 12288, 3072  # 24 weight tiles x 2 token tiles x 2 splits
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(N, K, generator=g) * 50).clamp(-448, 448).to(torch.float8_e4m3fn).to(DEV)
    L = native.lib()
    nbytes = (N * K * 2 + 255) // 256 * 256 - 256   # just below the decode route's need
    work = torch.empty(nbytes, dtype=torch.uint8, device=DEV)

    def run(ws_bytes):
        out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
        native._check(L.b200q_w8a16_linear(native._p(x), 0, K, native._p(w.view(torch.uint8)), K,
                                           None, None, 0, 0, native._p(out), 0, N, M, N, K,
                                           native._p(work), ws_bytes, native._stream(x)))
        return out
    assert L.b200q_w8a16_linear(native._p(x), 0, K, native._p(w.view(torch.uint8)), K, None, None,
                                0, 0, native._p(torch.empty(M, N, dtype=torch.bfloat16, device=DEV)),
                                0, N, M, N, K, None, 0, native._stream(x)) == 4, \
        "expected the split-K plan (no workspace -> B200Q_ERR_WORKSPACE)"
    o1, o2 = run(nbytes), run(nbytes)
    assert torch.equal(o1, o2)
    ref = oracle.w8a16_linear(x.cpu(), w.cpu(), None, None, None, out_dtype="fp32")
    assert oracle.elementwise_ulp_ratio(o1, ref) <= 1.0


def test_device_status_clean(native):
    torch.cuda.synchronize()
    assert native.device_status(reset=True) == 0
