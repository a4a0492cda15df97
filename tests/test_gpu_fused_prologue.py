"""GPU parity of the fused quant prologue (b200q_i8_linear_fused,
b200q_fp8_linear_fused): the activation quantization runs inside the GEMM
launch, so the codes, scales and outputs must be exactly those of the
two-launch route and of the CPU oracle.

INT8: codes, per-token scales and bf16/fp16 outputs bit-exact (the reference's
two-rounding epilogue, int8_gemm.mm:417-443, after its rowwise quant,
int8_gemm.mm:1337-1381).  FP8: codes and the per-tensor scale bit-exact against
the oracle's (x / s).to(e4m3); the GEMM output within FP8_RMS_TOL = 2% of the
reference RMS (fp32 output) and within 1 ULP elementwise (bf16 output).

The shapes cover both tile kernels (128-row tiles below M = 256 or N <= 128,
256-row CTA-pair tiles above), ragged bands (M % 128 != 0), one-row inputs,
strided activations, fp16 activations, the TMA-ineligible fallback (K % 16 != 0)
and CUDA-graph replay with the same sync buffer.
"""
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"
FP8_RMS_TOL = 0.02


def _gen(seed):
    return torch.Generator().manual_seed(seed)


@pytest.fixture(autouse=True)
def _fused_route(monkeypatch):
    """The ops below take the one-launch route unless a test switches it off."""
    monkeypatch.setenv("B200Q_FUSED_PROLOGUE", "1")


def _int8_inputs(g, M, K, N, dtype=torch.bfloat16, outliers=True):
    x = torch.randn(M, K, generator=g)
    if outliers:
        idx = torch.randperm(K, generator=g)[: max(1, K // 100)]
        x[:, idx] *= 20
    x = x.to(dtype)
    w = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int8)
    ws = torch.rand(N, generator=g) * 0.01 + 1e-3
    b = (torch.randn(N, generator=g) * 0.01).to(dtype)
    return x, w, ws, b


def _i8_fused_raw(native, x, w, ws, bias, out_dtype=torch.bfloat16, act="none", sync=None):
    """Calls the C ABI directly; returns (out, codes, scales)."""
    M, K = x.shape
    N = w.shape[0]
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty((M,), dtype=torch.float32, device=x.device)
    out = torch.empty((M, N), dtype=out_dtype, device=x.device)
    if sync is None:
        sync = native._sync_buffer(x, M)
    st = native.lib().b200q_i8_linear_fused(
        native._p(x), native._DT[x.dtype], x.stride(0), native._p(w), w.stride(0), native._p(ws),
        ws.numel(), native._p(bias), native.ACTS[act], native._p(out), native._DT[out_dtype], N, M,
        N, K, native._p(q), native._p(s), native._p(sync), sync.numel(), native._stream(x))
    native._check(st)
    return out, q, s


@pytest.mark.parametrize("M,K,N", [
    (1, 256, 512), (100, 512, 96), (128, 1024, 384), (129, 768, 640), (255, 1536, 1024),
    (256, 3072, 3072), (300, 2048, 200), (1000, 3072, 2304), (2048, 3072, 3072)])
def test_i8_linear_fused_bit_exact(native, M, K, N):
    g = _gen(3)
    x, w, ws, b = _int8_inputs(g, M, K, N)
    q_ref, s_ref = oracle.quantize_int8_rowwise(x)
    ref = oracle.int8_linear(x, w, ws, b)
    out, q, s = _i8_fused_raw(native, x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(q.cpu(), q_ref), "codes differ"
    assert torch.equal(s.cpu().reshape(-1, 1), s_ref), "scales differ"
    assert torch.equal(out.cpu(), ref), "outputs differ"


def _ulp_diff_16(a, b):
    """Elementwise distance in units of the last place between two 16-bit
    float tensors of the same dtype (sign-magnitude bit patterns mapped to a
    monotone integer line)."""
    def line(t):
        v = t.view(torch.int16).to(torch.int32)
        return torch.where(v < 0, -(v & 0x7FFF), v)
    return (line(a) - line(b)).abs()


def test_i8_linear_fused_fp16_and_gelu(native):
    """fp16 activations and output, GELU(tanh) after the two-rounding
    dequant (the block's up-projection epilogue): the dequant is exact, the
    GELU (fp32 on the GPU, float64 in the oracle) is within 1 ULP after rounding."""
    g = _gen(11)
    M, K, N = 520, 2048, 1536
    x, w, ws, b = _int8_inputs(g, M, K, N, dtype=torch.float16)
    ref = oracle.int8_linear(x, w, ws, b, torch.float16, "gelu_tanh")
    out = native.i8_linear(x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV), torch.float16, "gelu_tanh")
    assert out.dtype == torch.float16
    assert int(_ulp_diff_16(out.cpu(), ref).max()) <= 1
    plain = native.i8_linear(x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV), torch.float16)
    assert torch.equal(plain.cpu(), oracle.int8_linear(x, w, ws, b, torch.float16))


def test_i8_linear_fused_strided_activation(native):
    g = _gen(19)
    M, K, N = 384, 1024, 512
    x, w, ws, b = _int8_inputs(g, M, K + 64, N)
    xs = x[:, 8:8 + K]            # row stride K + 64, 16-byte aligned rows
    w = w[:, :K].contiguous()
    ref = oracle.int8_linear(xs.contiguous(), w, ws, b)
    xd = x.to(DEV)[:, 8:8 + K]
    out, q, s = _i8_fused_raw(native, xd, w.to(DEV), ws.to(DEV), b.to(DEV))
    assert torch.equal(out.cpu(), ref)


def test_i8_linear_fused_ragged_k_falls_back(native):
    g = _gen(23)
    M, K, N = 70, 100, 130      # K % 16 != 0: quant launch + SIMT GEMM inside the call
    x, w, ws, b = _int8_inputs(g, M, K, N)
    ref = oracle.int8_linear(x, w, ws, b)
    out = native.i8_linear(x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV))
    assert torch.equal(out.cpu(), ref)


def test_i8_linear_fused_matches_two_launch_route(native, monkeypatch):
    g = _gen(5)
    M, K, N = 2304, 3072, 4096
    x, w, ws, b = _int8_inputs(g, M, K, N)
    xd, wd, wsd, bd = x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV)
    fused = native.i8_linear(xd, wd, wsd, bd)
    monkeypatch.setenv("B200Q_FUSED_PROLOGUE", "0")
    two = native.i8_linear(xd, wd, wsd, bd)
    assert torch.equal(fused, two)


def test_sync_buffer_left_zero_and_reused(native):
    g = _gen(29)
    outs = []
    for M in (3000, 77, 513, 3000):
        x, w, ws, b = _int8_inputs(g, M, 1024, 768)
        out = native.i8_linear(x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV))
        outs.append((out, oracle.int8_linear(x, w, ws, b)))
    torch.cuda.synchronize()
    for out, ref in outs:
        assert torch.equal(out.cpu(), ref)
    key = (torch.cuda.current_device(), torch.cuda.current_stream().cuda_stream)
    assert int(native._SYNC[key].count_nonzero()) == 0


def _fp8_fused_raw(native, x, w, ws, bias, out_dtype, act="none"):
    M, K = x.shape
    N = w.shape[0]
    q = torch.empty((M, K), dtype=torch.uint8, device=x.device)
    s = torch.empty((1,), dtype=torch.float32, device=x.device)
    out = torch.empty((M, N), dtype=out_dtype, device=x.device)
    sync = native._sync_buffer(x, M)
    bdt = native._BIAS_DT[bias.dtype] if bias is not None else native.BIAS_NONE
    st = native.lib().b200q_fp8_linear_fused(
        native._p(x), native._DT[x.dtype], x.stride(0), native._p(w.view(torch.uint8)), w.stride(0),
        native._p(ws), ws.numel(), None, native._p(bias), bdt, native.ACTS[act], native._p(out),
        native._DT[out_dtype], N, M, N, K, native._p(q), native._p(s), native._p(sync), sync.numel(),
        native._stream(x))
    native._check(st)
    return out, q, s


@pytest.mark.parametrize("M,K,N", [(1, 512, 256), (100, 1024, 96), (333, 2048, 1024),
                                   (768, 5120, 1536), (512, 13824, 1280)])
@pytest.mark.parametrize("act", ["none", "gelu_tanh"])
def test_fp8_linear_fused(native, M, K, N, act):
    g = _gen(4)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    wq, wsc = oracle.quantize_fp8_tensorwise(w)
    ws = wsc.reshape(1)
    b = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16)
    q_ref, s_ref = oracle.quantize_fp8_tensorwise(x)
    ref = oracle.scaled_mm_fp8(q_ref, wq, s_ref.reshape(1), ws, None, b, None,
                               None if act == "none" else act)
    xd, wd, wsd, bd = x.to(DEV), wq.to(DEV), ws.to(DEV), b.to(DEV)
    out32, q, s = _fp8_fused_raw(native, xd, wd, wsd, bd, torch.float32, act)
    torch.cuda.synchronize()
    assert torch.equal(q.cpu(), q_ref.view(torch.uint8)), "codes differ"
    assert torch.equal(s.cpu().reshape(()), s_ref), "scale differs"
    assert oracle.fp8_errors(out32, ref)[0] <= FP8_RMS_TOL
    out = native.fp8_linear(xd, wd, wsd, bd, torch.bfloat16, act)
    assert oracle.elementwise_ulp_ratio(out, ref) <= 1.0
    assert torch.equal(out, out32.to(torch.bfloat16))


def test_fp8_linear_matches_two_launch_route(native, monkeypatch):
    g = _gen(41)
    M, K, N = 1536, 5120, 3072
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(DEV)
    wq, wsc = oracle.quantize_fp8_tensorwise((torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16))
    wd, ws = wq.to(DEV), wsc.reshape(1).to(DEV)
    fused = native.fp8_linear(x, wd, ws, None, torch.bfloat16, "gelu_tanh")
    monkeypatch.setenv("B200Q_FUSED_PROLOGUE", "0")
    two = native.fp8_linear(x, wd, ws, None, torch.bfloat16, "gelu_tanh")
    assert torch.equal(fused, two)


def test_fused_ops_replay_in_cuda_graphs(native):
    """Captured once, replayed with new input contents: the sync buffer is
    zeroed by each launch's last CTA, so every replay is exact."""
    g = _gen(31)
    M, K, N = 640, 1024, 768
    x0, w, ws, b = _int8_inputs(g, M, K, N)
    xf = torch.randn(M, K, generator=g).to(torch.bfloat16)
    wq, wsc = oracle.quantize_fp8_tensorwise((torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16))
    xi_d, xf_d = x0.to(DEV), xf.to(DEV)
    wd, wsd, bd, wqd, wsq = w.to(DEV), ws.to(DEV), b.to(DEV), wq.to(DEV), wsc.reshape(1).to(DEV)
    ops = torch.ops.b200q
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # warm-up outside capture
        ops.i8_linear(xi_d, wd, wsd, bd)
        ops.fp8_linear(xf_d, wqd, wsq, bd)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        yi = ops.i8_linear(xi_d, wd, wsd, bd)
        yf = ops.fp8_linear(xf_d, wqd, wsq, bd)
    for step in range(3):
        xi = _int8_inputs(_gen(100 + step), M, K, N)[0]
        xf = torch.randn(M, K, generator=_gen(200 + step)).to(torch.bfloat16)
        xi_d.copy_(xi)
        xf_d.copy_(xf)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(yi.cpu(), oracle.int8_linear(xi, w, ws, b))
        qf, sf = oracle.quantize_fp8_tensorwise(xf)
        ref = oracle.scaled_mm_fp8(qf, wq, sf.reshape(1), wsc.reshape(1), None, b, None)
        assert oracle.elementwise_ulp_ratio(yf, ref) <= 1.0
    del graph


def test_fused_device_status_clean(native):
    torch.cuda.synchronize()
    assert native.device_status() == 0
