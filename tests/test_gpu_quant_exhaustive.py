"""Exhaustive check of the quantizers' divide-free quotient (x * RN(1/s) with an
exact-divide fallback near rounding ties): every finite 16-bit value up to a
row's absmax goes through each quant path, and the codes must equal the
oracle's, which divides with numpy's correctly rounded fp32 division
(int8_gemm.mm:1363-1365 for INT8; (x / s).to(e4m3) for FP8).

Paths covered: the standalone rowwise INT8 kernel, the fused GEMM prologue
(i8_linear_fused, both tile kernels via the row count), the per-tensor FP8
quantize kernel and the fused FP8 prologue.
"""
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _all_values_up_to(amax, dtype):
    """Every finite value of `dtype` with |v| <= amax (both signs), plus amax itself."""
    if dtype == torch.bfloat16:
        bits = torch.arange(0, 0x7F80, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    else:
        bits = torch.arange(0, 0x7C00, dtype=torch.int32).to(torch.int16).view(torch.float16)
    v = bits.float()
    v = v[v <= amax]
    row = torch.cat([torch.tensor([amax]), v, -v]).to(dtype)
    pad = (-row.numel()) % 16
    return torch.cat([row, torch.zeros(pad, dtype=dtype)])


AMAXES = {torch.bfloat16: [1.0, 3.7, 0.0123, 448.0, 2.0e-20, 1.0e30],
          torch.float16: [1.0, 3.7, 0.0123, 448.0, 6.0e-5, 65504.0]}


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rowwise_int8_exhaustive(native, dtype):
    rows = [_all_values_up_to(a, dtype) for a in AMAXES[dtype]]
    K = max(r.numel() for r in rows)
    x = torch.zeros(len(rows), K, dtype=dtype)
    for i, r in enumerate(rows):
        x[i, : r.numel()] = r
    q_ref, s_ref = oracle.quantize_int8_rowwise(x)
    q, s = native.quant_rowwise_i8(x.to(DEV))
    assert torch.equal(s.cpu(), s_ref)
    assert torch.equal(q.cpu(), q_ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("copies", [1, 43])  # 43 x 6 = 258 rows: the CTA-pair tiles
def test_fused_prologue_int8_exhaustive(native, dtype, copies):
    rows = [_all_values_up_to(a, dtype) for a in AMAXES[dtype]] * copies
    K = max(r.numel() for r in rows)
    K += (-K) % 16
    x = torch.zeros(len(rows), K, dtype=dtype)
    for i, r in enumerate(rows):
        x[i, : r.numel()] = r
    M, N = x.shape[0], 256
    w = torch.zeros(N, K, dtype=torch.int8)
    w[:, 0] = 1
    ws = torch.ones(N)
    q_ref, s_ref = oracle.quantize_int8_rowwise(x)
    xd = x.to(DEV)
    q = torch.empty(M, K, dtype=torch.int8, device=DEV)
    s = torch.empty(M, dtype=torch.float32, device=DEV)
    out = torch.empty(M, N, dtype=dtype, device=DEV)
    sync = native._sync_buffer(xd, M)
    wd, wsd = w.to(DEV), ws.to(DEV)
    native._check(native.lib().b200q_i8_linear_fused(
        native._p(xd), native._DT[dtype], K, native._p(wd), K, native._p(wsd), N, None, 0,
        native._p(out), native._DT[dtype], N, M, N, K, native._p(q), native._p(s), native._p(sync),
        sync.numel(), native._stream(xd)))
    assert torch.equal(s.cpu().reshape(-1, 1), s_ref)
    assert torch.equal(q.cpu(), q_ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("amax", [1.0, 37.5, 3.0e-3])
def test_fp8_quant_exhaustive(native, dtype, amax):
    row = _all_values_up_to(amax, dtype)
    x = row.reshape(-1, 16)
    q_ref, s_ref = oracle.quantize_fp8_tensorwise(x)
    q, s = native.fp8_quant_tensorwise(x.to(DEV))
    assert torch.equal(s.cpu().reshape(()), s_ref)
    assert torch.equal(q.cpu().view(torch.uint8), q_ref.view(torch.uint8))
    # the fused prologue quantizes the same tensor (as [rows, 512] for the GEMM)
    x2 = row[: (row.numel() // 512) * 512].reshape(-1, 512)
    q_ref2, s_ref2 = oracle.quantize_fp8_tensorwise(x2)
    M, K, N = x2.shape[0], 512, 128
    w = torch.zeros(N, K).to(torch.float8_e4m3fn)
    xd = x2.to(DEV)
    qd = torch.empty(M, K, dtype=torch.uint8, device=DEV)
    sd = torch.empty(1, dtype=torch.float32, device=DEV)
    out = torch.empty(M, N, dtype=torch.float32, device=DEV)
    sync = native._sync_buffer(xd, M)
    wd = w.to(DEV)
    native._check(native.lib().b200q_fp8_linear_fused(
        native._p(xd), native._DT[dtype], K, native._p(wd.view(torch.uint8)), K, None, 0, None,
        None, 0, 0, native._p(out), native._DT[torch.float32], N, M, N, K, native._p(qd),
        native._p(sd), native._p(sync), sync.numel(), native._stream(xd)))
    assert torch.equal(sd.cpu().reshape(()), s_ref2)
    assert torch.equal(qd.cpu(), q_ref2.view(torch.uint8))
