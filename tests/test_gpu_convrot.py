"""GPU parity of the convrot rotation fused into the per-token INT8 quant
(b200q_quant_rowwise_i8_convrot).

Two oracles.  (1) The reference kernel's own fp32 butterflies, restated
(oracle.rotate_convrot_fwht, int8_gemm.mm:1463-1479): codes and scales must be
bit-identical.  (2) comfy's semantics, the exact rotation rounded once
(oracle.rotate_convrot): the fp32 sums can flip a rotated value's last bf16
ulp on a rare tie, moving one code by 1 or, via a flipped row absmax, a row's
scale by ~2^-8; the bounds are those of the reference's own test of its fused
rotate+quant kernel (tests/test_int8_linear_kernel.py:932-975): scale rel diff
< 6e-3, |code diff| <= 1, code mismatch fraction < 5e-3 (and >= 99% of rows
with identical scales).
"""
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _gen(seed):
    return torch.Generator().manual_seed(seed)


def _check_fwht_exact(q, s, x):
    q_ref, s_ref = oracle.quantize_int8_rowwise(oracle.rotate_convrot_fwht(x))
    assert torch.equal(s.cpu(), s_ref)
    assert torch.equal(q.cpu(), q_ref)


def _check_codes(q, s, q_ref, s_ref):
    srel = ((s.cpu() - s_ref).abs() / s_ref).max().item()
    assert srel < 6e-3, srel
    dq = (q.cpu().int() - q_ref.int()).abs()
    assert dq.max().item() <= 1
    assert (dq > 0).float().mean().item() < 5e-3
    assert (s.cpu() == s_ref).float().mean().item() >= 0.99


# merged [B*S, H*D] shapes of the reference test (B,H,S,D) plus its linear shapes
@pytest.mark.parametrize("M,K", [(777, 4608), (128, 4608), (256, 256), (5037, 1024),
                                 (257, 7168), (1, 6144), (512, 6144)])
def test_convrot_quant_matches_oracle(native, M, K):
    g = _gen(5)
    x = (torch.randn(M, K, generator=g) * 2).to(torch.bfloat16)
    q_ref, s_ref = oracle.quantize_int8_rowwise_convrot(x)
    q, s = native.quant_rowwise_i8_convrot(x.to(DEV))
    torch.cuda.synchronize()
    _check_codes(q, s, q_ref, s_ref)
    _check_fwht_exact(q, s, x)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_convrot_quant_outliers_fp16_strided(native, dtype):
    g = _gen(9)
    M, K = 300, 3072
    xf = torch.randn(M, K + 256, generator=g)
    xf[:, torch.randperm(K, generator=g)[:30]] *= 20  # outlier channels, as in BASELINE C4
    x = xf.to(dtype)
    xs = x[:, 128:128 + K]
    q_ref, s_ref = oracle.quantize_int8_rowwise_convrot(xs.contiguous())
    q, s = native.quant_rowwise_i8_convrot(x.to(DEV)[:, 128:128 + K])
    _check_codes(q, s, q_ref, s_ref)
    _check_fwht_exact(q, s, xs.contiguous())


def test_convrot_rejects_unsupported_groups(native):
    x = torch.randn(4, 384, device=DEV).to(torch.bfloat16)  # K % 256 != 0
    with pytest.raises(RuntimeError):
        native.quant_rowwise_i8_convrot(x)
    with pytest.raises(RuntimeError):
        native.quant_rowwise_i8_convrot(torch.randn(4, 512, device=DEV).to(torch.bfloat16), 128)


def test_convrot_linear_through_the_seam(native):
    """The int8_tensorwise convrot Linear (_int8_linear_kernel with convrot=True)
    against the oracle's rotate -> quant -> GEMM -> dequant on the same inputs."""
    from b200q._patches import int8_linear_kernel as seam
    seam._kernel = seam._NativeInt8Kernel()
    seam._act_cache = None
    g = _gen(3)
    M, K, N = 512, 6144, 2048
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int8)
    ws = torch.rand(N, generator=g) * 0.01 + 1e-3
    b = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16)
    out = seam._int8_linear_kernel(x.to(DEV), w.to(DEV), ws.to(DEV), b.to(DEV), torch.bfloat16,
                                   True, 256).cpu()
    ref = oracle.int8_linear(oracle.rotate_convrot(x), w, ws, b)
    # identical wherever the row's codes and scale match the oracle's
    q, s = native.quant_rowwise_i8_convrot(x.to(DEV))
    q_ref, s_ref = oracle.quantize_int8_rowwise_convrot(x)
    same_rows = ((q.cpu() == q_ref).all(dim=1) & (s.cpu() == s_ref).reshape(-1))
    assert same_rows.float().mean().item() >= 0.9
    assert torch.equal(out[same_rows], ref[same_rows])
    rel = ((out.float() - ref.float()).abs().max() / ref.float().abs().max()).item()
    assert rel < 0.02
    # against the reference kernel's own fp32 butterflies: identical everywhere
    ref_fwht = oracle.int8_linear(oracle.rotate_convrot_fwht(x), w, ws, b)
    assert torch.equal(out, ref_fwht)
