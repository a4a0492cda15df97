"""GPU parity of the QKV attention-layout epilogue and the in-place Q/K
RMSNorm + split-half RoPE.

* The QKV epilogue only changes storage: its q, k, v must equal the dense
  [M, 3HD] fused_cs output split and permuted to [B, H, S, D], byte for byte
  (the reference's test_channelwise_qkv_scatter_is_bit_exact,
  tests/test_int8_linear_kernel.py:334-360, batch 1; batch 2 extends it).
* RMSNorm + RoPE must equal the oracle's fp32 restatement of
  rms_rope_attention_partial (dit_kernels.mm:825-874), whose reduction order
  (torch_rms_sumsq, dit_kernels.mm:60-80) the kernel follows -- bit-exact.
  Shapes and rotary widths from the reference's fused-epilogue test
  (tests/test_int8_linear_kernel.py:363-411).
"""
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _gen(seed):
    return torch.Generator().manual_seed(seed)


@pytest.mark.parametrize("m", [65, 96, 128, 130, 300])
@pytest.mark.parametrize("heads,dim,batch", [(4, 32, 1), (4, 128, 1), (2, 128, 2)])
def test_qkv_scatter_is_bit_exact(native, m, heads, dim, batch):
    if m % batch:
        pytest.skip("rows must split evenly over the batch")
    g = _gen(31)
    kin = 512
    n = 3 * heads * dim
    a = torch.randint(-128, 128, (m, kin), generator=g, dtype=torch.int8).to(DEV)
    b = torch.randint(-128, 128, (n, kin), generator=g, dtype=torch.int8).to(DEV)
    rs = (torch.rand(m, generator=g) * 0.01).to(DEV)
    cs = (torch.rand(n, generator=g) * 0.01).to(DEV)
    bias = torch.randn(n, generator=g).to(torch.bfloat16).to(DEV)
    dense = native.i8_matmul_nt_fused_cs(a, b, rs, cs, bias)
    q, k, v = native.i8_matmul_nt_fused_cs_qkv(a, b, rs, cs, bias, heads, dim, batch)
    expected = oracle.qkv_scatter(dense.cpu(), heads, dim, batch)
    for got, ref in zip((q, k, v), expected):
        assert got.shape == ref.shape
        assert torch.equal(got.cpu(), ref)


def _rope_inputs(g, B, H, S, D, R):
    q = (torch.randn(B, H, S, D, generator=g) * 2).to(torch.bfloat16)
    k = (torch.randn(B, H, S, D, generator=g) * 2).to(torch.bfloat16)
    ang = torch.randn(B * S, R, generator=g)
    fr = torch.stack((ang.cos(), -ang.sin(), ang.sin(), ang.cos()), dim=-1).reshape(B * S, R, 2, 2)
    fr = fr.to(torch.bfloat16).contiguous()
    qw = torch.randn(D, generator=g).to(torch.bfloat16).float()
    kw = torch.randn(D, generator=g).to(torch.bfloat16).float()
    return q, k, fr, qw, kw


@pytest.mark.parametrize("S", [65, 259])
@pytest.mark.parametrize("R", [1, 16, 48, 64])
def test_rms_rope_matches_oracle_bit_exact(native, S, R):
    g = _gen(37)
    q, k, fr, qw, kw = _rope_inputs(g, 1, 4, S, 128, R)
    rq, rk = oracle.rms_rope_partial(q, k, fr, qw, kw, 1e-6)
    qd, kd = q.to(DEV).contiguous(), k.to(DEV).contiguous()
    native.rms_rope_partial_(qd, kd, fr.to(DEV), qw.to(DEV), kw.to(DEV), 1e-6)
    assert torch.equal(qd.cpu(), rq)
    assert torch.equal(kd.cpu(), rk)


@pytest.mark.parametrize("B,H,S,D,R", [(2, 3, 40, 64, 16), (1, 2, 33, 256, 100), (2, 2, 17, 128, 0)])
def test_rms_rope_other_head_dims(native, B, H, S, D, R):
    g = _gen(41)
    q, k, fr, qw, kw = _rope_inputs(g, B, H, S, D, max(R, 1))
    if R == 0:
        fr = fr[:, :0].contiguous()
    rq, rk = oracle.rms_rope_partial(q, k, fr, qw, kw, 1e-5)
    qd, kd = q.to(DEV).contiguous(), k.to(DEV).contiguous()
    native.rms_rope_partial_(qd, kd, fr.to(DEV), qw.to(DEV), kw.to(DEV), 1e-5)
    assert torch.equal(qd.cpu(), rq)
    assert torch.equal(kd.cpu(), rk)


def test_qkv_projection_norm_rope_chain(native):
    """The H3 chain: INT8 QKV projection into attention layout, then in-place
    Q/K norm + RoPE; V untouched (test_qkv_rms_rope_epilogue_matches_two_kernel_chain)."""
    g = _gen(43)
    m, kin, heads, dim, R = 259, 512, 4, 128, 48
    n = 3 * heads * dim
    a = torch.randint(-128, 128, (m, kin), generator=g, dtype=torch.int8)
    b = torch.randint(-128, 128, (n, kin), generator=g, dtype=torch.int8)
    rs = torch.rand(m, generator=g) * 0.01 + 1e-5
    cs = torch.rand(n, generator=g) * 0.01 + 1e-5
    bias = torch.randn(n, generator=g).to(torch.bfloat16)
    _, _, fr, qw, kw = _rope_inputs(g, 1, heads, m, dim, R)
    dense = oracle.int8_dequant_epilogue(oracle.int_mm(a, b.t()), rs.reshape(-1, 1), cs, bias)
    eq, ek, ev = oracle.qkv_scatter(dense, heads, dim, 1)
    eq, ek = oracle.rms_rope_partial(eq, ek, fr, qw, kw, 1e-6)
    q, k, v = native.i8_matmul_nt_fused_cs_qkv(a.to(DEV), b.to(DEV), rs.to(DEV), cs.to(DEV),
                                               bias.to(DEV), heads, dim, 1)
    native.rms_rope_partial_(q, k, fr.to(DEV), qw.to(DEV), kw.to(DEV), 1e-6)
    assert torch.equal(q.cpu(), eq)
    assert torch.equal(k.cpu(), ek)
    assert torch.equal(v.cpu(), ev)


# ----------------------------------------------------------------------------- fused epilogue
def _qkv_inputs(g, m, kin, heads, dim, bias):
    n = 3 * heads * dim
    a = torch.randint(-128, 128, (m, kin), generator=g, dtype=torch.int8)
    b = torch.randint(-128, 128, (n, kin), generator=g, dtype=torch.int8)
    rs = torch.rand(m, generator=g) * 0.01 + 1e-5
    cs = torch.rand(n, generator=g) * 0.01 + 1e-5
    bb = torch.randn(n, generator=g).to(torch.bfloat16) if bias else None
    return a, b, rs, cs, bb


@pytest.mark.parametrize("m,heads,R,batch,bias", [
    (130, 4, 48, 1, True),    # the reference test's shape class (single-CTA tiles)
    (259, 4, 64, 1, False),   # CTA-pair tiles, full rotary width
    (300, 3, 8, 2, True),     # odd head count: a tile holds the last Q and the first K head
    (96, 2, 0, 2, True),      # norm only
    (8193, 2, 32, 1, True),   # ragged last tile
])
def test_fused_qkv_norm_rope_epilogue_bit_exact(native, m, heads, R, batch, bias):
    """One launch (i8_matmul2d_nt_fused_cs_qkv_rms_rope) against the oracle chain
    (dense dequant -> attention layout -> RMSNorm + RoPE) and against the GPU's
    two-launch chain, bit for bit (test_qkv_rms_rope_epilogue_matches_two_kernel_chain,
    tests/test_int8_linear_kernel.py:363-411)."""
    g = _gen(47 + m)
    dim, kin = 128, 512
    a, b, rs, cs, bb = _qkv_inputs(g, m, kin, heads, dim, bias)
    S = m // batch
    _, _, fr, qw, kw = _rope_inputs(g, batch, heads, S, dim, max(R, 1))
    if R == 0:
        fr = fr[:, :0].contiguous()
    dense = oracle.int8_dequant_epilogue(oracle.int_mm(a, b.t()), rs.reshape(-1, 1), cs, bb)
    eq, ek, ev = oracle.qkv_scatter(dense, heads, dim, batch)
    eq, ek = oracle.rms_rope_partial(eq, ek, fr, qw, kw, 1e-6)
    dv = [t.to(DEV) if t is not None else None for t in (a, b, rs, cs, bb, fr, qw, kw)]
    q, k, v = native.i8_matmul_nt_fused_cs_qkv_rms_rope(*dv, heads, dim, 1e-6, batch)
    assert torch.equal(q.cpu(), eq)
    assert torch.equal(k.cpu(), ek)
    assert torch.equal(v.cpu(), ev)
    q2, k2, v2 = native.i8_matmul_nt_fused_cs_qkv(*dv[:5], heads, dim, batch)
    native.rms_rope_partial_(q2, k2, dv[5], dv[6], dv[7], 1e-6)
    assert torch.equal(q, q2) and torch.equal(k, k2) and torch.equal(v, v2)


def test_qkv_seams(native, monkeypatch):
    """int8_qkv_prequant / int8_qkv_rms_rope_prequant on an int8_tensorwise layer
    (rotary width 48 with the fused epilogue on and off; 20: always the scatter +
    norm/RoPE launches)."""
    import sys
    from types import ModuleType, SimpleNamespace
    from b200q._patches import int8_linear_kernel as seam

    class QT:
        def __init__(self, q, s):
            self._qdata, self._layout_cls = q, "TensorWiseINT8Layout"
            self._params = SimpleNamespace(scale=s, convrot=False, convrot_groupsize=256,
                                           transposed=False)

    ck, ckt = ModuleType("comfy_kitchen"), ModuleType("comfy_kitchen.tensor")
    ckt.QuantizedTensor = QT
    monkeypatch.setitem(sys.modules, "comfy_kitchen", ck)
    monkeypatch.setitem(sys.modules, "comfy_kitchen.tensor", ckt)
    monkeypatch.setattr(seam, "_kernel", seam._NativeInt8Kernel())
    monkeypatch.setattr(seam, "_act_cache", None)
    g = _gen(53)
    m, hidden, heads, dim = 259, 512, 2, 128
    x = (torch.randn(m, hidden, generator=g) * 0.5).to(torch.bfloat16)
    w = torch.randint(-128, 128, (3 * heads * dim, hidden), generator=g, dtype=torch.int8)
    ws = torch.rand(3 * heads * dim, generator=g) * 0.01 + 1e-4
    bias = torch.randn(3 * heads * dim, generator=g).to(torch.bfloat16)
    layer = SimpleNamespace(weight=QT(w.to(DEV), ws.to(DEV)), bias=bias.to(DEV), weight_function=[],
                            bias_function=[], _full_precision_mm=False,
                            comfy_force_cast_weights=False)
    xd = x.to(DEV)
    q8, xs = oracle.quantize_int8_rowwise(x)
    dense = oracle.int8_dequant_epilogue(oracle.int_mm(q8, w.t()), xs, ws, bias)
    eq, ek, ev = oracle.qkv_scatter(dense, heads, dim, 1)
    q, k, v = seam.int8_qkv_prequant(layer, xd, heads, dim)
    assert torch.equal(q.cpu(), eq) and torch.equal(k.cpu(), ek) and torch.equal(v.cpu(), ev)
    for R, fused in ((48, "1"), (48, "0"), (20, "1")):
        monkeypatch.setenv("B200Q_QKV_FUSED_NORM_ROPE", fused)
        _, _, fr, qw, kw = _rope_inputs(g, 1, heads, m, dim, R)
        rq, rk = oracle.rms_rope_partial(eq, ek, fr, qw, kw, 1e-6)
        out = seam.int8_qkv_rms_rope_prequant(layer, xd, fr.to(DEV), qw.to(DEV), kw.to(DEV), heads,
                                              dim, 1e-6)
        assert out is not None
        assert torch.equal(out[0].cpu(), rq) and torch.equal(out[1].cpu(), rk)
        assert torch.equal(out[2].cpu(), ev)
    monkeypatch.setenv("ASFP8_INT8_QKV_NORM_ROPE", "0")
    assert seam.int8_qkv_rms_rope_prequant(layer, xd, fr.to(DEV), qw.to(DEV), kw.to(DEV), heads,
                                           dim, 1e-6) is None
