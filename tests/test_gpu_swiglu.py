"""SwiGLU between FC1 and FC2 on the GPU against the oracle, bit for bit.

Covers the SwiGLU row kernels (silu_mul_split, i8_swiglu_rot, the fused
SwiGLU(+convrot)+quant pre-pass), FC1 with SwiGLU in the GEMM epilogue (both
tile kernels: M < 256 single-CTA, M >= 256 CTA pairs), the bridge
i8_mlp_bridge_prequant, and the comfy seams int8_mlp_bridge /
_try_int8_swiglu_forward.  The shapes and data follow the reference's bridge
tests (tests/test_int8_linear_kernel.py:660-825): int8 activations and weights
uniform in [-128, 128), scales uniform in [1e-4, 1.01e-2), bf16 normal bias.
Every finite bf16 gate value goes through the silu of each route (the rare
exact-silu fallback included).
"""
import sys
from types import ModuleType, SimpleNamespace

import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _same_bits(gpu, ref):
    g = gpu.cpu()
    if g.dtype == torch.bfloat16:
        return torch.equal(g.view(torch.int16), ref.view(torch.int16))
    return torch.equal(g, ref)


def _all_bf16_gates():
    bits = torch.arange(0, 0x10000, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    return bits[torch.isfinite(bits.float())]  # 65280 values


def _bridge_inputs(m, kin, ffn, seed, bias=True):
    g = torch.Generator().manual_seed(seed)
    a = torch.randint(-128, 128, (m, kin), generator=g, dtype=torch.int8)
    w = torch.randint(-128, 128, (2 * ffn, kin), generator=g, dtype=torch.int8)
    rs = torch.rand(m, generator=g) * 0.01 + 1.0e-4
    cs = torch.rand(2 * ffn, generator=g) * 0.01 + 1.0e-4
    b = torch.randn(2 * ffn, generator=g, dtype=torch.bfloat16) if bias else None
    return a, w, rs, cs, b


def _dev(*ts):
    return [t.to(DEV) if t is not None else None for t in ts]


# ----------------------------------------------------------------------------- row kernels
@pytest.mark.parametrize("unit_up", [True, False])
def test_silu_mul_split_every_bf16_gate(native, unit_up):
    F = 256
    gate = _all_bf16_gates().reshape(-1, F)
    gen = torch.Generator().manual_seed(5)
    up = torch.ones_like(gate) if unit_up else torch.randn(gate.shape, generator=gen).bfloat16()
    wide = torch.cat([gate, up], 1)
    assert _same_bits(native.silu_mul_split(wide.to(DEV)), oracle.swiglu(wide))


@pytest.mark.parametrize("M,F,pad", [(7, 100, 0), (33, 96, 24), (5, 1000, 8)])
def test_silu_mul_split_ragged_and_strided(native, M, F, pad):
    gen = torch.Generator().manual_seed(M + F)
    big = (torch.randn(M, 2 * F + pad, generator=gen) * 3).bfloat16()
    wide = big[:, : 2 * F]
    out = native.silu_mul_split(big.to(DEV)[:, : 2 * F])
    assert _same_bits(out, oracle.swiglu(wide))


@pytest.mark.parametrize("M,F", [(130, 512), (3, 14336), (64, 256)])
def test_swiglu_rot_matches_oracle(native, M, F):
    gen = torch.Generator().manual_seed(F)
    wide = (torch.randn(M, 2 * F, generator=gen) * 2).bfloat16()
    assert _same_bits(native.i8_swiglu_rot(wide.to(DEV)), oracle.swiglu_rot(wide))


@pytest.mark.parametrize("rotate", [True, False])
@pytest.mark.parametrize("M,F", [(130, 512), (3, 14336), (20, 768)])
def test_swiglu_quant_matches_oracle(native, rotate, M, F):
    gen = torch.Generator().manual_seed(M * F)
    wide = (torch.randn(M, 2 * F, generator=gen) * 2).bfloat16()
    wide[1] = 0                       # all-zero act row: the 1e-30 scale floor
    wide[2, :F] = 30.0                # silu(gate) ~ gate: large codes
    q, s = native.i8_swiglu_quant(wide.to(DEV), rotate)
    q_ref, s_ref = oracle.swiglu_quant(wide, rotate)
    assert _same_bits(s, s_ref)
    assert _same_bits(q, q_ref)


@pytest.mark.parametrize("rotate", [False, True])
def test_swiglu_quant_every_bf16_gate(native, rotate):
    """Every finite bf16 gate (rotated: every one below 2^119 in magnitude, so
    that a 256-group's butterfly sums stay finite; beyond that the rotation
    overflows to inf/NaN on any implementation)."""
    F = 256
    gate = _all_bf16_gates()
    if rotate:
        gate = gate[gate.float().abs() < 2.0 ** 119]
        gate = torch.cat([gate, torch.zeros((-gate.numel()) % F, dtype=gate.dtype)])
    gate = gate.reshape(-1, F)
    wide = torch.cat([gate, torch.ones_like(gate)], 1)
    q, s = native.i8_swiglu_quant(wide.to(DEV), rotate)
    q_ref, s_ref = oracle.swiglu_quant(wide, rotate)
    assert _same_bits(s, s_ref) and _same_bits(q, q_ref)


# ----------------------------------------------------------------------------- FC1 epilogue
@pytest.mark.parametrize("M,K,F,bias,cs_scalar", [
    (130, 512, 512, True, False),     # the reference's bridge test shape
    (300, 96, 256, False, False),     # CTA-pair tiles
    (300, 512, 200, True, False),     # F not a multiple of the tile or of 32
    (64, 256, 384, True, True),       # one column scale for all columns
    (1, 128, 256, True, False),
    (513, 64, 1000, True, False),
])
def test_fc1_swiglu_epilogue_matches_oracle(native, M, K, F, bias, cs_scalar):
    a, w, rs, cs, b = _bridge_inputs(M, K, F, seed=M + K + F, bias=bias)
    if cs_scalar:
        cs = cs[:1]
    act = native.i8_matmul_nt_fused_cs_swiglu(*_dev(a, w, rs, cs, b))
    assert _same_bits(act, oracle.fc1_swiglu(a, w, rs, cs, b))
    # the materialised route gives the same bytes
    wide = native.i8_matmul_nt_fused_cs(*_dev(a, w, rs, cs, b))
    assert torch.equal(act, native.silu_mul_split(wide))


@pytest.mark.parametrize("M", [4, 256])
def test_fc1_swiglu_epilogue_every_bf16_gate(native, M):
    """acc = 1 everywhere (a[:, 0] = w[:, 0] = 1), row scale 1: gate column f
    dequantizes to exactly col_scale[f], chosen as every finite bf16 value; the
    up columns are 1, so act = bf16(silu(gate))."""
    gates = _all_bf16_gates()
    F, K = gates.numel(), 16
    a = torch.zeros(M, K, dtype=torch.int8)
    a[:, 0] = 1
    w = torch.zeros(2 * F, K, dtype=torch.int8)
    w[:, 0] = 1
    rs = torch.ones(M)
    cs = torch.cat([gates.float(), torch.ones(F)])
    act = native.i8_matmul_nt_fused_cs_swiglu(*_dev(a, w, rs, cs, None))
    ref = oracle.swiglu(torch.cat([gates, torch.ones(F, dtype=torch.bfloat16)]).reshape(1, -1))
    assert _same_bits(act, ref.expand(M, -1).contiguous())


# ----------------------------------------------------------------------------- bridge
def _materialised(native, a, w, rs, cs, b, rotate=True):
    wide = native.i8_matmul_nt_fused_cs(a, w, rs, cs, b)
    return native.i8_swiglu_quant(wide, rotate)


@pytest.mark.parametrize("rotate", [True, False])
def test_bridge_matches_materialised_pipeline_and_oracle(native, rotate):
    a, w, rs, cs, b = _bridge_inputs(130, 512, 512, seed=41)
    ad, wd, rsd, csd, bd = _dev(a, w, rs, cs, b)
    q, s = native.i8_mlp_bridge_prequant(ad, wd, rsd, csd, bd, rotate)
    q2, s2 = _materialised(native, ad, wd, rsd, csd, bd, rotate)
    assert torch.equal(q, q2) and torch.equal(s, s2)
    q_ref, s_ref = oracle.mlp_bridge_prequant(a, w, rs, cs, b, rotate)
    assert _same_bits(s, s_ref) and _same_bits(q, q_ref)


@pytest.mark.parametrize("tile_rows", [0, 128, 1000])
def test_bridge_row_tiles(native, tile_rows):
    a, w, rs, cs, b = _bridge_inputs(8209, 96, 256, seed=43, bias=False)
    ad, wd, rsd, csd, _ = _dev(a, w, rs, cs, b)
    q, s = native.i8_mlp_bridge_prequant(ad, wd, rsd, csd, None, True, tile_rows)
    q2, s2 = _materialised(native, ad, wd, rsd, csd, None)
    assert torch.equal(q, q2) and torch.equal(s, s2)
    rows = torch.tensor([0, 1, 127, 128, 4095, 8191, 8192, 8208])
    q_ref, s_ref = oracle.mlp_bridge_prequant(a[rows], w, rs[rows], cs, None)
    assert _same_bits(q[rows.to(DEV)], q_ref) and _same_bits(s[rows.to(DEV)], s_ref)


def test_bridge_scratch_reuse_is_stream_ordered(native):
    """Back-to-back bridge calls on one stream, each reusing row-tiled scratch."""
    g = torch.Generator().manual_seed(45)
    m, kin, ffn = 385, 96, 256
    w = torch.randint(-128, 128, (2 * ffn, kin), generator=g, dtype=torch.int8).to(DEV)
    cs = (torch.rand(2 * ffn, generator=g) * 0.01 + 1.0e-4).to(DEV)
    inputs = []
    for _ in range(2):
        a = torch.randint(-128, 128, (m, kin), generator=g, dtype=torch.int8).to(DEV)
        rs = (torch.rand(m, generator=g) * 0.01 + 1.0e-4).to(DEV)
        inputs.append((a, rs))
    expected = [_materialised(native, a, w, rs, cs, None) for a, rs in inputs]
    actual = [native.i8_mlp_bridge_prequant(a, w, rs, cs, None, True, 128) for a, rs in inputs]
    torch.cuda.synchronize()
    for (q, s), (q2, s2) in zip(actual, expected):
        assert torch.equal(q, q2) and torch.equal(s, s2)


def test_bridge_h3_shape(native):
    """MiniMax H3's MLP (K 5376, F 14336) at 8193 rows: the bridge against the
    materialised route in full, and the oracle on sampled rows."""
    a, w, rs, cs, b = _bridge_inputs(8193, 5376, 14336, seed=47, bias=False)
    ad, wd, rsd, csd, _ = _dev(a, w, rs, cs, b)
    q, s = native.i8_mlp_bridge_prequant(ad, wd, rsd, csd, None)
    q2, s2 = _materialised(native, ad, wd, rsd, csd, None)
    assert torch.equal(q, q2) and torch.equal(s, s2)
    del q2, s2
    rows = torch.tensor([0, 255, 256, 8192])
    q_ref, s_ref = oracle.mlp_bridge_prequant(a[rows], w, rs[rows], cs, None)
    assert _same_bits(q[rows.to(DEV)], q_ref) and _same_bits(s[rows.to(DEV)], s_ref)


# ----------------------------------------------------------------------------- comfy seams
class _FakeQuantizedTensor:
    def __init__(self, qdata, scale, convrot=True):
        self._qdata = qdata
        self._layout_cls = "TensorWiseINT8Layout"
        self._params = SimpleNamespace(scale=scale, convrot=convrot, convrot_groupsize=256,
                                       transposed=False)
        self.shape = qdata.shape


def _layer(weight, scale, convrot=True, bias=None):
    return SimpleNamespace(weight=_FakeQuantizedTensor(weight, scale, convrot), bias=bias,
                           weight_function=[], bias_function=[], _full_precision_mm=False,
                           comfy_force_cast_weights=False)


@pytest.fixture
def seam(monkeypatch, native):
    from b200q._patches import int8_linear_kernel as k
    ck = ModuleType("comfy_kitchen")
    ck_t = ModuleType("comfy_kitchen.tensor")
    ck_t.QuantizedTensor = _FakeQuantizedTensor
    ck.tensor = ck_t
    monkeypatch.setitem(sys.modules, "comfy_kitchen", ck)
    monkeypatch.setitem(sys.modules, "comfy_kitchen.tensor", ck_t)
    monkeypatch.setattr(k, "_kernel", k._NativeInt8Kernel())
    monkeypatch.setattr(k, "_act_cache", None)
    return k


@pytest.mark.parametrize("fc1_convrot", [True, False])
def test_mlp_bridge_seam_matches_swiglu_route(seam, monkeypatch, fc1_convrot):
    """int8_mlp_bridge == FC1 through the INT8 route, then the SwiGLU FC2 route
    (the reference's test_h3_mlp_bridge_matches_existing_python_pipeline_bit_exact)."""
    g = torch.Generator().manual_seed(47)
    m, hidden, ffn, output = 130, 512, 512, 256
    x = (torch.randn((m, hidden), generator=g) * 0.25).to(DEV, torch.bfloat16).contiguous()
    w1 = torch.randint(-128, 128, (2 * ffn, hidden), generator=g, dtype=torch.int8).to(DEV)
    w2 = torch.randint(-128, 128, (output, ffn), generator=g, dtype=torch.int8).to(DEV)
    s1 = (torch.rand(2 * ffn, generator=g) * 0.01 + 1.0e-4).to(DEV)
    s2 = (torch.rand(output, generator=g) * 0.01 + 1.0e-4).to(DEV)
    b2 = torch.randn(output, generator=g, dtype=torch.bfloat16).to(DEV)
    fc1, fc2 = _layer(w1, s1, fc1_convrot), _layer(w2, s2, True, b2)
    wide = seam._int8_linear_kernel(x, w1, s1, None, torch.bfloat16, fc1_convrot, 256)
    reference = seam._try_int8_swiglu_forward(fc2, wide)
    assert reference is not None
    seam._act_cache = None
    actual = seam.int8_mlp_bridge(fc1, fc2, x)
    assert actual is not None and torch.equal(actual, reference)
    # the FC2 route itself against the oracle: quant of the rotated SwiGLU, then FC2
    q_ref, s_ref = oracle.swiglu_quant(wide.cpu(), True)
    c = oracle.int_mm(q_ref, w2.cpu().t())
    out_ref = oracle.int8_dequant_epilogue(c, s_ref, s2.cpu(), b2.cpu(), torch.bfloat16)
    assert _same_bits(reference, out_ref)
    monkeypatch.setenv("ASFP8_INT8_MLP_BRIDGE", "0")
    assert seam.int8_mlp_bridge(fc1, fc2, x) is None


def test_swiglu_forward_without_convrot(seam):
    g = torch.Generator().manual_seed(48)
    wide = (torch.randn((70, 2 * 320), generator=g) * 2).to(DEV, torch.bfloat16)
    w2 = torch.randint(-128, 128, (96, 320), generator=g, dtype=torch.int8).to(DEV)
    s2 = (torch.rand(96, generator=g) * 0.01 + 1.0e-4).to(DEV)
    out = seam._try_int8_swiglu_forward(_layer(w2, s2, convrot=False), wide)
    q_ref, s_ref = oracle.swiglu_quant(wide.cpu(), False)
    c = oracle.int_mm(q_ref, w2.cpu().t())
    assert _same_bits(out, oracle.int8_dequant_epilogue(c, s_ref, s2.cpu(), None, torch.bfloat16))
