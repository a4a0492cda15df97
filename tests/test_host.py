"""CPU tier: the C-ABI library, the seam patches' host logic (with fake comfy
modules, as the reference's tests do: tests/test_int8_linear_kernel.py:53-84,
tests/test_scaled_mm_fp8.py:103-145, tests/test_linear_fp8_w8a16.py:47-94),
and the multi-rank row sharding (gloo, world size 2).  No compute kernel runs."""
import ctypes
import os
import re
import sys
from types import ModuleType, SimpleNamespace

import pytest
import torch

import b200q
from b200q._patches import (_common, _native, int8_linear, int8_linear_kernel, int_mm,
                            linear_fp8, linear_fp8_w8a16, scaled_mm_fp8)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


# ----------------------------------------------------------------------------- C ABI
def _declared_symbols():
    hdr = open(os.path.join(ROOT, "include", "b200q.h")).read()
    return sorted(set(re.findall(r"B200Q_API\s+[\w\s\*]+?\b(b200q_\w+)\s*\(", hdr)))


def test_header_declares_the_abi():
    syms = _declared_symbols()
    for s in ("b200q_quant_rowwise_i8", "b200q_i8_matmul_nt", "b200q_i8_matmul_nt_dequant",
              "b200q_i8_linear", "b200q_fp8_scaled_mm", "b200q_fp8_quant_tensorwise",
              "b200q_w8a16_linear", "b200q_w8a16_workspace_size", "b200q_fp8_decode"):
        assert s in syms


def test_library_loads_and_exports_every_declared_symbol():
    path = _native.library_path()
    assert os.path.exists(path), "run __graft_entry__.build() first"
    lib = ctypes.CDLL(path)
    for s in _declared_symbols():
        assert hasattr(lib, s), s
    L = _native.lib()
    assert L.b200q_version() >= 1
    assert L.b200q_status_string(1) == b"invalid argument"


def test_abi_rejects_bad_arguments_without_a_gpu():
    """Argument validation happens on the host before any device query."""
    L = _native.lib()
    assert L.b200q_i8_matmul_nt(None, 16, None, 16, None, 16, 4, 4, 16, None) == 1
    assert L.b200q_quant_rowwise_i8(None, 0, 4, 16, 16, None, 16, None, None) == 1
    assert L.b200q_fp8_scaled_mm(None, 16, None, 16, None, 0, None, 0, None, None, 0, 0, None, 0,
                                 16, 4, 4, 16, None) == 1
    assert L.b200q_fp8_decode(None, 4, 0, None, 0, None) == 1
    assert L.b200q_silu_mul_split(None, 32, 4, 16, None, 16, None) == 1
    assert L.b200q_i8_swiglu_quant(None, 32, 4, 16, 1, None, 16, None, None) == 1
    assert L.b200q_i8_matmul_nt_dequant_swiglu(None, 16, None, 16, None, None, 1, None, None, 8,
                                               4, 15, 16, None) == 1
    assert L.b200q_i8_mlp_bridge_prequant(None, 16, None, 16, None, None, 1, None, 4, 512, 16, 1,
                                          0, None, None, 256, None, None) == 1
    assert L.b200q_i8_matmul_nt_dequant_qkv_rms_rope(None, 16, None, 16, None, None, 1, None, None,
                                                     None, None, 1, 1, None, 8, None, None, 1e-6,
                                                     4, 384, 16, None) == 1


def test_w8a16_workspace_size_follows_the_routes(monkeypatch):
    """The size query covers the route a call takes (a host query, no device
    work): the planes GEMV's planes + plane scales for M <= 4 (bf16, 2 planes;
    with B200Q_W8A16_PGEMV=1 also fp16's 3 planes for M <= 2), nothing for the
    decode-in-kernel GEMV (M 5..16 at K <= 4096), the planes route above 16."""
    L = _native.lib()
    N, K = 12288, 3072
    monkeypatch.delenv("B200Q_W8A16_PGEMV", raising=False)
    monkeypatch.delenv("B200Q_W8A16_PLANES", raising=False)
    for M in (1, 2, 3, 4):
        assert L.b200q_w8a16_workspace_size(M, N, K) == -(-2 * M * K // 256) * 256 + 2 * M * 4
    for M in (5, 8, 16):
        assert L.b200q_w8a16_workspace_size(M, N, K) == 0
    assert L.b200q_w8a16_workspace_size(17, N, K) > 0
    monkeypatch.setenv("B200Q_W8A16_PGEMV", "0")
    assert L.b200q_w8a16_workspace_size(1, N, K) == 0
    monkeypatch.setenv("B200Q_W8A16_PGEMV", "1")
    assert L.b200q_w8a16_workspace_size(2, N, K) == 3 * 2 * K + 3 * 2 * 4


def test_torch_ops_registered_with_fake_kernels():
    for name in ("quant_rowwise_i8", "int_mm", "i8_matmul_nt", "i8_matmul_nt_fused",
                 "i8_matmul_nt_fused_cs", "i8_linear", "fp8_quant_tensorwise", "fp8_scaled_mm",
                 "w8a16_linear", "fp8_decode", "silu_mul_split", "i8_swiglu_rot",
                 "i8_swiglu_quant", "i8_matmul_nt_fused_cs_swiglu", "i8_mlp_bridge_prequant",
                 "i8_matmul_nt_fused_cs_qkv_rms_rope"):
        assert hasattr(torch.ops.b200q, name)
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        x = torch.empty(5, 64, dtype=torch.bfloat16, device="cuda")
        w = torch.empty(32, 64, dtype=torch.float8_e4m3fn, device="cuda")
        assert torch.ops.b200q.w8a16_linear(x, w).shape == (5, 32)
        q, s = torch.ops.b200q.quant_rowwise_i8(x)
        assert q.dtype == torch.int8 and s.shape == (5, 1)
        q, s = torch.ops.b200q.i8_swiglu_quant(x)
        assert q.shape == (5, 32) and s.shape == (5, 1)
        a8 = torch.empty(5, 64, dtype=torch.int8, device="cuda")
        w1 = torch.empty(512, 64, dtype=torch.int8, device="cuda")
        rs, cs = torch.empty(5, device="cuda"), torch.empty(512, device="cuda")
        assert torch.ops.b200q.i8_matmul_nt_fused_cs_swiglu(a8, w1, rs, cs).shape == (5, 256)
        q, s = torch.ops.b200q.i8_mlp_bridge_prequant(a8, w1, rs, cs)
        assert q.shape == (5, 256) and q.dtype == torch.int8 and s.shape == (5, 1)


def test_ops_fail_loudly_off_gpu():
    with pytest.raises(RuntimeError):
        _native.quant_rowwise_i8(torch.zeros(2, 8, dtype=torch.bfloat16))


# ----------------------------------------------------------------------------- switches
def test_master_switch_implies_routes_and_explicit_wins():
    env = {"ASFP8_NATIVE": "1", "ASFP8_INT8_EXT": "0"}
    implied = _common.apply_native_master_switch(env)
    assert env["ASFP8_FP8_EXT"] == "1" and env["ASFP8_FP8_SGEMM"] == "1"
    assert env["ASFP8_INT8_EXT"] == "0" and "ASFP8_INT8_EXT" not in implied
    env = {"ASFP8_NATIVE": "0"}
    assert _common.apply_native_master_switch(env) == [] and "ASFP8_FP8_EXT" not in env


def test_master_switch_noop_without_b200(monkeypatch):
    monkeypatch.setattr(_common, "is_b200", lambda device=None: False)
    env = {}
    assert _common.apply_native_master_switch(env) == [] and env == {}


@pytest.mark.parametrize("mod,flag", [(int_mm, "ASFP8_INT8_EXT"), (scaled_mm_fp8, "ASFP8_FP8_EXT"),
                                      (linear_fp8, "ASFP8_FP8_EXT"), (int8_linear, "ASFP8_INT8_EXT"),
                                      (int8_linear_kernel, "ASFP8_INT8_EXT")])
def test_install_noop_without_flag(monkeypatch, mod, flag):
    monkeypatch.delenv(flag, raising=False)
    monkeypatch.setattr(mod, "_installed", False)
    mod.install()
    assert mod._installed is False


def test_install_noop_without_gpu(monkeypatch):
    """Flags set, but no B200: nothing is patched (the seams stay stock torch)."""
    for v in ("ASFP8_INT8_EXT", "ASFP8_FP8_EXT", "ASFP8_FP8_SGEMM"):
        monkeypatch.setenv(v, "1")
    orig = (torch._int_mm, torch._scaled_mm, torch.nn.functional.linear)
    for mod in (int_mm, scaled_mm_fp8, linear_fp8, linear_fp8_w8a16, int8_linear):
        monkeypatch.setattr(mod, "_installed", False)
        mod.install()
        assert mod._installed is False
    assert (torch._int_mm, torch._scaled_mm, torch.nn.functional.linear) == orig


def test_bootstrap_bisection(monkeypatch, capsys):
    monkeypatch.setenv("ASFP8_NATIVE", "0")
    monkeypatch.setenv("ASFP8_ENABLE_ONLY", "int_mm,scaled_mm_fp8")
    attempted = b200q.bootstrap()
    assert attempted == ["scaled_mm_fp8", "int_mm"]
    monkeypatch.delenv("ASFP8_ENABLE_ONLY")
    monkeypatch.setenv("ASFP8_DISABLE", "linear_fp8")
    assert "linear_fp8" not in b200q.bootstrap()


# ----------------------------------------------------------------------------- INT8 seam
def test_int8_wrapper_falls_back_off_cuda(monkeypatch):
    sentinel, called = object(), {}

    def fake_orig(x, w, ws, bias, out_dtype, convrot, gs):
        called["hit"] = True
        return sentinel

    monkeypatch.setattr(int8_linear_kernel, "_kernel", None)
    monkeypatch.setattr(int8_linear_kernel, "_orig_int8_linear", fake_orig)
    out = int8_linear_kernel._int8_linear_kernel(torch.zeros(4, 8), torch.zeros(8, 8, dtype=torch.int8),
                                                 torch.ones(1))
    assert out is sentinel and called["hit"]


@pytest.fixture
def fake_comfy(monkeypatch):
    comfy = ModuleType("comfy")
    ops = ModuleType("comfy.ops")
    comfy.ops = ops

    class Linear:
        def forward(self, input, *a, **k):
            return ("orig", input)

    def factory(quant_config=None, compute_dtype=torch.bfloat16, full_precision_mm=False,
                disabled=()):
        return type("Operations", (), {"_quant_config": quant_config,
                                       "_compute_dtype": compute_dtype,
                                       "_full_precision_mm": full_precision_mm,
                                       "_disabled": disabled, "Linear": Linear})

    ops.mixed_precision_ops = factory
    calls = []

    def lia(*args, **kwargs):
        calls.append((args, kwargs))
        return "lia"

    ops.linear_input_act = lia
    ck = ModuleType("comfy_kitchen")
    ck_be = ModuleType("comfy_kitchen.backends")
    ck_eager = ModuleType("comfy_kitchen.backends.eager")
    ck_q = ModuleType("comfy_kitchen.backends.eager.quantization")
    ck_q.int8_linear = lambda *a, **k: "eager"
    for name, m in (("comfy", comfy), ("comfy.ops", ops), ("comfy_kitchen", ck),
                    ("comfy_kitchen.backends", ck_be), ("comfy_kitchen.backends.eager", ck_eager),
                    ("comfy_kitchen.backends.eager.quantization", ck_q)):
        monkeypatch.setitem(sys.modules, name, m)
    monkeypatch.setattr(int8_linear_kernel, "_installed", False)
    monkeypatch.setattr(int8_linear_kernel, "_kernel", None)
    monkeypatch.setattr(int8_linear_kernel, "_load_kernel", lambda: object())
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setenv("ASFP8_INT8_EXT", "1")
    int8_linear_kernel.install()
    assert int8_linear_kernel._installed
    return ops, calls, Linear


@pytest.mark.parametrize("positional", [False, True])
@pytest.mark.parametrize("full_precision", [False, True])
def test_factory_enables_only_int8_and_preserves_precision_requests(fake_comfy, positional,
                                                                     full_precision):
    ops, _, _ = fake_comfy
    disabled = {"int8_tensorwise", "nvfp4", "convrot_w4a4"}
    qc = {"layer": {"full_precision_matrix_mult": True}}
    if positional:
        res = ops.mixed_precision_ops(qc, torch.float16, full_precision, disabled)
    else:
        res = ops.mixed_precision_ops(quant_config=qc, compute_dtype=torch.float16,
                                      full_precision_mm=full_precision, disabled=disabled)
    assert set(res._disabled) == {"nvfp4", "convrot_w4a4"}
    assert disabled == {"int8_tensorwise", "nvfp4", "convrot_w4a4"}
    assert res._full_precision_mm is full_precision and res._quant_config is qc
    assert res.Linear._asfp8_int8_patched


def test_factory_keeps_defaults_and_forward_falls_through(fake_comfy):
    ops, _, Linear = fake_comfy
    res = ops.mixed_precision_ops()
    assert res._disabled == () and res._full_precision_mm is False
    # plain (non-quantized) layer on CPU: the original forward answers
    assert res.Linear().forward("x") == ("orig", "x")


def test_linear_input_act_preserves_extended_contract(fake_comfy, monkeypatch):
    ops, calls, _ = fake_comfy
    native_calls = []
    monkeypatch.setattr(int8_linear_kernel, "_try_int8_swiglu_forward",
                        lambda *a: native_calls.append(a))
    lin, x = object(), object()
    assert ops.linear_input_act(lin, x, "rms_norm", "w", 1e-5) == "lia"
    assert ops.linear_input_act(lin, x, "swiglu", "w", 1e-5, "r", 0.5) == "lia"
    assert ops.linear_input_act(lin, x, "swiglu", residual="r") == "lia"
    assert len(calls) == 3 and native_calls == []
    # three-argument SwiGLU: the native route is tried, comfy's helper answers on None
    assert ops.linear_input_act(lin, x, "swiglu") == "lia"
    assert native_calls == [(lin, x)]


def test_linear_input_act_routes_three_argument_swiglu(fake_comfy, monkeypatch):
    ops, calls, _ = fake_comfy
    result = object()
    monkeypatch.setattr(int8_linear_kernel, "_try_int8_swiglu_forward", lambda *a: result)
    assert ops.linear_input_act(object(), object(), "swiglu") is result
    monkeypatch.setenv("ASFP8_INT8_SWIGLU", "0")
    assert ops.linear_input_act(object(), object(), "swiglu") == "lia"
    assert len(calls) == 1


class _FakeQT:
    def __init__(self, qdata, scale, convrot=True, layout="TensorWiseINT8Layout"):
        self._qdata, self._layout_cls = qdata, layout
        self._params = SimpleNamespace(scale=scale, convrot=convrot, convrot_groupsize=256,
                                       transposed=False)


def _fake_layer(w, s, convrot=True, **kw):
    d = dict(weight=_FakeQT(w, s, convrot), bias=None, weight_function=[], bias_function=[],
             _full_precision_mm=False, comfy_force_cast_weights=False)
    d.update(kw)
    return SimpleNamespace(**d)


def test_mlp_bridge_eligibility_and_call_sequence(monkeypatch):
    """int8_mlp_bridge's eligibility (int8_linear_kernel_mps.py:541-583) and its
    route: cached quant of x -> i8_mlp_bridge_prequant -> FC2 epilogue selection."""
    ck = ModuleType("comfy_kitchen")
    ck_t = ModuleType("comfy_kitchen.tensor")
    ck_t.QuantizedTensor = _FakeQT
    monkeypatch.setitem(sys.modules, "comfy_kitchen", ck)
    monkeypatch.setitem(sys.modules, "comfy_kitchen.tensor", ck_t)
    seen = []

    class K:
        def i8_quant_rowwise(self, x):
            seen.append("quant")
            return torch.zeros(x.shape, dtype=torch.int8), torch.ones(x.shape[0], 1)

        def i8_mlp_bridge_prequant(self, a, w1, rs, cs, bias=None):
            seen.append(("bridge", tuple(a.shape), tuple(w1.shape)))
            return torch.zeros(a.shape[0], w1.shape[0] // 2, dtype=torch.int8), torch.ones(
                a.shape[0], 1)

        def i8_matmul2d_nt_fused_cs(self, a, b, rs, cs, bias=None, *x, out_dtype=None):
            seen.append("fc2")
            return torch.zeros(a.shape[0], b.shape[0], dtype=out_dtype)

    monkeypatch.setattr(int8_linear_kernel, "_kernel", K())
    monkeypatch.setattr(int8_linear_kernel, "_act_cache", None)
    x = SimpleNamespace()  # replaced per case below
    w1, w2 = torch.zeros(1024, 64, dtype=torch.int8), torch.zeros(96, 512, dtype=torch.int8)
    fc1 = _fake_layer(w1, torch.ones(1024), convrot=False)
    fc2 = _fake_layer(w2, torch.ones(96))

    class CudaLike(torch.Tensor):
        """A CPU tensor that reports device cuda (the seam's eligibility only)."""
        @property
        def device(self):
            return torch.device("cuda")

    x = torch.zeros(10, 64, dtype=torch.bfloat16).as_subclass(CudaLike)
    out = int8_linear_kernel.int8_mlp_bridge(fc1, fc2, x)
    assert out is not None and tuple(out.shape) == (10, 96)
    assert seen == ["quant", ("bridge", (10, 64), (1024, 64)), "fc2"]
    # ineligible: FC2 without convrot, FC1 rows not a multiple of 512, env switch, CPU x
    assert int8_linear_kernel.int8_mlp_bridge(fc1, _fake_layer(w2, torch.ones(96), False), x) is None
    bad_w1 = torch.zeros(768, 64, dtype=torch.int8)
    assert int8_linear_kernel.int8_mlp_bridge(
        _fake_layer(bad_w1, torch.ones(768), False), _fake_layer(
            torch.zeros(96, 384, dtype=torch.int8), torch.ones(96)), x) is None
    assert int8_linear_kernel.int8_mlp_bridge(fc1, fc2, torch.zeros(10, 64, dtype=torch.bfloat16)) is None
    monkeypatch.setenv("ASFP8_INT8_MLP_BRIDGE", "0")
    assert int8_linear_kernel.int8_mlp_bridge(fc1, fc2, x) is None


def test_int8_epilogue_selection(monkeypatch):
    """Scalar scale -> fused tensorwise; [N,1] -> channelwise; f32 out -> int32 + chunked."""
    seen = []

    class K:
        def i8_matmul2d_nt_fused(self, a, b, rs, bias=None):
            seen.append("fused")
            return torch.zeros(a.shape[0], b.shape[0])

        def i8_matmul2d_nt_fused_cs(self, a, b, rs, cs, bias=None, *x, out_dtype=None):
            seen.append("cs")
            return torch.zeros(a.shape[0], b.shape[0])

        def i8_matmul2d_nt(self, a, b):
            seen.append("int32")
            return (a.long() @ b.long().t()).to(torch.int32)

    monkeypatch.setattr(int8_linear_kernel, "_kernel", K())
    x8, xs = torch.ones(3, 4, dtype=torch.int8), torch.ones(3, 1)
    w = torch.ones(5, 4, dtype=torch.int8)
    int8_linear_kernel._int8_linear_prequant(x8, xs, w, torch.ones(1), None, torch.bfloat16, (3, 4))
    int8_linear_kernel._int8_linear_prequant(x8, xs, w, torch.ones(5, 1), None, torch.bfloat16, (3, 4))
    out = int8_linear_kernel._int8_linear_prequant(x8, xs, w, torch.ones(5, 1), None,
                                                   torch.float32, (3, 4))
    assert seen == ["fused", "cs", "int32"]
    assert torch.equal(out, torch.full((3, 5), 4.0))


# ----------------------------------------------------------------------------- FP8 seams
def test_scaled_mm_eligibility(monkeypatch):
    monkeypatch.setenv("ASFP8_FP8_EXT", "1")
    a = torch.empty(4, 32, dtype=torch.float8_e4m3fn)
    b = torch.empty(32, 8, dtype=torch.float8_e4m3fn)
    assert not scaled_mm_fp8._fast_eligible(a, b)  # CPU tensors
    monkeypatch.delenv("ASFP8_FP8_EXT")
    assert not scaled_mm_fp8._fast_eligible(a, b)


def test_scaled_mm_passthrough_for_cpu(monkeypatch):
    called = {}

    def orig(*a, **k):
        called["k"] = k
        return "orig"

    monkeypatch.setattr(scaled_mm_fp8, "_original", orig)
    monkeypatch.setenv("ASFP8_FP8_EXT", "1")
    a = torch.empty(4, 32, dtype=torch.float8_e4m3fn)
    b = torch.empty(32, 8, dtype=torch.float8_e4m3fn)
    assert scaled_mm_fp8._cuda_scaled_mm(a, b, out_dtype=torch.bfloat16) == "orig"
    assert called["k"]["out_dtype"] == torch.bfloat16


def test_w8a16_eligibility_predicate():
    m = SimpleNamespace(weight=torch.empty(64, 32, dtype=torch.float8_e4m3fn), weight_function=[],
                        bias_function=[])
    x = torch.empty(3, 32, dtype=torch.bfloat16)
    assert not linear_fp8_w8a16._eligible(m, x)  # CPU weight
    m.weight = torch.empty(64, 32, dtype=torch.float8_e5m2)
    assert not linear_fp8_w8a16._eligible(m, x)


def test_linear_fp8_fast_path_untouched():
    x, w = torch.randn(2, 4), torch.randn(3, 4)
    assert torch.equal(linear_fp8._patched_linear(x, w), torch.nn.functional.linear(x, w))


def test_int8_fast_hook_patches_module(monkeypatch):
    mod = ModuleType("int8_quant")
    dyn = lambda *a: "dyn"
    mod.int8_forward_dynamic = dyn
    mod.int8_forward_dynamic_per_row = lambda *a: "dyn_pr"
    monkeypatch.setattr(int8_linear, "_patched", False)
    assert int8_linear.patch_module(mod)
    assert mod.int8_forward_dynamic.__wrapped__ is dyn
    assert not int8_linear.patch_module(mod)  # once per process
    # CPU call goes to the node's own function
    x, w, ws = torch.zeros(2, 4), torch.zeros(3, 4, dtype=torch.int8), torch.ones(1)
    assert mod.int8_forward_dynamic(x, w, ws, None, torch.bfloat16) == "dyn"
    assert mod.int8_forward_dynamic_per_row(x, w, ws, None, torch.bfloat16) == "dyn_pr"


def test_after_import_patches_a_module_imported_later(monkeypatch, tmp_path):
    """The deferred path: the target module is imported after the hook is set
    (int8-fast loading after this pack), from a package directory on disk."""
    pkg = tmp_path / "fake_int8_fast_pkg"
    pkg.mkdir()
    (pkg / "__init__.py").write_text("")
    (pkg / "int8_quant.py").write_text(
        "def int8_forward_dynamic(*a):\n    return 'dyn'\n"
        "def int8_forward_dynamic_per_row(*a):\n    return 'dyn_pr'\n")
    monkeypatch.syspath_prepend(str(tmp_path))
    monkeypatch.setattr(int8_linear, "_patched", False)
    monkeypatch.setattr(_common._HOOK, "pending", {})
    seen = []
    ran_now = _common.after_import("int8_quant", lambda m: seen.append(m) or
                                   int8_linear.patch_module(m), required=int8_linear.TARGETS)
    assert ran_now is False and seen == []
    try:
        import fake_int8_fast_pkg.int8_quant as iq
        assert seen == [iq] and iq.int8_forward_dynamic.__wrapped__.__name__ == "int8_forward_dynamic"
        assert iq.__loader__.__class__.__name__ != "_PatchingLoader"
        x, w, ws = torch.zeros(2, 4), torch.zeros(3, 4, dtype=torch.int8), torch.ones(1)
        assert iq.int8_forward_dynamic_per_row(x, w, ws, None, torch.bfloat16) == "dyn_pr"
    finally:
        for name in ("fake_int8_fast_pkg.int8_quant", "fake_int8_fast_pkg"):
            sys.modules.pop(name, None)
        if _common._HOOK in sys.meta_path:
            sys.meta_path.remove(_common._HOOK)


def test_abi_limits_match_the_bindings():
    hdr = open(os.path.join(ROOT, "include", "b200q.h")).read()
    assert f"#define B200Q_CONVROT_MAX_K {_native.CONVROT_MAX_K}" in hdr
    assert f"#define B200Q_SWIGLU_MAX_F {_native.SWIGLU_MAX_F}" in hdr


def test_wan_fp16_hook_eligibility(monkeypatch):
    """maybe_prequant declines without the opt-in, for CPU tensors, other shapes
    and a missing kernel method (reference tests/test_wan_fp16.py:95-99)."""
    from b200q._patches import wan_fp16
    x = torch.zeros(1, 5120, dtype=torch.int8)
    w = torch.zeros(5120, 5120, dtype=torch.int8)
    k = SimpleNamespace(i8_matmul2d_nt_fused_cs_half=lambda *a: pytest.fail("must not run"))
    with torch.inference_mode():
        monkeypatch.delenv("ASFP8_DIT_EXT", raising=False)
        assert wan_fp16.maybe_prequant(k, x, torch.ones(1), w, torch.ones(5120), None,
                                       (1, 1, 5120)) is None
        monkeypatch.setenv("ASFP8_DIT_EXT", "1")
        assert wan_fp16.maybe_prequant(None, x, torch.ones(1), w, torch.ones(5120), None,
                                       (1, 1, 5120)) is None
        assert wan_fp16.maybe_prequant(k, x, torch.ones(1), w, torch.ones(5120), None,
                                       (1, 1, 5120)) is None  # CPU tensors
        w2 = torch.zeros(4096, 5120, dtype=torch.int8)
        assert wan_fp16.maybe_prequant(k, x, torch.ones(1), w2, torch.ones(4096), None,
                                       (1, 1, 5120)) is None  # not a Wan shape


def test_library_source_makes_no_device_allocation():
    """The C ABI never allocates device memory (the caller passes every buffer;
    the allocation-free entry uses a static array): no allocation or free call
    appears in the library's sources."""
    csrc = os.path.join(ROOT, "comfyui-applesilicon-optimized_b200", "csrc")
    pat = re.compile(r"\b(cudaMalloc\w*|cudaFree\w*|cuMemAlloc\w*|cuMemFree\w*|cudaMallocAsync)\s*\(")
    for name in sorted(os.listdir(csrc)):
        if name.endswith((".cu", ".cuh", ".h")):
            text = open(os.path.join(csrc, name)).read()
            assert not pat.search(text), f"{name} allocates device memory"
