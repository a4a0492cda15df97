"""The allocation-free W8A16 entry point, called through the C ABI.

b200q_w8a16_linear_noalloc exists for callers that cannot allocate device
memory themselves (a host that only hands this library buffers it registered up
front, or a runtime whose device-memory budget is fixed before the model runs).
Its split-K scratch is a static device array inside the library.  These tests
check, through ctypes on the shared library, that two calls in a row match the
workspace-taking entry point within the tolerance the other W8A16 tests use,
that the calls allocate no device memory, and that an oversized shape is
rejected with the clear error status without launching anything.

The file name sorts last so that a run stopping at the first failure has
already run every other test; it also passes alone in a fresh process.
"""
import ctypes

import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

_vp, _i64, _int = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
B200Q_ERR_TOO_LARGE = 5
B200Q_NOALLOC_SCRATCH_BYTES = 16 << 20


@pytest.fixture(scope="module")
def abi(native):
    L = ctypes.CDLL(native.library_path())
    f = L.b200q_w8a16_linear_noalloc
    f.argtypes = [_vp, _int, _i64, _vp, _i64, _vp, _vp, _int, _int, _vp, _int, _i64, _i64, _i64,
                  _i64, _vp]
    f.restype = _int
    ws = L.b200q_w8a16_workspace_size
    ws.argtypes = [_i64, _i64, _i64]
    ws.restype = ctypes.c_size_t
    return L


def _call_noalloc(L, x, w, ws, bias, out):
    M, K = x.shape
    N = w.shape[0]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return L.b200q_w8a16_linear_noalloc(
        x.data_ptr(), 0, K, w.data_ptr(), K, ws.data_ptr(), bias.data_ptr(), 1, 1,
        out.data_ptr(), 0, N, M, N, K, stream)


def test_noalloc_matches_workspace_entry_point_twice(native, abi):
    g = torch.Generator().manual_seed(31)
    # a split-K plan of the weight-stationary kernel (256-token tiles), which the
    # allocation-free entry always uses: the call needs its static scratch
    M, K, N = 300, 12288, 3072
    assert abi.b200q_w8a16_workspace_size(M, N, K) > 0
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=g) * 100).clamp(-448, 448).to(torch.float8_e4m3fn).cuda()
    ws = torch.tensor([1e-4]).cuda()
    bias = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16).cuda()
    # the existing entry point (caller-provided workspace) is the comparison
    ref = native.w8a16_linear(x, w, ws, bias, "gelu_tanh")
    ref32 = native.w8a16_linear(x, w, ws, bias, "gelu_tanh", torch.float32)
    outs = [torch.empty(M, N, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    assert _call_noalloc(abi, x, w, ws, bias, outs[0]) == 0  # first call: per-device set-up
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for o in outs[1:]:
        assert _call_noalloc(abi, x, w, ws, bias, o) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0, "the no-alloc calls changed free device memory"
    assert oracle.elementwise_ulp_ratio(ref, ref32) <= 1.0
    for o in outs[1:]:
        # same tolerance as the other W8A16 tests: within 1 ULP of the fp32 result,
        # and within 1 ULP of the workspace entry point's own output
        assert oracle.elementwise_ulp_ratio(o, ref32) <= 1.0
        assert oracle.elementwise_ulp_ratio(o, ref.float()) <= 1.0
    assert native.device_status() == 0


def test_noalloc_rejects_shapes_beyond_the_static_scratch(native, abi):
    M, K, N = 300, 49152, 12288
    need = abi.b200q_w8a16_workspace_size(M, N, K)
    assert need > B200Q_NOALLOC_SCRATCH_BYTES
    x = torch.empty(M, K, dtype=torch.bfloat16, device="cuda")
    w = torch.empty(N, K, dtype=torch.float8_e4m3fn, device="cuda")
    ws = torch.ones(1, device="cuda")
    bias = torch.zeros(N, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    launches = native.launch_count()
    assert _call_noalloc(abi, x, w, ws, bias, out) == B200Q_ERR_TOO_LARGE
    assert native.launch_count() == launches
    assert b"static buffer" in native.lib().b200q_status_string(B200Q_ERR_TOO_LARGE)
