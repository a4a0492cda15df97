"""The allocation-free W8A16 entry point, called through the C ABI.

b200q_w8a16_linear_noalloc exists for callers that cannot allocate device
memory themselves (a host that only hands this library buffers it registered up
front, or a runtime whose device-memory budget is fixed before the model runs).
Its scratch is a static device array inside the library.  These tests check,
through ctypes on the shared library, that two calls in a row match the
workspace-taking entry point and the CPU oracle within the tolerance the other
W8A16 tests use, on the routes that use the array (the planes GEMV, the
small-M planes route and the split-K weight-stationary kernel); that the calls allocate no device
memory; that a shape whose route fits is accepted even when another route would
not fit; and that a shape whose route does not fit is rejected with the clear
error status without launching anything.

The file name sorts last so that a run stopping at the first failure has
already run every other test; it also passes alone in a fresh process.
"""
import ctypes

import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

_vp, _i64, _int = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
B200Q_BF16, B200Q_F16 = 0, 1
B200Q_ERR_INVALID, B200Q_ERR_TOO_LARGE = 1, 5
B200Q_NOALLOC_SCRATCH_BYTES = 16 << 20


@pytest.fixture(scope="module")
def abi(native):
    L = ctypes.CDLL(native.library_path())
    f = L.b200q_w8a16_linear_noalloc
    f.argtypes = [_vp, _int, _i64, _vp, _i64, _vp, _vp, _int, _int, _vp, _int, _i64, _i64, _i64,
                  _i64, _vp]
    f.restype = _int
    return L


def _call_noalloc(L, x, w, ws, bias, out):
    M, K = x.shape
    N = w.shape[0]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    xdt = B200Q_F16 if x.dtype == torch.float16 else B200Q_BF16
    bdt = 2 if bias.dtype == torch.float16 else 1
    odt = B200Q_F16 if out.dtype == torch.float16 else B200Q_BF16
    return L.b200q_w8a16_linear_noalloc(
        x.data_ptr(), xdt, K, w.data_ptr(), K, ws.data_ptr(), bias.data_ptr(), bdt, 1,
        out.data_ptr(), odt, N, M, N, K, stream)


def _kernel_splits(M, N, K, sms=148):
    """Split count of the weight-stationary kernel's plan for M > 256 tokens
    (256-token tiles): the fewest splits within 2% of the best wave efficiency,
    at most 8, >= 4 K blocks of 64 per split, and fp32 partials at most half the
    fp8 weight's bytes."""
    tiles = -(-N // 128) * -(-M // 256)
    num_kb = -(-K // 64)
    best, best_eff = 1, 0.0
    for s in range(1, 9):
        if s > 1 and (s * 4 > num_kb or s * M * N * 8.0 > 0.5 * N * K):
            break
        units = tiles * s
        eff = units / (-(-units // sms) * sms)
        if eff > best_eff + 0.02:
            best, best_eff = s, eff
    return best


def _inputs(g, M, K, N, dtype):
    x = torch.randn(M, K, generator=g).to(dtype)
    w = (torch.randn(N, K, generator=g) * 100).clamp(-448, 448).to(torch.float8_e4m3fn)
    ws = torch.tensor([1e-4])
    bias = (torch.randn(N, generator=g) * 0.01).to(dtype)
    return x, w, ws, bias


def _check_twice(native, abi, x, w, ws, bias):
    """Two no-alloc calls in a row against the workspace entry point and the
    oracle; returns the outputs."""
    M, N = x.shape[0], w.shape[0]
    dev = [t.cuda() for t in (x, w, ws, bias)]
    ref = native.w8a16_linear(*dev, "gelu_tanh")                 # existing entry point
    ref32 = oracle.w8a16_linear(x, w, ws, bias, "gelu_tanh", "fp32")   # CPU oracle
    outs = [torch.full((M, N), float("nan"), dtype=x.dtype, device="cuda") for _ in range(2)]
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    alloc0 = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
    for o in outs:
        assert _call_noalloc(abi, *dev, o) == 0
    torch.cuda.synchronize()
    # secondary evidence of no allocation (the primary one is the source check
    # in tests/test_host.py): torch's allocator made no allocation during the
    # calls and the device's free memory did not move
    assert torch.cuda.memory_stats().get("allocation.all.allocated", 0) == alloc0
    assert torch.cuda.mem_get_info()[0] == free0
    for o in outs:
        # same tolerance as the other W8A16 tests: within 1 ULP of the fp32
        # oracle value, and within 1 ULP of the workspace entry point's output
        assert oracle.elementwise_ulp_ratio(o, ref32) <= 1.0
        assert oracle.elementwise_ulp_ratio(o, ref.float()) <= 1.0
    assert native.device_status() == 0
    return outs


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,K,N", [(40, 3072, 3072), (200, 4096, 2048)])
def test_noalloc_planes_route_matches_twice(native, abi, dtype, M, K, N):
    """17 <= M <= 256: the planes route, its planes and plane scales in the
    static array (written by the planes pass, read by the GEMM)."""
    x, w, ws, bias = _inputs(torch.Generator().manual_seed(M + K), M, K, N, dtype)
    _check_twice(native, abi, x, w, ws, bias)


@pytest.mark.parametrize("M", [1, 4])
def test_noalloc_planes_gemv_matches_twice(native, abi, M):
    """bf16, M <= 4: the planes GEMV, its planes and plane scales in the static
    array (written by the planes pass, read by the GEMV's warps)."""
    x, w, ws, bias = _inputs(torch.Generator().manual_seed(M + 7), M, 3072, 4096, torch.bfloat16)
    _check_twice(native, abi, x, w, ws, bias)


def test_noalloc_split_k_kernel_matches_twice(native, abi):
    """M > 256: the weight-stationary kernel with split-K partials and tile
    counters in the static array (the counters are cleared on every call)."""
    M, K, N = 300, 12288, 3072
    assert _kernel_splits(M, N, K) == 2   # the call does use the array
    x, w, ws, bias = _inputs(torch.Generator().manual_seed(31), M, K, N, torch.bfloat16)
    a, b = _check_twice(native, abi, x, w, ws, bias)
    assert torch.equal(a, b)               # fixed-order split-K: reproducible


def test_noalloc_accepts_a_fitting_route_beside_a_large_plan(native, abi):
    """M = 200, K = 16384, N = 12288: the weight-stationary plan would need
    ~29 MB of partials, but the call takes the planes route, whose ~6.6 MB of
    planes fit, so it runs (and matches) instead of being rejected."""
    M, K, N = 200, 16384, 12288
    assert _kernel_splits(257, N, K) * 257 * N * 4 > B200Q_NOALLOC_SCRATCH_BYTES
    g = torch.Generator().manual_seed(7)
    x, w, ws, bias = _inputs(g, M, K, N, torch.bfloat16)
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    dev = [t.cuda() for t in (x, w, ws, bias)]
    assert _call_noalloc(abi, *dev, out) == 0
    ref32 = oracle.w8a16_linear(x[:64], w, ws, bias, "gelu_tanh", "fp32")
    assert oracle.elementwise_ulp_ratio(out[:64], ref32) <= 1.0


def test_noalloc_rejects_routes_beyond_the_static_scratch(native, abi):
    M, K, N = 300, 49152, 12288
    assert _kernel_splits(M, N, K) * M * N * 4 > B200Q_NOALLOC_SCRATCH_BYTES
    x = torch.empty(M, K, dtype=torch.bfloat16, device="cuda")
    w = torch.empty(N, K, dtype=torch.float8_e4m3fn, device="cuda")
    ws = torch.ones(1, device="cuda")
    bias = torch.zeros(N, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    launches = native.launch_count()
    assert _call_noalloc(abi, x, w, ws, bias, out) == B200Q_ERR_TOO_LARGE
    assert native.launch_count() == launches
    assert b"static buffer" in native.lib().b200q_status_string(B200Q_ERR_TOO_LARGE)
    # invalid arguments are reported as such, before any size decision
    bad = torch.empty(M, N, dtype=torch.float32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert abi.b200q_w8a16_linear_noalloc(x.data_ptr(), 7, K, w.data_ptr(), K, ws.data_ptr(),
                                          bias.data_ptr(), 1, 1, bad.data_ptr(), 0, N, M, N, K,
                                          stream) == B200Q_ERR_INVALID
