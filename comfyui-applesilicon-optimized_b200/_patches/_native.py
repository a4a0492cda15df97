"""Binding of the b200q C ABI (include/b200q.h) and the ``torch.ops.b200q`` ops.

The native library ``_lib/libb200q.so`` is built in-tree by ``csrc/build.py``.
This module loads it with ctypes, passes raw device pointers, element strides
and torch's current CUDA stream, and raises ``RuntimeError`` on any non-zero
status.  There is no CPU fallback: if the library is missing or the device is
not a B200 (sm_100), every op raises.

The ``b200q`` torch.library namespace mirrors the reference's native module
functions (pybind in the reference: _patches/int8_ext/int8_gemm.mm:2626-2715,
_patches/fp8_ext/fp8_matmul2d.mm:355-360, _patches/fp8s_ext/w8a16_gemm.mm:316-329):

  quant_rowwise_i8(x)                       -> (q int8 [M,K], scale f32 [M,1])
  quant_rowwise_i8_convrot(x, groupsize)    -> the same for the convrot-rotated rows
  int_mm(a [M,K] i8, b [K,N] i8)            -> int32 [M,N]      (torch._int_mm contract)
  i8_matmul_nt(a [M,K], w [N,K])            -> int32 [M,N]      (i8_matmul2d_nt)
  i8_matmul_nt_fused(a, w, row_scale, bias) -> bf16 [M,N]       (i8_matmul2d_nt_fused)
  i8_matmul_nt_fused_cs(a, w, row_scale, col_scale, bias, out_dtype) (i8_matmul2d_nt_fused_cs)
  i8_matmul_nt_fused_cs_qkv(a, w, rs, cs, bias, heads, head_dim, batch)
                                            -> q, k, v in [B, H, S, D] (i8_matmul2d_nt_fused_cs_qkv)
  rms_rope_partial_(q, k, freqs, qw, kw, eps) -> in-place RMSNorm + split-half RoPE
  i8_matmul_nt_fused_cs_qkv_rms_rope(a, w, rs, cs, bias, freqs, qw, kw, heads, head_dim, eps, batch)
                                            -> q, k, v with Q/K normalized + rotated in the epilogue
  silu_mul_split(x [M,2F] bf16)             -> act [M,F] = bf16(bf16(silu(gate)) * up)
  i8_swiglu_rot(x [M,2F] bf16)              -> convrot(act) [M,F] bf16   (i8_swiglu_rot)
  i8_swiglu_quant(x [M,2F], rotate)         -> (q int8 [M,F], scale [M,1]) of (rotated) act
  i8_matmul_nt_fused_cs_swiglu(a, w [2F,K], rs, cs, bias) -> act [M,F]  (FC1 + SwiGLU epilogue)
  i8_mlp_bridge_prequant(a, w1, rs, cs, bias, rotate, tile_rows)
                                            -> (q, scale) FC2 input      (i8_mlp_bridge_prequant)
  i8_linear(x, w, w_scale, bias, out_dtype) -> quant + GEMM + dequant epilogue
                                               (B200Q_FUSED_PROLOGUE=1: quant inside the GEMM)
  fp8_quant_tensorwise(x)                   -> (q e4m3 [M,K], scale f32 [])
  fp8_linear(x, w, w_scale, bias, out_dtype, act, scale_result)
                                            -> per-tensor e4m3 quant fused into fp8_scaled_mm
  fp8_scaled_mm(a, w_nk, scale_a, scale_b, scale_result, bias, out_dtype, act)
  w8a16_linear(x, w_nk e4m3, w_scale, bias, act, out_dtype)
  fp8_decode(t, out_dtype)
"""

import ctypes
import os

import torch

TAG = "[b200q]"

_LIB_PATH = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "_lib",
                         "libb200q.so")

B200Q_BF16, B200Q_F16, B200Q_F32, B200Q_I32 = 0, 1, 2, 3
BIAS_NONE, BIAS_BF16, BIAS_F16, BIAS_F32 = 0, 1, 2, 3
ACT_NONE, ACT_GELU_TANH, ACT_GELU_ERF = 0, 1, 2
ACTS = {None: ACT_NONE, "none": ACT_NONE, "gelu_tanh": ACT_GELU_TANH, "gelu": ACT_GELU_ERF}

_DT = {torch.bfloat16: B200Q_BF16, torch.float16: B200Q_F16, torch.float32: B200Q_F32}
_BIAS_DT = {torch.bfloat16: BIAS_BF16, torch.float16: BIAS_F16, torch.float32: BIAS_F32}

_lib = None

_vp, _i64, _int, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
_SIGNATURES = {
    "b200q_version": ([], _int),
    "b200q_status_string": ([_int], ctypes.c_char_p),
    "b200q_launch_count": ([], ctypes.c_uint64),
    "b200q_get_device_status": ([_vp, _int], _int),
    "b200q_quant_rowwise_i8": ([_vp, _int, _i64, _i64, _i64, _vp, _i64, _vp, _vp], _int),
    "b200q_quant_rowwise_i8_convrot": ([_vp, _int, _i64, _i64, _i64, _int, _vp, _i64, _vp, _vp],
                                       _int),
    "b200q_i8_matmul_nt": ([_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp], _int),
    "b200q_i8_matmul_nt_dequant_qkv": ([_vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _vp, _vp, _vp,
                                       _int, _i64, _i64, _i64, _i64, _i64, _i64, _vp], _int),
    "b200q_rms_rope_partial": ([_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                               ctypes.c_float, _vp], _int),
    "b200q_i8_matmul_nt_dequant_qkv_rms_rope": ([_vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _vp,
                                                 _vp, _vp, _i64, _i64, _vp, _i64, _vp, _vp,
                                                 ctypes.c_float, _i64, _i64, _i64, _vp], _int),
    "b200q_i8_matmul_nt_dequant": ([_vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _int, _vp, _int,
                                    _i64, _i64, _i64, _i64, _vp], _int),
    "b200q_i8_linear": ([_vp, _int, _i64, _vp, _i64, _vp, _i64, _vp, _int, _vp, _int, _i64, _i64,
                         _i64, _i64, _vp, _vp, _vp], _int),
    "b200q_fp8_scaled_mm": ([_vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _int, _int, _vp,
                             _int, _i64, _i64, _i64, _i64, _vp], _int),
    "b200q_fp8_scaled_mm_allgather": ([_vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _int,
                                       _int, _vp, _vp, _int, _int, _i64, _i64, _i64, _i64, _vp],
                                      _int),
    "b200q_ipc_export": ([_vp, _vp, ctypes.POINTER(ctypes.c_uint64)], _int),
    "b200q_ipc_import": ([_vp, ctypes.c_uint64, ctypes.POINTER(_vp), ctypes.POINTER(_vp)], _int),
    "b200q_ipc_close": ([_vp], _int),
    "b200q_fp8_scaled_mm_amax": ([_vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _int, _int,
                                  _vp, _int, _i64, _i64, _i64, _i64, _vp, _vp], _int),
    "b200q_fp8_quant_from_amax": ([_vp, _int, _i64, _i64, _i64, _vp, _vp, _i64, _vp, _vp], _int),
    "b200q_fp8_quant_tensorwise": ([_vp, _int, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _vp], _int),
    "b200q_prologue_sync_bytes": ([_i64], _sz),
    "b200q_i8_linear_fused": ([_vp, _int, _i64, _vp, _i64, _vp, _i64, _vp, _int, _vp, _int, _i64,
                               _i64, _i64, _i64, _vp, _vp, _vp, _sz, _vp], _int),
    "b200q_fp8_linear_fused": ([_vp, _int, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _int, _int, _vp,
                                _int, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _sz, _vp], _int),
    "b200q_w8a16_workspace_size": ([_i64, _i64, _i64], _sz),
    "b200q_w8a16_linear": ([_vp, _int, _i64, _vp, _i64, _vp, _vp, _int, _int, _vp, _int, _i64, _i64,
                            _i64, _i64, _vp, _sz, _vp], _int),
    "b200q_fp8_decode": ([_vp, _i64, _int, _vp, _int, _vp], _int),
    "b200q_silu_mul_split": ([_vp, _i64, _i64, _i64, _vp, _i64, _vp], _int),
    "b200q_i8_swiglu_rot": ([_vp, _i64, _i64, _i64, _vp, _i64, _vp], _int),
    "b200q_i8_swiglu_quant": ([_vp, _i64, _i64, _i64, _int, _vp, _i64, _vp, _vp], _int),
    "b200q_i8_matmul_nt_dequant_swiglu": ([_vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _vp, _i64,
                                           _i64, _i64, _i64, _vp], _int),
    "b200q_i8_mlp_bridge_prequant": ([_vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _i64, _i64, _i64,
                                      _int, _i64, _vp, _vp, _i64, _vp, _vp], _int),
}


def library_path():
    return _LIB_PATH


def lib():
    """The loaded C-ABI library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            raise RuntimeError(f"{TAG} native library missing at {_LIB_PATH}; run the build "
                               f"(__graft_entry__.build() or csrc/build.py)")
        L = ctypes.CDLL(_LIB_PATH)
        for name, (args, res) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def available():
    """True when the library is built and the current CUDA device is a B200."""
    if not os.path.exists(_LIB_PATH) or not torch.cuda.is_available():
        return False
    return torch.cuda.get_device_capability() == (10, 0)


def launch_count():
    return int(lib().b200q_launch_count())


def device_status(reset=False):
    v = ctypes.c_uint(0)
    _check(lib().b200q_get_device_status(ctypes.byref(v), int(bool(reset))))
    return int(v.value)


def _check(status):
    if status != 0:
        msg = lib().b200q_status_string(status).decode()
        raise RuntimeError(f"{TAG} native call failed: {msg} (status {status})")


def _stream(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _require_cuda(*ts):
    for t in ts:
        if t is not None and t.device.type != "cuda":
            raise RuntimeError(f"{TAG} expected CUDA tensors, got {t.device}")


def _rows_2d(t, name):
    """View as [rows, K] with unit inner stride (no copy when already so)."""
    if t.dim() != 2:
        raise RuntimeError(f"{TAG} {name} must be 2-D, got {tuple(t.shape)}")
    if t.stride(1) != 1:
        t = t.contiguous()
    return t


# ----------------------------------------------------------------------------- ops (eager)
def quant_rowwise_i8(x):
    _require_cuda(x)
    x = _rows_2d(x, "x")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise RuntimeError(f"{TAG} quant_rowwise_i8 expects bf16/f16, got {x.dtype}")
    M, K = x.shape
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty((M, 1), dtype=torch.float32, device=x.device)
    _check(lib().b200q_quant_rowwise_i8(_p(x), _DT[x.dtype], M, K, x.stride(0), _p(q), K, _p(s),
                                        _stream(x)))
    return q, s


CONVROT_MAX_K = 65536  # B200Q_CONVROT_MAX_K


def quant_rowwise_i8_convrot(x, groupsize=256):
    """Convrot (256-wide Hadamard) rotation fused into the per-token INT8 quant:
    x [M,K] bf16/f16 -> (q int8 [M,K], scale f32 [M,1]) of the rotated rows."""
    _require_cuda(x)
    x = _rows_2d(x, "x")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise RuntimeError(f"{TAG} quant_rowwise_i8_convrot expects bf16/f16, got {x.dtype}")
    M, K = x.shape
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty((M, 1), dtype=torch.float32, device=x.device)
    _check(lib().b200q_quant_rowwise_i8_convrot(_p(x), _DT[x.dtype], M, K, x.stride(0), int(groupsize),
                                                _p(q), K, _p(s), _stream(x)))
    return q, s


def i8_matmul_nt(a, w):
    _require_cuda(a, w)
    a, w = _rows_2d(a, "a"), _rows_2d(w, "w")
    if a.dtype != torch.int8 or w.dtype != torch.int8:
        raise RuntimeError(f"{TAG} i8_matmul_nt expects int8 operands")
    if a.shape[1] != w.shape[1]:
        raise RuntimeError(f"{TAG} K mismatch: a {tuple(a.shape)} w {tuple(w.shape)}")
    M, K = a.shape
    N = w.shape[0]
    c = torch.empty((M, N), dtype=torch.int32, device=a.device)
    _check(lib().b200q_i8_matmul_nt(_p(a), a.stride(0), _p(w), w.stride(0), _p(c), N, M, N, K,
                                    _stream(a)))
    return c


def int_mm(a, b):
    """torch._int_mm contract: a [M,K] int8 @ b [K,N] int8 -> int32 [M,N].

    b is consumed as W = b.t() ([N,K]); when b is the transpose view of a
    row-major weight (the common ``weight.T`` call) no copy is made."""
    if b.dim() != 2:
        raise RuntimeError(f"{TAG} int_mm expects 2-D b")
    return i8_matmul_nt(a, b.t())


def _out_dtype_code(dt, allowed):
    if dt not in allowed:
        raise RuntimeError(f"{TAG} unsupported out dtype {dt}")
    return _DT[dt]


def i8_matmul_nt_fused_cs(a, w, row_scale, col_scale, bias=None, out_dtype=torch.bfloat16,
                          act=None):
    _require_cuda(a, w, row_scale, col_scale, bias)
    a, w = _rows_2d(a, "a"), _rows_2d(w, "w")
    M, K = a.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise RuntimeError(f"{TAG} K mismatch")
    row_scale = row_scale.reshape(-1).float().contiguous()
    col_scale = col_scale.reshape(-1).float().contiguous()
    if row_scale.numel() != M or col_scale.numel() not in (1, N):
        raise RuntimeError(f"{TAG} scale numel mismatch: row {row_scale.numel()} (M={M}), "
                           f"col {col_scale.numel()} (N={N})")
    code = _out_dtype_code(out_dtype, (torch.bfloat16, torch.float16))
    if bias is not None:
        bias = bias.to(out_dtype).contiguous()
        if bias.numel() != N:
            raise RuntimeError(f"{TAG} bias numel {bias.numel()} != N {N}")
    out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    _check(lib().b200q_i8_matmul_nt_dequant(_p(a), a.stride(0), _p(w), w.stride(0), _p(row_scale),
                                            _p(col_scale), col_scale.numel(), _p(bias),
                                            ACTS[act], _p(out), code, N, M, N, K, _stream(a)))
    return out


def i8_matmul_nt_fused_cs_qkv(a, w, row_scale, col_scale, bias=None, heads=1, head_dim=128,
                              batch=1, out_dtype=torch.bfloat16):
    """INT8 QKV projection straight into attention layout: returns q, k, v, each
    [batch, heads, M // batch, head_dim] (i8_matmul2d_nt_fused_cs_qkv, batch 1)."""
    _require_cuda(a, w, row_scale, col_scale, bias)
    a, w = _rows_2d(a, "a"), _rows_2d(w, "w")
    M, K = a.shape
    N = w.shape[0]
    if w.shape[1] != K or N != 3 * heads * head_dim or M % batch:
        raise RuntimeError(f"{TAG} qkv shapes: M={M} K={K} N={N} heads={heads} head_dim={head_dim} "
                           f"batch={batch}")
    row_scale = row_scale.reshape(-1).float().contiguous()
    col_scale = col_scale.reshape(-1).float().contiguous()
    code = _out_dtype_code(out_dtype, (torch.bfloat16, torch.float16))
    if bias is not None:
        bias = bias.to(out_dtype).contiguous()
    S = M // batch
    outs = [torch.empty((batch, heads, S, head_dim), dtype=out_dtype, device=a.device) for _ in range(3)]
    _check(lib().b200q_i8_matmul_nt_dequant_qkv(
        _p(a), a.stride(0), _p(w), w.stride(0), _p(row_scale), _p(col_scale), col_scale.numel(),
        _p(bias), _p(outs[0]), _p(outs[1]), _p(outs[2]), code, heads, head_dim, batch, M, N, K,
        _stream(a)))
    return tuple(outs)


def i8_matmul_nt_fused_cs_qkv_rms_rope(a, w, row_scale, col_scale, bias, freqs, q_weight,
                                       k_weight, heads, head_dim=128, eps=1e-6, batch=1):
    """INT8 QKV projection into attention layout with Q/K RMSNorm + split-half
    RoPE applied in the GEMM epilogue (i8_matmul2d_nt_fused_cs_qkv_rms_rope):
    q, k, v [batch, heads, M // batch, 128] bf16; freqs [M, R, 2, 2] bf16 with
    R % 8 == 0 (use rms_rope_partial_ after the plain scatter otherwise)."""
    _require_cuda(a, w, row_scale, col_scale, bias, freqs, q_weight, k_weight)
    a, w = _rows_2d(a, "a"), _rows_2d(w, "w")
    M, K = a.shape
    N = w.shape[0]
    if head_dim != 128 or w.shape[1] != K or N != 3 * heads * head_dim or M % batch:
        raise RuntimeError(f"{TAG} qkv rms/rope shapes: M={M} K={K} N={N} heads={heads} "
                           f"head_dim={head_dim} batch={batch}")
    row_scale = row_scale.reshape(-1).float().contiguous()
    col_scale = col_scale.reshape(-1).float().contiguous()
    if bias is not None:
        bias = bias.to(torch.bfloat16).contiguous()
    fr = freqs.to(torch.bfloat16).contiguous()
    R = fr.shape[-3] if fr.dim() >= 3 else 0
    if fr.numel() != M * R * 4:
        raise RuntimeError(f"{TAG} freqs must hold [M, R, 2, 2] = {M} x R x 4 values")
    qw, kw = q_weight.float().contiguous(), k_weight.float().contiguous()
    S = M // batch
    outs = [torch.empty((batch, heads, S, head_dim), dtype=torch.bfloat16, device=a.device)
            for _ in range(3)]
    _check(lib().b200q_i8_matmul_nt_dequant_qkv_rms_rope(
        _p(a), a.stride(0), _p(w), w.stride(0), _p(row_scale), _p(col_scale), col_scale.numel(),
        _p(bias), _p(outs[0]), _p(outs[1]), _p(outs[2]), heads, batch, _p(fr), R, _p(qw), _p(kw),
        float(eps), M, N, K, _stream(a)))
    return tuple(outs)


def rms_rope_partial_(q, k, freqs, q_weight, k_weight, eps=1e-6):
    """In place: RMSNorm (fp32 weights) + split-half RoPE on the first 2R dims of
    bf16 q, k [B, H, S, D]; freqs [B*S, R, 2, 2] bf16 (any leading shape with that
    element count).  rms_rope_attention_partial (dit_kernels.mm:825-874, 1677)."""
    _require_cuda(q, k, freqs, q_weight, k_weight)
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or q.shape != k.shape or q.dim() != 4:
        raise RuntimeError(f"{TAG} rms_rope_partial_ expects bf16 q/k of one [B,H,S,D] shape")
    if not (q.is_contiguous() and k.is_contiguous()):
        raise RuntimeError(f"{TAG} rms_rope_partial_ works in place on contiguous q/k")
    B, H, S, D = q.shape
    fr = freqs.to(torch.bfloat16).contiguous()
    R = fr.shape[-3] if fr.dim() >= 3 else 0
    if fr.numel() != B * S * R * 4:
        raise RuntimeError(f"{TAG} freqs must hold [B*S, R, 2, 2] = {B * S} x R x 4 values")
    qw = q_weight.float().contiguous()
    kw = k_weight.float().contiguous()
    _check(lib().b200q_rms_rope_partial(_p(q), _p(k), _p(fr), _p(qw), _p(kw), B, H, S, D, R,
                                        float(eps), _stream(q)))


SWIGLU_MAX_F = 65536  # B200Q_SWIGLU_MAX_F


def _wide_2d(x, name):
    _require_cuda(x)
    x = _rows_2d(x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x, name)
    if x.dtype != torch.bfloat16:
        raise RuntimeError(f"{TAG} {name} must be bf16, got {x.dtype}")
    if x.shape[1] % 2:
        raise RuntimeError(f"{TAG} {name} width {x.shape[1]} is odd (expected [M, 2F])")
    return x, x.shape[0], x.shape[1] // 2


def silu_mul_split(x):
    """SwiGLU of a split-half bf16 [..., 2F] tensor -> [..., F] (silu_mul_split)."""
    shp = x.shape
    x2, M, F = _wide_2d(x, "x")
    out = torch.empty((M, F), dtype=torch.bfloat16, device=x.device)
    _check(lib().b200q_silu_mul_split(_p(x2), x2.stride(0), M, F, _p(out), F, _stream(x2)))
    return out.reshape(*shp[:-1], F)


def i8_swiglu_rot(x):
    """Convrot-rotated SwiGLU of a bf16 [M, 2F] tensor -> [M, F] bf16 (i8_swiglu_rot)."""
    x2, M, F = _wide_2d(x, "x")
    out = torch.empty((M, F), dtype=torch.bfloat16, device=x.device)
    _check(lib().b200q_i8_swiglu_rot(_p(x2), x2.stride(0), M, F, _p(out), F, _stream(x2)))
    return out


def i8_swiglu_quant(x, rotate=True):
    """Per-token INT8 quant of the (convrot-rotated) SwiGLU of a bf16 [M, 2F]
    tensor, in one pass: (q int8 [M, F], scale f32 [M, 1])."""
    x2, M, F = _wide_2d(x, "x")
    q = torch.empty((M, F), dtype=torch.int8, device=x.device)
    s = torch.empty((M, 1), dtype=torch.float32, device=x.device)
    _check(lib().b200q_i8_swiglu_quant(_p(x2), x2.stride(0), M, F, int(bool(rotate)), _p(q), F,
                                       _p(s), _stream(x2)))
    return q, s


def _fc1_args(a, w, row_scale, col_scale, bias):
    _require_cuda(a, w, row_scale, col_scale, bias)
    a, w = _rows_2d(a, "a"), _rows_2d(w, "w")
    if a.dtype != torch.int8 or w.dtype != torch.int8:
        raise RuntimeError(f"{TAG} FC1 operands must be int8")
    M, K = a.shape
    N2 = w.shape[0]
    if w.shape[1] != K or N2 % 2:
        raise RuntimeError(f"{TAG} FC1 shapes: a {tuple(a.shape)} w {tuple(w.shape)}")
    row_scale = row_scale.reshape(-1).float().contiguous()
    col_scale = col_scale.reshape(-1).float().contiguous()
    if row_scale.numel() != M or col_scale.numel() not in (1, N2):
        raise RuntimeError(f"{TAG} scale numel mismatch: row {row_scale.numel()} (M={M}), "
                           f"col {col_scale.numel()} (2F={N2})")
    if bias is not None:
        bias = bias.to(torch.bfloat16).contiguous()
        if bias.numel() != N2:
            raise RuntimeError(f"{TAG} FC1 bias numel {bias.numel()} != 2F {N2}")
    return a, w, row_scale, col_scale, bias, M, K, N2


def i8_matmul_nt_fused_cs_swiglu(a, w, row_scale, col_scale, bias=None):
    """FC1 (INT8 GEMM, channelwise two-rounding dequant + bias) with SwiGLU in the
    epilogue: a [M,K] int8, w [2F,K] int8 (rows [gate; up]) -> act [M,F] bf16."""
    a, w, rs, cs, bias, M, K, N2 = _fc1_args(a, w, row_scale, col_scale, bias)
    out = torch.empty((M, N2 // 2), dtype=torch.bfloat16, device=a.device)
    _check(lib().b200q_i8_matmul_nt_dequant_swiglu(_p(a), a.stride(0), _p(w), w.stride(0), _p(rs),
                                                   _p(cs), cs.numel(), _p(bias), _p(out), N2 // 2,
                                                   M, N2, K, _stream(a)))
    return out


BRIDGE_SCRATCH_BYTES = 1 << 30  # act scratch bound of the automatic row tiling


def i8_mlp_bridge_prequant(a, w1, row_scale, col_scale, bias=None, rotate=True, tile_rows=-1):
    """FC1 -> SwiGLU (-> convrot) -> per-token INT8 quant: the FC2 input
    (q int8 [M,F], scale f32 [M,1]) without FC1's [M,2F] output
    (i8_mlp_bridge_prequant).  tile_rows: rows per FC1 pass (0 = all rows,
    -1 = all rows unless the [rows, F] bf16 scratch would exceed 1 GiB)."""
    a, w1, rs, cs, bias, M, K, N2 = _fc1_args(a, w1, row_scale, col_scale, bias)
    F = N2 // 2
    if tile_rows < 0:
        tile_rows = 0 if M * F * 2 <= BRIDGE_SCRATCH_BYTES else max(
            256, (BRIDGE_SCRATCH_BYTES // (F * 2)) // 256 * 256)
    rows = M if tile_rows == 0 else min(M, int(tile_rows))
    scratch = torch.empty((max(rows, 1), F), dtype=torch.bfloat16, device=a.device)
    q = torch.empty((M, F), dtype=torch.int8, device=a.device)
    s = torch.empty((M, 1), dtype=torch.float32, device=a.device)
    _check(lib().b200q_i8_mlp_bridge_prequant(_p(a), a.stride(0), _p(w1), w1.stride(0), _p(rs),
                                              _p(cs), cs.numel(), _p(bias), M, N2, K,
                                              int(bool(rotate)), int(tile_rows), _p(scratch),
                                              _p(q), F, _p(s), _stream(a)))
    return q, s


def i8_matmul_nt_fused(a, w, row_scale, bias=None):
    """Tensorwise-weight variant: row_scale already holds weight_scale * x_scale."""
    one = torch.ones(1, dtype=torch.float32, device=a.device)
    return i8_matmul_nt_fused_cs(a, w, row_scale, one, bias, torch.bfloat16)


# Sync words of the fused-prologue launches (b200q_prologue_sync_bytes): one
# zero-initialised buffer per (device, stream), reused by every call ordered on
# that stream (each launch leaves it zeroed).  Buffers are never freed while the
# process runs: a CUDA graph captured with one keeps using its address.
_SYNC = {}
_SYNC_RETIRED = []
_SYNC_MIN_BYTES = 64 << 10


def _sync_buffer(t, M):
    need = int(lib().b200q_prologue_sync_bytes(M))
    key = (t.device.index, torch.cuda.current_stream(t.device).cuda_stream)
    buf = _SYNC.get(key)
    if buf is None or buf.numel() < need:
        if buf is not None:
            _SYNC_RETIRED.append(buf)
        buf = torch.zeros((max(need, _SYNC_MIN_BYTES),), dtype=torch.uint8, device=t.device)
        _SYNC[key] = buf
    return buf


def fused_prologue_enabled():
    """B200Q_FUSED_PROLOGUE=1 selects the one-launch route (quant inside the GEMM).

    Off by default: with two quantizer warps per SM the in-kernel quant is
    issue-bound and measured slower than its own launch on the BASELINE shapes."""
    return os.environ.get("B200Q_FUSED_PROLOGUE", "0") == "1"


def i8_linear(x, w, w_scale, bias=None, out_dtype=torch.bfloat16, act=None):
    """Per-token quant + INT8 GEMM + reference dequant epilogue; x [..., K].

    With B200Q_FUSED_PROLOGUE=1 the quantization runs inside the GEMM launch
    (b200q_i8_linear_fused); otherwise it is its own launch (b200q_i8_linear)."""
    _require_cuda(x, w, w_scale, bias)
    shp = x.shape
    x2 = _rows_2d(x.reshape(-1, shp[-1]), "x")
    M, K = x2.shape
    N = w.shape[0]
    w = _rows_2d(w, "w")
    ws = w_scale.reshape(-1).float().contiguous()
    if ws.numel() not in (1, N):
        raise RuntimeError(f"{TAG} weight scale numel {ws.numel()} not in (1, {N})")
    code = _out_dtype_code(out_dtype, (torch.bfloat16, torch.float16))
    if bias is not None:
        bias = bias.to(out_dtype).contiguous()
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty((M,), dtype=torch.float32, device=x.device)
    out = torch.empty((M, N), dtype=out_dtype, device=x.device)
    if fused_prologue_enabled():
        sync = _sync_buffer(x2, M)
        _check(lib().b200q_i8_linear_fused(_p(x2), _DT[x2.dtype], x2.stride(0), _p(w), w.stride(0),
                                           _p(ws), ws.numel(), _p(bias), ACTS[act], _p(out), code,
                                           N, M, N, K, _p(q), _p(s), _p(sync), sync.numel(),
                                           _stream(x2)))
    else:
        _check(lib().b200q_i8_linear(_p(x2), _DT[x2.dtype], x2.stride(0), _p(w), w.stride(0),
                                     _p(ws), ws.numel(), _p(bias), ACTS[act], _p(out), code, N, M,
                                     N, K, _p(q), _p(s), _stream(x2)))
    return out.reshape(*shp[:-1], N)


def fp8_quant_tensorwise(x):
    _require_cuda(x)
    x = _rows_2d(x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x, "x")
    M, K = x.shape
    q = torch.empty((M, K), dtype=torch.float8_e4m3fn, device=x.device)
    scale = torch.empty((), dtype=torch.float32, device=x.device)
    amax = torch.empty((1,), dtype=torch.int32, device=x.device)
    _check(lib().b200q_fp8_quant_tensorwise(_p(x), _DT[x.dtype], M, K, x.stride(0), _p(q), K,
                                            _p(scale), _p(amax), _stream(x)))
    return q, scale


def fp8_quant_from_amax(x, amax):
    """fp8_quant_tensorwise(x) given x's amax (float bits in an int32 [1] tensor,
    e.g. from fp8_scaled_mm_amax): the same codes and scale, no amax pass."""
    _require_cuda(x, amax)
    x = _rows_2d(x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x, "x")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise RuntimeError(f"{TAG} fp8_quant_from_amax expects bf16/f16, got {x.dtype}")
    M, K = x.shape
    q = torch.empty((M, K), dtype=torch.float8_e4m3fn, device=x.device)
    scale = torch.empty((), dtype=torch.float32, device=x.device)
    _check(lib().b200q_fp8_quant_from_amax(_p(x), _DT[x.dtype], M, K, x.stride(0), _p(amax), _p(q),
                                           K, _p(scale), _stream(x)))
    return q, scale


def _scale_arg(s, n_ok):
    if s is None:
        return None, 0
    s = s.reshape(-1).float().contiguous()
    if s.numel() not in n_ok:
        raise RuntimeError(f"{TAG} scale numel {s.numel()} not in {n_ok}")
    return s, s.numel()


def fp8_scaled_mm(a, w, scale_a=None, scale_b=None, scale_result=None, bias=None,
                  out_dtype=torch.bfloat16, act=None):
    """a [M,K] e4m3, w [N,K] e4m3 (i.e. torch._scaled_mm's ``other`` = w.t())."""
    _require_cuda(a, w, scale_a, scale_b, scale_result, bias)
    a, w = _rows_2d(a, "a"), _rows_2d(w, "w")
    M, K = a.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise RuntimeError(f"{TAG} K mismatch")
    sa, na = _scale_arg(scale_a, (1, M))
    sb, nb = _scale_arg(scale_b, (1, N))
    sr, _ = _scale_arg(scale_result, (1,))
    out_dtype = out_dtype or torch.bfloat16
    code = _out_dtype_code(out_dtype, (torch.bfloat16, torch.float16, torch.float32))
    bdt = BIAS_NONE
    if bias is not None:
        bias = bias.contiguous()
        if bias.dtype not in _BIAS_DT:
            bias = bias.float()
        bdt = _BIAS_DT[bias.dtype]
    out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    _check(lib().b200q_fp8_scaled_mm(_p(a), a.stride(0), _p(w), w.stride(0), _p(sa), na, _p(sb),
                                     nb, _p(sr), _p(bias), bdt, ACTS[act], _p(out), code, N, M, N,
                                     K, _stream(a)))
    return out


def fp8_scaled_mm_allgather(a, w, scale_a, scale_b, scale_result, bias, out, col0, peer_ptrs,
                            act=None):
    """Column-parallel fp8_scaled_mm: w [N,K] e4m3 holds this rank's output
    columns [col0, col0 + N) of the full-width bf16/f16 ``out`` [M, N_total];
    the result goes into ``out`` and, at the same position, into each peer copy
    whose device pointer (already at column col0, from ipc_import) is in
    ``peer_ptrs``.  Returns ``out``."""
    _require_cuda(a, w, scale_a, scale_b, scale_result, bias, out)
    a, w = _rows_2d(a, "a"), _rows_2d(w, "w")
    M, K = a.shape
    N = w.shape[0]
    if w.shape[1] != K or out.dim() != 2 or out.shape[0] != M or out.stride(1) != 1:
        raise RuntimeError(f"{TAG} fp8_scaled_mm_allgather: shape mismatch")
    if not 0 <= col0 <= out.shape[1] - N:
        raise RuntimeError(f"{TAG} fp8_scaled_mm_allgather: columns [{col0}, {col0 + N}) "
                           f"outside the output's {out.shape[1]}")
    if len(peer_ptrs) > 7:
        raise RuntimeError(f"{TAG} fp8_scaled_mm_allgather: at most 7 peer outputs")
    sa, na = _scale_arg(scale_a, (1, M))
    sb, nb = _scale_arg(scale_b, (1, N))
    sr, _ = _scale_arg(scale_result, (1,))
    code = _out_dtype_code(out.dtype, (torch.bfloat16, torch.float16))
    bdt = BIAS_NONE
    if bias is not None:
        bias = bias.contiguous()
        if bias.dtype not in _BIAS_DT:
            bias = bias.float()
        bdt = _BIAS_DT[bias.dtype]
    view = out[:, col0:]
    peers = (ctypes.c_void_p * max(1, len(peer_ptrs)))(*[int(p) for p in peer_ptrs])
    _check(lib().b200q_fp8_scaled_mm_allgather(
        _p(a), a.stride(0), _p(w), w.stride(0), _p(sa), na, _p(sb), nb, _p(sr), _p(bias), bdt,
        ACTS[act], ctypes.c_void_p(view.data_ptr()), peers, len(peer_ptrs), code, out.stride(0),
        M, N, K, _stream(a)))
    return out


def ipc_export(t):
    """(64-byte IPC handle, byte offset of t in its allocation) for a CUDA tensor."""
    _require_cuda(t)
    h = ctypes.create_string_buffer(64)
    off = ctypes.c_uint64(0)
    _check(lib().b200q_ipc_export(_p(t), h, ctypes.byref(off)))
    return h.raw, int(off.value)


def ipc_import(handle, offset):
    """Maps a peer process's allocation: (device pointer at offset, mapping base)."""
    if len(handle) != 64:
        raise RuntimeError(f"{TAG} IPC handles are 64 bytes")
    ptr, base = ctypes.c_void_p(0), ctypes.c_void_p(0)
    _check(lib().b200q_ipc_import(ctypes.create_string_buffer(bytes(handle), 64), int(offset),
                                  ctypes.byref(ptr), ctypes.byref(base)))
    return int(ptr.value), int(base.value)


def ipc_close(base):
    _check(lib().b200q_ipc_close(ctypes.c_void_p(int(base))))


def fp8_scaled_mm_amax(a, w, scale_a=None, scale_b=None, scale_result=None, bias=None,
                       out_dtype=torch.bfloat16, act=None):
    """fp8_scaled_mm (bf16/f16 out) plus max |out| as float bits in an int32 [1]
    tensor, taken in the GEMM epilogue on the CTA-pair route."""
    _require_cuda(a, w, scale_a, scale_b, scale_result, bias)
    a, w = _rows_2d(a, "a"), _rows_2d(w, "w")
    M, K = a.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise RuntimeError(f"{TAG} K mismatch")
    sa, na = _scale_arg(scale_a, (1, M))
    sb, nb = _scale_arg(scale_b, (1, N))
    sr, _ = _scale_arg(scale_result, (1,))
    code = _out_dtype_code(out_dtype or torch.bfloat16, (torch.bfloat16, torch.float16))
    bdt = BIAS_NONE
    if bias is not None:
        bias = bias.contiguous()
        if bias.dtype not in _BIAS_DT:
            bias = bias.float()
        bdt = _BIAS_DT[bias.dtype]
    out = torch.empty((M, N), dtype=out_dtype or torch.bfloat16, device=a.device)
    amax = torch.empty((1,), dtype=torch.int32, device=a.device)
    _check(lib().b200q_fp8_scaled_mm_amax(_p(a), a.stride(0), _p(w), w.stride(0), _p(sa), na,
                                          _p(sb), nb, _p(sr), _p(bias), bdt, ACTS[act], _p(out),
                                          code, N, M, N, K, _p(amax), _stream(a)))
    return out, amax


def fp8_linear(x, w, w_scale=None, bias=None, out_dtype=torch.bfloat16, act=None,
               scale_result=None):
    """bf16/f16 x [..., K] -> per-tensor e4m3 quant -> FP8 scaled GEMM with w [N,K] e4m3.

    Same result as fp8_quant_tensorwise(x) followed by fp8_scaled_mm(q, w, scale,
    w_scale, scale_result, bias, out_dtype, act).  With B200Q_FUSED_PROLOGUE=1 the
    quantization runs inside the GEMM launch after one amax-reduction launch
    (b200q_fp8_linear_fused)."""
    _require_cuda(x, w, w_scale, bias, scale_result)
    shp = x.shape
    x2 = _rows_2d(x.reshape(-1, shp[-1]), "x")
    if x2.dtype not in (torch.bfloat16, torch.float16):
        raise RuntimeError(f"{TAG} fp8_linear expects bf16/f16 activations, got {x2.dtype}")
    w = _rows_2d(w, "w")
    M, K = x2.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise RuntimeError(f"{TAG} K mismatch")
    sb, nb = _scale_arg(w_scale, (1, N))
    sr, _ = _scale_arg(scale_result, (1,))
    out_dtype = out_dtype or torch.bfloat16
    code = _out_dtype_code(out_dtype, (torch.bfloat16, torch.float16, torch.float32))
    bdt = BIAS_NONE
    if bias is not None:
        bias = bias.contiguous()
        if bias.dtype not in _BIAS_DT:
            bias = bias.float()
        bdt = _BIAS_DT[bias.dtype]
    if not fused_prologue_enabled():
        q, xs = fp8_quant_tensorwise(x2)
        out = fp8_scaled_mm(q, w, xs.reshape(1), w_scale, scale_result, bias, out_dtype, act)
        return out.reshape(*shp[:-1], N)
    q = torch.empty((M, K), dtype=torch.float8_e4m3fn, device=x.device)
    xs = torch.empty((1,), dtype=torch.float32, device=x.device)
    out = torch.empty((M, N), dtype=out_dtype, device=x.device)
    sync = _sync_buffer(x2, M)
    _check(lib().b200q_fp8_linear_fused(_p(x2), _DT[x2.dtype], x2.stride(0), _p(w), w.stride(0),
                                        _p(sb), nb, _p(sr), _p(bias), bdt, ACTS[act], _p(out), code,
                                        N, M, N, K, _p(q), _p(xs), _p(sync), sync.numel(),
                                        _stream(x2)))
    return out.reshape(*shp[:-1], N)


def w8a16_linear(x, w, w_scale=None, bias=None, act=None, out_dtype=None):
    """x [..., K] bf16/f16, w [N,K] e4m3 -> act(x . w^T * w_scale + bias)."""
    _require_cuda(x, w, w_scale, bias)
    shp = x.shape
    x2 = _rows_2d(x.reshape(-1, shp[-1]), "x")
    if x2.dtype not in (torch.bfloat16, torch.float16):
        raise RuntimeError(f"{TAG} w8a16 expects bf16/f16 activations, got {x2.dtype}")
    w = _rows_2d(w, "w")
    M, K = x2.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise RuntimeError(f"{TAG} K mismatch")
    ws, _ = _scale_arg(w_scale, (1,))
    out_dtype = out_dtype or x2.dtype
    code = _out_dtype_code(out_dtype, (torch.bfloat16, torch.float16, torch.float32))
    bdt = BIAS_NONE
    if bias is not None:
        bias = bias.contiguous()
        if bias.dtype not in _BIAS_DT:
            bias = bias.float()
        bdt = _BIAS_DT[bias.dtype]
    out = torch.empty((M, N), dtype=out_dtype, device=x.device)
    wsb = int(lib().b200q_w8a16_workspace_size(M, N, K))
    work = torch.empty((wsb,), dtype=torch.uint8, device=x.device) if wsb else None
    _check(lib().b200q_w8a16_linear(_p(x2), _DT[x2.dtype], x2.stride(0), _p(w), w.stride(0),
                                    _p(ws), _p(bias), bdt, ACTS[act], _p(out), code, N, M, N, K,
                                    _p(work), wsb, _stream(x2)))
    return out.reshape(*shp[:-1], N)


def fp8_decode(t, out_dtype=torch.float32):
    _require_cuda(t)
    kinds = {torch.float8_e4m3fn: 0, torch.float8_e5m2: 1}
    if t.dtype not in kinds:
        raise RuntimeError(f"{TAG} fp8_decode expects an FP8 tensor, got {t.dtype}")
    src = t.contiguous()
    code = _out_dtype_code(out_dtype, (torch.bfloat16, torch.float16, torch.float32))
    out = torch.empty(src.shape, dtype=out_dtype, device=t.device)
    _check(lib().b200q_fp8_decode(_p(src), src.numel(), kinds[t.dtype], _p(out), code,
                                  _stream(src)))
    return out


# ----------------------------------------------------------------------------- torch.library
_LIBRARY = None


def _register_ops():
    """Register the ``b200q`` namespace (CUDA kernels + shape-only fake kernels)."""
    global _LIBRARY
    if _LIBRARY is not None:
        return
    L = torch.library.Library("b200q", "DEF")
    L.define("quant_rowwise_i8(Tensor x) -> (Tensor, Tensor)")
    L.define("quant_rowwise_i8_convrot(Tensor x, int groupsize=256) -> (Tensor, Tensor)")
    L.define("int_mm(Tensor a, Tensor b) -> Tensor")
    L.define("i8_matmul_nt(Tensor a, Tensor w) -> Tensor")
    L.define("i8_matmul_nt_fused(Tensor a, Tensor w, Tensor row_scale, Tensor? bias=None) -> Tensor")
    L.define("i8_matmul_nt_fused_cs(Tensor a, Tensor w, Tensor row_scale, Tensor col_scale, "
             "Tensor? bias=None, ScalarType out_dtype=15, str act='none') -> Tensor")
    L.define("i8_matmul_nt_fused_cs_qkv(Tensor a, Tensor w, Tensor row_scale, Tensor col_scale, "
             "Tensor? bias, int heads, int head_dim, int batch=1, ScalarType out_dtype=15) "
             "-> (Tensor, Tensor, Tensor)")
    L.define("rms_rope_partial_(Tensor(a!) q, Tensor(b!) k, Tensor freqs, Tensor q_weight, "
             "Tensor k_weight, float eps=1e-06) -> ()")
    L.define("i8_matmul_nt_fused_cs_qkv_rms_rope(Tensor a, Tensor w, Tensor row_scale, "
             "Tensor col_scale, Tensor? bias, Tensor freqs, Tensor q_weight, Tensor k_weight, "
             "int heads, int head_dim=128, float eps=1e-06, int batch=1) -> (Tensor, Tensor, Tensor)")
    L.define("i8_linear(Tensor x, Tensor w, Tensor w_scale, Tensor? bias=None, "
             "ScalarType out_dtype=15, str act='none') -> Tensor")
    L.define("fp8_quant_tensorwise(Tensor x) -> (Tensor, Tensor)")
    L.define("fp8_quant_from_amax(Tensor x, Tensor amax) -> (Tensor, Tensor)")
    L.define("fp8_scaled_mm_amax(Tensor a, Tensor w, Tensor? scale_a=None, Tensor? scale_b=None, "
             "Tensor? scale_result=None, Tensor? bias=None, ScalarType out_dtype=15, "
             "str act='none') -> (Tensor, Tensor)")
    L.define("fp8_linear(Tensor x, Tensor w, Tensor? w_scale=None, Tensor? bias=None, "
             "ScalarType out_dtype=15, str act='none', Tensor? scale_result=None) -> Tensor")
    L.define("fp8_scaled_mm(Tensor a, Tensor w, Tensor? scale_a=None, Tensor? scale_b=None, "
             "Tensor? scale_result=None, Tensor? bias=None, ScalarType out_dtype=15, "
             "str act='none') -> Tensor")
    L.define("w8a16_linear(Tensor x, Tensor w, Tensor? w_scale=None, Tensor? bias=None, "
             "str act='none', ScalarType? out_dtype=None) -> Tensor")
    L.define("fp8_decode(Tensor t, ScalarType out_dtype=6) -> Tensor")
    L.define("silu_mul_split(Tensor x) -> Tensor")
    L.define("i8_swiglu_rot(Tensor x) -> Tensor")
    L.define("i8_swiglu_quant(Tensor x, bool rotate=True) -> (Tensor, Tensor)")
    L.define("i8_matmul_nt_fused_cs_swiglu(Tensor a, Tensor w, Tensor row_scale, Tensor col_scale, "
             "Tensor? bias=None) -> Tensor")
    L.define("i8_mlp_bridge_prequant(Tensor a, Tensor w1, Tensor row_scale, Tensor col_scale, "
             "Tensor? bias=None, bool rotate=True, int tile_rows=-1) -> (Tensor, Tensor)")

    impls = {
        "quant_rowwise_i8": quant_rowwise_i8,
        "quant_rowwise_i8_convrot": quant_rowwise_i8_convrot,
        "int_mm": int_mm,
        "i8_matmul_nt": i8_matmul_nt,
        "i8_matmul_nt_fused": i8_matmul_nt_fused,
        "i8_matmul_nt_fused_cs": i8_matmul_nt_fused_cs,
        "i8_linear": i8_linear,
        "i8_matmul_nt_fused_cs_qkv": i8_matmul_nt_fused_cs_qkv,
        "rms_rope_partial_": rms_rope_partial_,
        "i8_matmul_nt_fused_cs_qkv_rms_rope": i8_matmul_nt_fused_cs_qkv_rms_rope,
        "fp8_quant_tensorwise": fp8_quant_tensorwise,
        "fp8_quant_from_amax": fp8_quant_from_amax,
        "fp8_scaled_mm_amax": lambda a, w, sa=None, sb=None, sr=None, b=None, od=torch.bfloat16,
        act="none": fp8_scaled_mm_amax(a, w, sa, sb, sr, b, od, act),
        "fp8_linear": fp8_linear,
        "fp8_scaled_mm": lambda a, w, sa=None, sb=None, sr=None, b=None, od=torch.bfloat16,
        act="none": fp8_scaled_mm(a, w, sa, sb, sr, b, od, act),
        "w8a16_linear": w8a16_linear,
        "fp8_decode": fp8_decode,
        "silu_mul_split": silu_mul_split,
        "i8_swiglu_rot": i8_swiglu_rot,
        "i8_swiglu_quant": i8_swiglu_quant,
        "i8_matmul_nt_fused_cs_swiglu": i8_matmul_nt_fused_cs_swiglu,
        "i8_mlp_bridge_prequant": i8_mlp_bridge_prequant,
    }
    for name, fn in impls.items():
        L.impl(name, fn, "CUDA")

    def fake_quant(x):
        M = x.numel() // x.shape[-1]
        return (x.new_empty((M, x.shape[-1]), dtype=torch.int8),
                x.new_empty((M, 1), dtype=torch.float32))

    fakes = {
        "quant_rowwise_i8": fake_quant,
        "quant_rowwise_i8_convrot": lambda x, groupsize=256: fake_quant(x),
        "int_mm": lambda a, b: a.new_empty((a.shape[0], b.shape[1]), dtype=torch.int32),
        "i8_matmul_nt": lambda a, w: a.new_empty((a.shape[0], w.shape[0]), dtype=torch.int32),
        "i8_matmul_nt_fused": lambda a, w, rs, bias=None: a.new_empty((a.shape[0], w.shape[0]),
                                                                      dtype=torch.bfloat16),
        "i8_matmul_nt_fused_cs": lambda a, w, rs, cs, bias=None, od=torch.bfloat16, act="none":
        a.new_empty((a.shape[0], w.shape[0]), dtype=od),
        "i8_matmul_nt_fused_cs_qkv": lambda a, w, rs, cs, bias, heads, head_dim, batch=1,
        od=torch.bfloat16: tuple(a.new_empty((batch, heads, a.shape[0] // batch, head_dim), dtype=od)
                                 for _ in range(3)),
        "rms_rope_partial_": lambda q, k, fr, qw, kw, eps=1e-6: None,
        "i8_matmul_nt_fused_cs_qkv_rms_rope": lambda a, w, rs, cs, bias, fr, qw, kw, heads,
        head_dim=128, eps=1e-6, batch=1: tuple(
            a.new_empty((batch, heads, a.shape[0] // batch, head_dim), dtype=torch.bfloat16)
            for _ in range(3)),
        "i8_linear": lambda x, w, ws, bias=None, od=torch.bfloat16, act="none": x.new_empty(
            (*x.shape[:-1], w.shape[0]), dtype=od),
        "fp8_quant_tensorwise": lambda x: (x.new_empty((x.numel() // x.shape[-1], x.shape[-1]),
                                                       dtype=torch.float8_e4m3fn),
                                           x.new_empty((), dtype=torch.float32)),
        "fp8_scaled_mm": lambda a, w, sa=None, sb=None, sr=None, b=None, od=torch.bfloat16,
        act="none": a.new_empty((a.shape[0], w.shape[0]), dtype=od),
        "fp8_scaled_mm_amax": lambda a, w, sa=None, sb=None, sr=None, b=None, od=torch.bfloat16,
        act="none": (a.new_empty((a.shape[0], w.shape[0]), dtype=od),
                     a.new_empty((1,), dtype=torch.int32)),
        "fp8_quant_from_amax": lambda x, amax: (
            x.new_empty((x.numel() // x.shape[-1], x.shape[-1]), dtype=torch.float8_e4m3fn),
            x.new_empty((), dtype=torch.float32)),
        "fp8_linear": lambda x, w, ws=None, b=None, od=torch.bfloat16, act="none", sr=None:
        x.new_empty((*x.shape[:-1], w.shape[0]), dtype=od),
        "w8a16_linear": lambda x, w, ws=None, b=None, act="none", od=None: x.new_empty(
            (*x.shape[:-1], w.shape[0]), dtype=od or x.dtype),
        "fp8_decode": lambda t, od=torch.float32: t.new_empty(t.shape, dtype=od),
        "silu_mul_split": lambda x: x.new_empty((*x.shape[:-1], x.shape[-1] // 2)),
        "i8_swiglu_rot": lambda x: x.new_empty((x.shape[0], x.shape[1] // 2)),
        "i8_swiglu_quant": lambda x, rotate=True: (
            x.new_empty((x.shape[0], x.shape[1] // 2), dtype=torch.int8),
            x.new_empty((x.shape[0], 1), dtype=torch.float32)),
        "i8_matmul_nt_fused_cs_swiglu": lambda a, w, rs, cs, bias=None: a.new_empty(
            (a.shape[0], w.shape[0] // 2), dtype=torch.bfloat16),
        "i8_mlp_bridge_prequant": lambda a, w1, rs, cs, bias=None, rotate=True, tile_rows=-1: (
            a.new_empty((a.shape[0], w1.shape[0] // 2), dtype=torch.int8),
            a.new_empty((a.shape[0], 1), dtype=torch.float32)),
    }
    for name, fn in fakes.items():
        torch.library.register_fake(f"b200q::{name}", fn, lib=L)
    _LIBRARY = L


_register_ops()
