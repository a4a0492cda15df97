"""CPU oracle for the quantized DiT-linear path — TEST INFRASTRUCTURE ONLY.

A restatement, in numpy (+ torch CPU for the FP8 casts), of the reference's own
CPU-side / eager semantics for the three routes.  It is imported only by the
tests, by ``__graft_entry__.smoke()`` and by ``bench.py``'s CPU-baseline leg, and
only as the checker; the product path (the CUDA library behind the torch ops)
never calls it.

Pinning: the FP8 decode table and the INT8 dequant epilogue order are checked
against the reference's own Python code run in this container
(``tests/golden/make_golden.py`` -> ``tests/golden/*.npz``).  The INT8 rowwise
quant lives in comfy_kitchen (absent here); it is pinned through the
reference's restatement (int8_gemm.mm:1337-1381) and the known-answer cases of
its tests (zero and 1e-30 rows, corner codes, ragged K).  The convrot Hadamard
is likewise comfy_kitchen's; it is restated from the reference's fused kernel
(int8_gemm.mm:1417-1480) and checked for the properties that kernel relies on
(orthonormal, symmetric, entries +-2^-4) -- parity unpinned against
comfy_kitchen itself.

Reference citations are paths inside luix93/ComfyUI-AppleSilicon-Optimized.
"""

import numpy as np
import torch

BF16_TINY = np.float32(2.0 ** -126)
F16_TINY = np.float32(2.0 ** -14)


# ------------------------------------------------------------------ roundings
def round_bf16(a):
    """float32 -> nearest-even bf16, returned as float32 (NaN preserved)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> np.uint64(16)) & np.uint64(1)
    r = ((u + np.uint64(0x7FFF) + lsb) & np.uint64(0xFFFF0000)).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(a)
    out[nan] = np.nan
    return out


def round_f16(a):
    return np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float32)


def _rounder(dtype):
    if dtype == torch.bfloat16:
        return round_bf16, BF16_TINY
    if dtype == torch.float16:
        return round_f16, F16_TINY
    raise ValueError(f"unsupported dtype {dtype}")


def to_f32(t):
    """Exact widening of a bf16/f16/f32 tensor to a float32 numpy array."""
    return t.detach().to(torch.float32).cpu().numpy()


def from_f32(a, dtype):
    """float32 numpy values that are already representable in `dtype` -> tensor."""
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dtype)


# ------------------------------------------------------------------ INT8 route
def quantize_int8_rowwise(x):
    """Per-token symmetric INT8 quant (comfy_kitchen quantize_int8_rowwise with
    stochastic rounding off, as restated step by step at
    _patches/int8_ext/int8_gemm.mm:1337-1381):

      absmax = max|x| per row (exact)
      scale  = max(absmax / 127, 1e-30)  (fp32, correctly rounded)  -> returned [M,1]
      s      = x.dtype(scale); s == 0 -> finfo(x.dtype).tiny
      q      = int8(clamp(rint(x.dtype(x / s)), -128, 127))
    """
    rnd, tiny = _rounder(x.dtype)
    xf = to_f32(x.reshape(-1, x.shape[-1]))
    absmax = np.abs(xf).max(axis=1).astype(np.float32) if xf.shape[1] else np.zeros(xf.shape[0], np.float32)
    scale = np.maximum(absmax / np.float32(127.0), np.float32(1e-30)).astype(np.float32)
    s = rnd(scale)
    s = np.where(s == 0, tiny, s).astype(np.float32)
    d = rnd((xf / s[:, None]).astype(np.float32))
    q = np.clip(np.rint(d), -128, 127).astype(np.int8)
    return torch.from_numpy(q), torch.from_numpy(scale.reshape(-1, 1))


# ------------------------------------------------------------------ convrot
def hadamard_convrot(groupsize=256):
    """The convrot rotation matrix for groupsize 256, as the reference restates
    comfy_kitchen's _build_hadamard (absent here) in its fused kernel
    (_patches/int8_ext/int8_gemm.mm:1417-1480): the regular Hadamard
    H = H4 (x) H4 (x) H4 (x) H4 with H4 = [[1,1,1,-1],[1,1,-1,1],[1,-1,1,1],
    [-1,1,1,1]], scaled by 2^-4 (entries exactly +-1/16; symmetric; H @ H = I).
    Element (i, j) is the product over the four base-4 digits of i and j of
    H4[digit_i][digit_j]; the digit order is immaterial (each factor is the
    same symmetric matrix)."""
    if groupsize != 256:
        raise ValueError("convrot groupsize 256 only (the reference's fused kernels)")
    h4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], np.float64)
    h = np.ones((1, 1))
    for _ in range(4):
        h = np.kron(h, h4)
    return h / 16.0


def rotate_convrot(x, groupsize=256):
    """x [..., K] (K % 256 == 0) rotated group by group: x_g @ H, computed exactly
    (float64: bf16/fp16 values times +-2^-4, 256-term sums) and rounded once to
    x.dtype -- the value comfy's bf16 Hadamard matmul (_patches/
    int8_linear_kernel_mps.py:119-121) and the reference's fused FWHT
    (int8_gemm.mm:1479) both approximate, up to fp32 summation order."""
    rnd, _ = _rounder(x.dtype)
    shp = x.shape
    xf = to_f32(x.reshape(-1, shp[-1])).astype(np.float64)
    K = xf.shape[1]
    if K % groupsize:
        raise ValueError("K must be a multiple of the convrot groupsize")
    h = hadamard_convrot(groupsize)
    y = (xf.reshape(-1, K // groupsize, groupsize) @ h).reshape(-1, K)
    return from_f32(rnd(y.astype(np.float32)), x.dtype).reshape(shp)


def rotate_convrot_fwht(x, groupsize=256):
    """The reference's own fp32 evaluation of the convrot rotation (the fast
    Walsh-Hadamard butterflies of i8_swiglu_rot_bf16 and i8_merge_rot_quant,
    _patches/int8_ext/int8_gemm.mm:1533-1553 and :1463-1479): per 256-group, four
    radix-4 stages with strides 1, 4, 16, 64; at each stage the element with
    base-4 digit d (of its index, at that stride) becomes, in fp32 with this
    association,
        d=0: ((a0 + a1) + a2) - a3      d=1: ((a0 + a1) - a2) + a3
        d=2: ((a0 - a1) + a2) + a3      d=3: ((a1 - a0) + a2) + a3
    where a0..a3 are the four elements of its butterfly; finally * 2^-4 (exact)
    and one rounding to x.dtype.  Differs from rotate_convrot's single rounding
    of the exact product only where fp32 sums round across a last-ulp tie."""
    if groupsize != 256:
        raise ValueError("convrot groupsize 256 only (the reference's fused kernels)")
    rnd, _ = _rounder(x.dtype)
    shp = x.shape
    w = to_f32(x.reshape(-1, shp[-1]))
    K = w.shape[1]
    if K % groupsize:
        raise ValueError("K must be a multiple of the convrot groupsize")
    w = w.reshape(-1, K // groupsize, groupsize)
    for stride in (1, 4, 16, 64):
        v = w.reshape(w.shape[0], w.shape[1], groupsize // (4 * stride), 4, stride)
        a0, a1, a2, a3 = v[..., 0, :], v[..., 1, :], v[..., 2, :], v[..., 3, :]
        out = np.empty_like(v)
        out[..., 0, :] = ((a0 + a1) + a2) - a3
        out[..., 1, :] = ((a0 + a1) - a2) + a3
        out[..., 2, :] = ((a0 - a1) + a2) + a3
        out[..., 3, :] = ((a1 - a0) + a2) + a3
        w = out.reshape(w.shape)
    y = (w.reshape(-1, K) * np.float32(0.0625)).astype(np.float32)
    return from_f32(rnd(y), x.dtype).reshape(shp)


def quantize_int8_rowwise_convrot(x, groupsize=256):
    """Convrot rotation then per-token INT8 quant (_quant_cached,
    _patches/int8_linear_kernel_mps.py:97-140)."""
    return quantize_int8_rowwise(rotate_convrot(x, groupsize))


def int_mm(a, b):
    """Exact int8 x int8 -> int32: a [M,K] @ b [K,N].  float64 BLAS is exact here
    because |sum| <= 128*128*K < 2**53 for every K this library accepts."""
    af = a.numpy().astype(np.float64)
    bf = b.numpy().astype(np.float64)
    return torch.from_numpy((af @ bf).astype(np.int64).astype(np.int32))


def int8_dequant_epilogue(c, x_scale, w_scale, bias=None, out_dtype=torch.bfloat16, act=None):
    """The eager chunked epilogue of _patches/int8_linear_kernel_mps.py:203-215
    (== fused kernels int8_gemm.mm:96-122, 417-443):
      out = T( T(float(C) * (w_scale[n] * x_scale[m])) + T(bias[n]) )
    """
    rnd, _ = _rounder(out_dtype)
    cf = c.numpy().astype(np.float32)
    ws = to_f32(w_scale.reshape(-1))
    xs = to_f32(x_scale.reshape(-1, 1))
    s = (ws[None, :] * xs).astype(np.float32)  # [M,N] (or [M,1] for a scalar scale)
    out = rnd((cf * s).astype(np.float32))
    if bias is not None:
        b = to_f32(bias.to(out_dtype).reshape(-1))
        out = rnd((out + b[None, :]).astype(np.float32))
    if act == "gelu_tanh":  # BASELINE block extension: T(gelu(result))
        out = rnd(gelu_tanh(out))
    return from_f32(out, out_dtype)


def int8_linear(x, weight, weight_scale, bias=None, out_dtype=torch.bfloat16, act=None):
    """comfy_kitchen eager int8_linear without convrot (the oracle named at
    _patches/int8_linear_kernel_mps.py:218-263): rowwise quant -> int8 GEMM with
    the [N,K] weight -> chunked rescale -> bias."""
    shp = x.shape
    q, xs = quantize_int8_rowwise(x.reshape(-1, shp[-1]))
    c = int_mm(q, weight.t())
    out = int8_dequant_epilogue(c, xs, weight_scale, bias, out_dtype, act)
    return out.reshape(*shp[:-1], weight.shape[0])


def quantize_weight_int8_per_channel(w):
    """Symmetric per-output-channel int8 weight quant (BASELINE configs 1 and 4):
    s_w[n] = absmax_n / 127, q = rint(w / s_w) clamped (round-half-even)."""
    wf = to_f32(w)
    s = np.maximum(np.abs(wf).max(axis=1) / np.float32(127.0), np.float32(1e-30)).astype(np.float32)
    q = np.clip(np.rint(wf / s[:, None]), -128, 127).astype(np.int8)
    return torch.from_numpy(q), torch.from_numpy(s.reshape(-1, 1))


# ------------------------------------------------------------------ FP8 routes
def decode_fp8(t, out_dtype=torch.float32):
    """Exact FP8 -> float decode (every code, NaNs included); equal to the
    reference's LUT decode (_patches/_common.py:203-273)."""
    return t.cpu().to(out_dtype)


def quantize_fp8_tensorwise(x):
    """Per-tensor e4m3 activation quant: scale = max(amax/448, 1e-30),
    q = e4m3(x / scale) with saturation, round-to-nearest-even."""
    xf = to_f32(x.reshape(-1, x.shape[-1]))
    amax = np.float32(np.abs(xf).max()) if xf.size else np.float32(0)
    scale = np.float32(max(np.float32(amax / np.float32(448.0)), np.float32(1e-30)))
    v = np.clip((xf / scale).astype(np.float32), -448.0, 448.0)
    q = torch.from_numpy(v).to(torch.float8_e4m3fn)
    return q, torch.tensor(scale, dtype=torch.float32)


def gelu_tanh(v):
    """tanh-GELU 0.5 v (1 + tanh u), u = sqrt(2/pi) (v + 0.044715 v^3), in float64
    as the equal form v / (1 + exp(-2u)): 1 + tanh(u) cancels for v below about
    -5 (where the result is a tiny negative number), this form does not."""
    v = np.asarray(v, dtype=np.float64)
    u = 0.7978845608028654 * (v + 0.044715 * v ** 3)
    with np.errstate(over="ignore"):
        return (v / (1.0 + np.exp(-2.0 * u))).astype(np.float32)


def _apply_scale(acc, scale, axis):
    """acc * scale in fp32; scale numel 1 (tensorwise) or per-row/per-column."""
    v = to_f32(scale)
    if v.size == 1:
        return (acc * v.reshape(())).astype(np.float32)
    return (acc * (v.reshape(-1, 1) if axis == 0 else v.reshape(1, -1))).astype(np.float32)


def scaled_mm_fp8(a, w, scale_a=None, scale_b=None, scale_result=None, bias=None,
                  out_dtype=torch.bfloat16, act=None):
    """torch._scaled_mm on e4m3 operands with the arithmetic of the reference's
    native FP8 route (_fast_route, _patches/scaled_mm_fp8.py:123-146): exact
    fp32 product (fp8fp8_matmul2d_nt), then * scale_a, * scale_b,
    * scale_result and + bias in fp32, one cast to out_dtype.  `w` is the [N,K]
    weight (torch._scaled_mm's `other` is w.t()).  `act` ("gelu_tanh") is the
    BASELINE epilogue extension, applied after the bias.  out_dtype=None returns
    the fp32 value before the final cast (what parity is measured against)."""
    af = decode_fp8(a, torch.float32).numpy().astype(np.float64)
    wf = decode_fp8(w, torch.float32).numpy().astype(np.float64)
    out = (af @ wf.T).astype(np.float32)
    if scale_a is not None:
        out = _apply_scale(out, scale_a, 0)
    if scale_b is not None:
        out = _apply_scale(out, scale_b, 1)
    if scale_result is not None:
        out = _apply_scale(out, scale_result, 0)
    if bias is not None:
        out = (out + to_f32(bias).reshape(1, -1)).astype(np.float32)
    if act == "gelu_tanh":
        out = gelu_tanh(out)
    res = torch.from_numpy(np.ascontiguousarray(out, dtype=np.float32))
    return res if out_dtype is None else res.to(out_dtype)


def scaled_mm_fp8_decode_path(a, w, scale_a=None, scale_b=None, scale_result=None, bias=None,
                              out_dtype=torch.bfloat16):
    """The reference's decode fallback of _mps_scaled_mm (_patches/scaled_mm_fp8.py:178-207):
    decode to bf16, bf16 matmul (bf16 result), fp32 scales -> bf16, fp32 bias, cast.
    Three roundings, so it is looser than the fast route; used for reporting."""
    af = decode_fp8(a, torch.float32).numpy().astype(np.float64)
    wf = decode_fp8(w, torch.float32).numpy().astype(np.float64)
    out = round_bf16((af @ wf.T).astype(np.float32))
    if scale_a is not None or scale_b is not None or scale_result is not None:
        acc = out
        if scale_a is not None:
            acc = _apply_scale(acc, scale_a, 0)
        if scale_b is not None:
            acc = _apply_scale(acc, scale_b, 1)
        if scale_result is not None:
            acc = _apply_scale(acc, scale_result, 0)
        out = round_bf16(acc)
    if bias is not None:
        out = (out + to_f32(bias).reshape(1, -1)).astype(np.float32)
    return torch.from_numpy(np.ascontiguousarray(out, dtype=np.float32)).to(out_dtype)


def w8a16_linear(x, w, w_scale=None, bias=None, act=None, out_dtype=None):
    """FP8 weight-only linear: the reference decode path (decode W -> compute
    dtype -> F.linear; _patches/linear_fp8_w8a16.py:1-11, _common.py:249) in fp32,
    plus the BASELINE per-tensor weight scale and tanh-GELU epilogue.
    out_dtype="fp32" returns the fp32 value before the final cast."""
    shp = x.shape
    xf = to_f32(x.reshape(-1, shp[-1])).astype(np.float64)
    wf = decode_fp8(w, torch.float32).numpy().astype(np.float64)
    out = (xf @ wf.T).astype(np.float32)
    if w_scale is not None:
        out = (out * to_f32(w_scale).reshape(())).astype(np.float32)
    if bias is not None:
        out = (out + to_f32(bias).reshape(1, -1)).astype(np.float32)
    if act == "gelu_tanh":
        out = gelu_tanh(out)
    res = torch.from_numpy(np.ascontiguousarray(out))
    if out_dtype != "fp32":
        res = res.to(out_dtype or x.dtype)
    return res.reshape(*shp[:-1], w.shape[0])


def _plane_exponent(amax, used):
    """Per row: e with amax * 2^e in [128, 256) (amax normal), 0 for amax == 0 or
    NaN, clamped to [-120, 126 - used] (the GEMM's planes pass, plane_exponent)."""
    a = amax.astype(np.float32)
    E = ((a.view(np.uint32) >> 23) & 0xFF).astype(np.int64)
    e = 134 - E
    e = np.minimum(e, 126 - used)
    e = np.maximum(e, -120)
    return np.where(a > 0, e, 0)


def x_planes(x, planes):
    """Exact e4m3 plane split of activation rows (the small-M W8A16 route's
    planes pass, b200q's own design -- no reference counterpart; the reference
    decodes the weight instead): returns (codes uint8 [P, M, K], exponents int
    [P, M]) with x = sum_p decode(codes[p]) * 2^-exponents[p] (exact for bf16
    with P = 2 and fp16 with P = 3, up to elements far below the row maximum).
    Plane 0 is x * 2^e0 rounded (RNE) to e4m3; plane p+1 is the remainder of
    plane p times 2^(e_{p+1} - e_p), both exponents chosen so the maximum lands
    in [128, 256)."""
    xf = to_f32(x).reshape(-1, x.shape[-1]).astype(np.float32)
    with np.errstate(invalid="ignore"):
        amax = np.nanmax(np.abs(xf), axis=1) if xf.shape[1] else np.zeros(xf.shape[0], np.float32)
    amax = np.nan_to_num(amax, nan=0.0)
    used = _plane_exponent(amax, np.zeros_like(amax, dtype=np.int64))
    exps = [used.copy()]
    r = xf * np.exp2(used.astype(np.float64)).astype(np.float32)[:, None]
    codes = []
    for p in range(planes):
        q = torch.from_numpy(np.ascontiguousarray(r)).to(torch.float8_e4m3fn)
        codes.append(q.view(torch.uint8).numpy().copy())
        r = (r - q.float().numpy()).astype(np.float32)
        if p + 1 < planes:
            rmax = np.abs(r).max(axis=1) if r.shape[1] else np.zeros(r.shape[0], np.float32)
            e = _plane_exponent(np.nan_to_num(rmax, nan=0.0), used)
            used = used + e
            exps.append(used.copy())
            r = (r * np.exp2(e.astype(np.float64)).astype(np.float32)[:, None]).astype(np.float32)
    return np.stack(codes), np.stack(exps)


def x_planes_value(codes, exps):
    """sum_p decode(codes[p]) * 2^-exps[p] in float64 ([M, K])."""
    dec = decode_fp8(torch.from_numpy(codes).view(torch.float8_e4m3fn), torch.float32).numpy()
    return sum(dec[p].astype(np.float64) * np.exp2(-exps[p].astype(np.float64))[:, None]
               for p in range(codes.shape[0]))


# ------------------------------------------------------------------ error metrics
def fp8_errors(out, ref):
    """(max|d| / rms(ref), max|d| / max|ref|): the BASELINE bound and the
    reference's own rel_err (dev/bench_gemm.py; tests/test_scaled_mm_fp8.py:79)."""
    o = out.detach().float().cpu().numpy().astype(np.float64)
    r = ref.detach().float().cpu().numpy().astype(np.float64)
    d = np.abs(o - r).max() if o.size else 0.0
    rms = np.sqrt((r ** 2).mean()) if r.size else 1.0
    mx = np.abs(r).max() if r.size else 1.0
    return float(d / max(rms, 1e-30)), float(d / max(mx, 1e-30))


def ulp_size(v, dtype=torch.bfloat16):
    """Spacing of `dtype` at |v| (float32 numpy array in, float64 out)."""
    mant = 7 if dtype == torch.bfloat16 else 10
    min_exp = -126 if dtype == torch.bfloat16 else -14
    a = np.abs(np.asarray(v, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** min_exp)))
    return 2.0 ** (e - mant)


def elementwise_ulp_ratio(out, ref32, ulps=1.0, atol_rms=1e-3):
    """max over elements of |out - ref| / (ulps * ULP(ref) + atol_rms * rms(ref)).

    <= 1 means every element is within `ulps` ULPs of the fp32 oracle value, with
    an absolute slack of atol_rms * RMS for elements so close to zero that the
    accumulation order alone can move them by more than their own ULP."""
    o = out.detach().float().cpu().numpy().astype(np.float64)
    r = ref32.detach().float().cpu().numpy().astype(np.float64)
    if not r.size:
        return 0.0
    rms = np.sqrt((r ** 2).mean())
    tol = ulps * ulp_size(r, out.dtype) + atol_rms * rms
    return float((np.abs(o - r) / tol).max())


def ulp_vs_fp32(out, ref32):
    """Max distance, in ULPs of out's dtype (bf16/f16), between `out` and the
    fp32 oracle value rounded to that dtype."""
    ref = ref32.detach().float().cpu().to(out.dtype)
    return bf16_ulp_diff(out.detach().cpu(), ref)


def bf16_ulp_diff(a, b):
    """Max distance in bf16 ULPs (ordered bit patterns) between two bf16 tensors."""
    ia = a.contiguous().view(torch.int16).numpy().astype(np.int32)
    ib = b.contiguous().view(torch.int16).numpy().astype(np.int32)

    def ordered(i):
        i = i & 0xFFFF
        return np.where(i & 0x8000, 0x8000 - (i & 0x7FFF), 0x8000 + i)

    return int(np.abs(ordered(ia) - ordered(ib)).max()) if ia.size else 0


# ------------------------------------------------------------------ QKV layout, RMSNorm, RoPE
def qkv_scatter(dense, heads, head_dim, batch=1):
    """[M, 3*H*D] -> three [B, H, S, D] attention-layout tensors (M = B*S): the
    storage change of the reference's QKV epilogue (nax_frag_store_dequant_cs_qkv,
    _patches/int8_ext/int8_gemm.mm:445-474, whose layout is the B = 1 case
    [1, H, M, D]); values are untouched."""
    M = dense.shape[0]
    S = M // batch
    return tuple(part.reshape(batch, S, heads, head_dim).permute(0, 2, 1, 3).contiguous()
                 for part in dense.split(heads * head_dim, dim=-1))


def _rms_sumsq_f32(x):
    """Sum of squares of rows x [R, D] (float32) in the reduction order the
    reference restates for native F.rms_norm (torch_rms_sumsq,
    _patches/dit_ext/dit_kernels.mm:60-80): virtual thread vt sums elements
    4vt..4vt+3 in order (fp32 multiply, then add); each group of 32 vt is
    reduced across lanes, here by the xor butterfly (offsets 16, 8, 4, 2, 1);
    the group totals are then reduced the same way (zero-padded to 32)."""
    R, D = x.shape
    vt_count = 32 * ((((D + 3) // 4) + 31) // 32)
    acc = np.zeros((R, vt_count), np.float32)
    for i in range(4):
        idx = np.arange(vt_count) * 4 + i
        ok = idx < D
        v = np.zeros((R, vt_count), np.float32)
        v[:, ok] = x[:, idx[ok]]
        acc = (acc + (v * v).astype(np.float32)).astype(np.float32)

    def butterfly(a):  # a [R, 32] -> every lane holds the xor-tree total; return lane 0
        a = a.copy()
        for o in (16, 8, 4, 2, 1):
            a = (a + a[:, np.arange(32) ^ o]).astype(np.float32)
        return a[:, 0]

    groups = vt_count // 32
    sums = np.zeros((R, 32), np.float32)
    for gi in range(groups):
        sums[:, gi] = butterfly(acc[:, 32 * gi:32 * gi + 32])
    return butterfly(sums)


def rms_rope_partial(q, k, freqs, q_weight, k_weight, eps):
    """In-place semantics of rms_rope_attention_partial
    (_patches/dit_ext/dit_kernels.mm:825-874), returned as new tensors:
      y   = bf16((x * rsqrt(sumsq / D + eps)) * w[d])          per (b, h, s) row
      d >= 2R: out = y;  d < 2R: i = d mod R, r = d >= R, m = freqs[row][i][r]
      r = 0: bf16(bf16(m0 * y[i]) + m1 * y[i+R]);  r = 1: bf16(bf16(m1 * y[i+R]) + m0 * y[i])
    q, k [B, H, S, D] bf16; freqs [B*S, R, 2, 2] bf16 (rotation matrix rows per
    token row m = b*S + s); weights fp32 [D].  fp32 arithmetic throughout, the
    rsqrt correctly rounded."""
    B, H, S, D = q.shape
    fr = to_f32(freqs).reshape(B * S, -1, 2, 2)
    R = fr.shape[1]

    def one(t, w):
        x = to_f32(t).reshape(B, H, S, D)
        rows = x.reshape(-1, D)
        tot = _rms_sumsq_f32(rows)
        mean = (tot.astype(np.float64) / D).astype(np.float32)
        inv = (1.0 / np.sqrt((mean + np.float32(eps)).astype(np.float32).astype(np.float64))).astype(np.float32)
        wv = np.asarray(w, np.float32).reshape(1, D)
        y = round_bf16(((rows * inv[:, None]).astype(np.float32) * wv).astype(np.float32))
        y = y.reshape(B, H, S, D)
        out = y.copy()
        m_idx = (np.arange(B)[:, None] * S + np.arange(S)[None, :])  # [B, S]
        mat = fr[m_idx]  # [B, S, R, 2, 2]
        yi = y[..., :R]          # [B, H, S, R]
        yr = y[..., R:2 * R]
        m00 = mat[:, None, :, :, 0, 0]; m01 = mat[:, None, :, :, 0, 1]
        m10 = mat[:, None, :, :, 1, 0]; m11 = mat[:, None, :, :, 1, 1]
        out[..., :R] = round_bf16((round_bf16((m00 * yi).astype(np.float32)) + (m01 * yr).astype(np.float32)).astype(np.float32))
        out[..., R:2 * R] = round_bf16((round_bf16((m11 * yr).astype(np.float32)) + (m10 * yi).astype(np.float32)).astype(np.float32))
        return from_f32(out, torch.bfloat16)

    return one(q, q_weight), one(k, k_weight)


# ------------------------------------------------------------------ SwiGLU bridge
def silu_f32(a):
    """silu(a) = a / (1 + exp(-a)) evaluated as the reference's kernels do, in
    fp32 (silu_mul_split_bf16, _patches/dit_ext/dit_kernels.mm:724-737;
    i8_swiglu_rot_bf16, _patches/int8_ext/int8_gemm.mm:1521-1540), with exp
    correctly rounded to fp32 (float64 exp, then one rounding; overflow -> inf,
    so a < -88.7 gives -0 as the fp32 formula does) and the add and divide
    correctly rounded."""
    a = np.asarray(a, dtype=np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        e = np.exp(-a.astype(np.float64)).astype(np.float32)
        d = (np.float32(1.0) + e).astype(np.float32)
        return (a / d).astype(np.float32)


def swiglu(wide):
    """wide [..., 2F] (bf16) -> act [..., F] = bf16(bf16(silu(gate)) * up), gate
    = the first F columns, up = the last F (silu_mul_split_bf16; the same
    operation sequence as i8_swiglu_rot_bf16's first step).  The product of two
    bf16 values is exact in fp32, so it is rounded once."""
    w = to_f32(wide)
    F = w.shape[-1] // 2
    s = round_bf16(silu_f32(w[..., :F]))
    with np.errstate(over="ignore"):  # |product| > fp32 max -> inf, as on the device
        return from_f32(round_bf16((s * w[..., F:]).astype(np.float32)), torch.bfloat16)


def swiglu_rot(wide):
    """i8_swiglu_rot (_patches/int8_ext/int8_gemm.mm:1521-1555): the 256-group
    convrot rotation of swiglu(wide) with the reference kernel's fp32
    butterflies, bf16."""
    return rotate_convrot_fwht(swiglu(wide))


def swiglu_quant(wide, rotate=True):
    """The FC2 pre-pass of _try_int8_swiglu_forward
    (_patches/int8_linear_kernel_mps.py:757-773): per-token INT8 quant of the
    (rotated) SwiGLU activation -> (q int8 [M, F], scale f32 [M, 1])."""
    act = swiglu_rot(wide) if rotate else swiglu(wide)
    return quantize_int8_rowwise(act.reshape(-1, act.shape[-1]))


def fc1_swiglu(a, w, row_scale, col_scale, bias=None):
    """FC1 of the bridge: int8 GEMM + the channelwise two-rounding bf16 dequant
    (+ bias) of i8_matmul2d_nt_fused_cs (int8_gemm.mm:417-443), then swiglu.
    w [2F, K] has rows [gate; up]."""
    c = int_mm(a, w.t())
    wide = int8_dequant_epilogue(c, row_scale.reshape(-1, 1), col_scale.reshape(-1), bias,
                                 torch.bfloat16)
    return swiglu(wide)


def mlp_bridge_prequant(a, w, row_scale, col_scale, bias=None, rotate=True):
    """i8_mlp_bridge_prequant (int8_gemm.mm:2377-2537; rotate=True there): the
    FC2 input (q, scale) of FC1 -> SwiGLU -> convrot -> rowwise quant."""
    act = fc1_swiglu(a, w, row_scale, col_scale, bias)
    if rotate:
        act = rotate_convrot_fwht(act)
    return quantize_int8_rowwise(act)
