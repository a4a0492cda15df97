"""INT8 W8A8 comfy Linear route: comfy ``int8_tensorwise`` layers on the B200 kernels.

Mirrors the reference's _patches/int8_linear_kernel_mps.py: ``install()`` wraps
``comfy.ops.mixed_precision_ops`` so each generated ``Linear.forward`` tries
``_try_int8_kernel_forward`` first (eligibility :779-830), which runs
``_int8_linear_kernel`` (:218-263): rowwise activation quant (with the 1-slot
activation cache of :97-140), then the INT8 GEMM with the epilogue chosen as in
``_int8_linear_prequant`` (:152-215) — scalar weight scale -> fused tensorwise
epilogue, per-channel [N,1] -> fused channelwise epilogue, anything else -> raw
int32 GEMM + the chunked eager rescale.  Outputs are bit-identical to
comfy_kitchen's eager ``int8_linear`` (rowwise quant -> _int_mm -> chunked
rescale -> + bias).  ``_kernel`` exposes the reference's native-module method
names on top of ``torch.ops.b200q``.

Convrot (Hadamard-rotated) checkpoints rotate inside the fused rotate+quant
kernel (groupsize 256) or with comfy_kitchen's own helpers.

SwiGLU MLPs (:538-776): ``int8_mlp_bridge(fc1, fc2, x)`` runs FC1 with SwiGLU in
the GEMM epilogue, then the convrot quant of the [M, F] activation, then FC2 --
FC1's [M, 2F] output is never formed; ``_try_int8_swiglu_forward(linear, x)``
(the ``linear_input_act(..., "swiglu")`` route) quantizes the SwiGLU of an
already materialised [M, 2F] tensor in one pass.  Opt-in: ASFP8_INT8_EXT=1.
"""
import inspect
import os
import sys
import weakref

import torch

from . import _common

TAG = "[b200q/int8_kernel]"

_installed = False
_orig_int8_linear = None
_kernel = None
_act_cache = None  # (x_weakref, convrot, groupsize, x_8, x_scale)
_LINEAR_MAX_ELEMS = 2 ** 31 - 1


def half_epilogue_problem(a, b, row_scale, col_scale, bias=None):
    """Why i8_matmul2d_nt_fused_cs_half would reject these arguments, or None.

    The checks of the reference's host function (int8_gemm.mm:1965-1980):
    tensors on the GPU, 2-D int8 A [M,K] and B [N,K] with matching K, both
    contiguous; contiguous float32 row/column scales of M and N elements;
    positive M, N, K; a bias, when given, of N elements on the GPU."""
    ts = (a, b, row_scale, col_scale)
    if not all(isinstance(t, torch.Tensor) and t.device.type == "cuda" for t in ts):
        return "inputs must be on cuda"
    if a.dtype != torch.int8 or b.dtype != torch.int8 or a.dim() != 2 or b.dim() != 2:
        return "a/b must be 2D int8"
    if a.shape[1] != b.shape[1]:
        return "K mismatch: A[M,K], B[N,K]"
    if not (a.is_contiguous() and b.is_contiguous()):
        return "a/b must be contiguous"
    if not all(t.dtype == torch.float32 and t.is_contiguous() for t in (row_scale, col_scale)):
        return "row_scale / col_scale must be contiguous float32"
    if row_scale.numel() != a.shape[0] or col_scale.numel() != b.shape[0]:
        return "row_scale must have M and col_scale N elements"
    if min(a.shape[0], b.shape[0], a.shape[1]) <= 0:
        return "matrix dimensions must be positive"
    if bias is not None and (bias.device.type != "cuda" or bias.numel() != b.shape[0]):
        return "bias must be N cuda elements"
    return None


class _NativeInt8Kernel:
    """The reference's int8_ext module surface (int8_gemm.mm:2626-2715) on b200q ops."""

    @staticmethod
    def i8_quant_rowwise(x):
        return torch.ops.b200q.quant_rowwise_i8(x)

    @staticmethod
    def i8_matmul2d_nt(a, b):
        return torch.ops.b200q.i8_matmul_nt(a, b)

    @staticmethod
    def i8_matmul2d_nt_fused(a, b, row_scale, bias=None):
        return torch.ops.b200q.i8_matmul_nt_fused(a, b, row_scale, bias)

    @staticmethod
    def i8_matmul2d_nt_fused_cs(a, b, row_scale, col_scale, bias=None, split_tail=False,
                                long_schedule=True, moss_schedule=False, out_dtype=torch.bfloat16):
        # split_tail / long / moss are Apple tile schedules; the persistent tcgen05
        # kernel covers ragged M natively, and the bytes do not depend on them.
        return torch.ops.b200q.i8_matmul_nt_fused_cs(a, b, row_scale, col_scale, bias, out_dtype)

    @staticmethod
    def i8_matmul2d_nt_fused_cs_half(a, b, row_scale, col_scale, bias=None):
        """FP16 two-rounding epilogue (int8_gemm.mm:1965-2024), with the reference
        host's argument checks (half_epilogue_problem)."""
        problem = half_epilogue_problem(a, b, row_scale, col_scale, bias)
        if problem is not None:
            raise RuntimeError(problem)
        return torch.ops.b200q.i8_matmul_nt_fused_cs(a, b, row_scale, col_scale, bias,
                                                      torch.float16)

    @staticmethod
    def i8_matmul2d_nt_fused_cs_qkv(a, b, row_scale, col_scale, bias, H, D, long_schedule=True):
        """[1, H, M, D] Q/K/V straight from the epilogue (int8_gemm.mm:2028)."""
        return torch.ops.b200q.i8_matmul_nt_fused_cs_qkv(a, b, row_scale, col_scale, bias, H, D, 1)

    @staticmethod
    def i8_matmul2d_nt_fused_cs_qkv_rms_rope(a, b, row_scale, col_scale, bias, fr, qw, kw, H, D,
                                             eps, long_schedule=True):
        """Q/K/V with Q and K RMS-normalized and rotated (int8_gemm.mm:2111).  Default:
        the scatter epilogue, then the in-place norm + RoPE kernel (two launches).
        B200Q_QKV_FUSED_NORM_ROPE=1 runs the norm and RoPE inside the GEMM epilogue
        (rotary widths that are multiples of 8); both give the same bytes, and the
        two-launch route measured faster on B200."""
        R = fr.shape[-3] if fr.dim() >= 3 else 0
        if (os.environ.get("B200Q_QKV_FUSED_NORM_ROPE", "0") == "1" and D == 128
                and R % 8 == 0):
            return torch.ops.b200q.i8_matmul_nt_fused_cs_qkv_rms_rope(
                a, b, row_scale, col_scale, bias, fr, qw, kw, H, D, float(eps), 1)
        q, k, v = torch.ops.b200q.i8_matmul_nt_fused_cs_qkv(a, b, row_scale, col_scale, bias, H, D,
                                                            1)
        torch.ops.b200q.rms_rope_partial_(q, k, fr, qw, kw, float(eps))
        return q, k, v

    @staticmethod
    def i8_swiglu_rot(x):
        return torch.ops.b200q.i8_swiglu_rot(x)

    @staticmethod
    def i8_mlp_bridge_prequant(a_i8, fc1_weight, row_scale, fc1_col_scale, fc1_bias=None,
                               long_schedule=True, tile_rows=-1):
        # long_schedule is an Apple tile schedule; tile_rows bounds the act scratch.
        return torch.ops.b200q.i8_mlp_bridge_prequant(a_i8, fc1_weight, row_scale, fc1_col_scale,
                                                      fc1_bias, True, int(tile_rows))

    @staticmethod
    def warmup():
        return None


def _int8_linear_bounded(x, weight, weight_scale, bias, out_dtype, convrot, convrot_groupsize):
    """Row-chunk calls whose element count exceeds 2**31-1 (int8_linear_kernel_mps.py:75-94).
    The kernels use 64-bit offsets; chunking keeps the quant scratch bounded."""
    flat = x.reshape(-1, x.shape[-1])
    output = torch.empty((flat.shape[0], weight.shape[0]), device=x.device, dtype=out_dtype)
    rows = max(1, min(8192, _LINEAR_MAX_ELEMS // max(flat.shape[-1], weight.shape[0])))
    for start in range(0, flat.shape[0], rows):
        stop = min(start + rows, flat.shape[0])
        chunk = flat[start:stop]
        output[start:stop].copy_(_int8_linear_kernel(chunk, weight, weight_scale, bias, out_dtype,
                                                     convrot, convrot_groupsize))
    return output.reshape(*x.shape[:-1], weight.shape[0])


def _fused_convrot_ok(groupsize, K):
    """The fused rotate+quant kernel covers groupsize 256 (the only size the
    reference's fused kernels handle).  B200Q_CONVROT_FUSED=0 keeps comfy's eager
    bf16 Hadamard matmul instead (bit-identical to the eager path; the fused
    kernel may flip a rotated value's last bf16 ulp on rare ties)."""
    from . import _native
    return (os.environ.get("B200Q_CONVROT_FUSED", "1") != "0" and groupsize == 256
            and K % 256 == 0 and K <= _native.CONVROT_MAX_K)


def _quant_cached(x, convrot, convrot_groupsize):
    """Rotate (convrot) + rowwise quant, reusing the previous result for the same
    live tensor object and settings (int8_linear_kernel_mps.py:97-140)."""
    global _act_cache
    c = _act_cache
    if c is not None and c[0]() is x and c[1] == convrot and c[2] == convrot_groupsize:
        return c[3], c[4]
    K = x.shape[-1]
    if convrot and _fused_convrot_ok(convrot_groupsize, K):
        # One pass: Hadamard rotation + rowwise quant (int8_gemm.mm:1409-1505 numerics).
        x_8, x_scale = torch.ops.b200q.quant_rowwise_i8_convrot(x.reshape(-1, K), convrot_groupsize)
    else:
        xr = x
        if convrot:
            from comfy_kitchen.tensor.int8_utils import _build_hadamard, _rotate_activation
            h = _build_hadamard(convrot_groupsize, device=x.device, dtype=x.dtype)
            xr = _rotate_activation(xr, h, convrot_groupsize)
        x_8, x_scale = _kernel.i8_quant_rowwise(xr.reshape(-1, K))
    if os.environ.get("ASFP8_INT8_ACT_CACHE", "1") != "0":
        try:
            _act_cache = (weakref.ref(x), convrot, convrot_groupsize, x_8, x_scale)
        except TypeError:
            _act_cache = None
    return x_8, x_scale


def _int8_linear_prequant(x_8, x_scale, weight, weight_scale, bias, out_dtype, input_shape):
    """Epilogue selection of int8_linear_kernel_mps.py:152-215 (fp16 outputs first
    offered to the Wan fp16 hook, :157-162)."""
    weight_scale = weight_scale.reshape(-1)
    N = weight.shape[0]
    if out_dtype == torch.float16:
        from . import wan_fp16
        result = wan_fp16.maybe_prequant(_kernel, x_8, x_scale, weight, weight_scale, bias,
                                         input_shape)
        if result is not None:
            return result
    if out_dtype in (torch.bfloat16, torch.float16) and weight_scale.numel() in (1, N):
        if out_dtype == torch.bfloat16 and weight_scale.numel() == 1:
            row_scale = (weight_scale.float() * x_scale.reshape(-1).float()).contiguous()
            bias_arg = bias.to(torch.bfloat16) if bias is not None else None
            result = _kernel.i8_matmul2d_nt_fused(x_8, weight, row_scale, bias_arg)
        else:
            bias_arg = bias.to(out_dtype) if bias is not None else None
            result = _kernel.i8_matmul2d_nt_fused_cs(
                x_8, weight, x_scale.reshape(-1).float(), weight_scale.float(), bias_arg,
                out_dtype=out_dtype)
        return result.reshape(*input_shape[:-1], N)
    # Other output dtypes: exact int32 GEMM + the eager chunked rescale.
    result = _kernel.i8_matmul2d_nt(x_8, weight)
    m, n = result.shape
    chunk_size = max(1, min(m, 256 * 1024 * 1024 // (n * 4)))
    parts = []
    for i in range(0, m, chunk_size):
        end_i = min(i + chunk_size, m)
        chunk = result[i:end_i].float() * (weight_scale * x_scale[i:end_i])
        parts.append(chunk.to(out_dtype))
    result = torch.cat(parts, dim=0)
    if bias is not None:
        result = result + bias.to(device=result.device, dtype=result.dtype)
    return result.reshape(*input_shape[:-1], N)


def _int8_linear_kernel(x, weight, weight_scale, bias=None, out_dtype=torch.bfloat16,
                        convrot=False, convrot_groupsize=256):
    """Kernel-backed drop-in for comfy_kitchen eager int8_linear (same signature)."""
    if (_kernel is None or x.device.type != "cuda" or weight.device.type != "cuda"
            or weight.dtype != torch.int8 or x.dtype not in (torch.bfloat16, torch.float16)):
        return _orig_int8_linear(x, weight, weight_scale, bias, out_dtype, convrot,
                                 convrot_groupsize)
    rows = x.numel() // x.shape[-1]
    if x.numel() > _LINEAR_MAX_ELEMS or rows * weight.shape[0] > _LINEAR_MAX_ELEMS:
        return _int8_linear_bounded(x, weight, weight_scale, bias, out_dtype, convrot,
                                    convrot_groupsize)
    x_8, x_scale = _quant_cached(x, convrot, convrot_groupsize)
    return _int8_linear_prequant(x_8, x_scale, weight, weight_scale, bias, out_dtype, x.shape)


def _try_int8_kernel_forward(self, input):
    """Layer output via the kernel W8A8 path, or None to fall back to comfy's forward
    (eligibility of int8_linear_kernel_mps.py:779-830)."""
    if _kernel is None:
        return None
    try:
        from comfy_kitchen.tensor import QuantizedTensor
    except Exception:
        return None
    if not isinstance(input, torch.Tensor) or input.device.type != "cuda":
        return None
    if isinstance(input, QuantizedTensor):
        return None
    w = self.weight
    if not isinstance(w, QuantizedTensor) or getattr(w, "_layout_cls", None) != "TensorWiseINT8Layout":
        return None
    if getattr(self, "_full_precision_mm", False) or getattr(self, "comfy_force_cast_weights", False):
        return None
    if len(getattr(self, "weight_function", [])) or len(getattr(self, "bias_function", [])):
        return None
    params = w._params
    if getattr(params, "transposed", False):
        return None
    return _int8_linear_kernel(input, w._qdata, params.scale, self.bias, input.dtype,
                               getattr(params, "convrot", False),
                               getattr(params, "convrot_groupsize", 256))


def _int8_layer_ok(layer):
    """The weight / layer eligibility shared by the routes (:563-573, :726-737)."""
    try:
        from comfy_kitchen.tensor import QuantizedTensor
    except Exception:
        return False
    w = getattr(layer, "weight", None)
    if not isinstance(w, QuantizedTensor) or getattr(w, "_layout_cls", None) != "TensorWiseINT8Layout":
        return False
    if getattr(layer, "_full_precision_mm", False) or getattr(layer, "comfy_force_cast_weights", False):
        return False
    if len(getattr(layer, "weight_function", [])) or len(getattr(layer, "bias_function", [])):
        return False
    return not getattr(w._params, "transposed", False)


def _swiglu_activation(x):
    """Materialise SwiGLU once (int8_linear_kernel_mps.py:693-705): the b200q
    silu_mul_split kernel for bf16 CUDA tensors, comfy's eager expression for
    other dtypes (as the reference does for them)."""
    wide = x.shape[-1]
    half = wide // 2
    if (_kernel is not None and x.device.type == "cuda" and x.dtype == torch.bfloat16
            and os.environ.get("ASFP8_INT8_SWIGLU_EAGERACT") != "1"):
        return torch.ops.b200q.silu_mul_split(x.reshape(-1, wide)).reshape(*x.shape[:-1], half)
    return torch.nn.functional.silu(x[..., :half]) * x[..., half:]


def _try_int8_swiglu_forward(linear, x):
    """linear(swiglu(x)) for an INT8 ``linear`` (FC2) and a wide [..., 2F] x, or
    None (int8_linear_kernel_mps.py:708-776).  bf16 input: SwiGLU (+ convrot for
    convrot checkpoints) and the per-token quant in one kernel, then the INT8
    GEMM; otherwise SwiGLU, then the ordinary INT8 route."""
    if _kernel is None:
        return None
    try:
        from comfy_kitchen.tensor import QuantizedTensor
    except Exception:
        return None
    if not isinstance(x, torch.Tensor) or x.device.type != "cuda" or isinstance(x, QuantizedTensor):
        return None
    if not _int8_layer_ok(linear):
        return None
    w = linear.weight
    params = w._params
    wide = x.shape[-1]
    if wide % 2:
        return None
    half = wide // 2
    x2 = x.reshape(-1, wide)
    convrot = getattr(params, "convrot", False)
    groupsize = getattr(params, "convrot_groupsize", 256)
    from . import _native
    if (x.dtype == torch.bfloat16 and x2.is_contiguous() and half <= _native.SWIGLU_MAX_F
            and (not convrot or (os.environ.get("ASFP8_INT8_SWIGLU_ROT", "1") == "1"
                                 and groupsize == 256 and half % 256 == 0))):
        x_8, x_scale = torch.ops.b200q.i8_swiglu_quant(x2, bool(convrot))
        return _int8_linear_prequant(x_8, x_scale, w._qdata, params.scale, linear.bias, x.dtype,
                                     x.shape)
    act = _swiglu_activation(x)
    return _int8_linear_kernel(act, w._qdata, params.scale, linear.bias, x.dtype, convrot, groupsize)


def int8_mlp_bridge(fc1, fc2, x):
    """FC2(SwiGLU(FC1(x))) for INT8 FC1/FC2 without FC1's [M, 2F] output, or None
    (int8_mlp_bridge, int8_linear_kernel_mps.py:538-690).  Same eligibility:
    bf16 contiguous 2-D x, both weights TensorWiseINT8Layout, FC2 convrot with
    groupsize 256, FC1 rows a multiple of 512 and twice FC2's input width."""
    if (_kernel is None
            or os.environ.get("ASFP8_INT8_MLP_BRIDGE", "1") != "1"
            or os.environ.get("ASFP8_INT8_SWIGLU", "1") != "1"
            or os.environ.get("ASFP8_INT8_SWIGLU_ROT", "1") != "1"):
        return None
    try:
        if (not isinstance(x, torch.Tensor) or x.dim() != 2 or x.device.type != "cuda"
                or x.dtype != torch.bfloat16 or not x.is_contiguous()):
            return None
        if not (_int8_layer_ok(fc1) and _int8_layer_ok(fc2)):
            return None
        p1, p2 = fc1.weight._params, fc2.weight._params
        if not getattr(p2, "convrot", False) or getattr(p2, "convrot_groupsize", 256) != 256:
            return None
        w1, w2 = fc1.weight._qdata, fc2.weight._qdata
        if (w1.dim() != 2 or w2.dim() != 2 or w1.shape[0] % 512 or w1.shape[1] != x.shape[1]
                or w2.shape[1] * 2 != w1.shape[0]):
            return None
        from . import _native
        if w2.shape[1] > _native.CONVROT_MAX_K:
            return None
        s1, s2 = p1.scale.view(-1), p2.scale.view(-1)
        if s1.numel() != w1.shape[0] or s2.numel() != w2.shape[0]:
            return None
        x_8, x_scale = _quant_cached(x, getattr(p1, "convrot", False),
                                     getattr(p1, "convrot_groupsize", 256))
        bias1 = fc1.bias.to(torch.bfloat16) if fc1.bias is not None else None
        fc2_8, fc2_scale = _kernel.i8_mlp_bridge_prequant(
            x_8.contiguous(), w1.contiguous(), x_scale.reshape(-1).float().contiguous(),
            s1.float().contiguous(), bias1)
        return _int8_linear_prequant(fc2_8, fc2_scale, w2, s2, fc2.bias, x.dtype, x.shape)
    except Exception as e:
        print(f"{TAG} MLP bridge fell back ({e!r})")
        return None


def _int8_qkv_prequant(layer, x, heads, head_dim, norm_rope):
    """QKV projection straight to attention layout [1, H, S, D] (int8_linear_kernel_mps.py
    :266-412): ``norm_rope`` is None for the layout-only epilogue or (freqs, q_weight_fp32,
    k_weight_fp32, eps) for the D = 128 epilogue that also normalizes and rotates Q and K.
    Returns (q, k, v) or None (the caller keeps its own path)."""
    fused = norm_rope is not None
    name = "i8_matmul2d_nt_fused_cs_qkv_rms_rope" if fused else "i8_matmul2d_nt_fused_cs_qkv"
    if (_kernel is None or not hasattr(_kernel, name)
            or os.environ.get("ASFP8_INT8_QKV_SCATTER", "1") != "1"
            or (fused and os.environ.get("ASFP8_INT8_QKV_NORM_ROPE", "1") != "1")):
        return None
    try:
        if (not isinstance(x, torch.Tensor) or x.dim() != 2 or x.device.type != "cuda"
                or x.dtype != torch.bfloat16 or not x.is_contiguous()):
            return None
        if not _int8_layer_ok(layer):
            return None
        w = layer.weight
        params = w._params
        qdata = w._qdata
        if tuple(qdata.shape) != (3 * heads * head_dim, x.shape[1]):
            return None
        weight_scale = params.scale.view(-1)
        if weight_scale.numel() != qdata.shape[0]:
            return None
        x_8, x_scale = _quant_cached(x, getattr(params, "convrot", False),
                                     getattr(params, "convrot_groupsize", 256))
        bias_arg = layer.bias.to(torch.bfloat16) if layer.bias is not None else None
        common = (x_8, qdata.contiguous(), x_scale.reshape(-1).float().contiguous(),
                  weight_scale.float().contiguous(), bias_arg)
        if fused:
            freqs, q_weight, k_weight, eps = norm_rope
            if (head_dim != 128 or not isinstance(freqs, torch.Tensor)
                    or freqs.device.type != "cuda" or freqs.dtype != torch.bfloat16
                    or not freqs.is_contiguous() or freqs.dim() < 3
                    or freqs.numel() != x.shape[0] * freqs.shape[-3] * 4
                    or 2 * freqs.shape[-3] > head_dim
                    or any(not isinstance(t, torch.Tensor) or t.device.type != "cuda"
                           or t.dtype != torch.float32 or not t.is_contiguous()
                           or t.numel() != head_dim for t in (q_weight, k_weight))):
                return None
            return getattr(_kernel, name)(*common, freqs, q_weight, k_weight, heads, head_dim,
                                          float(eps))
        return getattr(_kernel, name)(*common, heads, head_dim)
    except Exception as e:
        route = "qkv norm/RoPE epilogue" if fused else "qkv scatter"
        print(f"{TAG} {route} fell back ({e!r})")
        return None


def int8_qkv_prequant(layer, x, heads, head_dim):
    """QKV projection directly to contiguous [1, H, S, D] Q/K/V (:409-414)."""
    return _int8_qkv_prequant(layer, x, heads, head_dim, None)


def int8_qkv_rms_rope_prequant(layer, x, freqs, q_weight, k_weight, heads, head_dim, eps):
    """INT8 QKV projection + Q/K RMSNorm / partial RoPE epilogue (:417-427)."""
    return _int8_qkv_prequant(layer, x, heads, head_dim, (freqs, q_weight, k_weight, eps))


def _load_kernel():
    if not (_common.is_b200() and _common.native_ready()):
        print(f"{TAG} b200q library unavailable or device is not a B200; route not installed.")
        return None
    return _NativeInt8Kernel()


def install():
    global _installed, _orig_int8_linear, _kernel
    if _installed:
        return
    if os.environ.get("ASFP8_INT8_EXT") != "1":
        return
    if not torch.cuda.is_available():
        return
    _kernel = _load_kernel()
    if _kernel is None:
        return
    try:
        from comfy_kitchen.backends.eager.quantization import int8_linear as _orig
        _orig_int8_linear = _orig
    except Exception as e:
        print(f"{TAG} could not import eager int8_linear: {e!r}")
        return
    try:
        import comfy.ops as ops
        orig_factory = ops.mixed_precision_ops
        if getattr(orig_factory, "_asfp8_wrapped", False):
            _installed = True
            return
        factory_signature = inspect.signature(orig_factory)

        def wrapped_factory(*a, **k):
            bound = factory_signature.bind(*a, **k)
            disabled = bound.arguments.get("disabled")
            if disabled is not None:
                # comfy's hardware probe does not know this route; keep every
                # other exclusion and precision request intact.
                bound.arguments["disabled"] = [f for f in disabled if f != "int8_tensorwise"]
            cls = orig_factory(*bound.args, **bound.kwargs)
            linear_cls = getattr(cls, "Linear", None)
            if linear_cls is not None and not getattr(linear_cls, "_asfp8_int8_patched", False):
                orig_forward = linear_cls.forward

                def forward(self, input, *args, **kwargs):
                    res = _try_int8_kernel_forward(self, input)
                    if res is not None:
                        return res
                    return orig_forward(self, input, *args, **kwargs)

                linear_cls.forward = forward
                linear_cls._asfp8_int8_patched = True
            return cls

        wrapped_factory._asfp8_wrapped = True
        ops.mixed_precision_ops = wrapped_factory

        if hasattr(ops, "linear_input_act") and not getattr(ops.linear_input_act, "_asfp8_wrapped", False):
            _orig_lia = ops.linear_input_act

            def linear_input_act_wrapped(linear, x, input_act, *args, **kwargs):
                # Extended contracts (norm weights / residual epilogues) stay on
                # comfy's helper; the three-argument SwiGLU contract takes the
                # fused SwiGLU-quant route; a plain merged projection goes
                # through Linear.forward, i.e. through this route.
                if args or kwargs:
                    return _orig_lia(linear, x, input_act, *args, **kwargs)
                if input_act == "swiglu" and os.environ.get("ASFP8_INT8_SWIGLU", "1") == "1":
                    res = _try_int8_swiglu_forward(linear, x)
                    if res is not None:
                        return res
                if (input_act is None and isinstance(linear, torch.nn.Module)
                        and os.environ.get("ASFP8_INT8_PLAIN_LIA", "1") == "1"):
                    return linear(x)
                return _orig_lia(linear, x, input_act)

            linear_input_act_wrapped._asfp8_wrapped = True
            ops.linear_input_act = linear_input_act_wrapped
    except Exception as e:
        print(f"{TAG} could not wrap mixed_precision_ops: {e!r}")
        return
    _installed = True
    print(f"{TAG} comfy int8_tensorwise Linear routed to the b200q W8A8 kernels "
          f"(rowwise quant -> tcgen05 int8 GEMM -> fused dequant epilogue).")
