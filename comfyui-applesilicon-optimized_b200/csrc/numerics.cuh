// Scalar numerics shared by every b200q kernel: rounding to 16-bit floats,
// FP8 (e4m3) encode/decode, GELU, and the element-wise GEMM epilogues.
//
// This translation unit is compiled WITHOUT --use_fast_math and every
// multiply/add that must reproduce the reference's fp32 arithmetic uses the
// explicit round-to-nearest intrinsics (__fmul_rn / __fadd_rn / __fdiv_rn), so
// the compiler cannot contract them into FMAs or approximate divides.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace b200q {

enum OutDtype : int { kOutBF16 = 0, kOutF16 = 1, kOutF32 = 2, kOutI32 = 3 };
enum BiasDtype : int { kBiasNone = 0, kBiasBF16 = 1, kBiasF16 = 2, kBiasF32 = 3 };
enum Act : int { kActNone = 0, kActGeluTanh = 1, kActGeluErf = 2 };

// float -> 16-bit float -> float, round to nearest even.
__device__ __forceinline__ float round_bf16(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}
__device__ __forceinline__ float round_f16(float v) { return __half2float(__float2half_rn(v)); }

// int32 -> fp32, round to nearest even, on the ALU/FMA pipes instead of the
// conversion unit (the INT8 epilogues are bound by that unit otherwise):
// c = hi * 2^11 + lo with |hi| < 2^20 and 0 <= lo < 2^11; both parts convert
// exactly through the 1.5 * 2^23 / 2^23 magic numbers, and one fma rounds the
// exact sum once -- the same value as __int2float_rn(c) for every int32.
__device__ __forceinline__ float i2f_rn(int32_t c) {
  const int32_t hi = c >> 11;
  const int32_t lo = c & 0x7FF;
  const float fh = __fsub_rn(__int_as_float(hi + 0x4B400000), 12582912.0f);
  const float fl = __fsub_rn(__int_as_float(lo + 0x4B000000), 8388608.0f);
  return __fmaf_rn(fh, 2048.0f, fl);
}

template <typename T>
__device__ __forceinline__ float to_float(T v);
template <>
__device__ __forceinline__ float to_float<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_float<__half>(__half v) {
  return __half2float(v);
}

// FP8 e4m3 (OCP "fn" variant: no infinities, 0x7F/0xFF are NaN).
__device__ __forceinline__ uint8_t encode_e4m3_sat(float v) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}
__device__ __forceinline__ float decode_e4m3(uint8_t b) {
  __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(b), __NV_E4M3);
  return __half2float(__half(h));
}
__device__ __forceinline__ float decode_e5m2(uint8_t b) {
  __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(b), __NV_E5M2);
  return __half2float(__half(h));
}

// Two e4m3 codes (low byte first) -> two bf16 packed in 32 bits.  Exact: every
// e4m3 value is an fp16 normal and a bf16 value.
__device__ __forceinline__ uint32_t e4m3x2_to_bf16x2(uint16_t two) {
  __half2_raw h2 = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two), __NV_E4M3);
  float2 f = __half22float2(__half2(h2));
  __nv_bfloat162 b = __float22bfloat162_rn(f);
  return *reinterpret_cast<uint32_t*>(&b);
}

// GELU with the tanh approximation (torch approximate="tanh") and exact erf GELU,
// written without cancellation: for negative x the textbook forms
// 0.5 x (1 + tanh(u)) and 0.5 x (1 + erf(x / sqrt 2)) subtract two numbers close
// to 1 and lose most of fp32's digits (several fp16 ULPs at x ~ -4).  Identities
// used: 1 + tanh(u) = 2 / (1 + exp(-2u)) and 1 + erf(z) = erfc(-z).  The tanh form
// is x / (1 + t) for u >= 0 and x t / (1 + t) for u < 0, with t = exp(-2|u|) in
// (0, 1], so nothing overflows (x / (1 + exp(-2u)) turned the tiny negative tail,
// x below about -10 and results near 1e-38, into -0) and the divisor lies in
// (1, 2]: the quotient is taken as a product with rcp.approx, within a few fp32
// ULP of the IEEE quotient there.  Every activated output is checked to one
// bf16/fp16 ULP of the reference after its rounding; the IEEE divide's slow-path
// branch had kept the independent columns of an epilogue chunk from overlapping
// (5 us of a 128-token W8A16 epilogue; an FP8 up projection's epilogue outlasted
// its mainloop).
__device__ __forceinline__ float rcp_approx_ftz(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float k1 = 0.044715f;
  const float u = k0 * (x + k1 * x * x * x);
  const float t = expf(-2.0f * fabsf(u));
  return (u >= 0.0f ? x : x * t) * rcp_approx_ftz(1.0f + t);
}
__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * erfcf(-x * 0.7071067811865476f);
}
// SiLU of the reference's SwiGLU kernels (silu_mul_split_bf16,
// dit_kernels.mm:724-737; i8_swiglu_rot_bf16, int8_gemm.mm:1521-1540):
//   s = a / (1 + exp(-a)) in fp32, then rounded to bf16.
// Defined here with exp correctly rounded to fp32 and the add and divide
// correctly rounded (silu_f32_exact), so the result is one well-defined number.
//
// Fast path: exp(-a) = 2^t, t = -a log2(e) carried as t_hi + t_lo (t_hi the
// rounded product, t_lo its exact residual plus the low part of log2(e)), so
// 2^t = ex2.approx(t_hi) * (1 + t_lo ln 2) to within ex2.approx's ~2^-22;
// then s = a * rcp.approx(1 + e).  Its relative distance from the exact
// definition is below 2^-21, i.e. at most 8 fp32 ulps of s.  Rounding to bf16
// can only tell the two apart when s lies that close to a bf16 tie (low 16 bits
// near 0x8000), so those inputs -- and a < -80, where exp(-a) nears fp32
// overflow -- take the exact route through a double-precision exp.  The input
// of every SwiGLU here is a bf16 value, so the whole input domain (65,280 finite
// values) is checked against the exact definition by the tests.
__device__ __forceinline__ float silu_f32_exact_inl(float a) {
  const float e = __double2float_rn(exp(-static_cast<double>(a)));
  return __fdiv_rn(a, __fadd_rn(1.0f, e));
}
__device__ __noinline__ float silu_f32_exact(float a) { return silu_f32_exact_inl(a); }
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float silu_f32_fast(float a) {
  const float kL2eHi = 1.44269502162933349609375f;  // log2(e) rounded to fp32
  const float kL2eLo = 1.925963033500011e-08f;      // log2(e) - kL2eHi
  const float kLn2 = 0.6931471805599453f;
  // a > 100: exp(-a) < 2^-144 and 1 + exp(-a) == 1, as with the clamped argument
  const float na = fmaxf(-a, -100.0f);
  const float th = __fmul_rn(na, kL2eHi);
  const float tl = __fmaf_rn(na, kL2eLo, __fmaf_rn(na, kL2eHi, -th));
  const float p = ex2_approx(th);
  const float e = __fmaf_rn(p, __fmul_rn(tl, kLn2), p);
  return __fmul_rn(a, rcp_approx(__fadd_rn(1.0f, e)));
}
// True when the fast s = silu_f32_fast(a) may round to a different bf16 than
// the exact definition.
__device__ __forceinline__ bool silu_needs_exact(float s, float a) {
  const int lo = static_cast<int>(__float_as_uint(s) & 0xFFFFu);
  return abs(lo - 0x8000) <= 24 || !(a > -80.0f);
}
__device__ __forceinline__ float silu_bf16(float a) {
  float s = silu_f32_fast(a);
  if (silu_needs_exact(s, a)) s = silu_f32_exact(a);
  return round_bf16(s);
}
// act = bf16(bf16(silu(gate)) * up): the product of two bf16 values is exact in fp32.
__device__ __forceinline__ float swiglu_bf16(float gate, float up) {
  return round_bf16(__fmul_rn(silu_bf16(gate), up));
}

__device__ __forceinline__ float apply_act(float v, int act) {
  if (act == kActGeluTanh) return gelu_tanh(v);
  if (act == kActGeluErf) return gelu_erf(v);
  return v;
}

__device__ __forceinline__ float load_bias(const void* bias, int dtype, int n) {
  if (dtype == kBiasBF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(bias)[n]);
  if (dtype == kBiasF16) return __half2float(static_cast<const __half*>(bias)[n]);
  if (dtype == kBiasF32) return static_cast<const float*>(bias)[n];
  return 0.0f;
}

// Everything an epilogue needs besides the accumulator.  Scale pointers may be
// null (factor 1, multiply skipped); *_vec = 0 broadcasts element 0.
struct EpiArgs {
  void* out;
  int64_t ldo;  // elements
  int out_dtype;
  const float* row_scale;
  int row_scale_vec;
  const float* col_scale;
  int col_scale_vec;
  const float* extra_scale;  // one scalar (scale_result / weight scale), or null
  const void* bias;
  int bias_dtype;
  int act;
  int M, N;
  // Attention-layout scatter (qkv_heads > 0): columns [kind*H*D + h*D + d] of
  // row m = b*S + s go to qkv[kind][((b*H + h)*S + s)*D + d] (kind 0/1/2 = Q/K/V),
  // instead of out[m*ldo + n].  Requires N == 3*H*D and D % 32 == 0.
  void* qkv[3];
  int qkv_heads, qkv_dim, qkv_seq;
  // Q/K RMSNorm + split-half RoPE in the QKV epilogue (kEpiI8QkvNormRope):
  // freqs [B*S, R, 2, 2] bf16, norm weights [D] fp32 for Q and K.
  const __nv_bfloat16* rope_freqs;
  const float* q_norm_w;
  const float* k_norm_w;
  int rope_r;
  float norm_eps;
  // Pair kernel, 16-bit row-major output: stage each 32 x 32 output block in
  // shared memory and write it with a TMA store (set by the host when the
  // output is 16-byte aligned with a row stride that is a multiple of 16 bytes).
  int tma_store;
  // Pair kernel: the epilogue warps sleep this long between probes of the
  // accumulator barrier (0 = spin on try_wait).
  unsigned int wait_sleep_ns;
  // Pair kernel, scaled / dequant epilogues: when set, max |out| over the
  // stored (rounded) outputs is folded into this word with atomicMax on the
  // float bits, so that a per-tensor quant of the output needs no amax pass.
  unsigned int* amax_out;
};

// Element pointer of output (m, n) for 16-bit outputs, in either layout.
__device__ __forceinline__ uint16_t* out_ptr16(const EpiArgs& e, int64_t m, int n) {
  if (e.qkv_heads > 0) {
    const int W = e.qkv_heads * e.qkv_dim;
    const int kind = n / W;
    const int inner = n - kind * W;
    const int h = inner / e.qkv_dim;
    const int d = inner - h * e.qkv_dim;
    const int64_t b = m / e.qkv_seq;
    const int64_t s = m - b * e.qkv_seq;
    // a select, not qkv[kind]: a runtime index would copy EpiArgs to local memory
    void* base = kind == 0 ? e.qkv[0] : (kind == 1 ? e.qkv[1] : e.qkv[2]);
    return static_cast<uint16_t*>(base) + ((b * e.qkv_heads + h) * e.qkv_seq + s) * e.qkv_dim + d;
  }
  return static_cast<uint16_t*>(e.out) + m * e.ldo + n;
}

// The INT8 W8A8 dequant epilogue of the reference (int8_gemm.mm:417-443 and the
// eager chunked path int8_linear_kernel_mps.py:203-215):
//   s = col_scale[n] * row_scale[m]           (fp32, this order)
//   r = OutT(float(C) * s)                    (round #1)
//   r = OutT(float(r) + float(bias[n]))       (round #2, bias already in OutT)
// OutT is bf16 (out_dtype 0) or fp16 (out_dtype 1).
__device__ __forceinline__ float epi_i8_dequant(int32_t c, float rs, float cs, const EpiArgs& e,
                                                int n) {
  const float s = __fmul_rn(cs, rs);
  float v = __fmul_rn(i2f_rn(c), s);
  if (e.out_dtype == kOutF16) {
    v = round_f16(v);
    if (e.bias_dtype != kBiasNone) v = round_f16(__fadd_rn(v, load_bias(e.bias, e.bias_dtype, n)));
  } else {
    v = round_bf16(v);
    if (e.bias_dtype != kBiasNone)
      v = round_bf16(__fadd_rn(v, load_bias(e.bias, e.bias_dtype, n)));
  }
  // Optional activation on the (already reference-exact) result; the store
  // rounds once more to OutT.
  return e.act == kActNone ? v : apply_act(v, e.act);
}

// The FP8 scaled epilogue (scaled_mm_fp8.py:136-146 order): fp32 accumulator
// times scale_a[m], scale_b[n], scale_result, plus fp32 bias, optional GELU,
// one rounding to the output type.
__device__ __forceinline__ float epi_scaled(float acc, float rs, float cs, float xs,
                                            const EpiArgs& e, int n) {
  float v = acc;
  if (e.row_scale) v = __fmul_rn(v, rs);
  if (e.col_scale) v = __fmul_rn(v, cs);
  if (e.extra_scale) v = __fmul_rn(v, xs);
  if (e.bias_dtype != kBiasNone) v = __fadd_rn(v, load_bias(e.bias, e.bias_dtype, n));
  return apply_act(v, e.act);
}

__device__ __forceinline__ void store_out(const EpiArgs& e, int64_t m, int n, float v) {
  const int64_t off = m * e.ldo + n;
  switch (e.out_dtype) {
    case kOutBF16:
      *reinterpret_cast<__nv_bfloat16*>(out_ptr16(e, m, n)) = __float2bfloat16_rn(v);
      break;
    case kOutF16:
      *reinterpret_cast<__half*>(out_ptr16(e, m, n)) = __float2half_rn(v);
      break;
    default:
      static_cast<float*>(e.out)[off] = v;
      break;
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&p);
}
__device__ __forceinline__ uint32_t pack_f16x2(float a, float b) {
  __half2 p = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&p);
}

}  // namespace b200q

namespace b200q {
// Round two floats to bf16 / fp16 (nearest even) with one packed conversion and
// widen them back exactly (bit moves).
__device__ __forceinline__ void round_bf16x2(float& a, float& b) {
  const uint32_t p = pack_bf16x2(a, b);  // low half = a, high half = b
  a = __uint_as_float(p << 16);
  b = __uint_as_float(p & 0xFFFF0000u);
}
__device__ __forceinline__ void round_f16x2(float& a, float& b) {
  const uint32_t p = pack_f16x2(a, b);
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&p));
  a = f.x;
  b = f.y;
}
}  // namespace b200q
