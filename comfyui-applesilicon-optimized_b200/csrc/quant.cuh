// Activation quantization kernels.
//
//  * quant_rowwise_i8: per-token symmetric INT8 quantization, bit-exact to the
//    reference's rowwise quant (int8_gemm.mm:1337-1381, which restates
//    comfy_kitchen quantize_int8_rowwise with stochastic rounding off):
//      absmax = max|x|                      (exact)
//      scale  = max(absmax / 127, 1e-30)    (correctly rounded fp32 divide) -> returned
//      s      = T(scale); s == 0 -> smallest normal of T
//      q      = int8(clamp(rint(T(x / s)), -128, 127))   (T = input dtype, RNE)
//    One CTA of 256 threads per row, 16-byte loads; the row stays in registers
//    between the absmax and the quantize pass (K <= 16384 for bf16/fp16), so HBM
//    sees one read of x and one write of q.  x / s is formed as x * RN(1/s) with
//    an exact-divide fallback near rounding ties (quotients8 below), which gives
//    the divide's result bit for bit at a fraction of its cost.
//
//  * fp8 per-tensor quant (the activation side of the FP8 W8A8 route):
//      amax = max|x| over the tensor; scale = max(amax / 448, 1e-30)
//      q = e4m3_satfinite_rne(x / scale)
//    Two launches: a grid-stride absmax reduction (atomicMax on the float's bit
//    pattern, valid because the values are non-negative) and the quantize pass.
#pragma once

#include "numerics.cuh"
#include "ptx.cuh"

namespace b200q {

constexpr int kQuantThreads = 256;
constexpr int kQuantMaxVec = 8;  // 16-byte vectors per thread kept in registers

template <typename T>
__device__ __forceinline__ float absmax8(const uint4& v) {
  const T* e = reinterpret_cast<const T*>(&v);
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(to_float<T>(e[i])));
  return m;
}

template <typename T>
__device__ __forceinline__ float round_to(float v);
template <>
__device__ __forceinline__ float round_to<__nv_bfloat16>(float v) {
  return round_bf16(v);
}
template <>
__device__ __forceinline__ float round_to<__half>(float v) {
  return round_f16(v);
}

template <typename T>
__device__ __forceinline__ float smallest_normal();
template <>
__device__ __forceinline__ float smallest_normal<__nv_bfloat16>() {
  return 1.1754943508222875e-38f;  // 2^-126
}
template <>
__device__ __forceinline__ float smallest_normal<__half>() {
  return 6.103515625e-05f;  // 2^-14
}

// The quotient x / s in the input dtype, rounded, clamped, as an int8 code.
template <typename T>
__device__ __forceinline__ int quant_code(float x, float s_math) {
  float d = round_to<T>(__fdiv_rn(x, s_math));
  d = rintf(d);
  d = fminf(fmaxf(d, -128.0f), 127.0f);
  return static_cast<int>(d);
}


__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------------------
// Quotients without a divide per element.
//
// The reference computes q = round(x / s) with a correctly rounded fp32 divide
// and then rounds that quotient to a coarser format F (bf16/fp16 before rint
// for int8, e4m3 for fp8).  Here y = RN(x * r) with r = RN(1/s):
//   y = (x/s)(1+d1)(1+d2), |d1|,|d2| <= 2^-24   =>   |y - RN(x/s)| <= 3 ulp.
// Rounding to F drops the low bits of the fp32 pattern and only changes
// outcome where those bits cross the tie pattern 100..0.  So when the dropped
// bits of y are more than 4 ulps away from the tie, y and RN(x/s) round to the
// same F value and y is used; otherwise (about 9 in 2^16 values for bf16) the
// exact __fdiv_rn quotient is taken.  The result is therefore identical to
// round_F(__fdiv_rn(x, s)) for every input.
//
// Range notes: for fp16 the 13-bit rule is only the tie rule in fp16's normal
// range; below it (|y| < 2^-14) rint gives 0 whichever way the quotient
// rounds, so the code is unaffected.  For e4m3 the 20-bit rule holds in the
// normal range (|y| >= 2^-6); nonzero quotients below it take the exact path.
template <typename T>
struct TieBits;
template <>
struct TieBits<__nv_bfloat16> {
  static constexpr uint32_t kMask = 0xFFFFu, kTie = 0x8000u;
};
template <>
struct TieBits<__half> {
  static constexpr uint32_t kMask = 0x1FFFu, kTie = 0x1000u;
};

template <typename T>
__device__ __forceinline__ bool near_tie(float y) {
  return (__float_as_uint(y) & TieBits<T>::kMask) - (TieBits<T>::kTie - 4u) <= 8u;
}

__device__ __forceinline__ bool near_tie_e4m3(float y) {
  const uint32_t b = __float_as_uint(y);
  const uint32_t mag = b & 0x7FFFFFFFu;
  return (mag < 0x3C800000u && mag != 0u) || (b & 0xFFFFFu) - (0x80000u - 4u) <= 8u;
}

// Eight quotients x[i] / s, each equal to __fdiv_rn(x[i], s) wherever the
// rounding to F could tell them apart (F = T, or e4m3 when E4M3 is true).  The
// exact divides sit in one rarely taken branch after the straight-line path.
template <typename T, bool E4M3>
__device__ __forceinline__ void quotients8(const uint4& v, float s, float r, float (&y)[8]) {
  const T* e = reinterpret_cast<const T*>(&v);
  uint32_t slow = 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    y[i] = __fmul_rn(to_float<T>(e[i]), r);
    const bool t = E4M3 ? near_tie_e4m3(y[i]) : near_tie<T>(y[i]);
    slow |= t ? (1u << i) : 0u;
  }
  if (slow) {  // fully unrolled: a runtime index would move y[] to local memory
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if ((slow >> i) & 1u) y[i] = __fdiv_rn(to_float<T>(e[i]), s);
  }
}

template <typename T>
__device__ __forceinline__ uint2 quant8_fast(const uint4& v, float s, float r) {
  float y[8];
  quotients8<T, false>(v, s, r, y);
  uint32_t w[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float d = fminf(fmaxf(rintf(round_to<T>(y[i])), -128.0f), 127.0f);
    w[i >> 2] |= (static_cast<uint32_t>(static_cast<int>(d)) & 0xFFu) << (8 * (i & 3));
  }
  return make_uint2(w[0], w[1]);
}

template <typename T>
__device__ __forceinline__ uint2 fp8_quant8_fast(const uint4& v, float s, float r) {
  float y[8];
  quotients8<T, true>(v, s, r, y);
  uint32_t w[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 8; ++i) w[i >> 2] |= static_cast<uint32_t>(encode_e4m3_sat(y[i])) << (8 * (i & 3));
  return make_uint2(w[0], w[1]);
}

// Row scale from the row's absmax; writes scales[row], returns s_math.
template <typename T>
__device__ __forceinline__ float row_scale_from_absmax(float amax, float* red, float* bcast,
                                                       float* scales, int row) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  amax = warp_max(amax);
  if (lane == 0) red[warp] = amax;
  __syncthreads();
  if (warp == 0) {
    float m = lane < kQuantThreads / 32 ? red[lane] : 0.0f;
    m = warp_max(m);
    if (lane == 0) {
      const float sc = fmaxf(__fdiv_rn(m, 127.0f), 1e-30f);
      scales[row] = sc;
      float s = round_to<T>(sc);
      if (s == 0.0f) s = smallest_normal<T>();
      *bcast = s;
    }
  }
  __syncthreads();
  return *bcast;
}

// Vector path: rows start 16-byte aligned and K % 8 == 0.
template <typename T>
__global__ void __launch_bounds__(kQuantThreads)
    quant_rowwise_i8_vec_kernel(const T* __restrict__ x, int64_t ldx, int8_t* __restrict__ q,
                                int64_t ldq, float* __restrict__ scales, int M, int K) {
  __shared__ float red[kQuantThreads / 32];
  __shared__ float bcast;
  const int nvec = K >> 3;
  for (int row = blockIdx.x; row < M; row += gridDim.x) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(row) * ldx);
    uint2* qr = reinterpret_cast<uint2*>(q + static_cast<int64_t>(row) * ldq);
    uint4 v[kQuantMaxVec];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < kQuantMaxVec; ++i) {
      const int idx = threadIdx.x + i * kQuantThreads;
      if (idx < nvec) {
        v[i] = __ldcs(xr + idx);
        amax = fmaxf(amax, absmax8<T>(v[i]));
      }
    }
    for (int idx = threadIdx.x + kQuantMaxVec * kQuantThreads; idx < nvec; idx += kQuantThreads)
      amax = fmaxf(amax, absmax8<T>(xr[idx]));
    const float s_math = row_scale_from_absmax<T>(amax, red, &bcast, scales, row);
    const float r_math = __frcp_rn(s_math);
#pragma unroll
    for (int i = 0; i < kQuantMaxVec; ++i) {
      const int idx = threadIdx.x + i * kQuantThreads;
      if (idx < nvec) qr[idx] = quant8_fast<T>(v[i], s_math, r_math);
    }
    for (int idx = threadIdx.x + kQuantMaxVec * kQuantThreads; idx < nvec; idx += kQuantThreads)
      qr[idx] = quant8_fast<T>(xr[idx], s_math, r_math);
    __syncthreads();  // red/bcast are reused by the next row
  }
}

// Scalar path for any K / alignment.
template <typename T>
__global__ void __launch_bounds__(kQuantThreads)
    quant_rowwise_i8_scalar_kernel(const T* __restrict__ x, int64_t ldx, int8_t* __restrict__ q,
                                   int64_t ldq, float* __restrict__ scales, int M, int K) {
  __shared__ float red[kQuantThreads / 32];
  __shared__ float bcast;
  for (int row = blockIdx.x; row < M; row += gridDim.x) {
    const T* xr = x + static_cast<int64_t>(row) * ldx;
    int8_t* qr = q + static_cast<int64_t>(row) * ldq;
    float amax = 0.0f;
    for (int i = threadIdx.x; i < K; i += kQuantThreads) amax = fmaxf(amax, fabsf(to_float<T>(xr[i])));
    const float s_math = row_scale_from_absmax<T>(amax, red, &bcast, scales, row);
    for (int i = threadIdx.x; i < K; i += kQuantThreads)
      qr[i] = static_cast<int8_t>(quant_code<T>(to_float<T>(xr[i]), s_math));
    __syncthreads();
  }
}

// ------------------------------------------------------------ convrot + INT8
// Convrot rotation fused into the per-token quant (the _quant_cached path with
// convrot, _patches/int8_linear_kernel_mps.py:97-140; the reference's fused
// form is i8_merge_rot_quant, _patches/int8_ext/int8_gemm.mm:1409-1505).
// Each 256-wide group of a row is multiplied by the regular Hadamard
// H = H4 (x) H4 (x) H4 (x) H4 / 16, H4 = [[1,1,1,-1],[1,1,-1,1],[1,-1,1,1],
// [-1,1,1,1]], as four radix-4 butterfly stages in fp32 (strides 1, 4, 16, 64,
// each output the row of H4 selected by its base-4 digit, evaluated in the
// reference's term order), then * 2^-4 (exact) and one rounding to the input
// dtype.  The rotated row stays in shared memory for the absmax and the
// quantize pass, which follow quant_rowwise_i8 exactly.  All groups of a row
// advance through a stage together (ping-pong buffers of K floats), so a row
// costs four block barriers whatever its width.
constexpr int kRotGroup = 256;

// Four radix-4 butterfly stages (strides 1, 4, 16, 64) of the unnormalised
// 256-point Hadamard over every 256-wide group of src[0, K), ping-ponging with
// dst; returns the buffer that holds the result.  Thread t owns position t of
// every group (kQuantThreads == kRotGroup).  The caller synchronises after
// filling src; the stages synchronise after each pass.
__device__ __forceinline__ float* convrot_stages(float* src, float* dst, int K) {
  const int t = threadIdx.x;
#pragma unroll
  for (int stride = 1; stride <= 64; stride *= 4) {
    const int digit = (t / stride) & 3;
    const int base = t - digit * stride;
    for (int g0 = 0; g0 < K; g0 += kRotGroup) {
      const float a0 = src[g0 + base];
      const float a1 = src[g0 + base + stride];
      const float a2 = src[g0 + base + 2 * stride];
      const float a3 = src[g0 + base + 3 * stride];
      float y;
      if (digit == 0) y = __fsub_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
      else if (digit == 1) y = __fadd_rn(__fsub_rn(__fadd_rn(a0, a1), a2), a3);
      else if (digit == 2) y = __fadd_rn(__fadd_rn(__fsub_rn(a0, a1), a2), a3);
      else y = __fadd_rn(__fadd_rn(__fsub_rn(a1, a0), a2), a3);
      dst[g0 + t] = y;
    }
    __syncthreads();
    float* tmp = src;
    src = dst;
    dst = tmp;
  }
  return src;
}

// Codes of one row whose values (already T-representable) sit in shared memory:
// the divide-free quotient with the exact fallback near T's rounding ties.
template <typename T>
__device__ __forceinline__ void quant_row_smem(const float* src, int K, float s_math, int8_t* qr,
                                               bool vec) {
  const int t = threadIdx.x;
  const float r_math = __frcp_rn(s_math);
  if (vec && (reinterpret_cast<uintptr_t>(qr) % 8 == 0)) {
    for (int i = t; i < (K >> 3); i += kQuantThreads) {
      float y[8];
      uint32_t w[2] = {0u, 0u};
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = src[8 * i + j];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float d = __fmul_rn(y[j], r_math);
        if (near_tie<T>(d)) d = __fdiv_rn(y[j], s_math);
        d = fminf(fmaxf(rintf(round_to<T>(d)), -128.0f), 127.0f);
        w[j >> 2] |= (static_cast<uint32_t>(static_cast<int>(d)) & 0xFFu) << (8 * (j & 3));
      }
      reinterpret_cast<uint2*>(qr)[i] = make_uint2(w[0], w[1]);
    }
  } else {
    for (int i = t; i < K; i += kQuantThreads) qr[i] = static_cast<int8_t>(quant_code<T>(src[i], s_math));
  }
}

template <typename T>
__global__ void __launch_bounds__(kQuantThreads)
    quant_rowwise_i8_rot_kernel(const T* __restrict__ x, int64_t ldx, int8_t* __restrict__ q,
                                int64_t ldq, float* __restrict__ scales, int M, int K) {
  extern __shared__ float rot_smem[];
  float* bufa = rot_smem;
  float* bufb = rot_smem + K;
  __shared__ float red[kQuantThreads / 32];
  __shared__ float bcast;
  const int t = threadIdx.x;  // position inside every 256-wide group
  const bool vec = (K % 8 == 0) && (ldx % 8 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0);
  for (int row = blockIdx.x; row < M; row += gridDim.x) {
    const T* xr = x + static_cast<int64_t>(row) * ldx;
    if (vec) {
      for (int i = t; i < (K >> 3); i += kQuantThreads) {
        const uint4 v = __ldcs(reinterpret_cast<const uint4*>(xr) + i);
        const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
        for (int j = 0; j < 8; ++j) bufa[8 * i + j] = to_float<T>(e[j]);
      }
    } else {
      for (int i = t; i < K; i += kQuantThreads) bufa[i] = to_float<T>(xr[i]);
    }
    __syncthreads();
    float* src = convrot_stages(bufa, bufb, K);
    // src holds the unscaled rotation; scale by 2^-4 (exact), round to T once.
    float amax = 0.0f;
    for (int i = t; i < K; i += kQuantThreads) {
      const float r = round_to<T>(src[i] * 0.0625f);
      src[i] = r;
      amax = fmaxf(amax, fabsf(r));
    }
    const float s_math = row_scale_from_absmax<T>(amax, red, &bcast, scales, row);
    quant_row_smem<T>(src, K, s_math, q + static_cast<int64_t>(row) * ldq, vec && (ldq % 8 == 0));
    __syncthreads();  // buffers and red/bcast are reused by the next row
  }
}

// ------------------------------------------------------------ SwiGLU rows
// One CTA per row (grid-stride) of a split-half [M, 2F] bf16 tensor x (gate =
// columns [0, F), up = [F, 2F)):
//   act = bf16(bf16(silu(gate)) * up)                       (silu_mul_split_bf16,
//                                                            dit_kernels.mm:724-737)
//   ROT:   act <- bf16(H256(act) * 2^-4) per 256-group     (i8_swiglu_rot_bf16,
//                                                            int8_gemm.mm:1521-1555)
//   QUANT: per-token INT8 codes + scale of act              (i8_quant_rowwise,
//                                                            int8_gemm.mm:1337-1381)
//   else:  act written to out [M, F] (bf16).
// Shared memory: ROT 2F floats, QUANT without ROT F floats, neither none.
template <bool ROT, bool QUANT>
__global__ void __launch_bounds__(kQuantThreads)
    swiglu_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int F,
                       __nv_bfloat16* __restrict__ out, int64_t ldo, int8_t* __restrict__ q,
                       int64_t ldq, float* __restrict__ scales, int M) {
  extern __shared__ float rot_smem[];
  float* bufa = rot_smem;
  float* bufb = rot_smem + F;
  __shared__ float red[kQuantThreads / 32];
  __shared__ float bcast;
  constexpr bool kSmem = ROT || QUANT;
  const int t = threadIdx.x;
  const bool vec = (F % 8 == 0) && (ldx % 8 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0);
  const bool vec_out = !kSmem && vec && (ldo % 8 == 0) && (reinterpret_cast<uintptr_t>(out) % 16 == 0);
  for (int row = blockIdx.x; row < M; row += gridDim.x) {
    const __nv_bfloat16* xr = x + static_cast<int64_t>(row) * ldx;
    __nv_bfloat16* orow = out + static_cast<int64_t>(row) * ldo;
    if (vec) {
      for (int i = t; i < (F >> 3); i += kQuantThreads) {
        const uint4 gv = __ldcs(reinterpret_cast<const uint4*>(xr) + i);
        const uint4 uv = __ldcs(reinterpret_cast<const uint4*>(xr + F) + i);
        const __nv_bfloat16* ge = reinterpret_cast<const __nv_bfloat16*>(&gv);
        const __nv_bfloat16* ue = reinterpret_cast<const __nv_bfloat16*>(&uv);
        float a[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) a[j] = swiglu_bf16(__bfloat162float(ge[j]), __bfloat162float(ue[j]));
        if constexpr (kSmem) {
#pragma unroll
          for (int j = 0; j < 8; ++j) bufa[8 * i + j] = a[j];
        } else if (vec_out) {
          reinterpret_cast<uint4*>(orow)[i] =
              make_uint4(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]), pack_bf16x2(a[4], a[5]),
                         pack_bf16x2(a[6], a[7]));
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) orow[8 * i + j] = __float2bfloat16_rn(a[j]);
        }
      }
    } else {
      for (int i = t; i < F; i += kQuantThreads) {
        const float a = swiglu_bf16(__bfloat162float(xr[i]), __bfloat162float(xr[F + i]));
        if constexpr (kSmem) bufa[i] = a;
        else orow[i] = __float2bfloat16_rn(a);
      }
    }
    if constexpr (kSmem) {
      __syncthreads();
      float* src = bufa;
      if constexpr (ROT) {
        src = convrot_stages(bufa, bufb, F);
        for (int i = t; i < F; i += kQuantThreads) src[i] = round_bf16(src[i] * 0.0625f);
      }
      if constexpr (QUANT) {
        float amax = 0.0f;
        for (int i = t; i < F; i += kQuantThreads) amax = fmaxf(amax, fabsf(src[i]));
        const float s_math = row_scale_from_absmax<__nv_bfloat16>(amax, red, &bcast, scales, row);
        quant_row_smem<__nv_bfloat16>(src, F, s_math, q + static_cast<int64_t>(row) * ldq,
                                      (F % 8 == 0) && (ldq % 8 == 0));
      } else {
        for (int i = t; i < F; i += kQuantThreads) orow[i] = __float2bfloat16_rn(src[i]);
      }
      __syncthreads();  // buffers and red/bcast are reused by the next row
    }
  }
}

// ------------------------------------------------------------ FP8 per-tensor
// Two addressing modes, chosen per launch: contiguous tensors (ldx == K) are
// walked as one flat array of 16-byte vectors; strided ones row by row (one
// CTA per row, grid-stride over rows).  No 64-bit division in either loop.
__device__ __forceinline__ void block_atomic_max(float m, unsigned int* amax_bits) {
  m = warp_max(m);
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    v = warp_max(v);
    if (threadIdx.x == 0) atomicMax(amax_bits, __float_as_uint(v));
  }
}

// amax_bits must be zeroed before the launch.  Rows of length K with stride ldx.
template <typename T>
__global__ void __launch_bounds__(256)
    absmax_kernel(const T* __restrict__ x, int64_t ldx, int64_t M, int K, unsigned int* amax_bits) {
  float m0 = 0.0f, m1 = 0.0f;
  const bool vec = (K % 8 == 0) && (ldx % 8 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0);
  if (vec && ldx == K) {
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    const int64_t nvec = (M * static_cast<int64_t>(K)) >> 3;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    for (; i + stride < nvec; i += 2 * stride) {
      const uint4 a = __ldcs(xv + i), b = __ldcs(xv + i + stride);
      m0 = fmaxf(m0, absmax8<T>(a));
      m1 = fmaxf(m1, absmax8<T>(b));
    }
    if (i < nvec) m0 = fmaxf(m0, absmax8<T>(__ldcs(xv + i)));
  } else {
    for (int64_t r = blockIdx.x; r < M; r += gridDim.x) {
      const T* xr = x + r * ldx;
      if (vec) {
        for (int c = threadIdx.x; c < (K >> 3); c += blockDim.x)
          m0 = fmaxf(m0, absmax8<T>(__ldcs(reinterpret_cast<const uint4*>(xr) + c)));
      } else {
        for (int c = threadIdx.x; c < K; c += blockDim.x) m0 = fmaxf(m0, fabsf(to_float<T>(xr[c])));
      }
    }
  }
  block_atomic_max(fmaxf(m0, m1), amax_bits);
}

__device__ __forceinline__ float fp8_scale_from_amax(unsigned int bits) {
  return fmaxf(__fdiv_rn(__uint_as_float(bits), 448.0f), 1e-30f);
}


template <typename T>
__global__ void __launch_bounds__(256)
    fp8_quantize_kernel(const T* __restrict__ x, int64_t ldx, int64_t M, int K,
                        const unsigned int* __restrict__ amax_bits, uint8_t* __restrict__ q,
                        int64_t ldq, float* __restrict__ scale_out) {
  const float s = fp8_scale_from_amax(*amax_bits);
  const float r = __frcp_rn(s);
  if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = s;
  const bool vec = (K % 8 == 0) && (ldx % 8 == 0) && (ldq % 8 == 0) &&
                   (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(q) % 8 == 0);
  if (vec && ldx == K && ldq == K) {
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    uint2* qv = reinterpret_cast<uint2*>(q);
    const int64_t nvec = (M * static_cast<int64_t>(K)) >> 3;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    for (; i + stride < nvec; i += 2 * stride) {
      const uint4 a = __ldcs(xv + i), b = __ldcs(xv + i + stride);
      qv[i] = fp8_quant8_fast<T>(a, s, r);
      qv[i + stride] = fp8_quant8_fast<T>(b, s, r);
    }
    if (i < nvec) qv[i] = fp8_quant8_fast<T>(__ldcs(xv + i), s, r);
  } else {
    for (int64_t r = blockIdx.x; r < M; r += gridDim.x) {
      const T* xr = x + r * ldx;
      uint8_t* qr = q + r * ldq;
      if (vec) {
        for (int c = threadIdx.x; c < (K >> 3); c += blockDim.x)
          reinterpret_cast<uint2*>(qr)[c] =
              fp8_quant8_fast<T>(__ldcs(reinterpret_cast<const uint4*>(xr) + c), s, r);
      } else {
        for (int c = threadIdx.x; c < K; c += blockDim.x)
          qr[c] = encode_e4m3_sat(__fdiv_rn(to_float<T>(xr[c]), s));
      }
    }
  }
}

// ------------------------------------------------------------ FP8 decode
// Exact FP8 -> bf16/fp16/fp32 decode (the F.linear / cast_bias_weight seams).
// kind 0 = e4m3fn, 1 = e5m2.  out_dtype: 0 bf16, 1 fp16, 2 fp32.
__global__ void __launch_bounds__(256)
    fp8_decode_kernel(const uint8_t* __restrict__ src, int64_t n, int kind, void* __restrict__ dst,
                      int out_dtype) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    const uint8_t b = src[i];
    const float v = kind == 0 ? decode_e4m3(b) : decode_e5m2(b);
    if (out_dtype == kOutBF16) {
      // fp16 -> fp32 -> bf16 keeps NaN payload semantics of a plain cast.
      static_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(v);
    } else if (out_dtype == kOutF16) {
      static_cast<__half*>(dst)[i] = __float2half_rn(v);
    } else {
      static_cast<float*>(dst)[i] = v;
    }
  }
}

}  // namespace b200q
