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
//    sees one read of x and one write of q.
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

template <typename T>
__device__ __forceinline__ uint2 quant8(const uint4& v, float s_math) {
  const T* e = reinterpret_cast<const T*>(&v);
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) lo |= (static_cast<uint32_t>(quant_code<T>(to_float<T>(e[i]), s_math)) & 0xFFu) << (8 * i);
#pragma unroll
  for (int i = 0; i < 4; ++i) hi |= (static_cast<uint32_t>(quant_code<T>(to_float<T>(e[i + 4]), s_math)) & 0xFFu) << (8 * i);
  return make_uint2(lo, hi);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
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
#pragma unroll
    for (int i = 0; i < kQuantMaxVec; ++i) {
      const int idx = threadIdx.x + i * kQuantThreads;
      if (idx < nvec) qr[idx] = quant8<T>(v[i], s_math);
    }
    for (int idx = threadIdx.x + kQuantMaxVec * kQuantThreads; idx < nvec; idx += kQuantThreads)
      qr[idx] = quant8<T>(xr[idx], s_math);
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
__device__ __forceinline__ uint2 fp8_quant8(const uint4& v, float s) {
  const T* e = reinterpret_cast<const T*>(&v);
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) lo |= static_cast<uint32_t>(encode_e4m3_sat(__fdiv_rn(to_float<T>(e[j]), s))) << (8 * j);
#pragma unroll
  for (int j = 0; j < 4; ++j) hi |= static_cast<uint32_t>(encode_e4m3_sat(__fdiv_rn(to_float<T>(e[j + 4]), s))) << (8 * j);
  return make_uint2(lo, hi);
}

template <typename T>
__global__ void __launch_bounds__(256)
    fp8_quantize_kernel(const T* __restrict__ x, int64_t ldx, int64_t M, int K,
                        const unsigned int* __restrict__ amax_bits, uint8_t* __restrict__ q,
                        int64_t ldq, float* __restrict__ scale_out) {
  const float s = fp8_scale_from_amax(*amax_bits);
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
      qv[i] = fp8_quant8<T>(a, s);
      qv[i + stride] = fp8_quant8<T>(b, s);
    }
    if (i < nvec) qv[i] = fp8_quant8<T>(__ldcs(xv + i), s);
  } else {
    for (int64_t r = blockIdx.x; r < M; r += gridDim.x) {
      const T* xr = x + r * ldx;
      uint8_t* qr = q + r * ldq;
      if (vec) {
        for (int c = threadIdx.x; c < (K >> 3); c += blockDim.x)
          reinterpret_cast<uint2*>(qr)[c] = fp8_quant8<T>(__ldcs(reinterpret_cast<const uint4*>(xr) + c), s);
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
