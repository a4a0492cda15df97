// In-place RMSNorm + partial split-half RoPE on attention-layout Q and K.
//
// The step that follows the QKV projection in the reference's DiT blocks
// (rms_rope_attention_partial, _patches/dit_ext/dit_kernels.mm:825-874; the
// same math fused into the INT8 QKV epilogue at int8_gemm.mm:672-862):
//   per row (b, h, s) of Q and of K, x = the row's D bf16 values:
//     y[d]  = bf16((x[d] * rsqrt(sum(x^2) / D + eps)) * w[d])
//     d >= 2R : out[d] = y[d]
//     d <  2R : i = d mod R, r = (d >= R), (m0, m1) = freqs[b*S + s][i][r]
//               r = 0: bf16(bf16(m0 * y[i]) + m1 * y[i+R])
//               r = 1: bf16(bf16(m1 * y[i+R]) + m0 * y[i])
// The sum of squares follows the order the reference restates for native
// F.rms_norm (torch_rms_sumsq, dit_kernels.mm:60-80): virtual thread vt sums
// elements 4vt..4vt+3 in order; groups of 32 vt are reduced across lanes (xor
// butterfly here), then the group totals the same way.  One warp per row:
// lane l holds vt = l + 32g.  fp32 throughout; rsqrt and the mean's divide are
// correctly rounded.  Needs 8-byte aligned q, k and 16-byte aligned weights
// (and freqs when R % 4 == 0); the host checks.
#pragma once

#include "numerics.cuh"

namespace b200q {

constexpr int kRrWarps = 8;

// Lane l of a warp holds elements 4(l + 32g) .. +3 of its row (g < GROUPS) and
// reads / writes them as one 8-byte vector; for R % 4 == 0 the rotation
// matrices of those four elements are two 16-byte loads.
template <int GROUPS>  // 1: D <= 128, 2: D <= 256
__global__ void __launch_bounds__(kRrWarps * 32)
    rms_rope_partial_kernel(__nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ k,
                            const __nv_bfloat16* __restrict__ fr, const float* __restrict__ qw,
                            const float* __restrict__ kw, int H, int S, int D, int R,
                            float eps) {
  __shared__ float ybuf[kRrWarps][256];
  // grid: x over blocks of kRrWarps sequence positions, y over (b, h), z: Q / K
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s = blockIdx.x * kRrWarps + warp;
  if (s >= S) return;
  const bool is_k = blockIdx.z != 0;
  const int bh = blockIdx.y;                   // b*H + h
  const int64_t row = static_cast<int64_t>(bh) * S + s;
  const int64_t m = static_cast<int64_t>(bh / H) * S + s;  // token row of the freqs table
  __nv_bfloat16* base = (is_k ? k : q) + row * D;
  const float* w = is_k ? kw : qw;

  float x[GROUPS][4];
  float gsum[GROUPS];
#pragma unroll
  for (int g = 0; g < GROUPS; ++g) {
    const int d0 = 4 * (lane + 32 * g);
    float acc = 0.0f;
    if (d0 < D) {
      const uint2 v = *reinterpret_cast<const uint2*>(base + d0);
      x[g][0] = __uint_as_float(v.x << 16);
      x[g][1] = __uint_as_float(v.x & 0xFFFF0000u);
      x[g][2] = __uint_as_float(v.y << 16);
      x[g][3] = __uint_as_float(v.y & 0xFFFF0000u);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) x[g][i] = 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) acc = __fadd_rn(acc, __fmul_rn(x[g][i], x[g][i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    gsum[g] = acc;
  }
  // GROUPS == 1: every lane already holds the row total.  GROUPS == 2: the group
  // totals are combined by the same butterfly (lanes other than 0 and 1 add +0).
  float total = gsum[0];
  if constexpr (GROUPS > 1) {
    total = 0.0f;
#pragma unroll
    for (int g = 0; g < GROUPS; ++g)
      if (lane == g) total = gsum[g];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) total = __fadd_rn(total, __shfl_xor_sync(0xffffffffu, total, o));
  }
  const float inv = __frsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(D)), eps));

  float y[GROUPS][4];
#pragma unroll
  for (int g = 0; g < GROUPS; ++g) {
    const int d0 = 4 * (lane + 32 * g);
    if (d0 < D) {
      const float4 wv = __ldg(reinterpret_cast<const float4*>(w + d0));
      const float wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        y[g][i] = round_bf16(__fmul_rn(__fmul_rn(x[g][i], inv), wa[i]));
        ybuf[warp][d0 + i] = y[g][i];
      }
    }
  }
  __syncwarp();
  const bool vec_fr = (R % 4) == 0;
#pragma unroll
  for (int g = 0; g < GROUPS; ++g) {
    const int d0 = 4 * (lane + 32 * g);
    if (d0 >= D) continue;
    float o[4] = {y[g][0], y[g][1], y[g][2], y[g][3]};
    if (d0 < 2 * R) {
      if (vec_fr) {
        // the four elements share r and use rotation rows i0 .. i0+3 (32 bytes)
        const int r = d0 < R ? 0 : 1;
        const int i0 = d0 - r * R;
        const uint4* mp = reinterpret_cast<const uint4*>(fr + (m * R + i0) * 4);
        const uint4 f0 = __ldg(mp), f1 = __ldg(mp + 1);
        const uint32_t fw[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t pr = fw[2 * i + r];  // (m_r0, m_r1) of row i0 + i
          const float m0 = __uint_as_float(pr << 16), m1 = __uint_as_float(pr & 0xFFFF0000u);
          const float p0 = __fmul_rn(m0, ybuf[warp][i0 + i]);
          const float p1 = __fmul_rn(m1, ybuf[warp][i0 + i + R]);
          o[i] = r == 0 ? round_bf16(__fadd_rn(round_bf16(p0), p1))
                        : round_bf16(__fadd_rn(round_bf16(p1), p0));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int d = d0 + i;
          if (d >= 2 * R) continue;
          const int ii = d < R ? d : d - R;
          const int r = d < R ? 0 : 1;
          const __nv_bfloat16* mat = fr + ((m * R + ii) * 2 + r) * 2;
          const float p0 = __fmul_rn(__bfloat162float(mat[0]), ybuf[warp][ii]);
          const float p1 = __fmul_rn(__bfloat162float(mat[1]), ybuf[warp][ii + R]);
          o[i] = r == 0 ? round_bf16(__fadd_rn(round_bf16(p0), p1))
                        : round_bf16(__fadd_rn(round_bf16(p1), p0));
        }
      }
    }
    *reinterpret_cast<uint2*>(base + d0) = make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
  }
}

}  // namespace b200q
