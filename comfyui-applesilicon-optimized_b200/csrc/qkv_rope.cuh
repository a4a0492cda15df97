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
// correctly rounded.
#pragma once

#include "numerics.cuh"

namespace b200q {

constexpr int kRrWarps = 8;

template <int GROUPS>  // 1: D <= 128, 2: D <= 256
__global__ void __launch_bounds__(kRrWarps * 32)
    rms_rope_partial_kernel(__nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ k,
                            const __nv_bfloat16* __restrict__ fr, const float* __restrict__ qw,
                            const float* __restrict__ kw, int B, int H, int S, int D, int R,
                            float eps) {
  __shared__ float ybuf[kRrWarps][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rows = static_cast<int64_t>(B) * H * S;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kRrWarps + warp;
  if (gw >= 2 * rows) return;
  const bool is_k = gw >= rows;
  const int64_t row = is_k ? gw - rows : gw;  // (b*H + h)*S + s
  const int64_t s = row % S;
  const int64_t b = (row / S) / H;
  const int64_t m = b * S + s;                 // token row of the freqs table
  __nv_bfloat16* base = (is_k ? k : q) + row * D;
  const float* w = is_k ? kw : qw;

  float x[GROUPS][4];
  float gsum[GROUPS];
#pragma unroll
  for (int g = 0; g < GROUPS; ++g) {
    const int vt = lane + 32 * g;
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int d = 4 * vt + i;
      const float v = d < D ? __bfloat162float(base[d]) : 0.0f;
      x[g][i] = v;
      acc = __fadd_rn(acc, __fmul_rn(v, v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    gsum[g] = acc;
  }
  float total = 0.0f;
#pragma unroll
  for (int g = 0; g < GROUPS; ++g)
    if (lane == g) total = gsum[g];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) total = __fadd_rn(total, __shfl_xor_sync(0xffffffffu, total, o));
  const float inv = __frsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(D)), eps));

  float y[GROUPS][4];
#pragma unroll
  for (int g = 0; g < GROUPS; ++g)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int d = 4 * (lane + 32 * g) + i;
      if (d < D) {
        y[g][i] = round_bf16(__fmul_rn(__fmul_rn(x[g][i], inv), __ldg(w + d)));
        ybuf[warp][d] = y[g][i];
      }
    }
  __syncwarp();
#pragma unroll
  for (int g = 0; g < GROUPS; ++g)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int d = 4 * (lane + 32 * g) + i;
      if (d >= D) continue;
      float o = y[g][i];
      if (d < 2 * R) {
        const int ii = d < R ? d : d - R;
        const int r = d < R ? 0 : 1;
        const __nv_bfloat16* mat = fr + ((m * R + ii) * 2 + r) * 2;
        const float p0 = __fmul_rn(__bfloat162float(mat[0]), ybuf[warp][ii]);
        const float p1 = __fmul_rn(__bfloat162float(mat[1]), ybuf[warp][ii + R]);
        o = r == 0 ? round_bf16(__fadd_rn(round_bf16(p0), p1)) : round_bf16(__fadd_rn(round_bf16(p1), p0));
      }
      base[d] = __float2bfloat16_rn(o);
    }
}

}  // namespace b200q
