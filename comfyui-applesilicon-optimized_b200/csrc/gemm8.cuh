// 8-bit x 8-bit GEMM on the sm_100a tensor cores:  C[M,N] = A[M,K] . W[N,K]^T
// (the "NT" layout of the reference, int8_gemm.mm:4), both operands K-major.
//
//  kind::i8      int8 x int8 -> int32 in TMEM   (INT8 W8A8 route, torch._int_mm)
//  kind::f8f6f4  e4m3 x e4m3 -> fp32 in TMEM    (FP8 W8A8 route, torch._scaled_mm)
//  kind::f16     bf16/f16 x bf16/f16 -> fp32     (W8A16 at large M on the decoded weight)
// The tiles are described in bytes (128-byte rows, 32 bytes of K per MMA), so a
// 16-bit operand is passed with K, row strides and extents in bytes.
//
// Structure (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: 128x128-byte A tile + BNx128-byte W tile per stage,
//               128-byte swizzle, STAGES-deep mbarrier ring.
//   warp 1      MMA issuer: one elected thread issues 4 tcgen05.mma (K=32 each)
//               per stage into a TMEM accumulator; tcgen05.commit frees the stage.
//   warp 2      TMEM allocator (2 x BN columns: double-buffered accumulator so the
//               epilogue of tile i overlaps the MMAs of tile i+1).
//   warps 4..11 epilogue: two warps per TMEM lane quarter, each taking half of
//               the tile's columns; tcgen05.ld 32 columns at a time with the
//               chunk's column scales / bias fetched by uniform vector loads
//               before the TMEM wait; element math (raw int32 / reference
//               two-rounding INT8 dequant / FP8 scaled + bias + GELU) and
//               16-byte global stores.
// With a quant prologue (PRO != kProNone, prologue.cuh) warps 2 and 3 quantize
// activation rows (bulk-copied into their shared-memory rings) while the tensor
// cores work, and the producer waits for a band's rows before loading it.
// Tiles are walked in groups of 16 M-tiles so the ~148 concurrently running
// tiles share A row panels and W column panels in L2.
#pragma once

#include "numerics.cuh"
#include "prologue.cuh"
#include "ptx.cuh"

namespace b200q {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 128;  // bytes = elements per k-block (one 128B swizzle atom)
constexpr int kGemmThreads = 384;  // 4 control warps + 8 epilogue warps
constexpr int kGemmGroupM = 16;

// kEpiI8SwiGLU: the INT8 dequant epilogue on an FC1 whose N = 2F rows are
// [gate; up]; each tile holds matching gate and up columns (the producer loads
// the two row ranges into the two halves of the B tile) and the epilogue writes
// act = swiglu(gate, up) [M, F] instead of the [M, 2F] output.
// kEpiI8QkvNormRope: the INT8 dequant epilogue storing Q/K/V in attention
// layout (EpiArgs.qkv*, head_dim 128) with Q and K RMS-normalized and rotated
// (split-half RoPE) before the store.
enum EpiMode : int { kEpiInt32 = 0, kEpiI8Dequant = 1, kEpiScaled = 2, kEpiI8SwiGLU = 3,
                     kEpiI8QkvNormRope = 4 };

template <int BN, int STAGES>
struct Gemm8Layout {
  static constexpr int kATile = kGemmBM * kGemmBK;
  static constexpr int kBTile = BN * kGemmBK;
  static constexpr int kStageBytes = kATile + kBTile;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  // full[S], empty[S], acc_full[2], acc_empty[2], tmem slot, abort flag
  static constexpr int kBarBytes = (2 * STAGES + 4) * 8 + 16;
  static constexpr int kSmemBytes = kBarOffset + kBarBytes + 1024;  // + alignment slack
  // Quant-prologue launches: the quantizer warps' bulk-copy rings follow.
  static constexpr int kQuantOffset = (kBarOffset + kBarBytes + 127) & ~127;
  static constexpr int kSmemBytesPro = kQuantOffset + kQSmemBytes + 1024;
  static constexpr uint32_t kTmemCols = 2 * BN;
};

// Tile order: groups of `group_m` M-tiles, M fastest inside a group.  group_m = 1
// is a plain N-fastest sweep (each A row panel is read once while the whole W
// stays in L2); the host picks it when W fits comfortably in L2.
__device__ __forceinline__ void gemm_tile_coords(int tile, int num_m, int num_n, int group_m,
                                                 int& mb, int& nb) {
  const int group_size = group_m * num_n;
  const int g = tile / group_size;
  const int first_m = g * group_m;
  const int gm = min(num_m - first_m, group_m);
  const int idx = tile - g * group_size;
  mb = first_m + idx % gm;
  nb = idx / gm;
}

// Column parameters of one 32-column chunk (scale and bias per output column),
// fetched with uniform vector loads: every lane of the warp reads the same
// addresses, so each load is one broadcast transaction.  Absent scales read as
// 1.0 (an exact multiply); bias presence is returned so the caller can skip the
// add (adding +0.0 would flip the sign of a -0.0 result).
__device__ __forceinline__ bool load_col_params(const EpiArgs& e, int n0, float (&cs)[32],
                                                float (&bi)[32]) {
  const bool full = n0 + 32 <= e.N;
  if (e.col_scale && e.col_scale_vec) {
    const float* p = e.col_scale + n0;
    if (full && ((reinterpret_cast<uintptr_t>(p) & 15) == 0)) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(p) + j);
        cs[4 * j] = v.x; cs[4 * j + 1] = v.y; cs[4 * j + 2] = v.z; cs[4 * j + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) cs[j] = __ldg(e.col_scale + min(n0 + j, e.N - 1));
    }
  } else {
    const float c = e.col_scale ? __ldg(e.col_scale) : 1.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) cs[j] = c;
  }
  if (e.bias_dtype == kBiasNone) return false;
  if (e.bias_dtype == kBiasF32) {
    const float* p = static_cast<const float*>(e.bias) + n0;
    if (full && ((reinterpret_cast<uintptr_t>(p) & 15) == 0)) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(p) + j);
        bi[4 * j] = v.x; bi[4 * j + 1] = v.y; bi[4 * j + 2] = v.z; bi[4 * j + 3] = v.w;
      }
      return true;
    }
  } else {
    const uint16_t* p = static_cast<const uint16_t*>(e.bias) + n0;
    if (full && ((reinterpret_cast<uintptr_t>(p) & 15) == 0)) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(p) + j);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint16_t lo = static_cast<uint16_t>(w[k] & 0xFFFFu), hi = static_cast<uint16_t>(w[k] >> 16);
          if (e.bias_dtype == kBiasBF16) {
            bi[8 * j + 2 * k] = __uint_as_float(static_cast<uint32_t>(lo) << 16);
            bi[8 * j + 2 * k + 1] = __uint_as_float(static_cast<uint32_t>(hi) << 16);
          } else {
            bi[8 * j + 2 * k] = __half2float(__ushort_as_half(lo));
            bi[8 * j + 2 * k + 1] = __half2float(__ushort_as_half(hi));
          }
        }
      }
      return true;
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) bi[j] = load_bias(e.bias, e.bias_dtype, min(n0 + j, e.N - 1));
  return true;
}

// Stores 32 values of row m at columns [n0, n0+32) (columns >= n_limit are
// dropped): 16-byte vector stores when the chunk is whole and aligned, element
// stores on ragged edges.
__device__ __forceinline__ void store_chunk(const EpiArgs& e, int64_t m, int n0, const float (&v)[32],
                                            int n_limit) {
  const bool full = n0 + 32 <= n_limit;
  if (e.out_dtype == kOutBF16 || e.out_dtype == kOutF16) {
    uint16_t* p16 = out_ptr16(e, m, n0);
    if (full && (e.qkv_heads > 0 || (e.ldo & 7) == 0) && ((reinterpret_cast<uintptr_t>(p16) & 15) == 0)) {
      uint4* o = reinterpret_cast<uint4*>(p16);
      if (e.out_dtype == kOutBF16) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          o[j] = make_uint4(pack_bf16x2(v[8 * j], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                            pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          o[j] = make_uint4(pack_f16x2(v[8 * j], v[8 * j + 1]), pack_f16x2(v[8 * j + 2], v[8 * j + 3]),
                            pack_f16x2(v[8 * j + 4], v[8 * j + 5]), pack_f16x2(v[8 * j + 6], v[8 * j + 7]));
      }
      return;
    }
  } else if (full && ((e.ldo & 3) == 0) && ((reinterpret_cast<uintptr_t>(e.out) & 15) == 0)) {
    float4* o = reinterpret_cast<float4*>(static_cast<float*>(e.out) + m * e.ldo + n0);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    return;
  }
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (n0 + j < n_limit) store_out(e, m, n0 + j, v[j]);
}

__device__ __forceinline__ void store_chunk_i32(const EpiArgs& e, int64_t m, int n0, const uint32_t (&r)[32]) {
  int32_t* out = static_cast<int32_t*>(e.out) + m * e.ldo;
  if (n0 + 32 <= e.N && ((e.ldo & 3) == 0) && ((reinterpret_cast<uintptr_t>(e.out) & 15) == 0)) {
    int4* o = reinterpret_cast<int4*>(out + n0);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      o[j] = make_int4(static_cast<int>(r[4 * j]), static_cast<int>(r[4 * j + 1]),
                       static_cast<int>(r[4 * j + 2]), static_cast<int>(r[4 * j + 3]));
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (n0 + j < e.N) out[n0 + j] = static_cast<int32_t>(r[j]);
  }
}

// Element math of one chunk.  Uniform flags are tested outside the unrolled loops.
template <int EPI, bool ACC_INT>
__device__ __forceinline__ void epilogue_math(const uint32_t (&r)[32], const float (&cs)[32],
                                              const float (&bi)[32], bool has_bias, float rs,
                                              float xs, const EpiArgs& e, float (&v)[32]) {
  if constexpr (EPI == kEpiI8Dequant || EPI == kEpiI8SwiGLU || EPI == kEpiI8QkvNormRope) {
    // Reference order (int8_gemm.mm:417-443): s = cs*rs; T(C*s); T(r + bias).
    // Without an activation the second rounding T(r + bias) is left to the
    // store's packed conversion (the same nearest-even rounding; every caller
    // of this path stores through store_chunk), saving a conversion per element.
    const bool round_bias = e.act != kActNone;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      v[j] = __fmul_rn(i2f_rn(static_cast<int32_t>(r[j])), __fmul_rn(cs[j], rs));
    if (e.out_dtype == kOutF16) {
#pragma unroll
      for (int j = 0; j < 32; j += 2) round_f16x2(v[j], v[j + 1]);
      if (has_bias) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], bi[j]);
        if (round_bias) {
#pragma unroll
          for (int j = 0; j < 32; j += 2) round_f16x2(v[j], v[j + 1]);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; j += 2) round_bf16x2(v[j], v[j + 1]);
      if (has_bias) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], bi[j]);
        if (round_bias) {
#pragma unroll
          for (int j = 0; j < 32; j += 2) round_bf16x2(v[j], v[j + 1]);
        }
      }
    }
  } else {
    // FP8 route order (scaled_mm_fp8.py:136-146): ((acc*sa)*sb)*sr + bias, fp32.
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float acc = ACC_INT ? i2f_rn(static_cast<int32_t>(r[j])) : __uint_as_float(r[j]);
      v[j] = __fmul_rn(__fmul_rn(__fmul_rn(acc, rs), cs[j]), xs);
    }
    if (has_bias) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], bi[j]);
    }
  }
  if (e.act == kActGeluTanh) {
    // The activation is checked to 1 ULP of the reference after the output
    // rounding (the INT8 dequant before it stays bit-exact): the branch-free
    // reciprocal form.  The IEEE divide's slow-path branch serialised the 32
    // columns, and an up projection's epilogue outlasted its mainloop.
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(v[j]);
  } else if (e.act == kActGeluErf) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = gelu_erf(v[j]);
  }
}

// Scale and bias of 8 consecutive columns n0.. (uniform loads; indices clamped
// to the last column on a ragged edge).  Returns whether a bias is present.
__device__ __forceinline__ bool load_col_params8(const EpiArgs& e, int n0, float (&cs)[8],
                                                 float (&bi)[8]) {
  const bool full = n0 + 8 <= e.N;
  if (e.col_scale_vec) {
    const float* p = e.col_scale + n0;
    if (full && ((reinterpret_cast<uintptr_t>(p) & 15) == 0)) {
      const float4 v0 = __ldg(reinterpret_cast<const float4*>(p));
      const float4 v1 = __ldg(reinterpret_cast<const float4*>(p) + 1);
      cs[0] = v0.x; cs[1] = v0.y; cs[2] = v0.z; cs[3] = v0.w;
      cs[4] = v1.x; cs[5] = v1.y; cs[6] = v1.z; cs[7] = v1.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) cs[j] = __ldg(e.col_scale + min(n0 + j, e.N - 1));
    }
  } else {
    const float c = __ldg(e.col_scale);
#pragma unroll
    for (int j = 0; j < 8; ++j) cs[j] = c;
  }
  if (e.bias_dtype == kBiasNone) return false;
  const uint16_t* p = static_cast<const uint16_t*>(e.bias) + n0;  // bf16
  if (full && ((reinterpret_cast<uintptr_t>(p) & 15) == 0)) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      bi[2 * k] = __uint_as_float(w[k] << 16);
      bi[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      bi[j] = __uint_as_float(static_cast<uint32_t>(__ldg(p - n0 + min(n0 + j, e.N - 1))) << 16);
  }
  return true;
}

// SwiGLU epilogue of one accumulator tile for one epilogue warp.  The tile's BN
// columns are BN/2 gate columns followed by the matching BN/2 up columns, both
// for output columns [f_base, f_base + BN/2).  Warp half `half` takes BN/128 of
// the 32-column gate chunks with their up partners, 8 columns at a time.  Each
// side gets the reference's bf16 two-rounding dequant (+ bias) at its own
// physical column (gate f, up F + f); then act = bf16(bf16(silu(gate)) * up).
// The rare exact-silu fallback runs once per warp iteration for every lane that
// still has one pending (a warp-uniform loop with a single inlined call site).
template <int BN>
__device__ __forceinline__ void swiglu_tile_epilogue(uint32_t taddr, int half, int f_base, int F,
                                                     int64_t m, bool row_ok, float rs,
                                                     const EpiArgs& ep) {
  constexpr int kPairs = BN / 128;
#pragma unroll 1
  for (int c = half * kPairs; c < (half + 1) * kPairs; ++c) {
    const int f0 = f_base + c * 32;
    uint32_t packed[16];
#pragma unroll
    for (int sb = 0; sb < 4; ++sb) {
      const int fs = f0 + sb * 8;
      uint32_t rg[8], ru[8];
      float csg[8], big[8], csu[8], biu[8];
      tmem_ld8(taddr + c * 32 + sb * 8, rg);
      tmem_ld8(taddr + BN / 2 + c * 32 + sb * 8, ru);
      const bool hb = load_col_params8(ep, fs, csg, big);
      load_col_params8(ep, F + fs, csu, biu);
      tmem_ld_wait();
      float g[8], u[8], a[8];
      uint32_t slow = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        g[j] = round_bf16(__fmul_rn(i2f_rn(static_cast<int32_t>(rg[j])), __fmul_rn(csg[j], rs)));
        u[j] = round_bf16(__fmul_rn(i2f_rn(static_cast<int32_t>(ru[j])), __fmul_rn(csu[j], rs)));
        if (hb) {
          g[j] = round_bf16(__fadd_rn(g[j], big[j]));
          u[j] = round_bf16(__fadd_rn(u[j], biu[j]));
        }
        a[j] = silu_f32_fast(g[j]);
        if (silu_needs_exact(a[j], g[j])) slow |= 1u << j;
      }
      while (__any_sync(0xffffffffu, slow != 0)) {
        const int jj = slow ? __ffs(slow) - 1 : 0;
        float gj = g[0];
#pragma unroll
        for (int j = 1; j < 8; ++j) gj = j == jj ? g[j] : gj;
        const float e = silu_f32_exact_inl(gj);
        if (slow) {
#pragma unroll
          for (int j = 0; j < 8; ++j) a[j] = j == jj ? e : a[j];
          slow &= slow - 1;
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k)
        packed[4 * sb + k] = pack_bf16x2(__fmul_rn(round_bf16(a[2 * k]), u[2 * k]),
                                         __fmul_rn(round_bf16(a[2 * k + 1]), u[2 * k + 1]));
    }
    if (row_ok && f0 < F) {
      uint16_t* p = static_cast<uint16_t*>(ep.out) + m * ep.ldo + f0;
      if (f0 + 32 <= F && (ep.ldo & 7) == 0 && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          reinterpret_cast<uint4*>(p)[k] =
              make_uint4(packed[4 * k], packed[4 * k + 1], packed[4 * k + 2], packed[4 * k + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (f0 + j < F) p[j] = static_cast<uint16_t>(packed[j >> 1] >> (16 * (j & 1)));
      }
    }
  }
}

// Eight columns of one row: tcgen05.ld of the accumulators at taddr, then the
// reference's bf16 two-rounding dequant (+ bias) at global columns n0 .. n0+7.
// Warp-collective (every lane of the warp calls it).
__device__ __forceinline__ void dequant8_bf16(uint32_t taddr, int n0, float rs, const EpiArgs& ep,
                                              float (&v)[8]) {
  uint32_t r[8];
  float cs[8], bi[8];
  tmem_ld8(taddr, r);
  const bool hb = load_col_params8(ep, n0, cs, bi);
  tmem_ld_wait();
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    v[j] = round_bf16(__fmul_rn(i2f_rn(static_cast<int32_t>(r[j])), __fmul_rn(cs[j], rs)));
    if (hb) v[j] = round_bf16(__fadd_rn(v[j], bi[j]));
  }
}

// One head (128 columns, TMEM columns taddr .. taddr+127, global columns
// n0 .. n0+127) of one row per thread, for a warp that owns the head:
// the reference's fused Q/K RMSNorm + partial split-half RoPE epilogue
// (int8_gemm.mm:672-862; rms_rope_attention_partial semantics,
// dit_kernels.mm:825-874).  V heads are stored as they are.
//  pass 1: dequant, sum of squares in the reference order (element groups
//          4vt..4vt+3 summed in order, then the 32 group sums combined by the
//          xor-butterfly tree of a warp-wide reduction, here inside one thread);
//  pass 2: TMEM read again (the same dequant values), y = bf16((x*inv)*w),
//          RoPE on column pairs (i, i+R) read together, stores of 8 columns.
__device__ __forceinline__ void qkv_norm_rope_head(uint32_t taddr, int n0, int64_t m, bool row_ok,
                                                   float rs, const EpiArgs& ep) {
  constexpr int D = 128;
  // The last tile's second half lies past N when the head count is odd (N = 384 H);
  // the whole warp skips it together, so no tcgen05.ld is left half-issued.
  if (n0 >= ep.N) return;
  const int kind = n0 / (ep.qkv_heads * D);
  if (kind == 2) {
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      uint32_t r[32];
      float cs[32], bi[32], v[32];
      const bool hb = load_col_params(ep, n0 + 32 * c, cs, bi);
      tmem_ld32(taddr + 32 * c, r);
      tmem_ld_wait();
      if (row_ok) {
        epilogue_math<kEpiI8Dequant, true>(r, cs, bi, hb, rs, 1.0f, ep, v);
        store_chunk(ep, m, n0 + 32 * c, v, ep.N);
      }
    }
    return;
  }
  float p[32];
#pragma unroll
  for (int s = 0; s < D / 8; ++s) {
    float x[8];
    dequant8_bf16(taddr + 8 * s, n0 + 8 * s, rs, ep, x);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float acc = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) acc = __fadd_rn(acc, __fmul_rn(x[4 * h + j], x[4 * h + j]));
      p[2 * s + h] = acc;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int i = 0; i < o; ++i) p[i] = __fadd_rn(p[i], p[i + o]);
  const float inv = __frsqrt_rn(__fadd_rn(__fdiv_rn(p[0], static_cast<float>(D)), ep.norm_eps));
  const float* w = kind == 0 ? ep.q_norm_w : ep.k_norm_w;
  const int R = ep.rope_r;
#pragma unroll 1
  for (int d0 = 0; d0 < D; d0 += 8) {
    if (d0 >= R && d0 < 2 * R) continue;  // stored with its partner d0 - R
    float ya[8];
    dequant8_bf16(taddr + d0, n0 + d0, rs, ep, ya);
    {
      const float4 w0 = __ldg(reinterpret_cast<const float4*>(w + d0));
      const float4 w1 = __ldg(reinterpret_cast<const float4*>(w + d0) + 1);
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) ya[j] = round_bf16(__fmul_rn(__fmul_rn(ya[j], inv), wv[j]));
    }
    if (d0 < R) {
      float yb[8];
      dequant8_bf16(taddr + d0 + R, n0 + d0 + R, rs, ep, yb);
      {
        const float4 w0 = __ldg(reinterpret_cast<const float4*>(w + d0 + R));
        const float4 w1 = __ldg(reinterpret_cast<const float4*>(w + d0 + R) + 1);
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) yb[j] = round_bf16(__fmul_rn(__fmul_rn(yb[j], inv), wv[j]));
      }
      if (row_ok) {
        // freqs[m][i][r][c] for i = d0 .. d0+7: 32 consecutive bf16
        const uint4* fp = reinterpret_cast<const uint4*>(ep.rope_freqs + (m * R + d0) * 4);
        float oa[8], ob[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 f = __ldg(fp + q);  // i = d0 + 2q, d0 + 2q + 1
          const uint32_t fw[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int j = 2 * q + t;
            const float m00 = __uint_as_float(fw[2 * t] << 16);
            const float m01 = __uint_as_float(fw[2 * t] & 0xFFFF0000u);
            const float m10 = __uint_as_float(fw[2 * t + 1] << 16);
            const float m11 = __uint_as_float(fw[2 * t + 1] & 0xFFFF0000u);
            oa[j] = round_bf16(__fadd_rn(round_bf16(__fmul_rn(m00, ya[j])), __fmul_rn(m01, yb[j])));
            ob[j] = round_bf16(__fadd_rn(round_bf16(__fmul_rn(m11, yb[j])), __fmul_rn(m10, ya[j])));
          }
        }
        uint4* pa = reinterpret_cast<uint4*>(out_ptr16(ep, m, n0 + d0));
        uint4* pb = reinterpret_cast<uint4*>(out_ptr16(ep, m, n0 + d0 + R));
        pa[0] = make_uint4(pack_bf16x2(oa[0], oa[1]), pack_bf16x2(oa[2], oa[3]),
                           pack_bf16x2(oa[4], oa[5]), pack_bf16x2(oa[6], oa[7]));
        pb[0] = make_uint4(pack_bf16x2(ob[0], ob[1]), pack_bf16x2(ob[2], ob[3]),
                           pack_bf16x2(ob[4], ob[5]), pack_bf16x2(ob[6], ob[7]));
      }
    } else if (row_ok) {
      uint4* pa = reinterpret_cast<uint4*>(out_ptr16(ep, m, n0 + d0));
      pa[0] = make_uint4(pack_bf16x2(ya[0], ya[1]), pack_bf16x2(ya[2], ya[3]),
                         pack_bf16x2(ya[4], ya[5]), pack_bf16x2(ya[6], ya[7]));
    }
  }
}

template <MmaKind KIND, int BN, int STAGES, int EPI, int PRO>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm8_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    int M, int N, int K, int group_m, EpiArgs ep, Prologue pro) {
  using L = Gemm8Layout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * L::kATile;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* exit_flag = reinterpret_cast<int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr bool kSwiGLU = EPI == kEpiI8SwiGLU;
  constexpr int kTileN = kSwiGLU ? BN / 2 : BN;  // output columns per tile
  const int F = N >> 1;                          // SwiGLU: gate rows [0, F), up rows [F, 2F)
  const int num_m = (M + kGemmBM - 1) / kGemmBM;
  const int num_n = ((kSwiGLU ? F : N) + kTileN - 1) / kTileN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + kGemmBK - 1) / kGemmBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8 * 32);
    }
    *abort_flag = 0;
    if constexpr (PRO != kProNone) {
      uint64_t* qfull = reinterpret_cast<uint64_t*>(smem + L::kQuantOffset + kQWarps * kQSlots * kQSlotBytes);
      for (int i = 0; i < kQWarps * kQSlots; ++i) mbar_init(&qfull[i], 1);
    }
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  float pro_s = 1.0f;  // per-tensor activation scale of the fp8 prologue
  if constexpr (PRO == kProFp8Tensor) {
    pro_s = pro_fp8_scale(pro);
    if (blockIdx.x == 0 && threadIdx.x == 0) pro.scales[0] = pro_s;
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int ready_band = -1;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int mb, nb;
        gemm_tile_coords(tile, num_m, num_n, group_m, mb, nb);
        if constexpr (PRO != kProNone) {
          if (mb != ready_band) {
            if (!pro_band_wait(pro, mb, M, abort_flag)) break;
            ready_band = mb;
          }
        }
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
          tma_load_2d(&tmA, &full[stage], sA + stage * L::kATile, kb * kGemmBK, mb * kGemmBM);
          if constexpr (kSwiGLU) {
            // B tile = [gate rows; up rows] of this tile's columns (tensor map box = BN/2 rows).
            tma_load_2d(&tmB, &full[stage], sB + stage * L::kBTile, kb * kGemmBK, nb * kTileN);
            tma_load_2d(&tmB, &full[stage], sB + stage * L::kBTile + kTileN * kGemmBK, kb * kGemmBK,
                        F + nb * kTileN);
          } else {
            tma_load_2d(&tmB, &full[stage], sB + stage * L::kBTile, kb * kGemmBK, nb * BN);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdesc = kind_idesc<KIND>(kGemmBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++it) {
        const int buf = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&acc_empty[buf], acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = make_sw128_desc(smem_u32(sA + stage * L::kATile));
          const uint64_t bdesc = make_sw128_desc(smem_u32(sB + stage * L::kBTile));
#pragma unroll
          for (int k = 0; k < kGemmBK / 32; ++k) {
            // +32 bytes along K inside the swizzle atom = +2 in the >>4 address field
            umma_ss<KIND>(d_tmem, adesc + 2 * k, bdesc + 2 * k, kIdesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
    }
    __syncwarp();
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------ quantizer warps
    if constexpr (PRO != kProNone) {
      if (pro.ring) {
        uint8_t* ring = smem + L::kQuantOffset + (warp - 2) * kQSlots * kQSlotBytes;
        uint64_t* qfull = reinterpret_cast<uint64_t*>(smem + L::kQuantOffset + kQWarps * kQSlots * kQSlotBytes) +
                          (warp - 2) * kQSlots;
        if (pro.x_f16) pro_ring_worker<PRO, __half>(pro, M, K, pro_s, ring, qfull, abort_flag);
        else pro_ring_worker<PRO, __nv_bfloat16>(pro, M, K, pro_s, ring, qfull, abort_flag);
      } else {
        pro_worker<PRO>(pro, M, K, pro_s);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    // 8 warps: warp w reads TMEM lane quarter (w % 4) and column half (w - 4) / 4.
    const int q = warp & 3;
    const int half = (warp - 4) >> 2;
    const int row_local = q * 32 + lane;
    const float xs = ep.extra_scale ? __ldg(ep.extra_scale) : 1.0f;
    constexpr bool kAccInt = KIND == MmaKind::I8;
    constexpr int kChunks = BN / 64;  // 32-column chunks per warp
    int it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      int mb, nb;
      gemm_tile_coords(tile, num_m, num_n, group_m, mb, nb);
      const int buf = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait_warp(&acc_full[buf], acc_phase, abort_flag)) break;
      tc_fence_after();
      const int64_t m = static_cast<int64_t>(mb) * kGemmBM + row_local;
      const bool row_ok = m < M;
      if constexpr (PRO == kProInt8Row) {
        // Row scales come from the quantizers: acquire the band before reading them.
        if (!__all_sync(0xffffffffu, pro_band_wait(pro, mb, M, abort_flag))) break;
      }
      float rs = 1.0f;
      if constexpr (PRO == kProFp8Tensor) {
        rs = pro_s;
      } else {
        if (EPI != kEpiInt32 && ep.row_scale && row_ok) rs = __ldcg(ep.row_scale + (ep.row_scale_vec ? m : 0));
      }
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
      if constexpr (kSwiGLU) {
        swiglu_tile_epilogue<BN>(taddr, half, nb * kTileN, F, m, row_ok, rs, ep);
      } else if constexpr (EPI == kEpiI8QkvNormRope) {
        // BN = 256: each warp half owns one 128-column head
        qkv_norm_rope_head(taddr + half * 128, nb * BN + half * 128, m, row_ok, rs, ep);
      } else {
#pragma unroll 1
        for (int c = half * kChunks; c < (half + 1) * kChunks; ++c) {
          const int n0 = nb * BN + c * 32;
          uint32_t r[32];
          if constexpr (EPI == kEpiInt32) {
            tmem_ld32(taddr + c * 32, r);
            tmem_ld_wait();
            if (row_ok && n0 < N) store_chunk_i32(ep, m, n0, r);
          } else {
            float cs[32], bi[32], v[32];
            const bool has_bias = n0 < N ? load_col_params(ep, n0, cs, bi) : false;
            tmem_ld32(taddr + c * 32, r);
            tmem_ld_wait();
            if (row_ok && n0 < N) {
              epilogue_math<EPI, kAccInt>(r, cs, bi, has_bias, rs, xs, ep, v);
              store_chunk(ep, m, n0, v, N);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem_base, L::kTmemCols);
  if constexpr (PRO != kProNone) pro_exit(pro, exit_flag);
}

// ---------------------------------------------------------------------------
// CTA-pair variant: a cluster of 2 CTAs computes 256x256 output tiles with
// tcgen05.mma.cta_group::2 (M=256).  Each CTA stages its own 128 A rows and
// 128 of the tile's 256 W rows, so per CTA and per K step the tensor core gets
// the same 128x256 work as the single-CTA kernel from 2/3 of the operand bytes
// (32 KB instead of 48 KB per 128-byte K block); the freed shared memory buys
// 6 pipeline stages.  The even CTA's warp 1 issues the MMAs; both CTAs' TMA
// loads complete on the even CTA's `full` barrier; each MMA batch's commit
// signals both CTAs' `empty` barriers; accumulators land in each CTA's own TMEM
// (its 128 rows x 256 columns) and each CTA runs its own epilogue.
// KATOMS 128-byte swizzle atoms of K per stage: one TMA box per atom and operand,
// 4 MMAs (K = 32 bytes each) per atom.  Measured on B200: the pipeline costs a
// roughly fixed ~1.1k cycles per stage hand-off beyond its MMAs, so a stage of
// one atom (4 MMAs = 512 tensor cycles) left the tensor pipe idle half the time;
// two atoms per stage (8 MMAs) amortise it.
// BN: output columns per tile (256, or 192 where the tile count fills the
// last wave better); each CTA stages BN / 2 of the tile's weight rows.
// Column-parallel all-gather in the pair kernel's TMA-store epilogue: every
// 32 x 32 output block also goes to up to kMaxPeerOuts more copies of the
// output (the other ranks' full-width buffers, reached over NVLink through
// peer mappings), each described by its own tensor map whose origin is this
// rank's first column there.  n = 0: a plain single-output GEMM.
constexpr int kMaxPeerOuts = 7;
struct PeerOuts {
  CUtensorMap map[kMaxPeerOuts];
  int n;
};

// max |v[j]| over the chunk's first `valid` columns into m (one FMNMX per
// element on whole chunks; the ragged last chunk of a row masks its tail).
__device__ __forceinline__ void chunk_amax(const float (&v)[32], int valid, float& m) {
  if (valid >= 32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) m = fmaxf(m, fabsf(v[j]));
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < valid) m = fmaxf(m, fabsf(v[j]));
  }
}

template <int STAGES, int KATOMS = 1, int BN = 256>
struct Gemm8PairLayout {
  static constexpr int kAtom = 128 * kGemmBK;            // one 128-row x 128-byte box (A)
  static constexpr int kBAtom = (BN / 2) * kGemmBK;      // this CTA's weight rows, one atom
  static constexpr int kATile = KATOMS * kAtom;          // this CTA's A rows
  static constexpr int kBTile = KATOMS * kBAtom;         // this CTA's half of the W rows
  static constexpr int kStageBytes = kATile + kBTile;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kBarBytes = (2 * STAGES + 4) * 8 + 16;
  static constexpr int kSmemBytes = kBarOffset + kBarBytes + 1024;
  static constexpr int kQuantOffset = (kBarOffset + kBarBytes + 127) & ~127;
  static constexpr int kSmemBytesPro = kQuantOffset + kQSmemBytes + 1024;
  // TMA-store epilogue: one 32 x 32 16-bit staging block per epilogue warp
  // (512-byte aligned for the 64-byte swizzle), then the tile's column scales
  // and biases as floats, double-buffered by tile.
  static constexpr int kEpiOffset = (kBarOffset + kBarBytes + 511) & ~511;
  static constexpr int kEpiBlock = 32 * 32 * 2;
  static constexpr int kParOffset = kEpiOffset + 8 * kEpiBlock;
  static constexpr int kParBarOffset = kParOffset + 2 * 2 * 256 * 4;  // 2 mbarriers
  static constexpr int kSmemBytesStore = kParBarOffset + 16 + 1024;
  static constexpr uint32_t kTmemCols = 512;  // 2 x 256-column accumulators
};

template <MmaKind KIND, int STAGES, int EPI, int PRO, int KATOMS = 1, int BN_ = 256>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm8_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ PeerOuts peers,
                     int M, int N, int K, int group_m, EpiArgs ep, Prologue pro) {
  static_assert(KATOMS == 1 || PRO == kProNone, "the quant prologue bands use one-atom stages");
  static_assert(BN_ == 256 || (BN_ == 192 && (EPI == kEpiInt32 || EPI == kEpiI8Dequant ||
                                               EPI == kEpiScaled)),
                "the SwiGLU and QKV epilogues use 256-column tiles");
  using L = Gemm8PairLayout<STAGES, KATOMS, BN_>;
  constexpr int kStageK = KATOMS * kGemmBK;  // K bytes per pipeline stage
  constexpr int BM = 256, BN = BN_;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * L::kATile;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* exit_flag = reinterpret_cast<int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = MMA-issuing CTA
  const uint32_t peer = rank ^ 1u;
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  constexpr bool kSwiGLU = EPI == kEpiI8SwiGLU;
  constexpr int kTileN = kSwiGLU ? BN / 2 : BN;  // output columns per tile
  const int F = N >> 1;                          // SwiGLU: gate rows [0, F), up rows [F, 2F)
  const int num_m = (M + BM - 1) / BM;
  const int num_n = ((kSwiGLU ? F : N) + kTileN - 1) / kTileN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + kStageK - 1) / kStageK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);   // the even CTA's producer arrives with both CTAs' bytes
      mbar_init(&empty[s], 1);  // one MMA commit per use
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * 8);  // 8 epilogue warps in each CTA
    }
    if constexpr ((EPI == kEpiI8Dequant || EPI == kEpiScaled) && PRO == kProNone) {
      if (ep.tma_store) {
        uint64_t* par_full = reinterpret_cast<uint64_t*>(smem + L::kParBarOffset);
        mbar_init(&par_full[0], 256);  // every epilogue thread stores one column's params
        mbar_init(&par_full[1], 256);
      }
    }
    *abort_flag = 0;
    if constexpr (PRO != kProNone) {
      uint64_t* qfull = reinterpret_cast<uint64_t*>(smem + L::kQuantOffset + kQWarps * kQSlots * kQSlotBytes);
      for (int i = 0; i < kQWarps * kQSlots; ++i) mbar_init(&qfull[i], 1);
    }
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, L::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Launched as a programmatic dependent of the kernel before it (the set-up
  // above overlaps that kernel's tail): no global memory is touched before it
  // has finished.
  griddep_wait();
  float pro_s = 1.0f;  // per-tensor activation scale of the fp8 prologue
  if constexpr (PRO == kProFp8Tensor) {
    pro_s = pro_fp8_scale(pro);
    if (blockIdx.x == 0 && threadIdx.x == 0) pro.scales[0] = pro_s;
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      const uint32_t leader_full0 = mapa_shared(smem_u32(&full[0]), 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int ready_band = -1;
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs) {
        int mb, nb;
        gemm_tile_coords(tile, num_m, num_n, group_m, mb, nb);
        const int a_row = mb * BM + static_cast<int>(rank) * 128;
        // SwiGLU: the even CTA loads the gate rows, the odd one the matching up
        // rows, so accumulator columns [0,128) are gate and [128,256) up.
        const int b_row = kSwiGLU ? (rank == 0 ? nb * kTileN : F + nb * kTileN)
                                  : nb * BN + static_cast<int>(rank) * (BN / 2);
        if constexpr (PRO != kProNone) {
          const int band = a_row / kBandRows;
          if (band != ready_band) {
            if (!pro_band_wait(pro, band, M, abort_flag)) break;
            ready_band = band;
          }
        }
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * L::kStageBytes);
          const uint32_t bar = leader_full0 + stage * 8;
#pragma unroll
          for (int a = 0; a < KATOMS; ++a) {
            // K past the end (a ragged last stage) reads as zeros
            const int x = kb * kStageK + a * kGemmBK;
            tma_load_2d_pair(&tmA, bar, sA + stage * L::kATile + a * L::kAtom, x, a_row);
            tma_load_2d_pair(&tmB, bar, sB + stage * L::kBTile + a * L::kBAtom, x, b_row);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t kIdesc = kind_idesc<KIND>(BM, BN);
      const uint32_t empty_self = smem_u32(&empty[0]);
      const uint32_t empty_peer = mapa_shared(empty_self, peer);
      const uint32_t accf_self = smem_u32(&acc_full[0]);
      const uint32_t accf_peer = mapa_shared(accf_self, peer);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs, ++it) {
        const int buf = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&acc_empty[buf], acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * 256u;  // accumulators 256 columns apart
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int a = 0; a < KATOMS; ++a) {
            const uint64_t adesc = make_sw128_desc(smem_u32(sA + stage * L::kATile + a * L::kAtom));
            const uint64_t bdesc = make_sw128_desc(smem_u32(sB + stage * L::kBTile + a * L::kBAtom));
#pragma unroll
            for (int k = 0; k < kGemmBK / 32; ++k)
              umma_ss_pair<KIND>(d_tmem, adesc + 2 * k, bdesc + 2 * k, kIdesc,
                                 (kb | a | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(empty_self + stage * 8);
          umma_commit_pair(empty_peer + stage * 8);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (ok) {
          umma_commit_pair(accf_self + buf * 8);
          umma_commit_pair(accf_peer + buf * 8);
        }
      }
    }
    __syncwarp();
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------ quantizer warps
    if constexpr (PRO != kProNone) {
      if (pro.ring) {
        uint8_t* ring = smem + L::kQuantOffset + (warp - 2) * kQSlots * kQSlotBytes;
        uint64_t* qfull = reinterpret_cast<uint64_t*>(smem + L::kQuantOffset + kQWarps * kQSlots * kQSlotBytes) +
                          (warp - 2) * kQSlots;
        if (pro.x_f16) pro_ring_worker<PRO, __half>(pro, M, K, pro_s, ring, qfull, abort_flag);
        else pro_ring_worker<PRO, __nv_bfloat16>(pro, M, K, pro_s, ring, qfull, abort_flag);
      } else {
        pro_worker<PRO>(pro, M, K, pro_s);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const int half = (warp - 4) >> 2;
    const int row_local = q * 32 + lane;
    const float xs = ep.extra_scale ? __ldg(ep.extra_scale) : 1.0f;
    const uint32_t acce_leader = mapa_shared(smem_u32(&acc_empty[0]), 0);
    constexpr bool kAccInt = KIND == MmaKind::I8;
    constexpr int kChunks = BN / 64;
    constexpr bool kStoreEpi = (EPI == kEpiI8Dequant || EPI == kEpiScaled) && PRO == kProNone;
    float amax_acc = 0.0f;  // max |out| of this thread's stored outputs (ep.amax_out)
    int it = 0;
    for (int tile = pair; tile < num_tiles; tile += num_pairs, ++it) {
      int mb, nb;
      gemm_tile_coords(tile, num_m, num_n, group_m, mb, nb);
      const int buf = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if constexpr (kStoreEpi) {
        if (ep.tma_store) {
          // this tile's 256 column scales and biases (as floats) into shared memory;
          // the buffer written here was last read two tiles ago, before every
          // epilogue warp passed the previous tile's barrier
          float* par = reinterpret_cast<float*>(smem + L::kParOffset) + (it & 1) * 512;
          uint64_t* par_full = reinterpret_cast<uint64_t*>(smem + L::kParBarOffset);
          const int et = threadIdx.x - 128;
          const int n = min(nb * BN + et, N - 1);
          par[et] = ep.col_scale ? __ldg(ep.col_scale + (ep.col_scale_vec ? n : 0)) : 1.0f;
          par[256 + et] = load_bias(ep.bias, ep.bias_dtype, n);
          mbar_arrive(&par_full[it & 1]);
          if (!mbar_wait_warp(&par_full[it & 1], (it >> 1) & 1, abort_flag)) break;
        }
      }
      if (ep.wait_sleep_ns) {
        if (!__all_sync(0xffffffffu, mbar_wait_sleepy(&acc_full[buf], acc_phase, abort_flag,
                                                       ep.wait_sleep_ns)))
          break;
      } else if (!mbar_wait_warp(&acc_full[buf], acc_phase, abort_flag)) {
        break;
      }
      tc_fence_after();
      const int64_t m = static_cast<int64_t>(mb) * BM + static_cast<int64_t>(rank) * 128 + row_local;
      const bool row_ok = m < M;
      if constexpr (PRO == kProInt8Row) {
        const int band = (mb * BM) / kBandRows + static_cast<int>(rank);
        if (!__all_sync(0xffffffffu, pro_band_wait(pro, band, M, abort_flag))) break;
      }
      float rs = 1.0f;
      if constexpr (PRO == kProFp8Tensor) {
        rs = pro_s;
      } else {
        if (EPI != kEpiInt32 && ep.row_scale && row_ok) rs = __ldcg(ep.row_scale + (ep.row_scale_vec ? m : 0));
      }
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * 256u;
      if constexpr (kStoreEpi) {
        if (ep.tma_store) {
          // Column params of the tile were staged above; each chunk goes
          // TMEM -> registers -> epilogue math -> 64B-swizzled staging block ->
          // TMA store of the warp's 32 rows x 32 columns (clipped at M and N).
          const float* par = reinterpret_cast<const float*>(smem + L::kParOffset) + (it & 1) * 512;
          uint8_t* stg = smem + L::kEpiOffset + (warp - 4) * L::kEpiBlock;
          const int y0 = mb * BM + static_cast<int>(rank) * 128 + q * 32;
          const bool has_bias = ep.bias_dtype != kBiasNone;
#pragma unroll 1
          for (int c = half * kChunks; c < (half + 1) * kChunks; ++c) {
            uint32_t r[32];
            float cs[32], bi[32], v[32];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 a = reinterpret_cast<const float4*>(par + c * 32)[j];
              cs[4 * j] = a.x; cs[4 * j + 1] = a.y; cs[4 * j + 2] = a.z; cs[4 * j + 3] = a.w;
              const float4 b = reinterpret_cast<const float4*>(par + 256 + c * 32)[j];
              bi[4 * j] = b.x; bi[4 * j + 1] = b.y; bi[4 * j + 2] = b.z; bi[4 * j + 3] = b.w;
            }
            tmem_ld32(taddr + c * 32, r);
            tmem_ld_wait();
            epilogue_math<EPI, kAccInt>(r, cs, bi, has_bias, rs, xs, ep, v);
            if (ep.amax_out && row_ok) chunk_amax(v, N - (nb * BN + c * 32), amax_acc);
            uint32_t pk[16];
#pragma unroll
            for (int j = 0; j < 16; ++j)
              pk[j] = ep.out_dtype == kOutF16 ? pack_f16x2(v[2 * j], v[2 * j + 1])
                                              : pack_bf16x2(v[2 * j], v[2 * j + 1]);
            if (lane == 0) bulk_wait_read_all();  // the previous block has left the buffer
            __syncwarp();
            uint8_t* row = stg + lane * 64;
#pragma unroll
            for (int j = 0; j < 4; ++j)
              *reinterpret_cast<uint4*>(row + ((j ^ ((lane >> 1) & 3)) << 4)) =
                  make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmOut, stg, nb * BN + c * 32, y0);
              for (int p = 0; p < peers.n; ++p)  // the same block into the peers' copies
                tma_store_2d(&peers.map[p], stg, nb * BN + c * 32, y0);
              bulk_commit_group();
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(acce_leader + buf * 8);
          continue;
        }
      }
      if constexpr (kSwiGLU) {
        swiglu_tile_epilogue<BN>(taddr, half, nb * kTileN, F, m, row_ok, rs, ep);
      } else if constexpr (EPI == kEpiI8QkvNormRope) {
        // BN = 256: each warp half owns one 128-column head
        qkv_norm_rope_head(taddr + half * 128, nb * BN + half * 128, m, row_ok, rs, ep);
      } else {
#pragma unroll 1
        for (int c = half * kChunks; c < (half + 1) * kChunks; ++c) {
          const int n0 = nb * BN + c * 32;
          uint32_t r[32];
          if constexpr (EPI == kEpiInt32) {
            tmem_ld32(taddr + c * 32, r);
            tmem_ld_wait();
            if (row_ok && n0 < N) store_chunk_i32(ep, m, n0, r);
          } else {
            float cs[32], bi[32], v[32];
            const bool has_bias = n0 < N ? load_col_params(ep, n0, cs, bi) : false;
            tmem_ld32(taddr + c * 32, r);
            tmem_ld_wait();
            if (row_ok && n0 < N) {
              epilogue_math<EPI, kAccInt>(r, cs, bi, has_bias, rs, xs, ep, v);
              store_chunk(ep, m, n0, v, N);
              if (ep.amax_out) chunk_amax(v, N - n0, amax_acc);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acce_leader + buf * 8);
    }
    if (ep.amax_out) {
      // the stored values are the outputs rounded to their type, and rounding
      // is monotonic: max |rounded| = rounded max |v|
      const float rm = ep.out_dtype == kOutF16 ? round_f16(amax_acc)
                       : ep.out_dtype == kOutBF16 ? round_bf16(amax_acc) : amax_acc;
      const unsigned int bits = __reduce_max_sync(0xffffffffu, __float_as_uint(rm));
      if (lane == 0 && bits != 0u) atomicMax(ep.amax_out, bits);
    }
    if constexpr (kStoreEpi) {
      if (ep.tma_store && lane == 0) {
        bulk_wait_all();  // stores done before the CTA exits
        if (peers.n > 0) __threadfence_system();  // peer writes performed system-wide
      }
    }
  }

  tc_fence_before();
  cluster_sync();  // the peer's shared memory and barriers stay alive until both are done
  tc_fence_after();
  if (warp == 2) tmem_dealloc_pair(tmem_base, L::kTmemCols);
  if constexpr (PRO != kProNone) pro_exit(pro, exit_flag);
}

template <int EPI>
__device__ __forceinline__ float epi_value(uint32_t raw, float rs, float cs, float xs,
                                           const EpiArgs& e, int n, bool acc_is_int) {
  if constexpr (EPI == kEpiI8Dequant) {
    return epi_i8_dequant(static_cast<int32_t>(raw), rs, cs, e, n);
  } else {
    const float acc = acc_is_int ? __int2float_rn(static_cast<int32_t>(raw)) : __uint_as_float(raw);
    return epi_scaled(acc, rs, cs, xs, e, n);
  }
}

// ---------------------------------------------------------------------------
// SIMT fallback for shapes the TMA path cannot describe (K or a row stride not a
// multiple of 16 bytes, unaligned base pointers).  Same epilogues; int8 sums are
// exact, fp8 sums accumulate in fp32.  64x64 tile, 256 threads, 4x4 per thread.
template <bool IS_FP8, int EPI>
__global__ void __launch_bounds__(256)
    gemm8_simt_kernel(const uint8_t* __restrict__ A, int64_t lda, const uint8_t* __restrict__ B,
                      int64_t ldb, int M, int N, int K, EpiArgs ep) {
  constexpr int T = 64, TK = 32;
  using Acc = typename std::conditional<IS_FP8, float, int32_t>::type;
  __shared__ Acc sa[TK][T + 1];
  __shared__ Acc sb[TK][T + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * T, n0 = blockIdx.x * T;
  Acc acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = Acc(0);
  for (int k0 = 0; k0 < K; k0 += TK) {
    for (int i = threadIdx.x; i < T * TK; i += 256) {
      const int r = i / TK, k = i % TK;
      const int gm = m0 + r, gn = n0 + r, gk = k0 + k;
      Acc va = Acc(0), vb = Acc(0);
      if (gm < M && gk < K) {
        const uint8_t b = A[static_cast<int64_t>(gm) * lda + gk];
        if constexpr (IS_FP8) va = decode_e4m3(b); else va = static_cast<int8_t>(b);
      }
      if (gn < N && gk < K) {
        const uint8_t b = B[static_cast<int64_t>(gn) * ldb + gk];
        if constexpr (IS_FP8) vb = decode_e4m3(b); else vb = static_cast<int8_t>(b);
      }
      sa[k][r] = va;
      sb[k][r] = vb;
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < TK; ++k) {
      Acc a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = sa[k][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = sb[k][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += a[i] * b[j];
    }
    __syncthreads();
  }
  const float xs = ep.extra_scale ? *ep.extra_scale : 1.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty + 16 * i;
    if (m >= M) continue;
    const float rs = ep.row_scale ? ep.row_scale[ep.row_scale_vec ? m : 0] : 1.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx + 16 * j;
      if (n >= N) continue;
      if constexpr (EPI == kEpiInt32) {
        static_cast<int32_t*>(ep.out)[static_cast<int64_t>(m) * ep.ldo + n] = static_cast<int32_t>(acc[i][j]);
      } else {
        const float cs = ep.col_scale ? ep.col_scale[ep.col_scale_vec ? n : 0] : 1.0f;
        uint32_t raw;
        if constexpr (IS_FP8) raw = __float_as_uint(static_cast<float>(acc[i][j]));
        else raw = static_cast<uint32_t>(acc[i][j]);
        store_out(ep, m, n, epi_value<EPI>(raw, rs, cs, xs, ep, n, !IS_FP8));
      }
    }
  }
}

}  // namespace b200q
