// FP8 weight-only W8A16 for small token counts without decoding the weight.
//
// At small M the W8A16 linear is bound by the e4m3 weight stream from HBM (one
// byte per weight; at M = 256 the tensor-core side takes over).  Decoding each weight to bf16 on the SMs costs ~4 ALU
// instructions per pair of weights, which at HBM rate takes about half of every
// SM's issue slots; instead, the activations (few rows) are split exactly into
// e4m3 "planes" and the tensor cores multiply the raw weight tile with them
// (tcgen05 kind::f8f6f4), so the weight goes TMA -> shared memory -> MMA with no
// instruction touching it:
//
//   x[t,k]   = sum_p q_p[t,k] * 2^-e_p[t]          q_p e4m3, e_p a per-row exponent
//   out[t,n] = act( (sum_p 2^-e_p[t] * sum_k W[n,k] q_p[t,k]) * w_scale + bias[n] )
//
// Plane 0 is x * 2^e_0 rounded to e4m3, with e_0 putting the row's |x| maximum in
// [128, 256); plane p+1 is the remainder of plane p, rescaled the same way by its
// own maximum.  A bf16 value has 8 significant bits and a rounded e4m3 plane
// keeps 4 of them, so two planes hold a bf16 row exactly (fp16: 11 bits, three
// planes) -- except for elements more than ~2^13 below the row maximum, whose
// last bits fall under e4m3's subnormal spacing; the part lost there is below
// 2^-21 of the row maximum, far under the fp32 rounding of the dot product.
//
// Kernels (one call = the planes pass, then the GEMM launched as its
// programmatic dependent, so the GEMM's CTAs start streaming weights while the
// planes are being written):
//   x_planes_kernel   one CTA per token row: |x| max, planes, plane scales.
//   w8a16_planes_kernel<NT>
//     weight-stationary tile: MMA M = 128 weight rows, N = NT = P x BT plane rows
//     (BT tokens padded to 16/32/64/128; more tokens are split into token tiles,
//     one CTA per (weight tile, token tile)), D^T[n, p*BT + t] in TMEM (fp32).
//     warp 0   TMA producer: 128 x 128 B weight tile + NT x 128 B plane tile per
//              stage, 128-byte swizzle; the weight loads of the first stages are
//              issued before griddepcontrol.wait, the plane loads after it.
//     warp 1   MMA issuer: 4 x kind::f8f6f4 (K = 32) per stage.
//     warp 2   TMEM allocator; warps 2..7 stage the plane scales during the
//              mainloop.
//     all 8 warps  epilogue once the accumulator is final: one thread per weight
//              row (TMEM lane), the two warp halves taking alternate 16-token
//              groups.  120 registers per thread let two CTAs share an SM.
//   Split-K for occupancy: a cluster of S CTAs shares a weight tile, CTA rank s
//   taking K blocks [s*nkb/S, (s+1)*nkb/S).  Ranks 1..S-1 dump their fp32
//   accumulators into their own (drained) ring memory; rank 0 adds them in rank
//   order through distributed shared memory (fixed order, so results are
//   bit-reproducible), combines the planes and runs the epilogue.  No global
//   workspace, counters or memset node is involved.
//   w8a16_pgemv_kernel<NG>
//     the planes GEMV for up to 8 * NG plane rows (a few tokens): the GEMV's
//     32-row CTAs and TMA weight ring, every warp multiplying its own K slice
//     on warp-level e4m3 MMAs (mma.sync m16n8k32) against the planes.
#pragma once

#include <type_traits>

#include "quant.cuh"  // warp_max
#include "w8a16.cuh"

namespace b200q {

constexpr int kWpBK = 128;          // K bytes per stage (one 128-byte swizzle atom)
constexpr int kWpThreads = 256;
constexpr int kWpMaxStages = 8;
constexpr int kWpPlaneThreads = 256;

__device__ __forceinline__ float ld_dsmem_f32(uint32_t cluster_addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
  return v;
}

template <int NT>
struct WpLayout {
  static constexpr int kWSlot = 128 * kWpBK;  // e4m3 weight tile
  static constexpr int kXSlot = NT * kWpBK;   // e4m3 plane tile
  static constexpr int kStage = kWSlot + kXSlot;
  static constexpr int kDump = NT * 128 * 4;  // fp32 accumulators, [column][row]
  static constexpr uint32_t kTmemCols = NT <= 32 ? 32 : NT <= 64 ? 64 : NT <= 128 ? 128 : 256;
  // bf16 tiles are 2 x {16,32,64,128} plane rows, fp16 tiles 3 x {16,32,64}.
  static constexpr int kPlanes = NT % 3 == 0 ? 3 : 2;
  // full[8], empty[8], acc_full, tmem slot, abort flag
  static constexpr int kBarBytes = (2 * kWpMaxStages + 1) * 8 + 16;
  __host__ __device__ static constexpr int ring_bytes(int stages) {
    return stages * kStage > kDump ? stages * kStage : kDump;
  }
  __host__ __device__ static constexpr int smem_bytes(int stages) {
    return ring_bytes(stages) + kBarBytes + 1024;
  }
};

struct WpArgs {
  int M, N, K;
  int bt;                 // tokens per plane and token tile (16, 32, 64 or 128)
  int ntt;                // token tiles: ceil(M / bt)
  int planes;             // P = 2 (bf16 activations) or 3 (fp16)
  int splits;             // cluster size S
  int stages;             // ring depth (<= kWpMaxStages)
  int katoms;             // 128-byte K atoms per stage (1 or 2): 4 MMAs per atom
  const float* pscale;    // [ntt][P][bt]: 2^-e_p[t]
};

// ---------------------------------------------------------------------------
// Planes of one activation row.  The row is read once from global memory into
// shared memory (16-byte vectors: K % 8 == 0 and 16-byte aligned rows, checked
// by the host; K <= kWpMaxK) and every pass (max; plane 0 and its remainder's
// max; plane 1 ...) reads it from there.  A row holding an infinity or NaN gets
// NaN plane scales, so its whole output row is NaN.
constexpr int kWpMaxK = 32768;  // 64 KB of bf16 / fp16 row in shared memory

// Largest e with max * 2^e < 256 and max * 2^e >= 128 for a normal max, clamped
// so that 2^(total) and 2^-(total) stay normal floats.
__device__ __forceinline__ int plane_exponent(float amax, int used) {
  if (!(amax > 0.0f)) return 0;
  const int E = static_cast<int>((__float_as_uint(amax) >> 23) & 0xFFu);  // biased exponent
  int e = 134 - E;                       // amax in [2^(E-127), 2^(E-126)) -> [128, 256)
  if (e > 126 - used) e = 126 - used;    // keep 2^-(used + e) a normal float
  if (e < -120) e = -120;
  return e;
}
__device__ __forceinline__ float exp2i(int e) {  // 2^e for -126 <= e <= 127
  return __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
}

template <typename XT>
__device__ __forceinline__ void unpack8f(const uint4 u, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<XT, __half>::value) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      const float2 f = __half22float2(h);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    } else {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
}

// e4m3 round-to-nearest-even of two floats (|v| <= 256 here, never saturates),
// returned as the code pair and as the decoded values.
__device__ __forceinline__ uint16_t e4m3x2_rn(float a, float b, float& da, float& db) {
  const __nv_fp8x2_storage_t c = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(c, __NV_E4M3);
  const float2 f = __half22float2(__half2(h));
  da = f.x;
  db = f.y;
  return static_cast<uint16_t>(c);
}

// Plane p of 8 consecutive row elements v (the row scaled by 2^e_tot[0] is
// split into planes 0..p; plane j's remainder is rescaled to plane j+1's range
// by 2^(e_tot[j+1] - e_tot[j]), all exact), packed as 8 e4m3 codes; rmax takes
// the largest remainder magnitude after plane p.
template <int P>
__device__ __forceinline__ uint2 plane_codes8(const float (&v)[8], float mult0,
                                              const int (&e_tot)[P], int p, float& rmax) {
  uint32_t codes[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    float r0 = v[i] * mult0, r1 = v[i + 1] * mult0;  // exact (power of two)
    uint16_t c = 0;
#pragma unroll
    for (int j = 0; j < P; ++j) {
      if (j > p) break;
      if (j > 0) {  // rescale the remainder to plane j's range (exact)
        const float s = exp2i(e_tot[j] - e_tot[j - 1]);
        r0 *= s;
        r1 *= s;
      }
      float d0, d1;
      c = e4m3x2_rn(r0, r1, d0, d1);
      r0 -= d0;  // exact: the remainder of a rounding to a coarser grid
      r1 -= d1;
    }
    codes[i >> 2] |= static_cast<uint32_t>(c) << ((i & 2) * 8);
    rmax = fmaxf(rmax, fmaxf(fabsf(r0), fabsf(r1)));
  }
  return make_uint2(codes[0], codes[1]);
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5;
  __syncthreads();  // red[] free from the previous use
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int w = 1; w < kWpPlaneThreads / 32; ++w) m = fmaxf(m, red[w]);
  return m;
}

// Grid: one CTA per token row t < M.  planes: [ntt][P][bt][K] bytes (token tile
// tt = t / bt holds its P planes' rows contiguously, one TMA box); pscale
// [ntt][P][bt].
template <typename XT, int P>
__global__ void __launch_bounds__(kWpPlaneThreads)
    x_planes_kernel(const XT* __restrict__ x, int64_t ldx, int K, int bt,
                    uint8_t* __restrict__ planes, float* __restrict__ pscale) {
  // Launched as a programmatic dependent of whatever ran before it: nothing of
  // that work is touched before griddepcontrol.wait, and the GEMM is released
  // only after it, so the GEMM's early weight loads never overtake a kernel
  // that wrote the weight.
  griddep_wait();
  griddep_launch_dependents();  // the GEMM may start streaming weights now
  __shared__ float red[kWpPlaneThreads / 32];
  extern __shared__ uint4 srow[];  // the row, K / 8 vectors
  const int t = blockIdx.x;
  const int tt = t / bt, tl = t - tt * bt;  // token tile, row inside it
  const uint4* row = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t) * ldx);
  const int64_t plane_stride = static_cast<int64_t>(bt) * K;
  uint8_t* out0 = planes + (static_cast<int64_t>(tt) * P * bt + tl) * K;
  const int nv = K / 8;

  // max |x|, and whether the row is finite; the row is kept in shared memory
  float amax = 0.0f;
  bool finite = true;
  for (int i = threadIdx.x; i < nv; i += kWpPlaneThreads) {
    const uint4 u = __ldg(row + i);
    srow[i] = u;
    float v[8];
    unpack8f<XT>(u, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float a = fabsf(v[i]);
      finite = finite && a <= 3.402823466e38f;
      amax = fmaxf(amax, a);
    }
  }
  const bool all_finite = __syncthreads_and(finite) != 0;
  amax = block_max(amax, red);
  int e_tot[P] = {};  // plane p holds x's remainder scaled by 2^e_tot[p]
  e_tot[0] = plane_exponent(amax, 0);
  int used = e_tot[0];
  const float mult0 = exp2i(e_tot[0]);

  // Plane p pass: recompute planes 0..p-1 (their remainders), write plane p,
  // and take the max of the remainder after it.
#pragma unroll
  for (int p = 0; p < P; ++p) {
    float rmax = 0.0f;
    for (int i = threadIdx.x; i < nv; i += kWpPlaneThreads) {
      float v[8];
      unpack8f<XT>(srow[i], v);
      *reinterpret_cast<uint2*>(out0 + p * plane_stride + i * 8) = plane_codes8<P>(v, mult0, e_tot, p, rmax);
    }
    if (p + 1 < P) {
      rmax = block_max(rmax, red);
      // The remainder is in plane p's units: its exponent adds to e_tot[p].
      used += plane_exponent(rmax, used);
      e_tot[p + 1] = used;
    }
  }
  if (threadIdx.x == 0) {
    const float nan = __uint_as_float(0x7FC00000u);
#pragma unroll
    for (int p = 0; p < P; ++p) pscale[(tt * P + p) * bt + tl] = all_finite ? exp2i(-e_tot[p]) : nan;
  }
}

// ---------------------------------------------------------------------------
// Rank 0's epilogue for one thread (weight row r of the tile, token tile tt):
// 16-token groups t0 = 16 * (2i + half).  Each group loads its P accumulator column groups with
// one TMEM wait, adds the peers' accumulators in rank order (distributed shared
// memory), combines the planes with their scales, applies w_scale (xs), bias
// and the activation (ACT fixed at compile time, so the 16 tokens are
// independent straight-line code) and stores tokens < M.  An absent scale is
// 1.0 and an absent bias -0.0: both exact, so no per-token branches remain.
template <int NT, int ACT>
__device__ __forceinline__ void wp_epilogue(const WpArgs& a, const EpiArgs& ep, int tile, int tt,
                                            int r, uint32_t taddr, int half, const float* s_pscale,
                                            uint32_t dump_base, float xs, float bias_v) {
  constexpr int P = WpLayout<NT>::kPlanes;
  constexpr int BT = NT / P;
  const int n = tile * 128 + r;
  const bool n_ok = n < a.N;
  const int S = a.splits;
  const int mt = a.M - tt * BT < BT ? a.M - tt * BT : BT;  // tokens of this tile
  const int64_t row0 = static_cast<int64_t>(tt) * BT;
#pragma unroll 1
  for (int t0 = 16 * half; t0 < mt; t0 += 32) {
    float acc[P][16];
    {
      uint32_t v[P][16];
#pragma unroll
      for (int p = 0; p < P; ++p) tmem_ld_cols<16>(taddr + p * BT + t0, v[p]);
      tmem_ld_wait();
#pragma unroll
      for (int p = 0; p < P; ++p)
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[p][j] = __uint_as_float(v[p][j]);
    }
    for (int s2 = 1; s2 < S; ++s2) {  // rank order: ((D_0 + D_1) + D_2) + ...
      const uint32_t peer = mapa_shared(dump_base, static_cast<uint32_t>(s2));
#pragma unroll
      for (int p = 0; p < P; ++p)
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (t0 + j < mt)  // peers dumped only the tile's tokens
            acc[p][j] = __fadd_rn(acc[p][j], ld_dsmem_f32(peer + ((p * BT + t0 + j) * 128 + r) * 4));
    }
    // Tokens t0 .. t0+15 < bt always index valid (if unused) plane columns and
    // scales; only the stores are limited to tokens < M.
    float out_v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float v = __fmul_rn(acc[0][j], s_pscale[t0 + j]);
#pragma unroll
      for (int p = 1; p < P; ++p) v = __fadd_rn(v, __fmul_rn(acc[p][j], s_pscale[p * BT + t0 + j]));
      v = __fadd_rn(__fmul_rn(v, xs), bias_v);
      out_v[j] = apply_act(v, ACT);
    }
    // Direct typed stores (32 lanes = 32 consecutive output features of one
    // token row); measured 2x faster here than the generic per-element store.
    if (n_ok) {
      if (ep.out_dtype == kOutF32) {
        float* o = static_cast<float*>(ep.out) + n;
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (t0 + j < mt) o[(row0 + t0 + j) * ep.ldo] = out_v[j];
      } else if (ep.out_dtype == kOutF16) {
        __half* o = static_cast<__half*>(ep.out) + n;
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (t0 + j < mt) o[(row0 + t0 + j) * ep.ldo] = __float2half_rn(out_v[j]);
      } else {
        __nv_bfloat16* o = static_cast<__nv_bfloat16*>(ep.out) + n;
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (t0 + j < mt) o[(row0 + t0 + j) * ep.ldo] = __float2bfloat16_rn(out_v[j]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// 120 registers per thread: two 256-thread CTAs fit an SM's register file
// (at 128 the occupancy calculator allowed only one).
template <int NT>
__global__ void __maxnreg__(120)
    w8a16_planes_kernel(const __grid_constant__ CUtensorMap tmW,
                        const __grid_constant__ CUtensorMap tmX, WpArgs a, EpiArgs ep) {
  using L = WpLayout<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int stages = a.stages;
  const int KA = a.katoms;
  // A stage holds KA weight atoms (128 rows x 128 bytes each) followed by KA
  // plane atoms (NT rows x 128 bytes each); every atom starts 1024-aligned.
  const int stage_bytes = KA * L::kStage;
  // Ring size exactly as the host sized the allocation: split ranks park their
  // accumulators in the ring afterwards, so with S > 1 it covers the dump too.
  const int ring = (a.splits > 1 && L::kDump > stages * stage_bytes) ? L::kDump : stages * stage_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + ring);
  uint64_t* empty = full + kWpMaxStages;
  uint64_t* acc_full = empty + kWpMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* dump = reinterpret_cast<float*>(smem);  // reuses the drained ring
  __shared__ float s_pscale[3 * 128];            // [P][bt] plane scales

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = a.splits;
  const int split = S > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int unit = blockIdx.x / S;  // (weight tile, token tile); the cluster's K-splits share it
  const int tile = unit / a.ntt;
  const int tt = unit - tile * a.ntt;
  const int nkb = (a.K + KA * kWpBK - 1) / (KA * kWpBK);  // stages of KA atoms along K
  const int kb0 = split * nkb / S, kb1 = (split + 1) * nkb / S;
  const int nst = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;
  // Epilogue operands that do not depend on this grid's inputs (written before
  // the planes pass ran): loaded now, consumed after the mainloop.
  const int q = warp & 3;
  const int r = q * 32 + lane;  // weight row in the tile = TMEM lane
  const float xs = ep.extra_scale ? __ldg(ep.extra_scale) : 1.0f;
  const float bias_v = (tile * 128 + r < a.N && ep.bias_dtype != kBiasNone)
                           ? load_bias(ep.bias, ep.bias_dtype, tile * 128 + r) : -0.0f;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const int pre = nst < stages ? nst : stages;
      // The weights were written before the planes pass started, so they may be
      // read before this grid's dependency on that pass resolves.
      // K past the end (a ragged last stage) reads as zeros.
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], stage_bytes);
        for (int at = 0; at < KA; ++at)
          tma_load_2d(&tmW, &full[i], smem + i * stage_bytes + at * L::kWSlot,
                      ((kb0 + i) * KA + at) * kWpBK, tile * 128);
      }
      griddep_wait();
      for (int i = 0; i < pre; ++i)
        for (int at = 0; at < KA; ++at)
          tma_load_2d(&tmX, &full[i], smem + i * stage_bytes + KA * L::kWSlot + at * L::kXSlot,
                      ((kb0 + i) * KA + at) * kWpBK, tt * NT);
      int issued = pre;
      bool ok = true;
      for (int i = pre; i < nst; ++i) {
        const int s = i % stages;
        const uint32_t ph = static_cast<uint32_t>(i / stages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) { ok = false; break; }
        mbar_arrive_expect_tx(&full[s], stage_bytes);
        uint8_t* dst = smem + s * stage_bytes;
        for (int at = 0; at < KA; ++at) {
          const int x = ((kb0 + i) * KA + at) * kWpBK;
          tma_load_2d(&tmW, &full[s], dst + at * L::kWSlot, x, tile * 128);
          tma_load_2d(&tmX, &full[s], dst + KA * L::kWSlot + at * L::kXSlot, x, tt * NT);
        }
        issued = i + 1;
      }
      if (!ok) {
        // Let the copies still in flight land before the ring is reused or freed.
        for (int i = issued - stages < 0 ? 0 : issued - stages; i < issued; ++i)
          mbar_wait_drain(&full[i % stages], static_cast<uint32_t>(i / stages) & 1u);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdesc = kind_idesc<MmaKind::F8F6F4>(128, NT);
      bool ok = true;
      for (int i = 0; i < nst; ++i) {
        const int s = i % stages;
        if (!mbar_wait(&full[s], static_cast<uint32_t>(i / stages) & 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        for (int at = 0; at < KA; ++at) {
          const uint64_t adesc = make_sw128_desc(smem_u32(smem + s * stage_bytes + at * L::kWSlot));
          const uint64_t bdesc =
              make_sw128_desc(smem_u32(smem + s * stage_bytes + KA * L::kWSlot + at * L::kXSlot));
#pragma unroll
          for (int k = 0; k < 4; ++k)  // K = 32 bytes per MMA = +2 in the >>4 address field
            umma_ss<MmaKind::F8F6F4>(tmem_d, adesc + 2 * k, bdesc + 2 * k, kIdesc,
                                     (i > 0 || at > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      if (ok) umma_commit(acc_full);
    }
    __syncwarp();
  } else if (split == 0) {
    // Warps 2..7 stage the plane scales while the mainloop runs.
    griddep_wait();
    for (int i = threadIdx.x - 64; i < L::kPlanes * (NT / L::kPlanes); i += kWpThreads - 64)
      s_pscale[i] = a.pscale[tt * NT + i];
  }

  // ------------------------------------------------------------ epilogue
  // All 8 warps, once the accumulator is final: warp w reads TMEM lane quarter
  // w % 4 (its weight rows) and takes every other 16-column group (w / 4).
  const int half = warp >> 2;
  const uint32_t taddr = tmem_d + (static_cast<uint32_t>(q * 32) << 16);
  const bool valid = mbar_wait_warp(acc_full, 0u, abort_flag);
  tc_fence_after();
  if (split > 0 && valid) {
    // Ranks 1..S-1: accumulators -> own shared memory, [column][row]; only the
    // 16-column groups holding tokens of this tile (rank 0 reads nothing else).
    constexpr int BT = NT / L::kPlanes;
    const int mt = a.M - tt * BT < BT ? a.M - tt * BT : BT;
#pragma unroll 1
    for (int c = 16 * half; c < NT; c += 32) {
      if (c % BT >= mt) continue;
      uint32_t v[16];
      tmem_ld_cols<16>(taddr + c, v);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; ++j) dump[(c + j) * 128 + r] = __uint_as_float(v[j]);
    }
  }

  if (S > 1) cluster_sync();  // every rank's dump is written and visible

  __syncthreads();  // the staged plane scales are visible
  if (split == 0 && valid && *abort_flag == 0) {
    const uint32_t db = smem_u32(dump);
    switch (ep.act) {
      case kActGeluTanh: wp_epilogue<NT, kActGeluTanh>(a, ep, tile, tt, r, taddr, half, s_pscale, db, xs, bias_v); break;
      case kActGeluErf: wp_epilogue<NT, kActGeluErf>(a, ep, tile, tt, r, taddr, half, s_pscale, db, xs, bias_v); break;
      default: wp_epilogue<NT, kActNone>(a, ep, tile, tt, r, taddr, half, s_pscale, db, xs, bias_v); break;
    }
  }

  if (S > 1) cluster_sync();  // rank 0 has read every peer's dump
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem_d, L::kTmemCols);
}

// ---------------------------------------------------------------------------
// Planes GEMV: 8 plane rows per MMA column group (4 bf16 tokens x 2 planes, 2 fp16
// tokens x 3), NG groups.
// The weight stream of the GEMV (32-row CTAs, the same TMA ring and 128-byte
// swizzle, three CTAs per SM) multiplied on warp-level e4m3 MMAs
// (mma.sync m16n8k32, fp32 accumulation) against the planes of the planes pass,
// so no instruction decodes a weight: 16 weight rows are the MMA's M, plane rows
// (plane p of token t is column p * M + t, the planes pass's layout with a token
// tile of M rows) its N = 8 columns.  Lane (g, q) reads 16 bytes of weight rows g
// and g + 8 of a 16-row group at K [16q, 16q + 16) of its warp's 64-byte slice;
// bytes 8kk .. 8kk + 3 and 8kk + 4 .. 8kk + 7 feed MMA kk (kk = 0, 1) as logical
// k 4q .. 4q + 3 and 16 + 4q .. 16 + 4q + 3, and the plane row's bytes at the
// same K positions form the B fragment (one 16-byte load per lane and column
// group), so the dot product is unchanged.  A stage's two MMAs start from zero
// and are added into fp32 sums, so the tensor core's own accumulation spans 64
// products.  The warps' sums meet in shared memory in warp order and the planes
// are combined as in the planes route's epilogue.
// The planes pass waited for every earlier kernel before it released this grid,
// so the weight is final when this grid starts: the first stages are issued
// before griddepcontrol.wait, which only guards the planes and their scales.
constexpr int kPgMaxCols = 16;  // NG <= 2

__device__ __forceinline__ void mma_e4m3_16832(float (&d)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// NG = 8-column groups (1: up to 8 plane rows, 2: up to 16).  Requires K % 16 ==
// 0 (whole 16-byte plane chunks) and P * M <= 8 * NG (the host checks).
template <int NG>
__global__ void __launch_bounds__(kGvThreads, 3)
    w8a16_pgemv_kernel(const __grid_constant__ CUtensorMap tmW, const uint8_t* __restrict__ planes,
                       const float* __restrict__ pscale, int P, int M, int N, int K, EpiArgs ep) {
  __shared__ float red[kGvWarps][NG * 8][kGvRows + 1];
  __shared__ float s_ps[kPgMaxCols];
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kGvStages * kGvStageBytes);
  uint64_t* empty = full + kGvStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kGvStages);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int n0 = blockIdx.x * kGvRows;
  const int nst = (K + kGvStageK - 1) / kGvStageK;
  const int cols = P * M;

  if (threadIdx.x == 0) {
    for (int s2 = 0; s2 < kGvStages; ++s2) {
      mbar_init(&full[s2], 1);
      mbar_init(&empty[s2], kGvWarps);
    }
    *abort_flag = 0;
    fence_mbarrier_init();
    tma_prefetch_desc(&tmW);
  }
  __syncthreads();
  auto issue = [&](int st) {  // thread 0: stage st into slot st % kGvStages
    const int slot = st % kGvStages;
    uint8_t* dst = ring + slot * kGvStageBytes;
    mbar_arrive_expect_tx(&full[slot], kGvStageBytes);
#pragma unroll
    for (int b = 0; b < kGvStageK / 128; ++b)
      tma_load_2d(&tmW, &full[slot], dst + b * (kGvRows * 128), st * kGvStageK + b * 128, n0);
  };
  if (threadIdx.x == 0)
    for (int st = 0; st < kGvStages && st < nst; ++st) issue(st);
  griddep_wait();  // the planes and plane scales of the planes pass
  griddep_launch_dependents();
  if (threadIdx.x < cols) s_ps[threadIdx.x] = __ldg(pscale + threadIdx.x);

  // Plane rows of this lane: column 8 ng + g; columns past P * M read as zero.
  const uint8_t* prow[NG];
  bool pok[NG];
#pragma unroll
  for (int ng = 0; ng < NG; ++ng) {
    const int c = 8 * ng + g;
    pok[ng] = c < cols;
    prow[ng] = planes + static_cast<int64_t>(pok[ng] ? c : 0) * K + 16 * q;
  }
  uint4 pa[NG], pn[NG];
  auto load_p = [&](int st, uint4 (&dst)[NG]) {
    const int k0 = st * kGvStageK + 64 * warp;
    const bool kin = st < nst && k0 + 16 * q < K;
#pragma unroll
    for (int ng = 0; ng < NG; ++ng)
      dst[ng] = (pok[ng] && kin) ? __ldg(reinterpret_cast<const uint4*>(prow[ng] + k0))
                                 : make_uint4(0u, 0u, 0u, 0u);
  };
  load_p(0, pn);
  float acc[2][NG][4];
#pragma unroll
  for (int rg = 0; rg < 2; ++rg)
#pragma unroll
    for (int ng = 0; ng < NG; ++ng)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[rg][ng][i] = 0.0f;
  const int box = warp >> 1;
  const int chunk = (warp & 1) * 4 + q;

  bool ok = true;
  for (int st = 0; st < nst && ok; ++st) {
    const int slot = st % kGvStages;
    const uint32_t ph = (st / kGvStages) & 1u;
#pragma unroll
    for (int ng = 0; ng < NG; ++ng) pa[ng] = pn[ng];
    load_p(st + 1, pn);
    if (!mbar_wait_warp(&full[slot], ph, abort_flag)) { ok = false; break; }
    const int k0 = st * kGvStageK + 64 * warp;
    if (k0 < K) {
      const uint8_t* sb = ring + slot * kGvStageBytes + box * (kGvRows * 128);
      uint4 wv[4];  // rows 8 gr + g
#pragma unroll
      for (int gr = 0; gr < 4; ++gr) {
        const int r = 8 * gr + g;
        wv[gr] = *reinterpret_cast<const uint4*>(sb + r * 128 + ((chunk ^ (r & 7)) << 4));
      }
#pragma unroll
      for (int rg = 0; rg < 2; ++rg)
#pragma unroll
        for (int ng = 0; ng < NG; ++ng) {
          float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          const uint4 lo = wv[2 * rg], hi = wv[2 * rg + 1];
          mma_e4m3_16832(d, lo.x, hi.x, lo.y, hi.y, pa[ng].x, pa[ng].y);
          mma_e4m3_16832(d, lo.z, hi.z, lo.w, hi.w, pa[ng].z, pa[ng].w);
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[rg][ng][i] += d[i];
        }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    if (threadIdx.x == 0 && st + kGvStages < nst) {
      if (!mbar_wait(&empty[slot], ph, abort_flag)) { ok = false; break; }
      issue(st + kGvStages);
    }
  }
  if (!ok && threadIdx.x == 0) {
    for (int s2 = 0; s2 < kGvStages; ++s2) mbar_wait_drain(&full[s2], 0);
  }

  // D fragment: acc[rg][ng][i] is weight row 16 rg + g + 8 (i >> 1), plane
  // column 8 ng + 2q + (i & 1).
#pragma unroll
  for (int rg = 0; rg < 2; ++rg)
#pragma unroll
    for (int ng = 0; ng < NG; ++ng)
#pragma unroll
      for (int i = 0; i < 4; ++i)
        red[warp][8 * ng + 2 * q + (i & 1)][16 * rg + g + 8 * (i >> 1)] = acc[rg][ng][i];
  __syncthreads();
  if (*abort_flag) return;
  const float xs = ep.extra_scale ? __ldg(ep.extra_scale) : 1.0f;
  for (int e = threadIdx.x; e < M * kGvRows; e += kGvThreads) {
    const int tok = e / kGvRows, r = e % kGvRows;
    const int n = n0 + r;
    if (n >= N) continue;
    float v = 0.0f;
    for (int p = 0; p < P; ++p) {
      const int c = p * M + tok;
      float s = red[0][c][r];
#pragma unroll
      for (int w2 = 1; w2 < kGvWarps; ++w2) s = __fadd_rn(s, red[w2][c][r]);
      v = p == 0 ? __fmul_rn(s, s_ps[c]) : __fadd_rn(v, __fmul_rn(s, s_ps[c]));
    }
    if (ep.extra_scale) v = __fmul_rn(v, xs);
    if (ep.bias_dtype != kBiasNone) v = __fadd_rn(v, load_bias(ep.bias, ep.bias_dtype, n));
    store_out(ep, tok, n, apply_act(v, ep.act));
  }
}

}  // namespace b200q
