// FP8 weight-only W8A16 linear on the sm_100a tensor cores:
//   out[M,N] = act( (X[M,K] . decode(W[N,K])^T) * w_scale + bias[N] )
// X is bf16 (or fp16), W is e4m3 bytes in the stored [N,K] layout (no per-call
// transpose or decode pass), w_scale is an optional per-tensor fp32 scale.
//
// The MMA runs "weight-stationary": tcgen05 M = 128 weight rows, N = BT tokens,
// so D^T[n, t] accumulates in TMEM with one lane per weight row.  That keeps
// small token counts (M = 1..256) on the tensor cores with a 16..256-wide N
// instead of padding M to 128, and makes the epilogue's stores coalesced along
// the output row (32 lanes write 32 consecutive output features).
//
//   warp 0      TMA producer: 128 x 64 fp8 weight bytes (no swizzle) and a
//               BT x 64 activation tile (128B swizzle) per stage.
//   warp 1      MMA issuer: 4 x tcgen05.mma kind::f16 (K=16) per stage.
//   warp 2      TMEM allocator (2 x BT columns).
//   warps 4..7  converters: e4m3 -> bf16/fp16 (exact), written into the
//               128B-swizzled K-major layout the MMA descriptor expects.
//   warps 8..11 epilogue: scale, bias, GELU, store; or, with split-K, fp32
//               partials to a workspace and a deterministic fixed-order
//               reduction by the last CTA to finish each tile.
// Split-K (small M only) spreads the weight stream over all SMs; the reduction
// order is fixed (split 0, 1, ...), so results are bit-reproducible run to run.
#pragma once

#include "numerics.cuh"
#include "ptx.cuh"

namespace b200q {

constexpr int kW16BM = 128;        // weight rows per tile (MMA M)
constexpr int kW16BK = 64;         // K elements per stage (one 128B bf16 swizzle atom)
constexpr int kW16Threads = 384;   // 12 warps

template <int BT>
struct W8A16Layout {
  static constexpr int kXStage = BT * kW16BK * 2;       // bf16 activation tile
  static constexpr int kCStage = kW16BM * kW16BK * 2;   // converted weight tile
  static constexpr int kWStage = kW16BM * kW16BK;       // raw fp8 weight tile
  static constexpr int kStageBytes = kXStage + kCStage + kWStage;
  static constexpr int kStages = (200 * 1024 / kStageBytes) > 8 ? 8 : (200 * 1024 / kStageBytes);
  static constexpr int kXOff = 0;
  static constexpr int kCOff = kStages * kXStage;
  static constexpr int kWOff = kCOff + kStages * kCStage;
  static constexpr int kBarOff = kWOff + kStages * kWStage;
  // full[S], empty[S], conv_full[S], acc_full[2], acc_empty[2], slot, abort, last flag
  static constexpr int kBarBytes = (3 * kStages + 4) * 8 + 16;
  static constexpr int kSmemBytes = kBarOff + kBarBytes + 1024;
  static constexpr uint32_t kTmemCols = 2 * BT < 32 ? 32 : 2 * BT;
};

template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[N]);
template <>
__device__ __forceinline__ void tmem_ld_cols<32>(uint32_t taddr, uint32_t (&r)[32]) {
  tmem_ld32(taddr, r);
}
template <>
__device__ __forceinline__ void tmem_ld_cols<16>(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Two e4m3 codes -> two fp16 packed (exact).
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t two) {
  __half2_raw h2 = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two), __NV_E4M3);
  return *reinterpret_cast<uint32_t*>(&h2);
}

__device__ __forceinline__ void w16_unit_coords(int u, int S, int num_t, int& nt, int& tt, int& sp) {
  sp = u % S;
  const int rest = u / S;
  tt = rest % num_t;
  nt = rest / num_t;
}

struct W8A16Args {
  int M, N, K;
  int splits;
  float* partial;            // [splits, M, N] fp32 (splits > 1)
  unsigned int* counters;    // one per (nt, tt) tile, zero on entry
};

template <int BT, bool X_F16>
__global__ void __launch_bounds__(kW16Threads, 1)
    w8a16_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                    W8A16Args a, EpiArgs ep) {
  using L = W8A16Layout<BT>;
  constexpr int S_ = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sX = smem + L::kXOff;
  uint8_t* sC = smem + L::kCOff;
  uint8_t* sW = smem + L::kWOff;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + S_;
  uint64_t* conv_full = empty + S_;
  uint64_t* acc_full = conv_full + S_;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_n = (a.N + kW16BM - 1) / kW16BM;
  const int num_t = (a.M + BT - 1) / BT;
  const int S = a.splits;
  const int num_units = num_n * num_t * S;
  const int num_kb = (a.K + kW16BK - 1) / kW16BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S_; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv_full[s], 128);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    *abort_flag = 0;
    *last_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        int nt, tt, sp;
        w16_unit_coords(u, S, num_t, nt, tt, sp);
        const int kb0 = sp * num_kb / S, kb1 = (sp + 1) * num_kb / S;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], L::kXStage + L::kWStage);
          tma_load_2d(&tmW, &full[stage], sW + stage * L::kWStage, kb * kW16BK, nt * kW16BM);
          tma_load_2d(&tmX, &full[stage], sX + stage * L::kXStage, kb * kW16BK, tt * BT);
          if (++stage == S_) { stage = 0; phase ^= 1u; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      // f32 accumulate; A = B = bf16 (format 1) or fp16 (format 0); M=128, N=BT.
      constexpr uint32_t kIdesc = X_F16 ? make_idesc(1, 0, 0, kW16BM, BT) : make_idesc(1, 1, 1, kW16BM, BT);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++it) {
        int nt, tt, sp;
        w16_unit_coords(u, S, num_t, nt, tt, sp);
        const int kb0 = sp * num_kb / S, kb1 = (sp + 1) * num_kb / S;
        const int buf = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&acc_empty[buf], acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BT;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&conv_full[stage], phase, abort_flag)) { ok = false; break; }
          if (!mbar_wait(&full[stage], phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = make_sw128_desc(smem_u32(sC + stage * L::kCStage));
          const uint64_t bdesc = make_sw128_desc(smem_u32(sX + stage * L::kXStage));
#pragma unroll
          for (int k = 0; k < kW16BK / 16; ++k)
            umma_ss<MmaKind::F16>(d_tmem, adesc + 2 * k, bdesc + 2 * k, kIdesc,
                                  (kb != kb0 || k != 0) ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == S_) { stage = 0; phase ^= 1u; }
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
    }
    __syncwarp();
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ converters
    const int t = threadIdx.x - 128;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
      int nt, tt, sp;
      w16_unit_coords(u, S, num_t, nt, tt, sp);
      const int kb0 = sp * num_kb / S, kb1 = (sp + 1) * num_kb / S;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag)) { ok = false; break; }
        const uint8_t* src = sW + stage * L::kWStage;
        uint8_t* dst = sC + stage * L::kCStage;
#pragma unroll
        for (int i = 0; i < (kW16BM * kW16BK / 8) / 128; ++i) {
          const int idx = i * 128 + t;
          const int r = idx >> 3, c = idx & 7;  // row, 16-byte output chunk
          const uint2 v = *reinterpret_cast<const uint2*>(src + r * kW16BK + c * 8);
          uint4 o;
          if constexpr (X_F16) {
            o.x = e4m3x2_to_f16x2(static_cast<uint16_t>(v.x & 0xFFFFu));
            o.y = e4m3x2_to_f16x2(static_cast<uint16_t>(v.x >> 16));
            o.z = e4m3x2_to_f16x2(static_cast<uint16_t>(v.y & 0xFFFFu));
            o.w = e4m3x2_to_f16x2(static_cast<uint16_t>(v.y >> 16));
          } else {
            o.x = e4m3x2_to_bf16x2(static_cast<uint16_t>(v.x & 0xFFFFu));
            o.y = e4m3x2_to_bf16x2(static_cast<uint16_t>(v.x >> 16));
            o.z = e4m3x2_to_bf16x2(static_cast<uint16_t>(v.y & 0xFFFFu));
            o.w = e4m3x2_to_bf16x2(static_cast<uint16_t>(v.y >> 16));
          }
          *reinterpret_cast<uint4*>(dst + r * 128 + ((c ^ (r & 7)) << 4)) = o;
        }
        fence_proxy_async_smem();
        mbar_arrive(&conv_full[stage]);
        if (++stage == S_) { stage = 0; phase ^= 1u; }
      }
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ epilogue
    constexpr int CH = BT < 32 ? BT : 32;
    const int q = warp & 3;
    const int et = threadIdx.x - 256;  // 0..127
    const float xs = ep.extra_scale ? __ldg(ep.extra_scale) : 1.0f;
    int it = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++it) {
      int nt, tt, sp;
      w16_unit_coords(u, S, num_t, nt, tt, sp);
      const int buf = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      // Never leave the loop early: the split-K hand-off below uses named
      // barriers that all 128 epilogue threads must reach the same number of times.
      const bool valid = mbar_wait_warp(&acc_full[buf], acc_phase, abort_flag);
      tc_fence_after();
      const int n = nt * kW16BM + q * 32 + lane;
      const bool n_ok = n < a.N;
      const float bias_v = (n_ok && ep.bias_dtype != kBiasNone) ? load_bias(ep.bias, ep.bias_dtype, n) : 0.0f;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BT;
#pragma unroll 1
      for (int c = 0; valid && c < BT / CH; ++c) {
        uint32_t r[CH];
        tmem_ld_cols<CH>(taddr + c * CH, r);
        tmem_ld_wait();
        const int t0 = tt * BT + c * CH;
        if (n_ok) {
#pragma unroll
          for (int j = 0; j < CH; ++j) {
            const int tok = t0 + j;
            if (tok < a.M) {
              const float acc = __uint_as_float(r[j]);
              if (S > 1) {
                a.partial[(static_cast<int64_t>(sp) * a.M + tok) * a.N + n] = acc;
              } else {
                float v = ep.extra_scale ? __fmul_rn(acc, xs) : acc;
                if (ep.bias_dtype != kBiasNone) v = __fadd_rn(v, bias_v);
                store_out(ep, tok, n, apply_act(v, ep.act));
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
      if (S > 1) {
        // Last CTA to finish this tile reduces the partials in split order.
        __threadfence();
        named_bar_sync(1, 128);
        if (et == 0) {
          const unsigned int old = atomicAdd(&a.counters[nt * num_t + tt], 1u);
          const int last = old == static_cast<unsigned int>(S - 1);
          if (last) a.counters[nt * num_t + tt] = 0u;
          *last_flag = last;
        }
        named_bar_sync(1, 128);
        const bool last = *last_flag != 0;
        named_bar_sync(1, 128);  // everyone has read last_flag before it is rewritten
        if (last && n_ok && valid) {
          __threadfence();
          const int tmax = min(BT, a.M - tt * BT);
          for (int j = 0; j < tmax; ++j) {
            const int tok = tt * BT + j;
            float v = 0.0f;
            for (int s2 = 0; s2 < S; ++s2)
              v = __fadd_rn(v, __ldcg(a.partial + (static_cast<int64_t>(s2) * a.M + tok) * a.N + n));
            if (ep.extra_scale) v = __fmul_rn(v, xs);
            if (ep.bias_dtype != kBiasNone) v = __fadd_rn(v, bias_v);
            store_out(ep, tok, n, apply_act(v, ep.act));
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem_base, L::kTmemCols);
}

// SIMT fallback (K % 16 != 0 or unaligned operands): one thread per output
// element block, fp32 accumulation over exactly decoded weights.
template <typename XT>
__global__ void __launch_bounds__(256)
    w8a16_simt_kernel(const XT* __restrict__ X, int64_t ldx, const uint8_t* __restrict__ W,
                      int64_t ldw, int M, int N, int K, EpiArgs ep) {
  constexpr int T = 32, TK = 32;
  __shared__ float sx[TK][T + 1];
  __shared__ float sw[TK][T + 1];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  const int m0 = blockIdx.y * T, n0 = blockIdx.x * T;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k0 = 0; k0 < K; k0 += TK) {
    for (int i = threadIdx.x; i < T * TK; i += 256) {
      const int r = i / TK, k = i % TK;
      const int gm = m0 + r, gn = n0 + r, gk = k0 + k;
      sx[k][r] = (gm < M && gk < K) ? to_float<XT>(X[static_cast<int64_t>(gm) * ldx + gk]) : 0.0f;
      sw[k][r] = (gn < N && gk < K) ? decode_e4m3(W[static_cast<int64_t>(gn) * ldw + gk]) : 0.0f;
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < TK; ++k) {
      const float w = sw[k][tx];
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] = fmaf(sx[k][ty + 8 * i], w, acc[i]);
    }
    __syncthreads();
  }
  const float xs = ep.extra_scale ? *ep.extra_scale : 1.0f;
  const int n = n0 + tx;
  if (n >= N) return;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty + 8 * i;
    if (m >= M) continue;
    float v = ep.extra_scale ? __fmul_rn(acc[i], xs) : acc[i];
    if (ep.bias_dtype != kBiasNone) v = __fadd_rn(v, load_bias(ep.bias, ep.bias_dtype, n));
    store_out(ep, m, n, apply_act(v, ep.act));
  }
}

}  // namespace b200q
