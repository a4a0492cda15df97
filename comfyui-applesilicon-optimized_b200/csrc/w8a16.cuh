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

constexpr int kW16MaxSplits = 8;

// Split-K fix-up run by the last CTA to finish a tile: sums the fp32 partials of
// tokens [t0, t0 + tcount) for output feature n in split order 0, 1, ... (fixed,
// so the result is bit-reproducible) and applies the epilogue.  Four tokens x up
// to kW16MaxSplits splits are loaded together so the L2 latencies overlap.
__device__ __forceinline__ void splitk_reduce_store(const W8A16Args& a, const EpiArgs& ep, int t0,
                                                    int tcount, int n, float xs, float bias_v) {
  const int64_t split_stride = static_cast<int64_t>(a.M) * a.N;
  const float* base = a.partial + static_cast<int64_t>(t0) * a.N + n;
  for (int j0 = 0; j0 < tcount; j0 += 4) {
    float p[kW16MaxSplits][4];
#pragma unroll
    for (int s2 = 0; s2 < kW16MaxSplits; ++s2)
#pragma unroll
      for (int jj = 0; jj < 4; ++jj)
        p[s2][jj] = (s2 < a.splits && j0 + jj < tcount)
                        ? __ldcg(base + s2 * split_stride + static_cast<int64_t>(j0 + jj) * a.N)
                        : 0.0f;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      if (j0 + jj >= tcount) break;
      float v = 0.0f;
#pragma unroll
      for (int s2 = 0; s2 < kW16MaxSplits; ++s2)
        if (s2 < a.splits) v = __fadd_rn(v, p[s2][jj]);
      if (ep.extra_scale) v = __fmul_rn(v, xs);
      if (ep.bias_dtype != kBiasNone) v = __fadd_rn(v, bias_v);
      store_out(ep, t0 + j0 + jj, n, apply_act(v, ep.act));
    }
  }
}

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
          splitk_reduce_store(a, ep, tt * BT, min(BT, a.M - tt * BT), n, xs, bias_v);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem_base, L::kTmemCols);
}

// ---------------------------------------------------------------------------
// Streaming variant for small token counts (BT <= 64), where the call is bound by
// the FP8 weight stream from HBM.  The dequantized weight tile never touches
// shared memory: converters read the raw e4m3 tile, convert to bf16 in registers
// and tcgen05.st it into a TMEM buffer, and the MMA takes its A operand from TMEM
// (tcgen05.mma ... [a_tmem], b_desc).  Shared-memory traffic per 16 KB weight
// block is then ~40 KB (TMA write + one read of the raw tile, the activation
// tile) instead of ~110 KB for a shared-memory converted operand -- on B200 the
// latter saturated the 128 B/clk shared-memory port before HBM.
//   W ring   RS slots x (128 rows x 128 B e4m3, 128B swizzle -> conflict-free reads)
//   X ring   RX slots x (BT x 128 bf16 as two 128B-swizzle atoms), read by the MMA
//   A ring   4 TMEM buffers x 64 columns (128 rows x 128 bf16)
//   warp 0   weight producer            warp 3   activation producer
//   warps 4..11 converters: warp w owns TMEM lane quarter w % 4 (the rows it may
//            access) and half of the block's K; one thread per weight row
//   warp 1   MMA: 8 x kind::f16 (bf16 x bf16 -> fp32), K=16 each, A from TMEM,
//            into one accumulator (back-to-back 128 x 16 x 16 MMAs on one
//            accumulator run at the tensor pipe's ~27 ns each, measured)
//   warps 12..15 epilogue (split-K protocol as in w8a16_tc_kernel)
constexpr int kWsBK = 128;
constexpr int kWsThreads = 512;
constexpr int kWsConv = 256;
constexpr int kWsSB = 2 * kWsBK;    // K per converter -> MMA handoff ("step": two blocks)
constexpr int kWsACols = kWsSB / 2;  // 256 bf16 per row = 128 32-bit columns

template <int BT>
struct W8A16StreamLayout {
  static constexpr int kRawSlot = kW16BM * kWsBK;        // 16 KB e4m3
  static constexpr int kXSlot = BT * kWsSB * 2;          // bf16 activations of one step (four atoms)
  static constexpr int kXSlots = BT <= 16 ? 4 : BT <= 32 ? 3 : 2;
  static constexpr int kFree = 204 * 1024 - kXSlots * kXSlot;
  static constexpr int kRawSlots = kFree / kRawSlot > 10 ? 10 : kFree / kRawSlot;
  static constexpr int kXOff = 0;
  static constexpr int kRawOff = kXSlots * kXSlot;
  static constexpr int kBarOff = kRawOff + kRawSlots * kRawSlot;
  // wfull/wempty[RS], xfull/xempty[RX], afull/aempty[4], acc_full/acc_empty[2], slot, abort, last
  // TMEM: double-buffered accumulators (2 x BT columns), then as many A buffers
  // of one step (128 columns) as fit in the 512 columns.
  static constexpr int kABufs = (512 - 2 * BT) / 128 > 3 ? 3 : (512 - 2 * BT) / 128;
  static constexpr int kBarBytes = (2 * kRawSlots + 2 * kXSlots + 2 * kABufs + 4) * 8 + 16;
  static constexpr int kSmemBytes = kBarOff + kBarBytes + 1024;
  static constexpr int kNacc = 1;
  static constexpr uint32_t kAccCols = 2 * kNacc * BT;
  static constexpr uint32_t kTmemCols = 512;  // accumulators + kABufs x 128 A columns
};

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
      "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]),
      "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]),
      "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// D(tmem) (+)= A(tmem) x B(smem desc)^T, kind::f16, one thread.
__device__ __forceinline__ void umma_ts_f16(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

template <int BT, bool X_F16>
__global__ void __launch_bounds__(kWsThreads, 1)
    w8a16_stream_kernel(const __grid_constant__ CUtensorMap tmX,
                        const __grid_constant__ CUtensorMap tmW, W8A16Args a, EpiArgs ep) {
  using L = W8A16StreamLayout<BT>;
  constexpr int RS = L::kRawSlots;
  constexpr int RX = L::kXSlots;
  constexpr int AB = L::kABufs;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sX = smem + L::kXOff;
  uint8_t* sW = smem + L::kRawOff;
  uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* wempty = wfull + RS;
  uint64_t* xfull = wempty + RS;
  uint64_t* xempty = xfull + RX;
  uint64_t* afull = xempty + RX;
  uint64_t* aempty = afull + AB;
  uint64_t* acc_full = aempty + AB;
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
  const int num_kb = (a.K + kWsBK - 1) / kWsBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < RS; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], kWsConv);
    }
    for (int s = 0; s < RX; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
    }
    for (int s = 0; s < AB; ++s) {
      mbar_init(&afull[s], kWsConv);
      mbar_init(&aempty[s], 1);
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
  const uint32_t tmem_a0 = tmem_base + L::kAccCols;  // A buffers follow the accumulators

  if (warp == 0) {
    // ------------------------------------------------------------ weight producer
    if (lane == 0) {
      int rs = 0;
      uint32_t rph = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        int nt, tt, sp;
        w16_unit_coords(u, S, num_t, nt, tt, sp);
        const int kb0 = sp * num_kb / S, kb1 = (sp + 1) * num_kb / S;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&wempty[rs], rph ^ 1u, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&wfull[rs], L::kRawSlot);
          tma_load_2d(&tmW, &wfull[rs], sW + rs * L::kRawSlot, kb * kWsBK, nt * kW16BM);
          if (++rs == RS) { rs = 0; rph ^= 1u; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 3) {
    // ------------------------------------------------------------ activation producer
    if (lane == 0) {
      int xs = 0;
      uint32_t xph = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        int nt, tt, sp;
        w16_unit_coords(u, S, num_t, nt, tt, sp);
        const int kb0 = sp * num_kb / S, kb1 = (sp + 1) * num_kb / S;
        for (int kb = kb0; kb < kb1; kb += 2) {
          const int nblk = min(2, kb1 - kb);  // 128-K blocks in this step
          if (!mbar_wait(&xempty[xs], xph ^ 1u, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&xfull[xs], static_cast<uint32_t>(nblk) * (L::kXSlot / 2));
          uint8_t* dst = sX + xs * L::kXSlot;
          for (int at = 0; at < 2 * nblk; ++at)  // 64-K swizzle atoms of BT rows
            tma_load_2d(&tmX, &xfull[xs], dst + at * (L::kXSlot / 4), kb * kWsBK + at * 64, tt * BT);
          if (++xs == RX) { xs = 0; xph ^= 1u; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      // f32 <- bf16 x bf16 (or fp16 x fp16), M=128, N=BT, both K-major.
      constexpr uint32_t kIdesc = X_F16 ? make_idesc(1, 0, 0, kW16BM, BT) : make_idesc(1, 1, 1, kW16BM, BT);
      int ab = 0, xs = 0;
      uint32_t aph = 0, xph = 0;
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
        const uint32_t d_tmem = tmem_base + buf * L::kNacc * BT;
        uint32_t acc = 0u;  // 0 for the unit's first MMA (overwrite), then accumulate
        for (int kb = kb0; kb < kb1; kb += 2) {
          const int nblk = min(2, kb1 - kb);
          if (!mbar_wait(&afull[ab], aph, abort_flag)) { ok = false; break; }
          if (!mbar_wait(&xfull[xs], xph, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_tmem = tmem_a0 + ab * kWsACols;
          for (int atom = 0; atom < 2 * nblk; ++atom) {
            const uint64_t bdesc = make_sw128_desc(smem_u32(sX + xs * L::kXSlot + atom * (L::kXSlot / 4)));
#pragma unroll
            for (int k = 0; k < 4; ++k) {  // K=16 per MMA = 8 TMEM columns of A, +32 B of B
              umma_ts_f16(d_tmem, a_tmem + (atom * 4 + k) * 8, bdesc + 2 * k, kIdesc, acc);
              acc = 1u;
            }
          }
          umma_commit(&aempty[ab]);
          umma_commit(&xempty[xs]);
          if (++ab == AB) { ab = 0; aph ^= 1u; }
          if (++xs == RX) { xs = 0; xph ^= 1u; }
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
    }
    __syncwarp();
  } else if (warp >= 4 && warp < 12) {
    // ------------------------------------------------------------ converters
    // Thread = weight row (TMEM lane q*32 + lane); `half` picks K 0..63 or 64..127.
    const int q = warp & 3;
    const int half = (warp - 4) >> 2;
    const int r = q * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    int rs = 0, ab = 0;
    uint32_t rph = 0, aph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
      int nt, tt, sp;
      w16_unit_coords(u, S, num_t, nt, tt, sp);
      const int kb0 = sp * num_kb / S, kb1 = (sp + 1) * num_kb / S;
      for (int kb = kb0; kb < kb1; kb += 2) {
        const int nblk = min(2, kb1 - kb);
        if (!mbar_wait_warp(&aempty[ab], aph ^ 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        for (int b = 0; b < nblk; ++b) {
          if (!mbar_wait_warp(&wfull[rs], rph, abort_flag)) { ok = false; break; }
          // Row r's 64 bytes: 16-byte chunks c = half*4 .. half*4+3, stored at chunk
          // position c ^ (r & 7) by the 128-byte TMA swizzle.
          const uint8_t* row = sW + rs * L::kRawSlot + r * kWsBK;
          uint32_t v[32];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int c = half * 4 + j;
            const uint4 w = *reinterpret_cast<const uint4*>(row + ((c ^ (r & 7)) << 4));
            const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              if constexpr (X_F16) {
                v[j * 8 + 2 * k] = e4m3x2_to_f16x2(static_cast<uint16_t>(wd[k] & 0xFFFFu));
                v[j * 8 + 2 * k + 1] = e4m3x2_to_f16x2(static_cast<uint16_t>(wd[k] >> 16));
              } else {
                v[j * 8 + 2 * k] = e4m3x2_to_bf16x2(static_cast<uint16_t>(wd[k] & 0xFFFFu));
                v[j * 8 + 2 * k + 1] = e4m3x2_to_bf16x2(static_cast<uint16_t>(wd[k] >> 16));
              }
            }
          }
          tmem_st32(tmem_a0 + lane_off + ab * kWsACols + b * (kWsBK / 2) + half * 32, v);
          mbar_arrive(&wempty[rs]);  // the raw slot's bytes are in registers / in flight to TMEM
          if (++rs == RS) { rs = 0; rph ^= 1u; }
        }
        if (!ok) break;
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&afull[ab]);
        if (++ab == AB) { ab = 0; aph ^= 1u; }
      }
    }
  } else if (warp >= 12) {
    // ------------------------------------------------------------ epilogue
    constexpr int CH = BT < 32 ? BT : 32;
    const int q = warp & 3;
    const int et = threadIdx.x - 384;
    const float xs = ep.extra_scale ? __ldg(ep.extra_scale) : 1.0f;
    int it = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++it) {
      int nt, tt, sp;
      w16_unit_coords(u, S, num_t, nt, tt, sp);
      const int buf = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      const bool valid = mbar_wait_warp(&acc_full[buf], acc_phase, abort_flag);
      tc_fence_after();
      const int n = nt * kW16BM + q * 32 + lane;
      const bool n_ok = n < a.N;
      const float bias_v = (n_ok && ep.bias_dtype != kBiasNone) ? load_bias(ep.bias, ep.bias_dtype, n) : 0.0f;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * L::kNacc * BT;
#pragma unroll 1
      for (int c = 0; valid && c < BT / CH; ++c) {
        uint32_t rr[CH];
        tmem_ld_cols<CH>(taddr + c * CH, rr);
        tmem_ld_wait();
#pragma unroll
        for (int j2 = 1; j2 < L::kNacc; ++j2) {  // fixed-order sum of the accumulators
          uint32_t r2[CH];
          tmem_ld_cols<CH>(taddr + j2 * BT + c * CH, r2);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < CH; ++j) rr[j] = __float_as_uint(__fadd_rn(__uint_as_float(rr[j]), __uint_as_float(r2[j])));
        }
        const int t0 = tt * BT + c * CH;
        if (n_ok) {
#pragma unroll
          for (int j = 0; j < CH; ++j) {
            const int tok = t0 + j;
            if (tok < a.M) {
              const float acc = __uint_as_float(rr[j]);
              if (S > 1) {
                a.partial[(static_cast<int64_t>(sp) * a.M + tok) * a.N + n] = acc;
              } else {
                float vv = ep.extra_scale ? __fmul_rn(acc, xs) : acc;
                if (ep.bias_dtype != kBiasNone) vv = __fadd_rn(vv, bias_v);
                store_out(ep, tok, n, apply_act(vv, ep.act));
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
      if (S > 1) {
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
        named_bar_sync(1, 128);
        if (last && n_ok && valid) {
          __threadfence();
          splitk_reduce_store(a, ep, tt * BT, min(BT, a.M - tt * BT), n, xs, bias_v);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem_base, L::kTmemCols);
}

// ---------------------------------------------------------------------------
// Weight-streaming GEMV for M <= 32 tokens: the HBM-bound regime, where every
// SM must pull its share of the FP8 weight (~44 GB/s per SM on B200) and the
// arithmetic is tiny.  A 128-row tcgen05 tile fed by one issuing thread cannot
// keep that pace at N = 16 tokens (a 2 KB weight step per MMA plus its
// barrier hand-offs, measured ~25 GB/s per SM), so here every warp converts
// e4m3 -> bf16/fp16 in registers and multiplies with warp-level m16n8k16 MMAs
// (fp32 accumulation), while TMA keeps the weight stream in flight.
//
// CTA = 8 warps on 32 weight rows (4 groups of 8), three CTAs per SM.  One
// thread streams the rows' K in stages of 512 bytes (4 TMA boxes of 32 rows x
// 128 B, 128-byte swizzle) through a kGvStages-deep shared-memory ring; in each
// stage warp w takes K [64w, 64w + 64).  The warps' partial sums are reduced
// through shared memory in warp order (deterministic).  Within a warp's 64-K
// slice, lane (g = lane/4, q = lane%4) reads W[row g of a group][16q .. 16q+15];
// byte 4t+j of that vector feeds MMA t (t = 0..3) at logical k = 2q + (j & 1)
// + 8 (j >> 1).  The activation operand uses the same per-lane permutation of K
// (X[m][16q + 4t + j], read from global memory through L1, one stage ahead), so
// the dot product is unchanged and no shuffles are needed.
// Measured alternatives that were slower on B200 (C2, 12288 x 3072): one
// persistent CTA per SM with a 12-16 stage ring (24.6 us per call vs 18.4 us),
// the same with 16 warps (22.5 us); the 3-CTA form keeps more warps resident to
// hide the activation loads and the per-warp MMA chain.
constexpr int kGvRows = 32;
constexpr int kGvWarps = 8;
constexpr int kGvThreads = kGvWarps * 32;
constexpr int kGvStageK = 64 * kGvWarps;              // 512 K bytes per stage
constexpr int kGvStageBytes = kGvRows * kGvStageK;    // 16 KB
constexpr int kGvStages = 3;
constexpr int kGvSmemBytes = kGvStages * kGvStageBytes + 2 * kGvStages * 8 + 16 + 1024;

__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1, bool f16) {
  if (f16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// MT = 16-token tiles (1: M <= 16, 2: M <= 32).  Requires K % 16 == 0, ldx % 8 == 0
// and a 16-byte-aligned X (the host checks; W goes through the tensor map).
template <int MT, bool X_F16>
__global__ void __launch_bounds__(kGvThreads, MT == 1 ? 3 : 2)
    w8a16_gemv_kernel(const __grid_constant__ CUtensorMap tmW, const uint16_t* __restrict__ X,
                      int64_t ldx, int M, int N, int K, EpiArgs ep) {
  __shared__ float red[kGvWarps][MT * 16][kGvRows + 1];
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
  // Launched as a programmatic dependent: the set-up above overlapped the kernel
  // before it; nothing in global memory is read before that kernel is done.
  // The next dependent may start its own set-up now (it waits for this grid).
  griddep_wait();
  griddep_launch_dependents();
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

  float acc[MT][4][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int gr = 0; gr < 4; ++gr)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[mt][gr][i] = 0.0f;
  // Activation rows of this lane: tokens g + 8h + 16mt; rows past M are zero.
  const uint16_t* xrow[MT][2];
  bool xok[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int m = 16 * mt + 8 * h + g;
      xok[mt][h] = m < M;
      xrow[mt][h] = X + static_cast<int64_t>(m < M ? m : 0) * ldx + 16 * q;
    }
  // Activation fragments are loaded one stage ahead, so their L2 round trip
  // overlaps the wait for the stage's weights.
  uint4 xa[MT][2][2], xn[MT][2][2];
  auto load_x = [&](int st, uint4 (&dst)[MT][2][2]) {
    const int k0 = st * kGvStageK + 64 * warp;
    const bool kin = st < nst && k0 + 16 * q < K;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int p = 0; p < 2; ++p)
          dst[mt][h][p] = (xok[mt][h] && kin)
                              ? __ldg(reinterpret_cast<const uint4*>(xrow[mt][h] + k0) + p)
                              : make_uint4(0u, 0u, 0u, 0u);
  };
  load_x(0, xn);
  // This warp's 16-byte chunk of each row inside the stage's box: box warp/2,
  // chunk (warp & 1) * 4 + q, stored at chunk ^ (row & 7) by the 128-byte swizzle.
  const int box = warp >> 1;
  const int chunk = (warp & 1) * 4 + q;

  bool ok = true;
  for (int st = 0; st < nst && ok; ++st) {
    const int slot = st % kGvStages;
    const uint32_t ph = (st / kGvStages) & 1u;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int p = 0; p < 2; ++p) xa[mt][h][p] = xn[mt][h][p];
    load_x(st + 1, xn);
    if (!mbar_wait_warp(&full[slot], ph, abort_flag)) { ok = false; break; }
    const int k0 = st * kGvStageK + 64 * warp;
    if (k0 < K) {
      const uint8_t* sb = ring + slot * kGvStageBytes + box * (kGvRows * 128);
      uint4 wv[4];
#pragma unroll
      for (int gr = 0; gr < 4; ++gr) {
        const int r = 8 * gr + g;
        wv[gr] = *reinterpret_cast<const uint4*>(sb + r * 128 + ((chunk ^ (r & 7)) << 4));
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        uint32_t a[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const uint32_t* r0 = reinterpret_cast<const uint32_t*>(&xa[mt][0][t >> 1]);
          const uint32_t* r1 = reinterpret_cast<const uint32_t*>(&xa[mt][1][t >> 1]);
          a[mt][0] = r0[(t & 1) * 2];
          a[mt][1] = r1[(t & 1) * 2];
          a[mt][2] = r0[(t & 1) * 2 + 1];
          a[mt][3] = r1[(t & 1) * 2 + 1];
        }
#pragma unroll
        for (int gr = 0; gr < 4; ++gr) {
          const uint32_t wd = (t == 0) ? wv[gr].x : (t == 1) ? wv[gr].y : (t == 2) ? wv[gr].z : wv[gr].w;
          const uint16_t lo = static_cast<uint16_t>(wd & 0xFFFFu), hi = static_cast<uint16_t>(wd >> 16);
          const uint32_t b0 = X_F16 ? e4m3x2_to_f16x2(lo) : e4m3x2_to_bf16x2(lo);
          const uint32_t b1 = X_F16 ? e4m3x2_to_f16x2(hi) : e4m3x2_to_bf16x2(hi);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) mma_16816(acc[mt][gr], a[mt], b0, b1, X_F16);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    if (threadIdx.x == 0 && st + kGvStages < nst) {
      // Refill this slot once every warp has released it.
      if (!mbar_wait(&empty[slot], ph, abort_flag)) { ok = false; break; }
      issue(st + kGvStages);
    }
  }
  if (!ok && threadIdx.x == 0) {
    // Let this CTA's in-flight stages land before its shared memory is released.
    for (int s2 = 0; s2 < kGvStages; ++s2) mbar_wait_drain(&full[s2], 0);
  }

  // D fragment: acc[mt][gr][i] is token 16mt + g + 8(i >> 1), row 8gr + 2q + (i & 1).
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int gr = 0; gr < 4; ++gr)
#pragma unroll
      for (int i = 0; i < 4; ++i)
        red[warp][16 * mt + g + 8 * (i >> 1)][8 * gr + 2 * q + (i & 1)] = acc[mt][gr][i];
  __syncthreads();
  if (*abort_flag) return;
  const float xs = ep.extra_scale ? __ldg(ep.extra_scale) : 1.0f;
  for (int e = threadIdx.x; e < MT * 16 * kGvRows; e += kGvThreads) {
    const int tok = e / kGvRows, r = e % kGvRows;
    const int n = n0 + r;
    if (tok >= M || n >= N) continue;
    float v = red[0][tok][r];
#pragma unroll
    for (int w2 = 1; w2 < kGvWarps; ++w2) v = __fadd_rn(v, red[w2][tok][r]);
    if (ep.extra_scale) v = __fmul_rn(v, xs);
    if (ep.bias_dtype != kBiasNone) v = __fadd_rn(v, load_bias(ep.bias, ep.bias_dtype, n));
    store_out(ep, tok, n, apply_act(v, ep.act));
  }
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
