// Activation quantization fused into the 8-bit GEMM launch ("quant prologue").
//
// The unfused route is two launches: quantize X [M,K] (bf16/fp16) into codes,
// then the GEMM over the codes.  The fused route is one GEMM launch that also
// does the quantization, overlapped with the tensor-core work instead of in
// front of it:
//
//  * Rows are quantized by warps 2 and 3 of every CTA, which have no other
//    work after setup.  A warp claims the next row from a global counter (rows
//    are claimed in increasing order, which is the order the tile raster needs
//    the 128-row bands in), quantizes it, and counts it into its band's
//    done-counter.  The row data reach the warp through a ring of shared-memory
//    slots filled by cp.async.bulk (pro_ring_worker): two warps per SM cannot
//    keep enough plain loads in flight to feed the tensor cores' appetite.
//  * The TMA producer, before loading the A tile of a band it has not used
//    yet, waits (bounded) until that band's counter reaches the band's row count.
//  * Nobody who quantizes ever waits on anything, so progress needs no
//    co-residency of the grid (no grid barrier anywhere).
//
// Modes:
//  * kProInt8Row: per-token int8, the same arithmetic as quant_rowwise_i8
//    (bit-exact to the reference's rowwise quant, int8_gemm.mm:1337-1381), the
//    row scales go to `scales[M]` and feed the epilogue's row scale.
//  * kProFp8Tensor: per-tensor e4m3 with the amax already reduced into
//    sync[kSyncAmax] by an absmax launch earlier on the stream;
//    scale = max(amax / 448, 1e-30) is written to scales[0].
//
// Memory ordering: the codes are written by generic-proxy stores and read by
// TMA (async proxy) in other CTAs.  Writer: stores; fence.proxy.async.global;
// __syncwarp; lane 0: __threadfence + atomicAdd on the band counter (release).
// Reader: ld.acquire.gpu of the counter; fence.proxy.async.global; TMA.
// The epilogue reads row scales after its own acquire of the band counter.
//
// `sync` (uint32 words): [0] row-claim counter, [1] CTA-exit counter,
// [2] amax bits (fp8 mode), [3] unused, [4 + b] rows done in band b.
// It must be zero before the first launch; the last CTA to exit zeroes it again,
// so back-to-back launches (and CUDA-graph replays) on one stream can share it.
#pragma once

#include "numerics.cuh"
#include "ptx.cuh"
#include "quant.cuh"

namespace b200q {

enum PrologueMode : int { kProNone = 0, kProInt8Row = 1, kProFp8Tensor = 2 };

constexpr int kSyncClaim = 0;
constexpr int kSyncExit = 1;
constexpr int kSyncAmax = 2;
constexpr int kSyncBands = 4;
constexpr int kBandRows = 128;

struct Prologue {
  const void* x;       // [M, K] bf16 / fp16, row stride ldx elements
  int64_t ldx;
  uint8_t* q;          // [M, K] codes, row stride K (the GEMM's A operand)
  float* scales;       // [M] per-token scales (int8) or [1] per-tensor scale (fp8)
  unsigned int* sync;  // see the header comment
  int x_f16;           // 1 = fp16 input, 0 = bf16
  int nbands;          // band counters to clear at exit
  int ring;            // 1 = bulk-copy quantizer (pro_ring_worker), 0 = register path (pro_worker)
};

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const unsigned int* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Warp-uniform row claim; -1 once every row has been handed out.
__device__ __forceinline__ int pro_claim(const Prologue& p, int M) {
  unsigned int row = 0;
  if ((threadIdx.x & 31) == 0) row = atomicAdd(&p.sync[kSyncClaim], 1u);
  row = __shfl_sync(0xffffffffu, row, 0);
  return row < static_cast<unsigned int>(M) ? static_cast<int>(row) : -1;
}

// Register-path quantizers (pro_worker: inputs the bulk-copy ring cannot take,
// i.e. rows that are not 16-byte aligned).  One warp, one row, int8 per token:
// up to kRowRegs 16-byte vectors per lane stay in registers between the absmax
// and the quantize pass; the rest of a longer row is read again (from L2).
template <typename T>
__device__ __forceinline__ void quant_row_i8_warp(const T* __restrict__ xr, int K,
                                                  int8_t* __restrict__ qr, float* scale_out,
                                                  int lane) {
  constexpr int kRowRegs = 4;
  const bool vec = (K % 8 == 0) && ((reinterpret_cast<uintptr_t>(xr) & 15) == 0);
  float amax = 0.0f;
  if (vec) {
    const int nvec = K >> 3;
    const uint4* xv = reinterpret_cast<const uint4*>(xr);
    uint4 v[kRowRegs];
#pragma unroll
    for (int i = 0; i < kRowRegs; ++i) {
      const int idx = lane + 32 * i;
      if (idx < nvec) {
        v[i] = __ldcs(xv + idx);
        amax = fmaxf(amax, absmax8<T>(v[i]));
      }
    }
#pragma unroll 4
    for (int idx = lane + 32 * kRowRegs; idx < nvec; idx += 32) amax = fmaxf(amax, absmax8<T>(xv[idx]));
    amax = warp_max(amax);
    const float sc = fmaxf(__fdiv_rn(amax, 127.0f), 1e-30f);
    float s = round_to<T>(sc);
    if (s == 0.0f) s = smallest_normal<T>();
    const float r = __frcp_rn(s);
    if (lane == 0) *scale_out = sc;
    uint2* qv = reinterpret_cast<uint2*>(qr);
#pragma unroll
    for (int i = 0; i < kRowRegs; ++i) {
      const int idx = lane + 32 * i;
      if (idx < nvec) qv[idx] = quant8_fast<T>(v[i], s, r);
    }
#pragma unroll 4
    for (int idx = lane + 32 * kRowRegs; idx < nvec; idx += 32) qv[idx] = quant8_fast<T>(__ldcs(xv + idx), s, r);
  } else {
    for (int i = lane; i < K; i += 32) amax = fmaxf(amax, fabsf(to_float<T>(xr[i])));
    amax = warp_max(amax);
    const float sc = fmaxf(__fdiv_rn(amax, 127.0f), 1e-30f);
    float s = round_to<T>(sc);
    if (s == 0.0f) s = smallest_normal<T>();
    if (lane == 0) *scale_out = sc;
    for (int i = lane; i < K; i += 32) qr[i] = static_cast<int8_t>(quant_code<T>(to_float<T>(xr[i]), s));
  }
}

// One warp, one row, e4m3 with the per-tensor scale s (r = RN(1/s)).
template <typename T>
__device__ __forceinline__ void quant_row_fp8_warp(const T* __restrict__ xr, int K,
                                                   uint8_t* __restrict__ qr, float s, float r,
                                                   int lane) {
  if ((K % 8 == 0) && ((reinterpret_cast<uintptr_t>(xr) & 15) == 0)) {
    const int nvec = K >> 3;
    const uint4* xv = reinterpret_cast<const uint4*>(xr);
    uint2* qv = reinterpret_cast<uint2*>(qr);
#pragma unroll 4
    for (int idx = lane; idx < nvec; idx += 32) qv[idx] = fp8_quant8_fast<T>(__ldcs(xv + idx), s, r);
  } else {
    for (int i = lane; i < K; i += 32) qr[i] = encode_e4m3_sat(__fdiv_rn(to_float<T>(xr[i]), s));
  }
}

// Quantizes row `row` with the calling warp and publishes it to its band
// (register path).  Kept out of line: it is the rarely used fallback.
template <int MODE>
__device__ __noinline__ void pro_quant_row(const Prologue& p, int row, int K, float fp8_s) {
  const int lane = threadIdx.x & 31;
  const int64_t xo = static_cast<int64_t>(row) * p.ldx;
  uint8_t* qr = p.q + static_cast<int64_t>(row) * K;
  if constexpr (MODE == kProInt8Row) {
    if (p.x_f16)
      quant_row_i8_warp<__half>(static_cast<const __half*>(p.x) + xo, K, reinterpret_cast<int8_t*>(qr),
                                p.scales + row, lane);
    else
      quant_row_i8_warp<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(p.x) + xo, K,
                                       reinterpret_cast<int8_t*>(qr), p.scales + row, lane);
  } else {
    if (p.x_f16)
      quant_row_fp8_warp<__half>(static_cast<const __half*>(p.x) + xo, K, qr, fp8_s, __frcp_rn(fp8_s), lane);
    else
      quant_row_fp8_warp<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(p.x) + xo, K, qr, fp8_s,
                                        __frcp_rn(fp8_s), lane);
  }
  fence_proxy_async_global();
  __syncwarp();
  if (lane == 0) {
    __threadfence();
    atomicAdd(&p.sync[kSyncBands + row / kBandRows], 1u);
  }
}

// Claims and quantizes rows until none are left (dedicated quantizer warps).
template <int MODE>
__device__ __forceinline__ void pro_worker(const Prologue& p, int M, int K, float fp8_s) {
  while (true) {
    const int row = pro_claim(p, M);
    if (row < 0) return;
    pro_quant_row<MODE>(p, row, K, fp8_s);
  }
}

// ---------------------------------------------------------------------------
// Bulk-copy quantizer.  Each quantizer warp owns a ring of kQSlots shared-memory
// slots of kQSlotBytes; its lane 0 streams row segments into the ring with
// cp.async.bulk (so one warp keeps kQSlots x kQSlotBytes of activation in
// flight without spending registers on it) and the whole warp converts from
// shared memory.  Work is a sequence of units: for fp8 the segments of each
// claimed row; for int8 the segments twice (absmax pass, then quantize pass,
// the second read served by L2).  Units are consumed in issue order, so a row's
// absmax is complete before its quantize units.  Needs K % 8 == 0, ldx % 8 == 0
// and a 16-byte-aligned x (the host checks; otherwise pro_worker is used).
constexpr int kQWarps = 2;         // warps 2 and 3
constexpr int kQSlots = 4;
constexpr int kQSlotBytes = 4096;  // 2048 bf16 / fp16 elements
constexpr int kQSmemBytes = kQWarps * kQSlots * (kQSlotBytes + 8);

struct QuantSeg {
  int nseg, seg;  // segments per row, elements per segment (multiple of 8)
};

__device__ __forceinline__ QuantSeg quant_segments(int K) {
  QuantSeg g;
  g.nseg = (K * 2 + kQSlotBytes - 1) / kQSlotBytes;
  g.seg = ((K + g.nseg - 1) / g.nseg + 7) & ~7;
  return g;
}

template <int MODE, typename T>
__device__ __forceinline__ void pro_ring_worker(const Prologue& p, int M, int K, float fp8_s,
                                                uint8_t* ring, uint64_t* full, volatile int* abort) {
  const int lane = threadIdx.x & 31;
  const QuantSeg g = quant_segments(K);
  const int units_per_row = MODE == kProInt8Row ? 2 * g.nseg : g.nseg;
  const T* x = static_cast<const T*>(p.x);
  // Issue side (warp-uniform): the row being issued and the next unit in it.
  int i_row = -1, i_k = 0;
  bool i_done = false;
  // Descriptor of the unit in each slot (row < 0: empty) and the slot parities.
  int d_row[kQSlots], d_k[kQSlots];
  uint32_t parity = 0u;
  // Consume side: the current row's scale (int8).
  float amax = 0.0f, s = 1.0f, r = 1.0f;
  if constexpr (MODE == kProFp8Tensor) {
    s = fp8_s;
    r = __frcp_rn(fp8_s);
  }

  auto issue = [&](int sl) {
    if (!i_done && i_row < 0) {
      i_row = pro_claim(p, M);
      i_k = 0;
      if (i_row < 0) i_done = true;
    }
    if (i_done) {
      d_row[sl] = -1;
      return;
    }
    const int sg = i_k % g.nseg;
    const int e0 = sg * g.seg;
    const int ne = min(g.seg, K - e0);
    if (lane == 0) {
      fence_proxy_async_smem();  // this slot's previous generic reads before the async write
      mbar_arrive_expect_tx(&full[sl], static_cast<uint32_t>(ne) * 2u);
      bulk_load(ring + sl * kQSlotBytes, x + static_cast<int64_t>(i_row) * p.ldx + e0,
                static_cast<uint32_t>(ne) * 2u, &full[sl]);
    }
    d_row[sl] = i_row;
    d_k[sl] = i_k;
    if (++i_k == units_per_row) i_row = -1;
  };

#pragma unroll
  for (int sl = 0; sl < kQSlots; ++sl) issue(sl);

  bool failed = false;
  while (!failed) {
    bool any = false;
#pragma unroll
    for (int sl = 0; sl < kQSlots; ++sl) {
      if (d_row[sl] < 0 || failed) continue;
      any = true;
      const uint32_t ph = (parity >> sl) & 1u;
      if (!__all_sync(0xffffffffu, mbar_wait(&full[sl], ph, abort))) {
        failed = true;
        continue;
      }
      parity ^= 1u << sl;
      const int row = d_row[sl], k = d_k[sl];
      const bool absmax_pass = MODE == kProInt8Row && k < g.nseg;
      const int sg = k % g.nseg;
      const int e0 = sg * g.seg;
      const int nvec = min(g.seg, K - e0) >> 3;
      const uint4* sv = reinterpret_cast<const uint4*>(ring + sl * kQSlotBytes);
      if (absmax_pass) {
        for (int i = lane; i < nvec; i += 32) amax = fmaxf(amax, absmax8<T>(sv[i]));
        if (sg == g.nseg - 1) {
          amax = warp_max(amax);
          const float sc = fmaxf(__fdiv_rn(amax, 127.0f), 1e-30f);
          s = round_to<T>(sc);
          if (s == 0.0f) s = smallest_normal<T>();
          r = __frcp_rn(s);
          if (lane == 0) p.scales[row] = sc;
          amax = 0.0f;
        }
      } else {
        uint2* qv = reinterpret_cast<uint2*>(p.q + static_cast<int64_t>(row) * K + e0);
        for (int i = lane; i < nvec; i += 32)
          qv[i] = MODE == kProInt8Row ? quant8_fast<T>(sv[i], s, r) : fp8_quant8_fast<T>(sv[i], s, r);
        if (sg == g.nseg - 1) {  // the row is complete: publish it to its band
          fence_proxy_async_global();
          __syncwarp();
          if (lane == 0) {
            __threadfence();
            atomicAdd(&p.sync[kSyncBands + row / kBandRows], 1u);
          }
        }
      }
      __syncwarp();
      issue(sl);
    }
    if (!any) break;
  }
  if (failed) {
    // Let this warp's own copies land before the CTA's shared memory is reused.
#pragma unroll
    for (int sl = 0; sl < kQSlots; ++sl)
      if (d_row[sl] >= 0 && lane == 0) mbar_wait_drain(&full[sl], (parity >> sl) & 1u);
    __syncwarp();
  }
}

// Waits (bounded) until every row of `band` has been quantized and published;
// afterwards this thread's TMA loads and plain loads see the band's codes and
// scales.  Returns false on timeout/abort.
__device__ __forceinline__ bool pro_band_wait(const Prologue& p, int band, int M, volatile int* abort) {
  const int need = min(kBandRows, M - band * kBandRows);
  if (need <= 0) return true;
  const unsigned int* f = p.sync + kSyncBands + band;
  if (ld_acquire_gpu(f) < static_cast<unsigned int>(need)) {
    const unsigned long long t0 = globaltimer_ns();
    uint32_t polls = 0;
    while (ld_acquire_gpu(f) < static_cast<unsigned int>(need)) {
      __nanosleep(32);
      if ((++polls & 63u) == 0u) {
        if (*abort) return false;
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
          atomicOr(&g_device_status, kStatusWaitTimeout);
          *abort = 1;
          return false;
        }
      }
    }
  }
  fence_proxy_async_global();
  return true;
}

// Per-tensor e4m3 scale from the amax reduced before this launch.
__device__ __forceinline__ float pro_fp8_scale(const Prologue& p) {
  return fp8_scale_from_amax(__ldcg(p.sync + kSyncAmax));
}

// Called by every thread of the CTA after all of its work (and after its last
// block-wide barrier): the last CTA of the grid to get here zeroes `sync`.
__device__ __forceinline__ void pro_exit(const Prologue& p, int* smem_flag) {
  if (threadIdx.x == 0) {
    __threadfence();
    *smem_flag = atomicAdd(&p.sync[kSyncExit], 1u) == gridDim.x - 1 ? 1 : 0;
    __threadfence();
  }
  __syncthreads();
  if (*smem_flag) {
    for (int i = threadIdx.x; i < p.nbands; i += blockDim.x) p.sync[kSyncBands + i] = 0u;
    if (threadIdx.x == 0) {
      p.sync[kSyncClaim] = 0u;
      p.sync[kSyncAmax] = 0u;
      p.sync[kSyncExit] = 0u;
    }
  }
}

}  // namespace b200q
