// C ABI launch layer of the b200q kernels (declarations: include/b200q.h).
//
// Host-side responsibilities: validate every pointer/shape/stride before a
// launch, pick the tensor-core (TMA) path when the operands satisfy TMA's
// 16-byte rules and the SIMT path otherwise, encode the TMA descriptors, size
// persistent grids to the SM count, and launch on the caller's stream.  No
// device memory is allocated here and no call synchronises the device (except
// b200q_get_device_status, which exists to read the device status word).
#include <atomic>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/b200q.h"
#include "gemm8.cuh"
#include "qkv_rope.cuh"
#include "quant.cuh"
#include "w8a16.cuh"
#include "w8a16_planes.cuh"

using namespace b200q;

namespace {

std::atomic<uint64_t> g_launches{0};

struct DeviceInfo {
  bool init = false;
  bool sm100 = false;
  int num_sms = 0;
};
DeviceInfo g_dev[64];
std::mutex g_dev_mu;

// Returns nullptr if the current device cannot run sm_100a code.
const DeviceInfo* current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.init) {
    int major = 0, minor = 0, sms = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    d.sm100 = (major == 10 && minor == 0);
    d.num_sms = sms > 0 ? sms : 148;
    d.init = true;
  }
  return d.sm100 ? &d : nullptr;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// 2-D row-major tensor [rows, cols] with row stride `ld_bytes`; box = box_cols x box_rows.
bool make_tmap(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t cols,
               uint64_t rows, uint64_t ld_bytes, uint32_t box_cols, uint32_t box_rows,
               CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int finish_launch() {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    fprintf(stderr, "[b200q] launch failed: %s\n", cudaGetErrorString(e));
    return B200Q_ERR_CUDA;
  }
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return B200Q_OK;
}

template <typename Kern>
bool set_smem(Kern kern, int bytes) {
  // Idempotent and cheap; done per call so multi-device processes stay correct.
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) ==
         cudaSuccess;
}

bool valid_dims(int64_t M, int64_t N, int64_t K) {
  return M >= 0 && N >= 0 && K >= 0 && M < (int64_t(1) << 31) && N < (int64_t(1) << 31) &&
         K < (int64_t(1) << 31);
}

// Raster choice: when the weight is small enough to stay in L2 next to the
// streaming activations, sweep N fastest (A row panels are read from HBM once);
// otherwise walk groups of 16 M-tiles so concurrent tiles share both operands'
// panels.  The threshold is measured, not derived: B200's L2 is split between
// the two dies, and a 70-80 MB weight swept N-fastest was re-read 4-5x from HBM
// (C5 qkv/up/down), while <= 38 MB weights (C3, C4, C5 out-proj) gained.
// For the grouped order the group is at most 16 M-tiles and at most ~28 MB of
// A panels (256 rows x K bytes each), so the group's A stays in L2 while the
// weight streams past it: at K = 13,824 a 16-tile group (56 MB of A next to a
// 71 MB weight) re-read its A panels about 3x.  B200Q_GROUP_M overrides.
int raster_group_m(int64_t lda, int64_t ldw, int64_t M, int64_t N, int64_t K) {
  (void)M;
  static const int forced = [] {
    const char* e = getenv("B200Q_GROUP_M");
    return e ? atoi(e) : 0;
  }();
  if (forced > 0) return forced;
  const double w_bytes = double(N) * double(ldw);
  if (w_bytes <= 40.0 * 1024 * 1024) return 1;
  const double a_panel = 256.0 * double(lda > K ? lda : K);
  int g = kGemmGroupM;
  while (g > 4 && g * a_panel > 28.0 * 1024 * 1024) g >>= 1;
  return g;
}

// ------------------------------------------------------------ 8-bit GEMM dispatch
template <MmaKind KIND, int BN, int STAGES, int EPI, int PRO>
int launch_gemm8_tc(const DeviceInfo* d, const void* a, int64_t lda, const void* w, int64_t ldw,
                    int M, int N, int K, const EpiArgs& ep, const Prologue& pro, cudaStream_t st) {
  CUtensorMap ta, tb;
  if (!make_tmap(&ta, a, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, M, lda, kGemmBK, kGemmBM,
                 CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap(&tb, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, N, ldw, kGemmBK,
                 EPI == kEpiI8SwiGLU ? BN / 2 : BN, CU_TENSOR_MAP_SWIZZLE_128B))
    return B200Q_ERR_CUDA;
  auto kern = gemm8_tc_kernel<KIND, BN, STAGES, EPI, PRO>;
  constexpr int smem = PRO != kProNone ? Gemm8Layout<BN, STAGES>::kSmemBytesPro
                                       : Gemm8Layout<BN, STAGES>::kSmemBytes;
  if (!set_smem(kern, smem)) return B200Q_ERR_CUDA;
  const int64_t tiles = int64_t((M + kGemmBM - 1) / kGemmBM) * ((N + BN - 1) / BN);
  const int grid = static_cast<int>(tiles < d->num_sms ? tiles : d->num_sms);
  kern<<<grid, kGemmThreads, smem, st>>>(ta, tb, M, N, K, raster_group_m(lda, ldw, M, N, K), ep, pro);
  return finish_launch();
}

// Programmatic dependent launch for the CTA-pair GEMM and the warp-per-row
// quant (read per call; B200Q_PDL=0 launches them plainly).
bool pdl_launch_on() {
  const char* e = getenv("B200Q_PDL");
  return !(e && e[0] == '0');
}

// A plain 1-D launch of `kern` as a programmatic dependent (when enabled).
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), int grid, int block, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(static_cast<unsigned>(block));
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_launch_on() ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kern, args...);
  return finish_launch();
}

// CTA-pair kernel: clusters of 2, grid = 2 x min(tiles, SMs / 2).
// B200Q_TMA_STORE=0 keeps the per-thread global stores in the pair kernel's
// epilogue (A/B runs).
bool tma_store_enabled() {
  static const bool on = [] {
    const char* e = getenv("B200Q_TMA_STORE");
    return !(e && e[0] == '0');
  }();
  return on;
}

// B200Q_EPI_SLEEP_NS: nanoseconds the pair kernel's epilogue warps sleep between
// probes of the accumulator barrier (default 0: spin).
unsigned int epilogue_sleep_ns() {
  static const unsigned int v = [] {
    const char* e = getenv("B200Q_EPI_SLEEP_NS");
    return e ? static_cast<unsigned int>(atoi(e)) : 0u;
  }();
  return v;
}

template <MmaKind KIND, int STAGES, int EPI, int PRO, int KATOMS = 1, int BN = 256>
int launch_gemm8_tc2(const DeviceInfo* d, const void* a, int64_t lda, const void* w, int64_t ldw,
                     int M, int N, int K, const EpiArgs& ep_in, const Prologue& pro, cudaStream_t st,
                     const PeerOuts* peers = nullptr) {
  using L = Gemm8PairLayout<STAGES, KATOMS, BN>;
  CUtensorMap ta, tb, to;
  if (!make_tmap(&ta, a, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, M, lda, kGemmBK, 128,
                 CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap(&tb, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, N, ldw, kGemmBK, BN / 2,
                 CU_TENSOR_MAP_SWIZZLE_128B))
    return B200Q_ERR_CUDA;
  // 16-bit row-major outputs leave through TMA stores of 32 x 32 blocks
  EpiArgs ep = ep_in;
  constexpr bool kStoreEpi = (EPI == kEpiI8Dequant || EPI == kEpiScaled) && PRO == kProNone;
  ep.tma_store = 0;
  // The TMA store clips a box at the row's end only to 16-byte granularity (a
  // 16-bit row of N = 300 got columns 300..303 written), so ragged widths keep
  // the per-thread stores.
  if (kStoreEpi && tma_store_enabled() && ep.qkv_heads == 0 &&
      (ep.out_dtype == kOutBF16 || ep.out_dtype == kOutF16) && aligned16(ep.out) &&
      (ep.ldo * 2) % 16 == 0 && (int64_t(N) * 2) % 16 == 0 &&
      make_tmap(&to, ep.out,
                ep.out_dtype == kOutF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                uint64_t(N), uint64_t(M), uint64_t(ep.ldo) * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
    ep.tma_store = 1;
  if (!ep.tma_store) to = ta;  // unused by the kernel
  PeerOuts po;
  po.n = 0;
  if (peers && peers->n > 0) {
    if (!ep.tma_store) return B200Q_ERR_INVALID;  // peer copies leave through the TMA stores
    po = *peers;
  }
  ep.wait_sleep_ns = epilogue_sleep_ns();
  auto kern = gemm8_tc2_kernel<KIND, STAGES, EPI, PRO, KATOMS, BN>;
  constexpr int smem = PRO != kProNone ? L::kSmemBytesPro
                       : kStoreEpi     ? L::kSmemBytesStore
                                       : L::kSmemBytes;
  if (!set_smem(kern, smem)) return B200Q_ERR_CUDA;
  const int64_t tiles = int64_t((M + 255) / 256) * ((N + BN - 1) / BN);
  const int64_t pairs = tiles < d->num_sms / 2 ? tiles : d->num_sms / 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // the set-up (barriers, TMEM, descriptor prefetch) overlaps the previous
  // kernel's tail; the kernel waits for it before touching memory
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_launch_on() ? 2 : 1;
  const cudaError_t le =
      cudaLaunchKernelEx(&cfg, kern, ta, tb, to, po, M, N, K, raster_group_m(lda, ldw, M, N, K), ep, pro);
  if (le != cudaSuccess) {
    cudaGetLastError();
    fprintf(stderr, "[b200q] cluster launch failed: %s\n", cudaGetErrorString(le));
    return B200Q_ERR_CUDA;
  }
  return finish_launch();
}

template <bool IS_FP8, int EPI>
int launch_gemm8_simt(const void* a, int64_t lda, const void* w, int64_t ldw, int M, int N, int K,
                      const EpiArgs& ep, cudaStream_t st) {
  dim3 grid((N + 63) / 64, (M + 63) / 64);
  if (grid.y > 65535u) return B200Q_ERR_INVALID;
  gemm8_simt_kernel<IS_FP8, EPI><<<grid, 256, 0, st>>>(static_cast<const uint8_t*>(a), lda,
                                                        static_cast<const uint8_t*>(w), ldw, M, N,
                                                        K, ep);
  return finish_launch();
}

// Pair-kernel stage shape: two K atoms (256 bytes, 8 MMAs) per stage in three
// stages by default; B200Q_PAIR_KATOMS=1 selects six one-atom stages (A/B runs).
bool pair_two_atoms() {
  static const bool on = [] {
    const char* e = getenv("B200Q_PAIR_KATOMS");
    return !(e && e[0] == '1');
  }();
  return on;
}
// Tile width of the pair kernel: 192 instead of 256 columns when its tile count
// fills the last wave of CTA pairs clearly better (e.g. 8192 x 3072: 384 tiles =
// 5.19 waves at 256, 512 tiles = 6.92 waves at 192).  B200Q_PAIR_BN=256/192 forces.
int pair_tile_n(const DeviceInfo* d, int M, int N) {
  static const int forced = [] {
    const char* e = getenv("B200Q_PAIR_BN");
    return e ? atoi(e) : 0;
  }();
  if (forced == 256 || forced == 192) return forced;
  const int pairs = d->num_sms / 2;
  auto eff = [&](int bn) {
    const int64_t nt = (N + bn - 1) / bn;
    const int64_t tiles = int64_t((M + 255) / 256) * nt;
    const int64_t waves = (tiles + pairs - 1) / pairs;
    // useful fraction of the launched tile slots, times the column fill of the
    // last (ragged) N tile, times a small charge for 192's extra operand bytes
    const double fill = double(N) / double(nt * bn);
    return double(tiles) / double(waves * pairs) * fill * (bn == 192 ? 0.97 : 1.0);
  };
  return eff(192) > eff(256) + 0.02 ? 192 : 256;
}

template <MmaKind KIND, int EPI, int PRO>
int launch_pair(const DeviceInfo* d, const void* a, int64_t lda, const void* w, int64_t ldw,
                int M, int N, int K, const EpiArgs& ep, const Prologue& pro, cudaStream_t st,
                const PeerOuts* peers = nullptr) {
  if constexpr (PRO == kProNone) {
    if (pair_two_atoms()) {
      if constexpr (EPI == kEpiInt32 || EPI == kEpiI8Dequant || EPI == kEpiScaled) {
        if (pair_tile_n(d, M, N) == 192)
          return launch_gemm8_tc2<KIND, 3, EPI, kProNone, 2, 192>(d, a, lda, w, ldw, M, N, K, ep,
                                                                   pro, st, peers);
      }
      return launch_gemm8_tc2<KIND, 3, EPI, kProNone, 2>(d, a, lda, w, ldw, M, N, K, ep, pro, st,
                                                         peers);
    }
  }
  return launch_gemm8_tc2<KIND, 6, EPI, PRO, 1>(d, a, lda, w, ldw, M, N, K, ep, pro, st, peers);
}

// B200Q_PAIR_GEMM=0 selects the single-CTA kernel everywhere (A/B measurements).
bool pair_kernels_enabled() {
  static const bool on = [] {
    const char* e = getenv("B200Q_PAIR_GEMM");
    return !(e && e[0] == '0');
  }();
  return on;
}

bool gemm8_tc_eligible(const void* a, int64_t lda, const void* w, int64_t ldw, int64_t K) {
  return K > 0 && (K % 16 == 0) && (lda % 16 == 0) && (ldw % 16 == 0) && aligned16(a) && aligned16(w);
}

// Tensor-core dispatch; PRO != kProNone means `a` is the code buffer that the
// launch's own quant prologue fills (gemm8_tc_eligible must hold).
template <MmaKind KIND, int EPI, int PRO = kProNone>
int gemm8(const void* a, int64_t lda, const void* w, int64_t ldw, int64_t M, int64_t N, int64_t K,
          const EpiArgs& ep, cudaStream_t st, const Prologue& pro = Prologue{}) {
  const DeviceInfo* d = current_device();
  if (!d) return B200Q_ERR_UNSUPPORTED;
  if (M == 0 || N == 0) return B200Q_OK;
  constexpr bool kFp8 = KIND == MmaKind::F8F6F4;
  if (!gemm8_tc_eligible(a, lda, w, ldw, K)) {
    if constexpr (PRO != kProNone) return B200Q_ERR_INVALID;
    else return launch_gemm8_simt<kFp8, EPI>(a, lda, w, ldw, int(M), int(N), int(K), ep, st);
  }
  if (N <= 128)
    return launch_gemm8_tc<KIND, 128, 6, EPI, PRO>(d, a, lda, w, ldw, int(M), int(N), int(K), ep, pro, st);
  if (M >= 256 && pair_kernels_enabled())
    return launch_pair<KIND, EPI, PRO>(d, a, lda, w, ldw, int(M), int(N), int(K), ep, pro, st);
  return launch_gemm8_tc<KIND, 256, 4, EPI, PRO>(d, a, lda, w, ldw, int(M), int(N), int(K), ep, pro, st);
}

// FC1 with the SwiGLU epilogue: N2 = 2F weight rows [gate; up].  TMA path only
// (both kernels split the B tile between the gate and up row ranges).
int gemm8_swiglu(const void* a, int64_t lda, const void* w, int64_t ldw, int64_t M, int64_t N2,
                 int64_t K, const EpiArgs& ep, cudaStream_t st) {
  const DeviceInfo* d = current_device();
  if (!d) return B200Q_ERR_UNSUPPORTED;
  if (M == 0 || N2 == 0) return B200Q_OK;
  if (!gemm8_tc_eligible(a, lda, w, ldw, K)) return B200Q_ERR_INVALID;
  if (M >= 256 && pair_kernels_enabled())
    return launch_pair<MmaKind::I8, kEpiI8SwiGLU, kProNone>(d, a, lda, w, ldw, int(M), int(N2), int(K), ep, Prologue{}, st);
  return launch_gemm8_tc<MmaKind::I8, 256, 4, kEpiI8SwiGLU, kProNone>(d, a, lda, w, ldw, int(M), int(N2), int(K), ep, Prologue{}, st);
}

// Grouped row kernel: one resident wave of CTAs (occupancy-sized), each looping
// over rows.
template <typename T, bool SWIGLU, bool ROT, bool QUANT>
int launch_rows(const DeviceInfo* d, const void* x, int64_t ldx, int64_t M, int64_t K, void* out,
                int64_t ldo, int8_t* q, int64_t ldq, float* scales, cudaStream_t st) {
  auto kern = rows_kernel<T, SWIGLU, ROT, QUANT>;
  const int smem = rows_smem_bytes(static_cast<int>(K), ROT, QUANT);
  if (!set_smem(kern, smem)) return B200Q_ERR_CUDA;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kRowThreads, smem) !=
          cudaSuccess ||
      per_sm < 1)
    return B200Q_ERR_CUDA;
  const int64_t wave = int64_t(d->num_sms) * per_sm;
  const int grid = static_cast<int>(M < wave ? M : wave);
  kern<<<grid, kRowThreads, smem, st>>>(static_cast<const T*>(x), ldx, int(K), static_cast<T*>(out),
                                         ldo, q, ldq, scales, int(M));
  return finish_launch();
}

template <bool ROT, bool QUANT>
int launch_swiglu_rows(const DeviceInfo* d, const void* x, int64_t ldx, int64_t M, int64_t F,
                       void* out, int64_t ldo, int8_t* q, int64_t ldq, float* scales,
                       cudaStream_t st) {
  return launch_rows<__nv_bfloat16, true, ROT, QUANT>(d, x, ldx, M, F, out, ldo, q, ldq, scales, st);
}

// GEMM on 16-bit operands (kind::f16) through the 8-bit tile kernels: the tiles
// are byte-described, so K, the row strides and the tensor-map extents are passed
// in bytes.  Needs 16-byte aligned operands and K % 8 == 0.
template <MmaKind KIND, int EPI>
int gemm16(const DeviceInfo* d, const void* a, int64_t lda, const void* w, int64_t ldw, int64_t M,
           int64_t N, int64_t K, const EpiArgs& ep, cudaStream_t st) {
  const int64_t kb = 2 * K, la = 2 * lda, lw = 2 * ldw;
  if (N <= 128)
    return launch_gemm8_tc<KIND, 128, 6, EPI, kProNone>(d, a, la, w, lw, int(M), int(N), int(kb), ep, Prologue{}, st);
  if (M >= 256 && pair_kernels_enabled())
    return launch_pair<KIND, EPI, kProNone>(d, a, la, w, lw, int(M), int(N), int(kb), ep, Prologue{}, st);
  return launch_gemm8_tc<KIND, 256, 4, EPI, kProNone>(d, a, la, w, lw, int(M), int(N), int(kb), ep, Prologue{}, st);
}

EpiArgs make_epi(void* out, int64_t ldo, int out_dtype, int64_t M, int64_t N) {
  EpiArgs e{};
  e.out = out;
  e.ldo = ldo;
  e.out_dtype = out_dtype;
  e.bias_dtype = kBiasNone;
  e.act = kActNone;
  e.M = static_cast<int>(M);
  e.N = static_cast<int>(N);
  return e;
}

// ------------------------------------------------------------ W8A16 planning
struct W16Plan {
  int bt;
  int splits;
  size_t partial_bytes;
  size_t counter_bytes;
};

// W8A16 at M >= 128: the weight is decoded to the activation's 16-bit type once
// per call (exact) into the caller's workspace and the product runs on the 8-bit
// tile kernels as kind::f16.  The in-kernel conversion of the weight-stationary
// kernels repeats per token tile (M / 256 times); the decode costs one pass of
// 3 bytes per weight element.  Measured crossover on B200 (K x N = 3072 x 12288,
// 5120 x 5120, 5120 x 13824): the decoded route is ahead from M = 65..192 and
// 1.6-2.6x ahead at M >= 512; B200Q_W8A16_DECODE_MIN_M overrides the threshold.
int64_t w8a16_decode_min_m() {
  static const int64_t v = [] {
    const char* e = getenv("B200Q_W8A16_DECODE_MIN_M");
    return e ? static_cast<int64_t>(atoll(e)) : static_cast<int64_t>(128);
  }();
  return v;
}
bool w8a16_decode_selected(int64_t M, int64_t N, int64_t K) {
  return M >= w8a16_decode_min_m() && K % 16 == 0 && N > 0 && N <= 65535;
}
size_t w8a16_decode_bytes(int64_t N, int64_t K) {
  return (static_cast<size_t>(N) * static_cast<size_t>(K) * 2 + 255) & ~size_t(255);
}

W16Plan w8a16_plan(int num_sms, int64_t M, int64_t N, int64_t K) {
  W16Plan p{};
  // Token tiles up to 64 run the TMEM-operand streaming kernel; larger M runs the
  // shared-memory-operand kernel (128- or 256-token tiles).  A 128-token
  // streaming tile was measured no faster at M = 128..256 (its X stream and
  // the single MMA issuer bind first).
  p.bt = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  const int64_t num_n = (N + kW16BM - 1) / kW16BM;
  const int64_t num_t = (M + p.bt - 1) / p.bt;
  const int64_t tiles = num_n * num_t;
  const int64_t num_kb = (K + kW16BK - 1) / kW16BK;
  int best = 1;
  double best_eff = 0.0;
  // Token tiles of <= 64 run the streaming kernel as one tile per CTA: its
  // split-K fix-up (one dependent L2 round trip per 4 tokens) cost more than the
  // idle SMs it would fill (measured: S = 2 turned 34 us into 74 us at M = 64).
  const int max_splits = p.bt <= 64 ? 1 : kW16MaxSplits;
  for (int s = 1; s <= max_splits; ++s) {
    if (s > 1 && s * 4 > num_kb) break;
    // fp32 partial write + read must stay small next to the fp8 weight stream
    if (s > 1 && double(s) * M * N * 8.0 > 0.5 * double(N) * K) break;
    const int64_t units = tiles * s;
    const int64_t waves = (units + num_sms - 1) / num_sms;
    const double eff = double(units) / double(waves * num_sms);
    if (eff > best_eff + 0.02) {
      best_eff = eff;
      best = s;
    }
  }
  // Tuning override (B200Q_W8A16_SPLITS=n) for measurements; clamped to the plan's limits.
  static const int forced = [] {
    const char* e = getenv("B200Q_W8A16_SPLITS");
    return e ? atoi(e) : 0;
  }();
  if (forced > 0) {
    best = forced > kW16MaxSplits ? kW16MaxSplits : forced;
    while (best > 1 && best * 2 > num_kb) --best;
  }
  p.splits = best;
  if (best > 1) {
    p.partial_bytes = size_t(best) * size_t(M) * size_t(N) * sizeof(float);
    p.counter_bytes = size_t(tiles) * sizeof(unsigned int);
  }
  return p;
}

template <int BT, bool XF16>
int launch_w8a16_tc(const DeviceInfo* d, const void* x, int64_t ldx, const uint8_t* w, int64_t ldw,
                    const W8A16Args& args, const EpiArgs& ep, cudaStream_t st) {
  CUtensorMap tx, tw;
  const CUtensorMapDataType xdt = XF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (!make_tmap(&tx, x, xdt, args.K, args.M, ldx * 2, kW16BK, BT, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap(&tw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, args.K, args.N, ldw, kW16BK, kW16BM,
                 CU_TENSOR_MAP_SWIZZLE_NONE))
    return B200Q_ERR_CUDA;
  auto kern = w8a16_tc_kernel<BT, XF16>;
  constexpr int smem = W8A16Layout<BT>::kSmemBytes;
  if (!set_smem(kern, smem)) return B200Q_ERR_CUDA;
  const int64_t units = int64_t((args.N + kW16BM - 1) / kW16BM) * ((args.M + BT - 1) / BT) * args.splits;
  const int grid = static_cast<int>(units < d->num_sms ? units : d->num_sms);
  kern<<<grid, kW16Threads, smem, st>>>(tx, tw, args, ep);
  return finish_launch();
}

// Small token counts: the streaming kernel (deep raw-weight ring, 128-byte boxes).
template <int BT, bool XF16>
int launch_w8a16_stream(const DeviceInfo* d, const void* x, int64_t ldx, const uint8_t* w,
                        int64_t ldw, const W8A16Args& args, const EpiArgs& ep, cudaStream_t st) {
  CUtensorMap tx, tw;
  const CUtensorMapDataType xdt = XF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (!make_tmap(&tx, x, xdt, args.K, args.M, ldx * 2, 64, BT, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap(&tw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, args.K, args.N, ldw, kWsBK, kW16BM,
                 CU_TENSOR_MAP_SWIZZLE_128B))
    return B200Q_ERR_CUDA;
  auto kern = w8a16_stream_kernel<BT, XF16>;
  constexpr int smem = W8A16StreamLayout<BT>::kSmemBytes;
  if (!set_smem(kern, smem)) return B200Q_ERR_CUDA;
  const int64_t units = int64_t((args.N + kW16BM - 1) / kW16BM) * ((args.M + BT - 1) / BT) * args.splits;
  const int grid = static_cast<int>(units < d->num_sms ? units : d->num_sms);
  kern<<<grid, kWsThreads, smem, st>>>(tx, tw, args, ep);
  return finish_launch();
}

template <bool XF16>
int dispatch_w8a16_tc(const DeviceInfo* d, int bt, const void* x, int64_t ldx, const uint8_t* w,
                      int64_t ldw, const W8A16Args& args, const EpiArgs& ep, cudaStream_t st) {
  switch (bt) {
    case 16: return launch_w8a16_stream<16, XF16>(d, x, ldx, w, ldw, args, ep, st);
    case 32: return launch_w8a16_stream<32, XF16>(d, x, ldx, w, ldw, args, ep, st);
    case 64: return launch_w8a16_stream<64, XF16>(d, x, ldx, w, ldw, args, ep, st);
    case 128: return launch_w8a16_tc<128, XF16>(d, x, ldx, w, ldw, args, ep, st);
    default: return launch_w8a16_tc<256, XF16>(d, x, ldx, w, ldw, args, ep, st);
  }
}

// The prologue's bulk-copy quantizer reads 16-byte row segments of x.
bool ring_ok(const void* x, int64_t ldx, int64_t K) {
  return aligned16(x) && K % 8 == 0 && ldx % 8 == 0;
}

template <int MT, bool XF16>
int launch_w8a16_gemv(const void* x, int64_t ldx, const uint8_t* w, int64_t ldw, int64_t M,
                      int64_t N, int64_t K, const EpiArgs& ep, cudaStream_t st) {
  CUtensorMap tw;
  if (!make_tmap(&tw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, N, ldw, 128, kGvRows,
                 CU_TENSOR_MAP_SWIZZLE_128B))
    return B200Q_ERR_CUDA;
  auto kern = w8a16_gemv_kernel<MT, XF16>;
  if (!set_smem(kern, kGvSmemBytes)) return B200Q_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((N + kGvRows - 1) / kGvRows));
  cfg.blockDim = dim3(kGvThreads);
  cfg.dynamicSmemBytes = kGvSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_launch_on() ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kern, tw, static_cast<const uint16_t*>(x), ldx, int(M), int(N), int(K),
                     ep);
  return finish_launch();
}

// W8A16 with <= 32 tokens takes the weight-streaming GEMV when the operands are
// 16-byte aligned (the caller checks) and neither the planes GEMV nor the planes
// route took the call.  B200Q_W8A16_GEMV=0 turns it off (A/B runs).
bool w8a16_gemv_selected(int64_t M) {
  static const bool on = [] {
    const char* e = getenv("B200Q_W8A16_GEMV");
    return !(e && e[0] == '0');
  }();
  return on && M <= 32;
}

// Sync words of a fused-prologue launch: 16-byte aligned, large enough for M rows.
bool sync_ok(const unsigned int* sync, size_t sync_bytes, int64_t M) {
  return sync && (reinterpret_cast<uintptr_t>(sync) & 15) == 0 &&
         sync_bytes >= b200q_prologue_sync_bytes(M);
}

// ---------------------------------------------------------------------------
// W8A16 planes route (w8a16_planes.cuh): M <= 128 bf16 / M <= 64 fp16 tokens,
// raw e4m3 weight tiles x exact e4m3 activation planes on kind::f8f6f4.
// B200Q_W8A16_PLANES=0 turns it off (A/B runs); B200Q_W8A16_PLANES_SPLITS=n
// forces the cluster size; B200Q_PDL=0 launches the GEMM without the
// programmatic dependency on the planes pass.
struct WpPlan {
  bool ok = false;
  int bt = 0, P = 0, nt = 0, ntt = 1, S = 1, stages = 0, smem = 0, katoms = 1;
};

bool env_flag(const char* name, bool dflt) {
  const char* e = getenv(name);
  return e ? e[0] != '0' : dflt;
}
// Read per call (a getenv), so tests can switch routes inside one process.
// B200Q_W8A16_PLANES: unset = where the planes route measured at least level
// with the decode-in-kernel kernels on B200 (back-to-back calls, weights larger
// than L2): every M > 16; for bf16 activations also M <= 16 when K > 4096 (at
// K = 3072 the GEMV is ~8% ahead there); fp16 activations keep the GEMV for
// M <= 16 at every K (its e4m3 -> fp16 decode is one instruction per pair: 10.6
// vs 13.6 us at 3072 x 12288, 15.1 vs 18.9 us at 5120 x 13824); "1" = every
// eligible call, "0" = never.
bool w8a16_planes_for(int64_t M, int64_t K, bool f16) {
  const char* e = getenv("B200Q_W8A16_PLANES");
  if (e) return e[0] != '0';
  return M > 16 || (!f16 && K > 4096);
}
bool pdl_on() { return env_flag("B200Q_PDL", true); }
// Tokens per plane tile: 16/32/64 for M up to 16/32/128 and 128 above (bf16),
// at most 64 for fp16 (three planes: P x bt <= 192 plane rows per MMA); M is
// split into ntt = ceil(M / bt) token tiles.
constexpr int64_t kWpMaxM = 256;
// Measured on B200 at 3072 x 12288: 65..128 tokens as two 64-token tiles (192
// CTAs, half the epilogue each) beat one 128-token tile (96 CTAs) by ~4%
// (21.9 vs 22.8 us at M = 128); above 128 tokens 128-token tiles stay ahead
// (31.7 vs 45.6 us at M = 256).
int wp_bt(int64_t M, int P) {
  const int cap = P == 3 ? 64 : 128;
  const int bt = M <= 16 ? 16 : M <= 32 ? 32 : M <= 128 ? 64 : 128;
  return bt < cap ? bt : cap;
}
int wp_ntt(int64_t M, int bt) { return static_cast<int>((M + bt - 1) / bt); }
size_t wp_plane_bytes(int P, int bt, int ntt, int64_t K) {
  return (size_t(ntt) * size_t(P) * size_t(bt) * size_t(K) + 255) & ~size_t(255);
}
size_t wp_workspace_bytes(int P, int bt, int ntt, int64_t K) {
  return wp_plane_bytes(P, bt, ntt, K) + size_t(ntt) * size_t(P) * size_t(bt) * sizeof(float);
}
// Workspace of the planes route for either activation type (the size query
// does not know the type): 0 when M is out of its range.
size_t wp_workspace_any(int64_t M, int64_t K) {
  if (M < 1 || M > kWpMaxM || K % 16 != 0 || K > kWpMaxK) return 0;
  size_t best = 0;
  for (int P = 2; P <= 3; ++P) {
    if (!w8a16_planes_for(M, K, P == 3)) continue;
    const int bt = wp_bt(M, P);
    const size_t b = wp_workspace_bytes(P, bt, wp_ntt(M, bt), K);
    if (b > best) best = b;
  }
  return best;
}

// Plan: the weight's 128-row tiles times the token tiles times S K-splits (one
// cluster of S CTAs per (weight tile, token tile)), with the ring sized for 1 or
// 2 CTAs per SM.  Cost model, from B200 measurements of this kernel: a CTA
// streams its share at ~45 GB/s with its ring full (so 96 weight tiles stream
// faster as 192 half-K CTAs than as 96), the GPU at ~6 TB/s (a
// weight tile is read from HBM once; its other token tiles run next to it and
// hit L2), the tensor cores at ~1.3e15 e4m3 MAC/s (twice the measured
// sustained bf16 rate); every split adds a reduction
// step.  Only
// plans that are resident in one wave are taken; two CTAs per SM were measured
// to co-reside (the occupancy calculator reports one), and with clusters of
// S > 1 about 10% of the slots are lost to cluster placement (S = 3 at 2 per SM
// did not fit 288 CTAs on 148 SMs).
WpPlan w8a16_planes_plan(const DeviceInfo* d, int64_t M, int64_t N, int64_t K, bool f16) {
  WpPlan best;
  if (!w8a16_planes_for(M, K, f16) || M < 1 || M > kWpMaxM || K % 16 != 0 || K > kWpMaxK ||
      N < 1 || N > (int64_t(1) << 24))
    return best;
  const int P = f16 ? 3 : 2;
  int bt = wp_bt(M, P);
  {  // measurement switch: a smaller token tile (more CTAs per weight tile)
    const char* fb = getenv("B200Q_W8A16_PLANES_BT");
    const int want = fb ? atoi(fb) : 0;
    if ((want == 16 || want == 32 || want == 64) && want < bt) bt = want;
  }
  const int ntt = wp_ntt(M, bt);
  const int nt = P * bt;
  const int dump = nt * 128 * 4;
  const int tmem = nt <= 32 ? 32 : nt <= 64 ? 64 : nt <= 128 ? 128 : 256;
  const int bar = (2 * kWpMaxStages + 1) * 8 + 16 + 1024;
  const int64_t tiles = (N + 127) / 128;
  const char* fs = getenv("B200Q_W8A16_PLANES_SPLITS");
  const int forced_s = fs ? atoi(fs) : 0;
  const char* fc = getenv("B200Q_W8A16_PLANES_CTAS");  // CTAs per SM the ring is sized for
  const int forced_c = fc ? atoi(fc) : 0;
  // K atoms per stage (1 or 2): B200Q_W8A16_PLANES_KATOMS forces one, otherwise
  // both are costed.  A stage hand-off costs a CTA ~0.36 us whatever the stage
  // holds (measured: one 16 KB atom per stage streamed ~45 GB/s per CTA), so
  // two atoms halve the hand-offs but need twice the ring per stage.
  const char* fk = getenv("B200Q_W8A16_PLANES_KATOMS");
  const int forced_k = fk ? atoi(fk) : 0;
  double best_cost = 1e30;
  for (int KA = 2; KA >= 1; --KA) {  // two-atom stages first: they win ties (fewer hand-offs)
    if (forced_k > 0 && KA != forced_k) continue;
    const int stage = KA * (128 * kWpBK + nt * kWpBK);
    const int nkb = static_cast<int>((K + KA * kWpBK - 1) / (KA * kWpBK));  // stages along K
    const double t_hbm = double(tiles) * double(K) * 128.0 / 6.0e6;        // us
    const double t_mma = double(tiles) * ntt * double(K) * 128.0 * nt / 1.3e9;  // us
    for (int c = 1; c <= 2; ++c) {
      if (c * tmem > 512 || (forced_c > 0 && c != forced_c)) continue;
      const int budget = (c == 1 ? 232448 : 233472 / c - 1024);  // per-CTA dynamic smem
      int stages = (budget - bar) / stage;
      if (stages > kWpMaxStages) stages = kWpMaxStages;
      if (stages < 2) continue;
      for (int S = 1; S <= 8 && S <= nkb; ++S) {
        if (forced_s > 0 && S != forced_s) continue;
        if (S > 1 && dump + bar > budget) continue;  // split ranks park accumulators in the ring
        const int ring = (S > 1 && dump > stages * stage) ? dump : stages * stage;
        const int smem = ring + bar;
        const int64_t ctas = tiles * ntt * S;
        const double slots = double(c) * d->num_sms * (S > 1 ? 0.9 : 1.0);
        if (double(ctas) > slots && forced_s == 0) continue;
        // a second CTA per SM only pays when one per SM cannot hold the grid
        // (its ring is half as deep)
        if (c == 2 && ctas <= d->num_sms && forced_c == 0) continue;
        // A CTA streams its share at ~45 GB/s whatever its stage size (measured:
        // 96 CTAs of two-atom stages moved the 37.7 MB of 3072 x 12288 in ~9.7 us),
        // and pays ~0.36 us per stage hand-off.
        const double t_bytes = 128.0 * double(K) / S / 45.0e3;  // us, weight bytes (planes hit L2)
        const double t_handoff = double((nkb + S - 1) / S) * 0.364;          // us
        const double t_cta = t_bytes > t_handoff ? t_bytes : t_handoff;
        double cost = t_cta > t_hbm ? t_cta : t_hbm;
        if (t_mma > cost) cost = t_mma;
        // Rank 0 adds the other ranks' accumulators of the tile's tokens over
        // distributed shared memory and runs the whole epilogue: ~0.045 us per
        // (rank, plane, token) column (3072 x 12288: two K-halves win at 16
        // tokens, one CTA per weight tile from 24 tokens on: 14.3 vs 15.1 us at
        // 32, 15.7 vs 18.5 us at 48).
        const int mt = static_cast<int>(M < bt ? M : bt);
        cost += (S > 1 ? 0.3 : 0.0) + 0.1 * S + 0.045 * (S - 1) * P * mt;
        if (env_flag("B200Q_DEBUG_PLAN", false))
          fprintf(stderr, "[b200q] planes plan M %lld N %lld K %lld: ka %d c %d S %d stages %d smem %d cost %.2f\n",
                  (long long)M, (long long)N, (long long)K, KA, c, S, stages, smem, cost);
        if (cost < best_cost - 1e-9) {
          best_cost = cost;
          best.ok = true;
          best.bt = bt;
          best.P = P;
          best.nt = nt;
          best.ntt = ntt;
          best.S = S;
          best.stages = stages;
          best.smem = smem;
          best.katoms = KA;
        }
      }
    }
  }
  return best;
}

template <int NT>
int launch_planes_gemm(const WpPlan& p, const CUtensorMap& tw, const CUtensorMap& tx,
                       const WpArgs& args, const EpiArgs& ep, cudaStream_t st) {
  auto kern = w8a16_planes_kernel<NT>;
  if (!set_smem(kern, p.smem)) return B200Q_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((args.N + 127) / 128 * p.ntt * p.S));
  cfg.blockDim = dim3(kWpThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(p.smem);
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  int na = 0;
  if (pdl_on()) {
    at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (p.S > 1) {
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = static_cast<unsigned>(p.S);
    at[na].val.clusterDim.y = 1;
    at[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = at;
  cfg.numAttrs = na;
  cudaLaunchKernelEx(&cfg, kern, tw, tx, args, ep);  // errors surface in finish_launch
  return finish_launch();
}

int launch_planes_gemm_nt(const WpPlan& p, const uint8_t* w, int64_t ldw, uint8_t* planes,
                          float* pscale, int64_t M, int64_t N, int64_t K, const EpiArgs& ep,
                          cudaStream_t st);

// The planes pass over M token rows (token tiles of bt rows): a programmatic
// dependent of the previous kernel on the stream too, it waits for it
// (griddepcontrol.wait) before touching memory.
int launch_x_planes(const void* x, int x_dtype, int64_t ldx, int64_t M, int64_t K, int bt,
                    uint8_t* planes, float* pscale, cudaStream_t st) {
  const int row_smem = static_cast<int>(K) * 2;
  cudaLaunchConfig_t pcfg = {};
  pcfg.gridDim = dim3(static_cast<unsigned>(M));
  pcfg.blockDim = dim3(kWpPlaneThreads);
  pcfg.dynamicSmemBytes = static_cast<size_t>(row_smem);
  pcfg.stream = st;
  cudaLaunchAttribute pat[1];
  pat[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pat[0].val.programmaticStreamSerializationAllowed = 1;
  pcfg.attrs = pat;
  pcfg.numAttrs = pdl_on() ? 1 : 0;
  if (x_dtype == B200Q_F16) {
    if (!set_smem(x_planes_kernel<__half, 3>, row_smem)) return B200Q_ERR_CUDA;
    cudaLaunchKernelEx(&pcfg, x_planes_kernel<__half, 3>, static_cast<const __half*>(x), ldx,
                       int(K), bt, planes, pscale);
  } else {
    if (!set_smem(x_planes_kernel<__nv_bfloat16, 2>, row_smem)) return B200Q_ERR_CUDA;
    cudaLaunchKernelEx(&pcfg, x_planes_kernel<__nv_bfloat16, 2>,
                       static_cast<const __nv_bfloat16*>(x), ldx, int(K), bt, planes, pscale);
  }
  return finish_launch();
}

int launch_w8a16_planes(const WpPlan& p, const void* x, int x_dtype, int64_t ldx, const uint8_t* w,
                        int64_t ldw, int64_t M, int64_t N, int64_t K, const EpiArgs& ep,
                        void* workspace, cudaStream_t st) {
  uint8_t* planes = static_cast<uint8_t*>(workspace);
  float* pscale = reinterpret_cast<float*>(planes + wp_plane_bytes(p.P, p.bt, p.ntt, K));
  const int s = launch_x_planes(x, x_dtype, ldx, M, K, p.bt, planes, pscale, st);
  if (s != B200Q_OK) return s;
  return launch_planes_gemm_nt(p, w, ldw, planes, pscale, M, N, K, ep, st);
}

// Planes GEMV (w8a16_pgemv_kernel): one 8-column MMA group of plane rows, i.e.
// M <= 4 bf16 or M <= 2 fp16 tokens, one token tile of M rows.  Measured on
// B200 at 3072 x 12288 (back-to-back calls in a CUDA graph, weights larger than
// L2) against the decode-in-kernel GEMV: bf16 10.5 vs 12.2 us per call at M = 1,
// 10.8 vs 12.3 at M = 4; fp16 10.6 vs 10.3 (its GEMV decodes with one
// instruction per weight pair); two column groups (bf16 M = 8) 13.9 vs 12.5, so
// the kernel's NG = 2 form is not routed.  B200Q_W8A16_PGEMV: unset = bf16
// activations only, "1" = fp16 too, "0" = never (read per call).
int pg_planes(int x_dtype) { return x_dtype == B200Q_F16 ? 3 : 2; }
bool w8a16_pgemv_for(int64_t M, int P, int64_t K) {
  const char* e = getenv("B200Q_W8A16_PGEMV");
  const bool on = e ? e[0] != '0' : P == 2;
  return on && M >= 1 && P * M <= 8 && K % 16 == 0 && K <= kWpMaxK;
}
size_t pg_workspace_bytes(int P, int64_t M, int64_t K) {
  return wp_workspace_bytes(P, static_cast<int>(M), 1, K);
}

int launch_w8a16_pgemv(const void* x, int x_dtype, int64_t ldx, const uint8_t* w, int64_t ldw,
                       int64_t M, int64_t N, int64_t K, const EpiArgs& ep, void* workspace,
                       cudaStream_t st) {
  const int P = pg_planes(x_dtype);
  uint8_t* planes = static_cast<uint8_t*>(workspace);
  float* pscale = reinterpret_cast<float*>(planes + wp_plane_bytes(P, int(M), 1, K));
  CUtensorMap tw;
  if (!make_tmap(&tw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, N, ldw, 128, kGvRows,
                 CU_TENSOR_MAP_SWIZZLE_128B))
    return B200Q_ERR_CUDA;
  int s = launch_x_planes(x, x_dtype, ldx, M, K, int(M), planes, pscale, st);
  if (s != B200Q_OK) return s;
  auto kern = w8a16_pgemv_kernel<1>;
  if (!set_smem(kern, kGvSmemBytes)) return B200Q_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((N + kGvRows - 1) / kGvRows));
  cfg.blockDim = dim3(kGvThreads);
  cfg.dynamicSmemBytes = kGvSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_on() ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kern, tw, static_cast<const uint8_t*>(planes),
                     static_cast<const float*>(pscale), P, int(M), int(N), int(K), ep);
  return finish_launch();
}

int launch_planes_gemm_nt(const WpPlan& p, const uint8_t* w, int64_t ldw, uint8_t* planes,
                          float* pscale, int64_t M, int64_t N, int64_t K, const EpiArgs& ep,
                          cudaStream_t st) {
  CUtensorMap tw, tx;
  if (!make_tmap(&tw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, N, ldw, kWpBK, 128,
                 CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap(&tx, planes, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, uint64_t(p.ntt) * p.P * p.bt, K,
                 kWpBK, p.nt, CU_TENSOR_MAP_SWIZZLE_128B))
    return B200Q_ERR_CUDA;
  WpArgs args{};
  args.M = int(M);
  args.N = int(N);
  args.K = int(K);
  args.bt = p.bt;
  args.ntt = p.ntt;
  args.planes = p.P;
  args.splits = p.S;
  args.stages = p.stages;
  args.katoms = p.katoms;
  args.pscale = pscale;
  switch (p.nt) {
    case 32: return launch_planes_gemm<32>(p, tw, tx, args, ep, st);
    case 48: return launch_planes_gemm<48>(p, tw, tx, args, ep, st);
    case 64: return launch_planes_gemm<64>(p, tw, tx, args, ep, st);
    case 96: return launch_planes_gemm<96>(p, tw, tx, args, ep, st);
    case 128: return launch_planes_gemm<128>(p, tw, tx, args, ep, st);
    case 192: return launch_planes_gemm<192>(p, tw, tx, args, ep, st);
    case 256: return launch_planes_gemm<256>(p, tw, tx, args, ep, st);
    default: return B200Q_ERR_INVALID;
  }
}

// Warp-per-row INT8 quant: VPL 16-byte vectors per lane, the smallest
// instantiated count covering K / 8 vectors over 32 lanes (K <= 8192).
template <typename T>
int launch_quant_warp(int grid, const void* x, int64_t ldx, int8_t* q, int64_t ldq, float* scales,
                      int64_t M, int64_t K, cudaStream_t st) {
  const T* xp = static_cast<const T*>(x);
  const int need = static_cast<int>((K / 8 + 31) / 32);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kQuantWarpRows * 32);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_launch_on() ? 1 : 0;
  const int Mi = int(M), Ki = int(K);
  if (need <= 4) cudaLaunchKernelEx(&cfg, quant_rowwise_i8_warp_kernel<T, 4>, xp, ldx, q, ldq, scales, Mi, Ki);
  else if (need <= 8) cudaLaunchKernelEx(&cfg, quant_rowwise_i8_warp_kernel<T, 8>, xp, ldx, q, ldq, scales, Mi, Ki);
  else if (need <= 12) cudaLaunchKernelEx(&cfg, quant_rowwise_i8_warp_kernel<T, 12>, xp, ldx, q, ldq, scales, Mi, Ki);
  else if (need <= 16) cudaLaunchKernelEx(&cfg, quant_rowwise_i8_warp_kernel<T, 16>, xp, ldx, q, ldq, scales, Mi, Ki);
  else if (need <= 20) cudaLaunchKernelEx(&cfg, quant_rowwise_i8_warp_kernel<T, 20>, xp, ldx, q, ldq, scales, Mi, Ki);
  else if (need <= 24) cudaLaunchKernelEx(&cfg, quant_rowwise_i8_warp_kernel<T, 24>, xp, ldx, q, ldq, scales, Mi, Ki);
  else cudaLaunchKernelEx(&cfg, quant_rowwise_i8_warp_kernel<T, 32>, xp, ldx, q, ldq, scales, Mi, Ki);
  return finish_launch();
}

int grid_for(int64_t work, int per_block, const DeviceInfo* d) {
  int64_t g = (work + per_block - 1) / per_block;
  const int64_t cap = int64_t(d->num_sms) * 8;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

}  // namespace

// =====================================================================  C ABI
extern "C" {

int b200q_version(void) { return 1; }

const char* b200q_status_string(int s) {
  switch (s) {
    case B200Q_OK: return "ok";
    case B200Q_ERR_INVALID: return "invalid argument";
    case B200Q_ERR_UNSUPPORTED: return "unsupported device (b200q kernels need sm_100 / B200)";
    case B200Q_ERR_CUDA: return "CUDA error";
    case B200Q_ERR_WORKSPACE: return "workspace too small";
    case B200Q_ERR_TOO_LARGE:
      return "shape needs more split-K scratch than the allocation-free entry point's static "
             "buffer (B200Q_NOALLOC_SCRATCH_BYTES) holds; use b200q_w8a16_linear with a workspace";
    default: return "unknown status";
  }
}

uint64_t b200q_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int b200q_get_device_status(unsigned int* status, int reset) {
  if (!status) return B200Q_ERR_INVALID;
  if (cudaMemcpyFromSymbol(status, g_device_status, sizeof(unsigned int)) != cudaSuccess)
    return B200Q_ERR_CUDA;
  if (reset) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(g_device_status, &zero, sizeof(unsigned int)) != cudaSuccess)
      return B200Q_ERR_CUDA;
  }
  return B200Q_OK;
}

int b200q_quant_rowwise_i8(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                           int8_t* q, int64_t ldq, float* scales, void* stream) {
  if (!x || !q || !scales || M < 0 || K <= 0 || ldx < K || ldq < K || M >= (int64_t(1) << 31) ||
      (x_dtype != B200Q_BF16 && x_dtype != B200Q_F16))
    return B200Q_ERR_INVALID;
  const DeviceInfo* d = current_device();
  if (!d) return B200Q_ERR_UNSUPPORTED;
  if (M == 0) return B200Q_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = static_cast<int>(M < int64_t(d->num_sms) * 16 ? M : int64_t(d->num_sms) * 16);
  const bool vec = (K % 8 == 0) && (ldx % 8 == 0) && (ldq % 8 == 0) && aligned16(x) &&
                   (reinterpret_cast<uintptr_t>(q) % 8 == 0);
  if (vec && K <= 8192 && env_flag("B200Q_QUANT_WARP_ROWS", true)) {
    const int wgrid = static_cast<int>((M + kQuantWarpRows - 1) / kQuantWarpRows);
    return x_dtype == B200Q_BF16
               ? launch_quant_warp<__nv_bfloat16>(wgrid, x, ldx, q, ldq, scales, M, K, st)
               : launch_quant_warp<__half>(wgrid, x, ldx, q, ldq, scales, M, K, st);
  }
  if (x_dtype == B200Q_BF16) {
    auto* xp = static_cast<const __nv_bfloat16*>(x);
    if (vec) quant_rowwise_i8_vec_kernel<__nv_bfloat16><<<grid, kQuantThreads, 0, st>>>(xp, ldx, q, ldq, scales, int(M), int(K));
    else quant_rowwise_i8_scalar_kernel<__nv_bfloat16><<<grid, kQuantThreads, 0, st>>>(xp, ldx, q, ldq, scales, int(M), int(K));
  } else {
    auto* xp = static_cast<const __half*>(x);
    if (vec) quant_rowwise_i8_vec_kernel<__half><<<grid, kQuantThreads, 0, st>>>(xp, ldx, q, ldq, scales, int(M), int(K));
    else quant_rowwise_i8_scalar_kernel<__half><<<grid, kQuantThreads, 0, st>>>(xp, ldx, q, ldq, scales, int(M), int(K));
  }
  return finish_launch();
}

int b200q_quant_rowwise_i8_convrot(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                                   int groupsize, int8_t* q, int64_t ldq, float* scales,
                                   void* stream) {
  if (!x || !q || !scales || M < 0 || K <= 0 || ldx < K || ldq < K || M >= (int64_t(1) << 31) ||
      (x_dtype != B200Q_BF16 && x_dtype != B200Q_F16))
    return B200Q_ERR_INVALID;
  if (groupsize != kRotGroup || K % kRotGroup != 0 || K > B200Q_CONVROT_MAX_K)
    return B200Q_ERR_UNSUPPORTED;
  const DeviceInfo* d = current_device();
  if (!d) return B200Q_ERR_UNSUPPORTED;
  if (M == 0) return B200Q_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (x_dtype == B200Q_BF16)
    return launch_rows<__nv_bfloat16, false, true, true>(d, x, ldx, M, K, nullptr, 0, q, ldq, scales, st);
  return launch_rows<__half, false, true, true>(d, x, ldx, M, K, nullptr, 0, q, ldq, scales, st);
}

int b200q_i8_matmul_nt(const int8_t* a, int64_t lda, const int8_t* w, int64_t ldw, int32_t* c,
                       int64_t ldc, int64_t M, int64_t N, int64_t K, void* stream) {
  if (!a || !w || !c || !valid_dims(M, N, K) || K == 0 || lda < K || ldw < K || ldc < N)
    return B200Q_ERR_INVALID;
  EpiArgs ep = make_epi(c, ldc, kOutI32, M, N);
  return gemm8<MmaKind::I8, kEpiInt32>(a, lda, w, ldw, M, N, K, ep, static_cast<cudaStream_t>(stream));
}

int b200q_i8_matmul_nt_dequant(const int8_t* a, int64_t lda, const int8_t* w, int64_t ldw,
                               const float* row_scale, const float* col_scale,
                               int64_t col_scale_numel, const void* bias, int act, void* out,
                               int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K,
                               void* stream) {
  if (!a || !w || !out || !row_scale || !col_scale || !valid_dims(M, N, K) || K == 0 || lda < K ||
      ldw < K || ldo < N || (col_scale_numel != 1 && col_scale_numel != N) ||
      (out_dtype != B200Q_BF16 && out_dtype != B200Q_F16) || act < B200Q_ACT_NONE ||
      act > B200Q_ACT_GELU_ERF)
    return B200Q_ERR_INVALID;
  EpiArgs ep = make_epi(out, ldo, out_dtype, M, N);
  ep.row_scale = row_scale;
  ep.row_scale_vec = 1;
  ep.col_scale = col_scale;
  ep.col_scale_vec = col_scale_numel == N && N != 1 ? 1 : 0;
  if (col_scale_numel == 1) ep.col_scale_vec = 0;
  ep.bias = bias;
  ep.bias_dtype = bias ? (out_dtype == B200Q_BF16 ? kBiasBF16 : kBiasF16) : kBiasNone;
  ep.act = act;
  return gemm8<MmaKind::I8, kEpiI8Dequant>(a, lda, w, ldw, M, N, K, ep, static_cast<cudaStream_t>(stream));
}

int b200q_i8_linear(const void* x, int x_dtype, int64_t ldx, const int8_t* w, int64_t ldw,
                    const float* col_scale, int64_t col_scale_numel, const void* bias, int act,
                    void* out, int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K,
                    int8_t* q_scratch, float* scale_scratch, void* stream) {
  int s = b200q_quant_rowwise_i8(x, x_dtype, M, K, ldx, q_scratch, K, scale_scratch, stream);
  if (s != B200Q_OK) return s;
  return b200q_i8_matmul_nt_dequant(q_scratch, K, w, ldw, scale_scratch, col_scale,
                                    col_scale_numel, bias, act, out, out_dtype, ldo, M, N, K,
                                    stream);
}

int b200q_i8_matmul_nt_dequant_qkv(const int8_t* a, int64_t lda, const int8_t* w, int64_t ldw,
                                   const float* row_scale, const float* col_scale,
                                   int64_t col_scale_numel, const void* bias, void* q_out,
                                   void* k_out, void* v_out, int out_dtype, int64_t heads,
                                   int64_t head_dim, int64_t batch, int64_t M, int64_t N, int64_t K,
                                   void* stream) {
  if (!a || !w || !row_scale || !col_scale || !q_out || !k_out || !v_out || !valid_dims(M, N, K) ||
      K == 0 || lda < K || ldw < K || heads <= 0 || head_dim <= 0 || head_dim % 32 != 0 ||
      batch <= 0 || M % batch != 0 || N != 3 * heads * head_dim ||
      (col_scale_numel != 1 && col_scale_numel != N) ||
      (out_dtype != B200Q_BF16 && out_dtype != B200Q_F16) || !aligned16(q_out) ||
      !aligned16(k_out) || !aligned16(v_out))
    return B200Q_ERR_INVALID;
  EpiArgs ep = make_epi(q_out, N, out_dtype, M, N);
  ep.row_scale = row_scale;
  ep.row_scale_vec = 1;
  ep.col_scale = col_scale;
  ep.col_scale_vec = col_scale_numel == N && N != 1 ? 1 : 0;
  ep.bias = bias;
  ep.bias_dtype = bias ? (out_dtype == B200Q_BF16 ? kBiasBF16 : kBiasF16) : kBiasNone;
  ep.qkv[0] = q_out;
  ep.qkv[1] = k_out;
  ep.qkv[2] = v_out;
  ep.qkv_heads = static_cast<int>(heads);
  ep.qkv_dim = static_cast<int>(head_dim);
  ep.qkv_seq = static_cast<int>(M / batch);
  return gemm8<MmaKind::I8, kEpiI8Dequant>(a, lda, w, ldw, M, N, K, ep, static_cast<cudaStream_t>(stream));
}

int b200q_i8_matmul_nt_dequant_swiglu(const int8_t* a, int64_t lda, const int8_t* w, int64_t ldw,
                                      const float* row_scale, const float* col_scale,
                                      int64_t col_scale_numel, const void* bias, void* act_out,
                                      int64_t ldo, int64_t M, int64_t N2, int64_t K, void* stream) {
  if (!a || !w || !row_scale || !col_scale || !act_out || !valid_dims(M, N2, K) || K == 0 ||
      lda < K || ldw < K || N2 <= 0 || N2 % 2 != 0 || ldo < N2 / 2 ||
      (col_scale_numel != 1 && col_scale_numel != N2))
    return B200Q_ERR_INVALID;
  EpiArgs ep = make_epi(act_out, ldo, B200Q_BF16, M, N2);
  ep.row_scale = row_scale;
  ep.row_scale_vec = 1;
  ep.col_scale = col_scale;
  ep.col_scale_vec = col_scale_numel == N2 ? 1 : 0;
  ep.bias = bias;
  ep.bias_dtype = bias ? kBiasBF16 : kBiasNone;
  return gemm8_swiglu(a, lda, w, ldw, M, N2, K, ep, static_cast<cudaStream_t>(stream));
}

static int swiglu_rows_args_ok(const void* x, int64_t ldx, int64_t M, int64_t F) {
  return x && M >= 0 && M < (int64_t(1) << 31) && F > 0 && F <= B200Q_SWIGLU_MAX_F &&
         ldx >= 2 * F;
}

int b200q_silu_mul_split(const void* x, int64_t ldx, int64_t M, int64_t F, void* out, int64_t ldo,
                         void* stream) {
  if (!swiglu_rows_args_ok(x, ldx, M, F) || !out || ldo < F) return B200Q_ERR_INVALID;
  const DeviceInfo* d = current_device();
  if (!d) return B200Q_ERR_UNSUPPORTED;
  if (M == 0) return B200Q_OK;
  return launch_swiglu_rows<false, false>(d, x, ldx, M, F, out, ldo, nullptr, 0, nullptr,
                                          static_cast<cudaStream_t>(stream));
}

int b200q_i8_swiglu_rot(const void* x, int64_t ldx, int64_t M, int64_t F, void* out, int64_t ldo,
                        void* stream) {
  if (!swiglu_rows_args_ok(x, ldx, M, F) || !out || ldo < F) return B200Q_ERR_INVALID;
  if (F % kRotGroup != 0) return B200Q_ERR_UNSUPPORTED;
  const DeviceInfo* d = current_device();
  if (!d) return B200Q_ERR_UNSUPPORTED;
  if (M == 0) return B200Q_OK;
  return launch_swiglu_rows<true, false>(d, x, ldx, M, F, out, ldo, nullptr, 0, nullptr,
                                         static_cast<cudaStream_t>(stream));
}

int b200q_i8_swiglu_quant(const void* x, int64_t ldx, int64_t M, int64_t F, int rotate, int8_t* q,
                          int64_t ldq, float* scales, void* stream) {
  if (!swiglu_rows_args_ok(x, ldx, M, F) || !q || !scales || ldq < F) return B200Q_ERR_INVALID;
  if (rotate && F % kRotGroup != 0) return B200Q_ERR_UNSUPPORTED;
  const DeviceInfo* d = current_device();
  if (!d) return B200Q_ERR_UNSUPPORTED;
  if (M == 0) return B200Q_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rotate) return launch_swiglu_rows<true, true>(d, x, ldx, M, F, nullptr, 0, q, ldq, scales, st);
  return launch_swiglu_rows<false, true>(d, x, ldx, M, F, nullptr, 0, q, ldq, scales, st);
}

int b200q_i8_mlp_bridge_prequant(const int8_t* a, int64_t lda, const int8_t* w1, int64_t ldw,
                                 const float* row_scale, const float* col_scale,
                                 int64_t col_scale_numel, const void* bias, int64_t M, int64_t N2,
                                 int64_t K, int rotate, int64_t tile_rows, void* act_scratch,
                                 int8_t* q, int64_t ldq, float* scales, void* stream) {
  const int64_t F = N2 / 2;
  if (!a || !w1 || !row_scale || !col_scale || !act_scratch || !q || !scales ||
      !valid_dims(M, N2, K) || K == 0 || lda < K || ldw < K || N2 <= 0 || N2 % 2 != 0 ||
      ldq < F || tile_rows < 0 || (col_scale_numel != 1 && col_scale_numel != N2))
    return B200Q_ERR_INVALID;
  if (rotate && (F % kRotGroup != 0 || F > B200Q_CONVROT_MAX_K)) return B200Q_ERR_UNSUPPORTED;
  if (M == 0) return B200Q_OK;
  const int64_t rows = tile_rows == 0 || tile_rows > M ? M : tile_rows;
  auto* act = static_cast<__nv_bfloat16*>(act_scratch);
  for (int64_t r0 = 0; r0 < M; r0 += rows) {
    const int64_t mr = M - r0 < rows ? M - r0 : rows;
    int s = b200q_i8_matmul_nt_dequant_swiglu(a + r0 * lda, lda, w1, ldw, row_scale + r0,
                                              col_scale, col_scale_numel, bias, act, F, mr, N2,
                                              K, stream);
    if (s != B200Q_OK) return s;
    s = rotate ? b200q_quant_rowwise_i8_convrot(act, B200Q_BF16, mr, F, F, kRotGroup, q + r0 * ldq,
                                                ldq, scales + r0, stream)
               : b200q_quant_rowwise_i8(act, B200Q_BF16, mr, F, F, q + r0 * ldq, ldq,
                                        scales + r0, stream);
    if (s != B200Q_OK) return s;
  }
  return B200Q_OK;
}

int b200q_i8_matmul_nt_dequant_qkv_rms_rope(
    const int8_t* a, int64_t lda, const int8_t* w, int64_t ldw, const float* row_scale,
    const float* col_scale, int64_t col_scale_numel, const void* bias, void* q_out, void* k_out,
    void* v_out, int64_t heads, int64_t batch, const void* freqs, int64_t rot_half,
    const float* q_weight, const float* k_weight, float eps, int64_t M, int64_t N, int64_t K,
    void* stream) {
  constexpr int64_t D = 128;
  if (!a || !w || !row_scale || !col_scale || !q_out || !k_out || !v_out || !q_weight ||
      !k_weight || !valid_dims(M, N, K) || K == 0 || lda < K || ldw < K || heads <= 0 ||
      batch <= 0 || M % batch != 0 || N != 3 * heads * D ||
      (col_scale_numel != 1 && col_scale_numel != N) || rot_half < 0 || rot_half % 8 != 0 ||
      2 * rot_half > D || (rot_half > 0 && (!freqs || !aligned16(freqs))) ||
      !aligned16(q_out) || !aligned16(k_out) || !aligned16(v_out) || !aligned16(q_weight) ||
      !aligned16(k_weight) || !gemm8_tc_eligible(a, lda, w, ldw, K))
    return B200Q_ERR_INVALID;
  const DeviceInfo* d = current_device();
  if (!d) return B200Q_ERR_UNSUPPORTED;
  if (M == 0) return B200Q_OK;
  EpiArgs ep = make_epi(q_out, N, B200Q_BF16, M, N);
  ep.row_scale = row_scale;
  ep.row_scale_vec = 1;
  ep.col_scale = col_scale;
  ep.col_scale_vec = col_scale_numel == N ? 1 : 0;
  ep.bias = bias;
  ep.bias_dtype = bias ? kBiasBF16 : kBiasNone;
  ep.qkv[0] = q_out;
  ep.qkv[1] = k_out;
  ep.qkv[2] = v_out;
  ep.qkv_heads = static_cast<int>(heads);
  ep.qkv_dim = static_cast<int>(D);
  ep.qkv_seq = static_cast<int>(M / batch);
  ep.rope_freqs = static_cast<const __nv_bfloat16*>(freqs);
  ep.q_norm_w = q_weight;
  ep.k_norm_w = k_weight;
  ep.rope_r = static_cast<int>(rot_half);
  ep.norm_eps = eps;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (M >= 256 && pair_kernels_enabled())
    return launch_pair<MmaKind::I8, kEpiI8QkvNormRope, kProNone>(d, a, lda, w, ldw, int(M), int(N), int(K), ep, Prologue{}, st);
  return launch_gemm8_tc<MmaKind::I8, 256, 4, kEpiI8QkvNormRope, kProNone>(d, a, lda, w, ldw, int(M), int(N), int(K), ep, Prologue{}, st);
}

int b200q_rms_rope_partial(void* q, void* k, const void* freqs, const float* q_weight,
                           const float* k_weight, int64_t batch, int64_t heads, int64_t seq,
                           int64_t head_dim, int64_t rot_half, float eps, void* stream) {
  if (!q || !k || !q_weight || !k_weight || batch <= 0 || heads <= 0 || seq <= 0 ||
      head_dim <= 0 || head_dim % 32 != 0 || head_dim > 256 || rot_half < 0 ||
      2 * rot_half > head_dim || (rot_half > 0 && !freqs) ||
      batch * heads * seq >= (int64_t(1) << 30) ||
      (reinterpret_cast<uintptr_t>(q) & 7) != 0 || (reinterpret_cast<uintptr_t>(k) & 7) != 0 ||
      !aligned16(q_weight) || !aligned16(k_weight) ||
      (rot_half > 0 && rot_half % 4 == 0 && !aligned16(freqs)))
    return B200Q_ERR_INVALID;
  const DeviceInfo* d = current_device();
  if (!d) return B200Q_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (batch * heads > 65535) return B200Q_ERR_INVALID;
  const dim3 grid(static_cast<unsigned>((seq + kRrWarps - 1) / kRrWarps),
                  static_cast<unsigned>(batch * heads), 2);
  auto* qp = static_cast<__nv_bfloat16*>(q);
  auto* kp = static_cast<__nv_bfloat16*>(k);
  auto* fp = static_cast<const __nv_bfloat16*>(freqs);
  if (head_dim <= 128)
    rms_rope_partial_kernel<1><<<grid, kRrWarps * 32, 0, st>>>(qp, kp, fp, q_weight, k_weight, int(heads), int(seq), int(head_dim), int(rot_half), eps);
  else
    rms_rope_partial_kernel<2><<<grid, kRrWarps * 32, 0, st>>>(qp, kp, fp, q_weight, k_weight, int(heads), int(seq), int(head_dim), int(rot_half), eps);
  return finish_launch();
}

size_t b200q_prologue_sync_bytes(int64_t M) {
  const int64_t bands = M > 0 ? (M + kBandRows - 1) / kBandRows : 0;
  return static_cast<size_t>(((kSyncBands + bands) * 4 + 255) & ~int64_t(255));
}

int b200q_i8_linear_fused(const void* x, int x_dtype, int64_t ldx, const int8_t* w, int64_t ldw,
                          const float* col_scale, int64_t col_scale_numel, const void* bias,
                          int act, void* out, int out_dtype, int64_t ldo, int64_t M, int64_t N,
                          int64_t K, int8_t* q_scratch, float* scale_scratch, unsigned int* sync,
                          size_t sync_bytes, void* stream) {
  if (!x || !w || !out || !col_scale || !q_scratch || !scale_scratch || !valid_dims(M, N, K) ||
      K == 0 || ldx < K || ldw < K || ldo < N || (col_scale_numel != 1 && col_scale_numel != N) ||
      (x_dtype != B200Q_BF16 && x_dtype != B200Q_F16) ||
      (out_dtype != B200Q_BF16 && out_dtype != B200Q_F16) || act < B200Q_ACT_NONE ||
      act > B200Q_ACT_GELU_ERF)
    return B200Q_ERR_INVALID;
  if (!sync_ok(sync, sync_bytes, M)) return B200Q_ERR_WORKSPACE;
  const DeviceInfo* d = current_device();
  if (!d) return B200Q_ERR_UNSUPPORTED;
  if (M == 0 || N == 0) return B200Q_OK;
  // Shapes the TMA path cannot take run as quant launch + SIMT GEMM.
  if (!gemm8_tc_eligible(q_scratch, K, w, ldw, K))
    return b200q_i8_linear(x, x_dtype, ldx, w, ldw, col_scale, col_scale_numel, bias, act, out,
                           out_dtype, ldo, M, N, K, q_scratch, scale_scratch, stream);
  EpiArgs ep = make_epi(out, ldo, out_dtype, M, N);
  ep.row_scale = scale_scratch;
  ep.row_scale_vec = 1;
  ep.col_scale = col_scale;
  ep.col_scale_vec = col_scale_numel == N && N != 1 ? 1 : 0;
  ep.bias = bias;
  ep.bias_dtype = bias ? (out_dtype == B200Q_BF16 ? kBiasBF16 : kBiasF16) : kBiasNone;
  ep.act = act;
  Prologue pro{};
  pro.x = x;
  pro.ldx = ldx;
  pro.q = reinterpret_cast<uint8_t*>(q_scratch);
  pro.scales = scale_scratch;
  pro.sync = sync;
  pro.x_f16 = x_dtype == B200Q_F16 ? 1 : 0;
  pro.nbands = static_cast<int>((M + kBandRows - 1) / kBandRows);
  pro.ring = ring_ok(x, ldx, K) ? 1 : 0;
  return gemm8<MmaKind::I8, kEpiI8Dequant, kProInt8Row>(q_scratch, K, w, ldw, M, N, K, ep,
                                                        static_cast<cudaStream_t>(stream), pro);
}

int b200q_fp8_linear_fused(const void* x, int x_dtype, int64_t ldx, const uint8_t* w, int64_t ldw,
                           const float* scale_b, int64_t scale_b_numel, const float* scale_result,
                           const void* bias, int bias_dtype, int act, void* out, int out_dtype,
                           int64_t ldo, int64_t M, int64_t N, int64_t K, uint8_t* q_scratch,
                           float* scale_out, unsigned int* sync, size_t sync_bytes, void* stream) {
  if (!x || !w || !out || !q_scratch || !scale_out || !valid_dims(M, N, K) || K == 0 || ldx < K ||
      ldw < K || ldo < N || (scale_b && scale_b_numel != 1 && scale_b_numel != N) ||
      (x_dtype != B200Q_BF16 && x_dtype != B200Q_F16) ||
      (out_dtype != B200Q_BF16 && out_dtype != B200Q_F16 && out_dtype != B200Q_F32) ||
      bias_dtype < B200Q_BIAS_NONE || bias_dtype > B200Q_BIAS_F32 ||
      (bias_dtype != B200Q_BIAS_NONE && !bias) || act < B200Q_ACT_NONE || act > B200Q_ACT_GELU_ERF)
    return B200Q_ERR_INVALID;
  if (!sync_ok(sync, sync_bytes, M)) return B200Q_ERR_WORKSPACE;
  const DeviceInfo* d = current_device();
  if (!d) return B200Q_ERR_UNSUPPORTED;
  if (M == 0) return B200Q_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned int* amax = sync + kSyncAmax;
  if (N == 0 || !gemm8_tc_eligible(q_scratch, K, w, ldw, K)) {
    // Two-launch route; the quant's amax word is cleared again afterwards so
    // the sync buffer stays all-zero between calls.
    int s = b200q_fp8_quant_tensorwise(x, x_dtype, M, K, ldx, q_scratch, K, scale_out, amax, stream);
    if (s == B200Q_OK && N > 0)
      s = b200q_fp8_scaled_mm(q_scratch, K, w, ldw, scale_out, 1, scale_b, scale_b_numel,
                              scale_result, bias, bias_dtype, act, out, out_dtype, ldo, M, N, K,
                              stream);
    if (cudaMemsetAsync(amax, 0, sizeof(unsigned int), st) != cudaSuccess && s == B200Q_OK)
      s = B200Q_ERR_CUDA;
    return s;
  }
  const int grid = grid_for(M * K / 8 + 1, 256, d);
  if (x_dtype == B200Q_BF16)
    absmax_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), ldx, M, int(K), amax);
  else
    absmax_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(x), ldx, M, int(K), amax);
  const int s = finish_launch();
  if (s != B200Q_OK) return s;
  EpiArgs ep = make_epi(out, ldo, out_dtype, M, N);
  ep.col_scale = scale_b;
  ep.col_scale_vec = scale_b && scale_b_numel == N && N != 1 ? 1 : 0;
  ep.extra_scale = scale_result;
  ep.bias = bias;
  ep.bias_dtype = bias ? bias_dtype : kBiasNone;
  ep.act = act;
  Prologue pro{};
  pro.x = x;
  pro.ldx = ldx;
  pro.q = q_scratch;
  pro.scales = scale_out;
  pro.sync = sync;
  pro.x_f16 = x_dtype == B200Q_F16 ? 1 : 0;
  pro.nbands = static_cast<int>((M + kBandRows - 1) / kBandRows);
  pro.ring = ring_ok(x, ldx, K) ? 1 : 0;
  return gemm8<MmaKind::F8F6F4, kEpiScaled, kProFp8Tensor>(q_scratch, K, w, ldw, M, N, K, ep, st, pro);
}

int b200q_fp8_scaled_mm(const uint8_t* a, int64_t lda, const uint8_t* w, int64_t ldw,
                        const float* scale_a, int64_t scale_a_numel, const float* scale_b,
                        int64_t scale_b_numel, const float* scale_result, const void* bias,
                        int bias_dtype, int act, void* out, int out_dtype, int64_t ldo, int64_t M,
                        int64_t N, int64_t K, void* stream) {
  if (!a || !w || !out || !valid_dims(M, N, K) || K == 0 || lda < K || ldw < K || ldo < N ||
      (scale_a && scale_a_numel != 1 && scale_a_numel != M) ||
      (scale_b && scale_b_numel != 1 && scale_b_numel != N) ||
      (out_dtype != B200Q_BF16 && out_dtype != B200Q_F16 && out_dtype != B200Q_F32) ||
      bias_dtype < B200Q_BIAS_NONE || bias_dtype > B200Q_BIAS_F32 || (bias_dtype != B200Q_BIAS_NONE && !bias) ||
      act < B200Q_ACT_NONE || act > B200Q_ACT_GELU_ERF)
    return B200Q_ERR_INVALID;
  EpiArgs ep = make_epi(out, ldo, out_dtype, M, N);
  ep.row_scale = scale_a;
  ep.row_scale_vec = scale_a && scale_a_numel == M && M != 1 ? 1 : 0;
  ep.col_scale = scale_b;
  ep.col_scale_vec = scale_b && scale_b_numel == N && N != 1 ? 1 : 0;
  ep.extra_scale = scale_result;
  ep.bias = bias;
  ep.bias_dtype = bias ? bias_dtype : kBiasNone;
  ep.act = act;
  return gemm8<MmaKind::F8F6F4, kEpiScaled>(a, lda, w, ldw, M, N, K, ep, static_cast<cudaStream_t>(stream));
}

// b200q_fp8_scaled_mm that also leaves max |out| (of the rounded outputs) in
// *amax_bits as float bits: on the CTA-pair route the epilogue folds it in while
// storing; other routes take it with the absmax pass over the output.
int b200q_fp8_scaled_mm_amax(const uint8_t* a, int64_t lda, const uint8_t* w, int64_t ldw,
                             const float* scale_a, int64_t scale_a_numel, const float* scale_b,
                             int64_t scale_b_numel, const float* scale_result, const void* bias,
                             int bias_dtype, int act, void* out, int out_dtype, int64_t ldo,
                             int64_t M, int64_t N, int64_t K, unsigned int* amax_bits,
                             void* stream) {
  if (!amax_bits || (out_dtype != B200Q_BF16 && out_dtype != B200Q_F16) || !a || !w || !out ||
      !valid_dims(M, N, K) || K == 0 || lda < K || ldw < K || ldo < N ||
      (scale_a && scale_a_numel != 1 && scale_a_numel != M) ||
      (scale_b && scale_b_numel != 1 && scale_b_numel != N) ||
      bias_dtype < B200Q_BIAS_NONE || bias_dtype > B200Q_BIAS_F32 ||
      (bias_dtype != B200Q_BIAS_NONE && !bias) || act < B200Q_ACT_NONE || act > B200Q_ACT_GELU_ERF)
    return B200Q_ERR_INVALID;
  const DeviceInfo* d = current_device();
  if (!d) return B200Q_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(amax_bits, 0, sizeof(unsigned int), st) != cudaSuccess) return B200Q_ERR_CUDA;
  if (M == 0 || N == 0) return B200Q_OK;
  EpiArgs ep = make_epi(out, ldo, out_dtype, M, N);
  ep.row_scale = scale_a;
  ep.row_scale_vec = scale_a && scale_a_numel == M && M != 1 ? 1 : 0;
  ep.col_scale = scale_b;
  ep.col_scale_vec = scale_b && scale_b_numel == N && N != 1 ? 1 : 0;
  ep.extra_scale = scale_result;
  ep.bias = bias;
  ep.bias_dtype = bias ? bias_dtype : kBiasNone;
  ep.act = act;
  const bool pair = gemm8_tc_eligible(a, lda, w, ldw, K) && N > 128 && M >= 256 &&
                    pair_kernels_enabled();
  if (pair) {
    ep.amax_out = amax_bits;
    return launch_pair<MmaKind::F8F6F4, kEpiScaled, kProNone>(d, a, lda, w, ldw, int(M), int(N),
                                                              int(K), ep, Prologue{}, st);
  }
  const int s = gemm8<MmaKind::F8F6F4, kEpiScaled>(a, lda, w, ldw, M, N, K, ep, st);
  if (s != B200Q_OK) return s;
  const int grid = grid_for(M * N / 8 + 1, 256, d);
  if (out_dtype == B200Q_BF16)
    absmax_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(out), ldo,
                                                       M, int(N), amax_bits);
  else
    absmax_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(out), ldo, M, int(N),
                                                amax_bits);
  return finish_launch();
}

// Per-tensor e4m3 quant of x with an amax already taken (the second half of
// b200q_fp8_quant_tensorwise).
int b200q_fp8_quant_from_amax(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                              const unsigned int* amax_bits, uint8_t* q, int64_t ldq,
                              float* scale, void* stream) {
  if (!x || !q || !scale || !amax_bits || M < 0 || K <= 0 || ldx < K || ldq < K ||
      (x_dtype != B200Q_BF16 && x_dtype != B200Q_F16))
    return B200Q_ERR_INVALID;
  const DeviceInfo* d = current_device();
  if (!d) return B200Q_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = grid_for(M * K / 8 + 1, 256, d);
  if (x_dtype == B200Q_BF16)
    return launch_pdl(fp8_quantize_kernel<__nv_bfloat16>, grid, 256, st,
                      static_cast<const __nv_bfloat16*>(x), ldx, M, int(K), amax_bits, q, ldq, scale);
  return launch_pdl(fp8_quantize_kernel<__half>, grid, 256, st, static_cast<const __half*>(x), ldx,
                    M, int(K), amax_bits, q, ldq, scale);
}

// Column-parallel FP8 GEMM with the all-gather in its epilogue.  This rank owns
// output columns [c0, c0 + N) of an [M, N_total] output held in full by every
// rank; `out` and peer_outs[i] point at column c0 of this rank's and of the
// peers' copies.  On the CTA-pair route with TMA stores every 32 x 32 output
// block leaves shared memory once per copy, so the NVLink transfer of a tile
// overlaps the MMAs of the next; other shapes run the plain GEMM into `out` and
// then copy the block to each peer (one cudaMemcpy2DAsync per peer).
int b200q_fp8_scaled_mm_allgather(const uint8_t* a, int64_t lda, const uint8_t* w, int64_t ldw,
                                  const float* scale_a, int64_t scale_a_numel, const float* scale_b,
                                  int64_t scale_b_numel, const float* scale_result, const void* bias,
                                  int bias_dtype, int act, void* out, void* const* peer_outs,
                                  int n_peer_outs, int out_dtype, int64_t ldo, int64_t M, int64_t N,
                                  int64_t K, void* stream) {
  if (n_peer_outs < 0 || n_peer_outs > kMaxPeerOuts || (n_peer_outs > 0 && !peer_outs) ||
      (out_dtype != B200Q_BF16 && out_dtype != B200Q_F16))
    return B200Q_ERR_INVALID;
  for (int i = 0; i < n_peer_outs; ++i)
    if (!peer_outs[i]) return B200Q_ERR_INVALID;
  if (n_peer_outs == 0)
    return b200q_fp8_scaled_mm(a, lda, w, ldw, scale_a, scale_a_numel, scale_b, scale_b_numel,
                               scale_result, bias, bias_dtype, act, out, out_dtype, ldo, M, N, K,
                               stream);
  if (!a || !w || !out || !valid_dims(M, N, K) || K == 0 || lda < K || ldw < K || ldo < N ||
      (scale_a && scale_a_numel != 1 && scale_a_numel != M) ||
      (scale_b && scale_b_numel != 1 && scale_b_numel != N) ||
      bias_dtype < B200Q_BIAS_NONE || bias_dtype > B200Q_BIAS_F32 ||
      (bias_dtype != B200Q_BIAS_NONE && !bias) || act < B200Q_ACT_NONE || act > B200Q_ACT_GELU_ERF)
    return B200Q_ERR_INVALID;
  const DeviceInfo* d = current_device();
  if (!d) return B200Q_ERR_UNSUPPORTED;
  if (M == 0 || N == 0) return B200Q_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  EpiArgs ep = make_epi(out, ldo, out_dtype, M, N);
  ep.row_scale = scale_a;
  ep.row_scale_vec = scale_a && scale_a_numel == M && M != 1 ? 1 : 0;
  ep.col_scale = scale_b;
  ep.col_scale_vec = scale_b && scale_b_numel == N && N != 1 ? 1 : 0;
  ep.extra_scale = scale_result;
  ep.bias = bias;
  ep.bias_dtype = bias ? bias_dtype : kBiasNone;
  ep.act = act;
  bool fused = gemm8_tc_eligible(a, lda, w, ldw, K) && N > 128 && M >= 256 &&
               pair_kernels_enabled() && tma_store_enabled() && aligned16(out) &&
               (ldo * 2) % 16 == 0 && (N * 2) % 16 == 0;
  PeerOuts po;
  po.n = n_peer_outs;
  const CUtensorMapDataType odt =
      out_dtype == B200Q_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  for (int i = 0; i < n_peer_outs && fused; ++i)
    fused = aligned16(peer_outs[i]) &&
            make_tmap(&po.map[i], peer_outs[i], odt, uint64_t(N), uint64_t(M), uint64_t(ldo) * 2,
                      32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
  if (fused)
    return launch_pair<MmaKind::F8F6F4, kEpiScaled, kProNone>(d, a, lda, w, ldw, int(M), int(N),
                                                              int(K), ep, Prologue{}, st, &po);
  const int s = gemm8<MmaKind::F8F6F4, kEpiScaled>(a, lda, w, ldw, M, N, K, ep, st);
  if (s != B200Q_OK) return s;
  const size_t row_bytes = size_t(ldo) * 2;
  for (int i = 0; i < n_peer_outs; ++i)
    if (cudaMemcpy2DAsync(peer_outs[i], row_bytes, out, row_bytes, size_t(N) * 2, size_t(M),
                          cudaMemcpyDefault, st) != cudaSuccess)
      return B200Q_ERR_CUDA;
  return B200Q_OK;
}

// Peer mappings for the column-parallel all-gather: the 64-byte CUDA IPC
// handle of the allocation holding a device pointer, and the pointer's offset
// in it; opening a handle maps that allocation into this process (peer access
// over NVLink enabled lazily).
namespace {
using MemGetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
MemGetAddressRangeFn address_range_fn() {
  static MemGetAddressRangeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<MemGetAddressRangeFn>(nullptr);
    return reinterpret_cast<MemGetAddressRangeFn>(p);
  }();
  return fn;
}
}  // namespace

int b200q_ipc_export(const void* dev_ptr, void* handle_out, uint64_t* offset_out) {
  if (!dev_ptr || !handle_out || !offset_out) return B200Q_ERR_INVALID;
  MemGetAddressRangeFn range = address_range_fn();
  if (!range) return B200Q_ERR_CUDA;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return B200Q_ERR_INVALID;  // not a device allocation
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) {
    cudaGetLastError();
    return B200Q_ERR_CUDA;
  }
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return B200Q_OK;
}

int b200q_ipc_import(const void* handle, uint64_t offset, void** dev_ptr_out, void** base_out) {
  if (!handle || !dev_ptr_out || !base_out) return B200Q_ERR_INVALID;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return B200Q_ERR_CUDA;
  }
  *base_out = base;
  *dev_ptr_out = static_cast<uint8_t*>(base) + offset;
  return B200Q_OK;
}

int b200q_ipc_close(void* base) {
  if (!base) return B200Q_ERR_INVALID;
  if (cudaIpcCloseMemHandle(base) != cudaSuccess) {
    cudaGetLastError();
    return B200Q_ERR_CUDA;
  }
  return B200Q_OK;
}

int b200q_fp8_quant_tensorwise(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                               uint8_t* q, int64_t ldq, float* scale, unsigned int* amax_scratch,
                               void* stream) {
  if (!x || !q || !scale || !amax_scratch || M < 0 || K <= 0 || ldx < K || ldq < K ||
      (x_dtype != B200Q_BF16 && x_dtype != B200Q_F16))
    return B200Q_ERR_INVALID;
  const DeviceInfo* d = current_device();
  if (!d) return B200Q_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(amax_scratch, 0, sizeof(unsigned int), st) != cudaSuccess) return B200Q_ERR_CUDA;
  const int64_t total = M * K;
  const int grid = grid_for(total / 8 + 1, 256, d);
  // both passes as programmatic dependents (each waits for the kernel before it)
  if (x_dtype == B200Q_BF16) {
    auto* xp = static_cast<const __nv_bfloat16*>(x);
    int s = launch_pdl(absmax_kernel<__nv_bfloat16>, grid, 256, st, xp, ldx, M, int(K), amax_scratch);
    if (s) return s;
    return launch_pdl(fp8_quantize_kernel<__nv_bfloat16>, grid, 256, st, xp, ldx, M, int(K),
                      static_cast<const unsigned int*>(amax_scratch), q, ldq, scale);
  }
  auto* xp = static_cast<const __half*>(x);
  int s = launch_pdl(absmax_kernel<__half>, grid, 256, st, xp, ldx, M, int(K), amax_scratch);
  if (s) return s;
  return launch_pdl(fp8_quantize_kernel<__half>, grid, 256, st, xp, ldx, M, int(K),
                    static_cast<const unsigned int*>(amax_scratch), q, ldq, scale);
}

}  // extern "C"
namespace {
// Workspace of the weight-stationary kernels alone (split-K partials + counters).
size_t w8a16_kernel_workspace(int64_t M, int64_t N, int64_t K) {
  const DeviceInfo* d = current_device();
  const int sms = d ? d->num_sms : 148;
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if (w8a16_gemv_selected(M)) return 0;
  const W16Plan p = w8a16_plan(sms, M, N, K);
  if (p.splits <= 1) return 0;
  return ((p.partial_bytes + 255) & ~size_t(255)) + p.counter_bytes;
}
}  // namespace
extern "C" {

size_t b200q_w8a16_workspace_size(int64_t M, int64_t N, int64_t K) {
  size_t ws = w8a16_kernel_workspace(M, N, K);
  if (M <= 0 || N <= 0 || K <= 0) return ws;
  const size_t planes = wp_workspace_any(M, K);
  if (planes > ws) ws = planes;
  for (int P = 2; P <= 3; ++P)
    if (w8a16_pgemv_for(M, P, K) && pg_workspace_bytes(P, M, K) > ws) ws = pg_workspace_bytes(P, M, K);
  if (!w8a16_decode_selected(M, N, K)) return ws;
  const size_t dec = w8a16_decode_bytes(N, K);
  return dec > ws ? dec : ws;
}

}  // extern "C"
namespace {
bool w8a16_args_valid(const void* x, int x_dtype, int64_t ldx, const uint8_t* w, int64_t ldw,
                      const void* bias, int bias_dtype, int act, const void* out, int out_dtype,
                      int64_t ldo, int64_t M, int64_t N, int64_t K) {
  return x && w && out && valid_dims(M, N, K) && K > 0 && ldx >= K && ldw >= K && ldo >= N &&
         (x_dtype == B200Q_BF16 || x_dtype == B200Q_F16) &&
         (out_dtype == B200Q_BF16 || out_dtype == B200Q_F16 || out_dtype == B200Q_F32) &&
         bias_dtype >= B200Q_BIAS_NONE && bias_dtype <= B200Q_BIAS_F32 &&
         (bias_dtype == B200Q_BIAS_NONE || bias) && act >= B200Q_ACT_NONE &&
         act <= B200Q_ACT_GELU_ERF;
}

bool w8a16_tc_operands(const void* x, int64_t ldx, const uint8_t* w, int64_t ldw, int64_t K) {
  return (K % 16 == 0) && (ldw % 16 == 0) && (ldx % 8 == 0) && aligned16(x) && aligned16(w);
}

int w8a16_linear_impl(const void* x, int x_dtype, int64_t ldx, const uint8_t* w, int64_t ldw,
                      const float* w_scale, const void* bias, int bias_dtype, int act, void* out,
                      int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K, void* workspace,
                      size_t workspace_bytes, bool allow_decode, void* stream) {
  if (!w8a16_args_valid(x, x_dtype, ldx, w, ldw, bias, bias_dtype, act, out, out_dtype, ldo, M, N, K))
    return B200Q_ERR_INVALID;
  const DeviceInfo* d = current_device();
  if (!d) return B200Q_ERR_UNSUPPORTED;
  if (M == 0 || N == 0) return B200Q_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  EpiArgs ep = make_epi(out, ldo, out_dtype, M, N);
  ep.extra_scale = w_scale;
  ep.bias = bias;
  ep.bias_dtype = bias ? bias_dtype : kBiasNone;
  ep.act = act;
  const bool tc = w8a16_tc_operands(x, ldx, w, ldw, K);
  if (!tc) {
    dim3 grid((N + 31) / 32, (M + 31) / 32);
    if (grid.y > 65535u) return B200Q_ERR_INVALID;
    if (x_dtype == B200Q_BF16)
      w8a16_simt_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), ldx, w, ldw, int(M), int(N), int(K), ep);
    else
      w8a16_simt_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(x), ldx, w, ldw, int(M), int(N), int(K), ep);
    return finish_launch();
  }
  if (workspace && aligned16(workspace) && w8a16_pgemv_for(M, pg_planes(x_dtype), K) &&
      workspace_bytes >= pg_workspace_bytes(pg_planes(x_dtype), M, K))
    return launch_w8a16_pgemv(x, x_dtype, ldx, w, ldw, M, N, K, ep, workspace, st);
  if (workspace && aligned16(workspace)) {
    const WpPlan wp = w8a16_planes_plan(d, M, N, K, x_dtype == B200Q_F16);
    if (wp.ok && workspace_bytes >= wp_workspace_bytes(wp.P, wp.bt, wp.ntt, K))
      return launch_w8a16_planes(wp, x, x_dtype, ldx, w, ldw, M, N, K, ep, workspace, st);
  }
  if (w8a16_gemv_selected(M)) {
    if (M <= 16)
      return x_dtype == B200Q_F16 ? launch_w8a16_gemv<1, true>(x, ldx, w, ldw, M, N, K, ep, st)
                                  : launch_w8a16_gemv<1, false>(x, ldx, w, ldw, M, N, K, ep, st);
    return x_dtype == B200Q_F16 ? launch_w8a16_gemv<2, true>(x, ldx, w, ldw, M, N, K, ep, st)
                                : launch_w8a16_gemv<2, false>(x, ldx, w, ldw, M, N, K, ep, st);
  }
  if (allow_decode && w8a16_decode_selected(M, N, K) && workspace &&
      workspace_bytes >= w8a16_decode_bytes(N, K) && aligned16(workspace)) {
    const dim3 dgrid(static_cast<unsigned>((K / 16 + 127) / 128), static_cast<unsigned>(N));
    if (x_dtype == B200Q_F16) {
      auto* wd = static_cast<__half*>(workspace);
      e4m3_rows_to16_kernel<__half><<<dgrid, 128, 0, st>>>(w, ldw, int(N), int(K), wd);
      int s = finish_launch();
      if (s != B200Q_OK) return s;
      return gemm16<MmaKind::F16, kEpiScaled>(d, x, ldx, wd, K, M, N, K, ep, st);
    }
    auto* wd = static_cast<__nv_bfloat16*>(workspace);
    e4m3_rows_to16_kernel<__nv_bfloat16><<<dgrid, 128, 0, st>>>(w, ldw, int(N), int(K), wd);
    int s = finish_launch();
    if (s != B200Q_OK) return s;
    return gemm16<MmaKind::BF16, kEpiScaled>(d, x, ldx, wd, K, M, N, K, ep, st);
  }
  const W16Plan p = w8a16_plan(d->num_sms, M, N, K);
  W8A16Args args{};
  args.M = int(M);
  args.N = int(N);
  args.K = int(K);
  args.splits = p.splits;
  if (p.splits > 1) {
    const size_t part = (p.partial_bytes + 255) & ~size_t(255);
    if (!workspace || workspace_bytes < part + p.counter_bytes || !aligned16(workspace))
      return B200Q_ERR_WORKSPACE;
    args.partial = static_cast<float*>(workspace);
    args.counters = reinterpret_cast<unsigned int*>(static_cast<uint8_t*>(workspace) + part);
    if (cudaMemsetAsync(args.counters, 0, p.counter_bytes, st) != cudaSuccess) return B200Q_ERR_CUDA;
  }
  if (x_dtype == B200Q_F16) return dispatch_w8a16_tc<true>(d, p.bt, x, ldx, w, ldw, args, ep, st);
  return dispatch_w8a16_tc<false>(d, p.bt, x, ldx, w, ldw, args, ep, st);
}
}  // namespace
extern "C" {

int b200q_w8a16_linear(const void* x, int x_dtype, int64_t ldx, const uint8_t* w, int64_t ldw,
                       const float* w_scale, const void* bias, int bias_dtype, int act, void* out,
                       int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K,
                       void* workspace, size_t workspace_bytes, void* stream) {
  return w8a16_linear_impl(x, x_dtype, ldx, w, ldw, w_scale, bias, bias_dtype, act, out,
                           out_dtype, ldo, M, N, K, workspace, workspace_bytes, true, stream);
}

// ---------------------------------------------------------------------------
// Allocation-free W8A16.  The split-K partials and tile counters live in this
// file-scope device array instead of a caller workspace.  In host code the name
// g_noalloc_scratch is only a host-side stand-in for the symbol, never a device
// address: the device address is looked up once per device with
// cudaGetSymbolAddress (with that device current) and cached.
}  // extern "C"

static __device__ __align__(256) unsigned char g_noalloc_scratch[B200Q_NOALLOC_SCRATCH_BYTES];

namespace {
// Per device: the context the address was looked up in, and the address.  A
// device reset (or a torn-down and re-created primary context) reloads the
// module, so a cached address is only reused inside the context it came from.
struct NoallocSlot {
  CUcontext ctx = nullptr;
  void* addr = nullptr;
};
NoallocSlot g_noalloc_slot[64];
std::mutex g_noalloc_mu;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<CtxGetCurrentFn>(nullptr);
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  return fn;
}

int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return B200Q_ERR_CUDA;
  CUcontext ctx = nullptr;
  if (CtxGetCurrentFn f = ctx_get_current_fn()) f(&ctx);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoallocSlot& slot = g_noalloc_slot[dev];
  if (!slot.addr || slot.ctx != ctx) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      fprintf(stderr, "[b200q] cudaGetSymbolAddress(noalloc scratch) failed: %s\n",
              cudaGetErrorString(e));
      return B200Q_ERR_CUDA;
    }
    slot.addr = p;
    slot.ctx = ctx;
  }
  *out = slot.addr;
  return B200Q_OK;
}

// Scratch bytes the call will use, following w8a16_linear_impl's route order
// with the decoded-weight route off: SIMT kernel (unaligned operands) -> none;
// planes GEMV (up to 8 plane rows) -> its planes; planes route when planned and
// its planes fit the static array; GEMV (M <= 32) -> none; otherwise the weight-stationary kernel's split-K partials + tile
// counters (0 when it runs unsplit).  B200Q_NOALLOC_SCRATCH_BYTES + 1 means the
// route needs more than the array holds.
size_t noalloc_route_bytes(const DeviceInfo* d, const void* x, int x_dtype, int64_t ldx,
                           const uint8_t* w, int64_t ldw, int64_t M, int64_t N, int64_t K) {
  if (M == 0 || N == 0 || !w8a16_tc_operands(x, ldx, w, ldw, K)) return 0;
  if (w8a16_pgemv_for(M, pg_planes(x_dtype), K)) return pg_workspace_bytes(pg_planes(x_dtype), M, K);
  const WpPlan wp = w8a16_planes_plan(d, M, N, K, x_dtype == B200Q_F16);
  if (wp.ok) {
    const size_t b = wp_workspace_bytes(wp.P, wp.bt, wp.ntt, K);
    if (b <= B200Q_NOALLOC_SCRATCH_BYTES) return b;
  }
  if (w8a16_gemv_selected(M)) return 0;
  const W16Plan p = w8a16_plan(d->num_sms, M, N, K);
  if (p.splits <= 1) return 0;
  const size_t need = ((p.partial_bytes + 255) & ~size_t(255)) + p.counter_bytes;
  return need <= B200Q_NOALLOC_SCRATCH_BYTES ? need : size_t(B200Q_NOALLOC_SCRATCH_BYTES) + 1;
}
}  // namespace

extern "C" {

int b200q_w8a16_linear_noalloc(const void* x, int x_dtype, int64_t ldx, const uint8_t* w,
                               int64_t ldw, const float* w_scale, const void* bias, int bias_dtype,
                               int act, void* out, int out_dtype, int64_t ldo, int64_t M, int64_t N,
                               int64_t K, void* stream) {
  if (!w8a16_args_valid(x, x_dtype, ldx, w, ldw, bias, bias_dtype, act, out, out_dtype, ldo, M, N, K))
    return B200Q_ERR_INVALID;
  const DeviceInfo* d = current_device();
  if (!d) return B200Q_ERR_UNSUPPORTED;
  const size_t need = noalloc_route_bytes(d, x, x_dtype, ldx, w, ldw, M, N, K);
  if (need > B200Q_NOALLOC_SCRATCH_BYTES) return B200Q_ERR_TOO_LARGE;
  void* scratch = nullptr;
  if (need) {
    const int st = noalloc_scratch(&scratch);
    if (st != B200Q_OK) return st;
  }
  // Nothing in the array needs clearing by this entry: the split-K route clears
  // its tile counters on `stream` before the kernel and every split writes its
  // partial slice before it is read; the planes pass writes the planes and
  // plane scales of every token the GEMM's epilogue uses (the padding rows of a
  // token tile feed only accumulator columns that are never read).
  return w8a16_linear_impl(x, x_dtype, ldx, w, ldw, w_scale, bias, bias_dtype, act, out,
                           out_dtype, ldo, M, N, K, scratch,
                           need ? size_t(B200Q_NOALLOC_SCRATCH_BYTES) : 0, false, stream);
}

int b200q_fp8_decode(const uint8_t* src, int64_t n, int fp8_kind, void* dst, int out_dtype,
                     void* stream) {
  if (!src || !dst || n < 0 || (fp8_kind != B200Q_FP8_E4M3 && fp8_kind != B200Q_FP8_E5M2) ||
      (out_dtype != B200Q_BF16 && out_dtype != B200Q_F16 && out_dtype != B200Q_F32))
    return B200Q_ERR_INVALID;
  const DeviceInfo* d = current_device();
  if (!d) return B200Q_ERR_UNSUPPORTED;
  if (n == 0) return B200Q_OK;
  fp8_decode_kernel<<<grid_for(n, 256, d), 256, 0, static_cast<cudaStream_t>(stream)>>>(src, n, fp8_kind, dst, out_dtype);
  return finish_launch();
}

}  // extern "C"
