// Host side of the C ABI declared in include/busfill.h: argument checks,
// TMA descriptor encoding, the choice of the K split (cluster size), the
// per-(device, stream) error words and the kernel launches (programmatic
// dependent launch by default).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <map>
#include <mutex>
#include <type_traits>
#include <utility>

#include "busfill.h"
#include "decode_gemm.cuh"
#include "prefill_gemm.cuh"
#include "prefill_pair_gemm.cuh"
#include "sweep_gemm.cuh"
#include "dequant.cuh"

using namespace busfill;

// Scratch of busfill_gemm_q4k_noalloc: the device error word and the first
// failure record, 256 bytes on every GPU that loads this library, held until
// the process exits. Host code must not use this name as a pointer: in host
// code it is only a stand-in for the device array, so the device address is
// looked up with cudaGetSymbolAddress (static_scratch()).
constexpr size_t kStaticScratchBytes = 256;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

namespace {

constexpr int kVersion = 100;  // 0.1.0
// detail word of the last device failure read by busfill_stream_status_ex
std::atomic<unsigned> g_last_detail{0};
std::atomic<int> g_use_pdl{1};
std::atomic<int> g_force_ksplit{0};  // 0 = automatic
// Batch size from which GEMMs take the prefill kernel (one pass over the
// weights for all rows) instead of the decode kernel (64 rows a launch).
// 0 = automatic:
//  * with the stream-K workspace (plain GEMMs): M > kStreamKMinM, or M > 32
//    when N <= K and K >= kPrefillMinK. Measured on B200 (Q4_K, us, decode vs
//    prefill, M = 33 / 64): K = N = 5120 14.2 / 14.5 vs 15.1 / 15.8; N = 5120,
//    K = 8192 18.8 / 19.2 vs 19.7 / 20.1; N = 5120, K = 17408 32.1 / 32.5 vs
//    29.9 / 30.3; N = 10240, K = 5120 19.1 / 19.7 vs 23.0 / 24.1; at M = 96
//    the prefill kernel wins on every shape (17.5 vs 25.0 at 5120^2).
//  * without it (SwiGLU pairs, the no-allocation entry point, a first call
//    inside a graph capture): M >= 128 and at least kPrefillMinItems work
//    items, since whole items go one per SM (measured: M = 128, N = 5120,
//    K = 17408 takes 157 us as 20 items, 93 us as four decode launches).
constexpr int kStreamKMinM = 64;
constexpr int kPrefillMinK = 12288;
constexpr int kPrefillMinItems = 64;
std::atomic<int> g_prefill_min_m{0};

// Batch rows per prefill work item (prefill_gemm.cuh, Geo): 256 (one weight
// tile, MMA N = 256, half the dequant per flop) from kWideMinM rows, else 128
// (two weight tiles); SwiGLU pairs always 128 (gate and up accumulators).
// BUSFILL_OPT_PREFILL_BATCH_TILE forces 128 or 256.
constexpr int kWideMinM = 256;
std::atomic<int> g_prefill_bt{0};

int prefill_bt(int M, bool swiglu) {
  if (swiglu) return 128;
  const int forced = g_prefill_bt.load();
  if (forced) return forced;
  return M >= kWideMinM ? 256 : 128;
}

// CTA pairs (prefill_pair_gemm.cuh: items of 256 weight rows x 256 batch
// rows on the two CTAs of a cluster, each loading half of the batch rows):
// by default from kPairMinM rows (measured on B200, us one CTA / pairs:
// M = 128, N = 17408, K = 5120 37.7 / 42.3; M = 160 56.7 / 43.6; M = 224
// 58.9 / 46.5; N = 5120, K = 17408, M = 192 51.8 / 40.1);
// BUSFILL_OPT_PREFILL_PAIR 1 forces them for every prefill GEMM but the
// SwiGLU pairs, 2 turns them off.
constexpr int kPairMinM = 129;
std::atomic<int> g_prefill_pair{0};
std::atomic<int> g_sweep_ctas{0};   // BUSFILL_OPT_SWEEP_CTAS: 0 = one CTA per SM
std::atomic<int> g_sweep_unmet{0};  // BUSFILL_OPT_SWEEP_UNMET_DEP (failure-detection tests)

bool prefill_pairs(int M, bool swiglu) {
  if (swiglu) return false;
  const int mode = g_prefill_pair.load();
  if (mode == 1) return true;
  if (mode == 2) return false;
  return M >= kPairMinM;
}

// work items of a prefill launch: weight-row groups x batch tiles
long long prefill_items(int M, int N, bool swiglu) {
  if (prefill_pairs(M, swiglu)) return (long long)((N + 255) / 256) * ((M + 255) / 256);
  const int bt = prefill_bt(M, swiglu);
  const int item_rows = swiglu ? kTileRows : bt == 128 ? 2 * kTileRows : kTileRows;  // SwiGLU: gate tile j + up tile j
  return (long long)((N + item_rows - 1) / item_rows) * ((M + bt - 1) / bt);
}

bool use_prefill(int M, int N, int K, bool swiglu = false, bool stream_k = false) {
  const int forced = g_prefill_min_m.load();
  if (forced > 0) return M >= forced;
  if (stream_k && !swiglu) return M > kStreamKMinM || (M > 32 && N <= K && K >= kPrefillMinK);
  // SwiGLU pairs: the decode kernel takes them 32 rows a launch; one fused
  // prefill launch of whole items is faster from M = 33 (N = 17408, K = 5120,
  // M = 64: 70 us as two decode launches; M = 96: 104 us as three; one
  // prefill launch, 54 us at M = 128)
  if (swiglu) return M > 32 && prefill_items(M, N, swiglu) >= kPrefillMinItems;
  return M >= 128 && prefill_items(M, N, swiglu) >= kPrefillMinItems;
}

// ---------------------------------------------------------------------------
// device properties (cached)
// ---------------------------------------------------------------------------
struct DeviceInfo {
  int sm_count = 0;
  int major = 0, minor = 0;
  bool ok = false;
};

std::mutex g_mu;
std::map<int, DeviceInfo> g_devices;

int current_device(DeviceInfo* out, int* dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return BUSFILL_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_devices.find(dev);
  if (it == g_devices.end()) {
    DeviceInfo di;
    if (cudaDeviceGetAttribute(&di.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&di.major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&di.minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
      return BUSFILL_ERR_CUDA;
    di.ok = (di.major == 10 && di.minor == 0);  // the kernels are built for sm_100a only
    it = g_devices.emplace(dev, di).first;
  }
  *out = it->second;
  *dev_out = dev;
  return it->second.ok ? BUSFILL_OK : BUSFILL_ERR_UNSUPPORTED_DEVICE;
}

// ---------------------------------------------------------------------------
// TMA descriptors (driver entry point fetched through the runtime, so the
// library does not link libcuda directly)
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

bool make_tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t dim0, uint64_t dim1,
                  uint64_t row_stride_bytes, uint32_t box0, uint32_t box1, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {dim0, dim1};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box0, box1};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Activations [rows, K] fp16 row-major seen as 3-D (64 values, rows, K/64
// chunks) so that one box brings `chunks` consecutive 64-value chunks of
// `box_rows` rows, landing chunk-major with the 128-byte swizzle.
bool make_tmap_act3d(CUtensorMap* m, const void* base, uint64_t rows, uint64_t K, uint32_t box_rows,
                     uint32_t chunks) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {64, rows, K / 64};
  const cuuint64_t strides[2] = {K * 2, 128};
  const cuuint32_t box[3] = {64, box_rows, chunks};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ---------------------------------------------------------------------------
// per-(device, stream) device words: [0] error bits, [1] first failure record.
// Zeroed at allocation; busfill_stream_status clears them after a failure.
// ---------------------------------------------------------------------------
constexpr size_t kErrorWordsBytes = 256;

std::map<std::pair<int, cudaStream_t>, unsigned*> g_err;
// device allocations this library made on its own (error words, stream-K
// workspaces; not busfill_ipc_alloc), for busfill_internal_allocations
std::atomic<unsigned> g_internal_allocs{0};

// true if `s` is capturing a graph (or the query failed): no allocation then,
// since a cudaMalloc would invalidate the capture
bool capturing(cudaStream_t s) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cs) != cudaSuccess) {
    cudaGetLastError();
    return true;
  }
  return cs != cudaStreamCaptureStatusNone;
}

int get_error_words(int dev, cudaStream_t s, unsigned** out) {
  // caller holds g_mu
  unsigned*& w = g_err[{dev, s}];
  if (!w) {
    // the first call on a stream makes its words; inside a graph capture that
    // would end the capture, so it fails cleanly instead
    if (capturing(s)) return BUSFILL_ERR_ALLOC;
    if (cudaMalloc(&w, kErrorWordsBytes) != cudaSuccess) {
      cudaGetLastError();
      w = nullptr;
      return BUSFILL_ERR_ALLOC;
    }
    ++g_internal_allocs;
    if (cudaMemsetAsync(w, 0, kErrorWordsBytes, s) != cudaSuccess) return BUSFILL_ERR_CUDA;
  }
  *out = w;
  return BUSFILL_OK;
}

// The prefill kernel's stream-K partial tiles: two fp32 tiles of 32768
// values (batch tile x item rows) per CTA, one workspace per (device, stream) so that
// GEMMs on different streams never share one. Allocated on first use; never
// while the stream is capturing a graph (an allocation would end the
// capture), in which case the kernel runs without stream-K.
std::map<std::pair<int, cudaStream_t>, float*> g_part;

float* prefill_workspace(int dev, cudaStream_t s, int sm_count) {
  std::lock_guard<std::mutex> lk(g_mu);
  float*& w = g_part[{dev, s}];
  if (!w) {
    if (capturing(s)) return nullptr;
    if (cudaMalloc(&w, (size_t)2 * sm_count * prefill::kPartElems * sizeof(float)) != cudaSuccess) {
      cudaGetLastError();
      w = nullptr;
    } else {
      ++g_internal_allocs;
    }
  }
  return w;
}

// The layer-sweep kernel's workspace, one per (device, stream): its counter
// words (zeroed here; the kernel leaves them zero) and the partial tiles of
// up to sm_count CTAs per op. Never made while the stream is capturing.
std::map<std::pair<int, cudaStream_t>, unsigned*> g_sweep;

unsigned* sweep_workspace(int dev, cudaStream_t s, int sm_count) {
  // caller holds g_mu
  unsigned*& w = g_sweep[{dev, s}];
  if (!w) {
    if (capturing(s)) return nullptr;
    const size_t bytes = (size_t)sweep::kFlagWords * 4 + (size_t)sweep::kMaxOps * sm_count * sweep::kSlotsPerCta *
                                                               kTileRows * sweep::kMaxNB * sizeof(float);
    if (cudaMalloc(&w, bytes) != cudaSuccess) {
      cudaGetLastError();
      w = nullptr;
      return nullptr;
    }
    ++g_internal_allocs;
    if (cudaMemsetAsync(w, 0, (size_t)sweep::kFlagWords * 4, s) != cudaSuccess) {
      cudaGetLastError();
      cudaFree(w);
      w = nullptr;
    }
  }
  return w;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

cudaError_t launch(const void* func, dim3 grid, dim3 block, size_t smem, cudaStream_t s, void** args, bool pdl,
                   int cluster = 1) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = (unsigned)cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelExC(&cfg, func, args);
}

// ---------------------------------------------------------------------------
// decode GEMM launch
// ---------------------------------------------------------------------------
template <WFmt FMT, int NB, typename OutT, bool SW = false, bool GA = false>
const void* decode_kernel_ptr() {
  return reinterpret_cast<const void*>(decode_gemm_kernel<FMT, NB, OutT, SW, GA>);
}

// Raise the kernel's dynamic shared memory limit, once per device.
template <WFmt FMT, int NB, typename OutT, bool SW = false, bool GA = false>
bool decode_smem_attr(int dev) {
  static std::once_flag once[64];
  static cudaError_t err[64];
  std::call_once(once[dev & 63], [&] {
    err[dev & 63] = cudaFuncSetAttribute(decode_kernel_ptr<FMT, NB, OutT, SW, GA>(),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, DecodeSmem<NB, FMT>::kAlloc);
  });
  return err[dev & 63] == cudaSuccess;
}

// Largest number of clusters of `csize` CTAs that can be resident at once
// (one CTA per SM); cached per device, kernel and cluster size.
template <WFmt FMT, int NB, typename OutT>
int max_active_clusters(int dev, int csize, int sm_count) {
  static std::mutex mu;
  static std::map<std::pair<int, int>, int> cache;
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find({dev, csize});
  if (it != cache.end()) return it->second;
  int v = sm_count / csize;
  if (!decode_smem_attr<FMT, NB, OutT>(dev)) return v;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(csize * std::max(1, sm_count / csize)));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = DecodeSmem<NB, FMT>::kAlloc;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, decode_kernel_ptr<FMT, NB, OutT>(), &cfg) == cudaSuccess && n > 0)
    v = std::min(v, n);
  else
    cudaGetLastError();
  cache[{dev, csize}] = v;
  return v;
}

struct DecodeSchedule {
  int csize = 1;      // CTAs per cluster = K split of every tile
  int nclusters = 1;  // clusters in the grid
};

// Pick the K split c (1..max_cluster) with the shortest estimated time. A
// cluster takes R = ceil(T / G) tiles in turn, each `segs` x ceil(S / c)
// units (segs = 2 for SwiGLU gate/up pairs), so a CTA runs U = R x segs x
// ceil(S / c) units. The estimate, fitted to CUDA-event times of Q4_K GEMMs
// on B200 (M = 1 and 32; N, K in {5120, 8192, 10240, 17408}; every c):
//   t = 7.2 us + 0.51 us x U + 4 us x (R - 1)
// A unit costs ~0.5 us once the dequant pipeline runs, whatever the K split;
// a launch costs ~7 us (set-up, the first boxes, the last tile's reduction
// and exit); every further round of tiles adds a drain and refill of the
// pipeline and a cluster reduction (N = 10240, K = 5120, M = 32: 15.5 us as
// 80 one-CTA tiles, 18.3 us as two rounds of 3-CTA clusters; a bandwidth-only
// model preferred the latter). Ties go to the smaller c.
template <WFmt FMT, int NB, typename OutT>
DecodeSchedule choose_schedule(int dev, int T, int S, int sm_count, int segs) {
  constexpr double kLaunchUs = 7.2, kUnitUs = 0.51, kRoundUs = 4.0;
  DecodeSchedule best;
  double best_us = 1e300;
  const int forced = g_force_ksplit.load();
  const int cmax = std::min(max_cluster<NB>(), S);
  for (int c = 1; c <= cmax; ++c) {
    if (forced > 0 && forced <= cmax && c != forced) continue;
    const int cap = c == 1 ? sm_count : max_active_clusters<FMT, NB, OutT>(dev, c, sm_count);
    const int ncl = std::min(T, cap);
    if (ncl < 1) continue;
    const long long rounds = (T + ncl - 1) / ncl;
    const long long units = rounds * segs * ((S + c - 1) / c);
    const double us = kLaunchUs + kUnitUs * (double)units + kRoundUs * (double)(rounds - 1);
    if (us < best_us - 1e-9) {
      best_us = us;
      best.csize = c;
      best.nclusters = ncl;
    }
  }
  return best;
}

template <WFmt FMT, int NB, typename OutT, bool SW = false, bool GA = false>
int launch_decode_nb(const DeviceInfo& di, const CUtensorMap& tw, const CUtensorMap& tws, const CUtensorMap& ta,
                     const DecodeParams& p, cudaStream_t s) {
  const void* kern = decode_kernel_ptr<FMT, NB, OutT, SW, GA>();
  constexpr int smem = DecodeSmem<NB, FMT>::kAlloc;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!decode_smem_attr<FMT, NB, OutT, SW, GA>(dev)) return BUSFILL_ERR_LAUNCH;
  const int grid = p.nclusters * p.csize;
  void* args[] = {const_cast<CUtensorMap*>(&tw), const_cast<CUtensorMap*>(&tws), const_cast<CUtensorMap*>(&ta),
                  const_cast<DecodeParams*>(&p)};
  if (launch(kern, dim3(grid), dim3(kThreads), smem, s, args, g_use_pdl.load() != 0, p.csize) != cudaSuccess) {
    cudaGetLastError();
    return BUSFILL_ERR_LAUNCH;
  }
  return BUSFILL_OK;
}

// Checks shared by every GEMM entry point.
template <WFmt FMT>
int check_gemm_args(const uint8_t* w, const uint16_t* ws, const uint16_t* a, const void* c, int M, int N, int K) {
  if (!w || !a || !c || ((FMT == WFmt::Q4_0 || FMT == WFmt::Q6K) && !ws)) return BUSFILL_ERR_INVALID_ARG;
  if (M < 1 || N < 1 || K < kUnitK || K % kUnitK != 0) return BUSFILL_ERR_SHAPE;
  if (FMT == WFmt::Q6K && N % 8 != 0) return BUSFILL_ERR_SHAPE;  // the d plane's rows: 16-byte multiples
  if (!aligned16(w) || !aligned16(a) || (ws && !aligned16(ws))) return BUSFILL_ERR_ALIGNMENT;
  return BUSFILL_OK;
}

// Launches the decode kernel once per 32 rows of A; `error` points at the two
// device words the kernels report failures to.
// With `w_up` (144-byte formats only) the GEMM is the SwiGLU pair:
// C = silu(A deq(w)^T) * (A deq(w_up)^T).
template <WFmt FMT, typename OutT>
int run_decode(const DeviceInfo& di, int dev, const uint8_t* w, const uint16_t* ws, const uint16_t* a, void* c,
               int M, int N, int K, unsigned* error, cudaStream_t s, const uint8_t* w_up = nullptr,
               const busfill_gather* gather = nullptr) {
  const int S = K / kUnitK;
  const int T = (N + kTileRows - 1) / kTileRows;
  const int swiglu = w_up ? 1 : 0;

  CUtensorMap tw, tws, ta;
  std::memset(&tws, 0, sizeof(tws));
  if constexpr (aos_rows<FMT>()) {
    // whole block rows: 144 bytes per 256 values (one block_q4_K, eight
    // block_q4_0) or 176 (one block_q5_K)
    constexpr int ub = unit_row_bytes<FMT>();
    const uint64_t row = (uint64_t)S * ub;
    if (!make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, row, (uint64_t)N, row, ub, kTileRows,
                      CU_TENSOR_MAP_SWIZZLE_NONE))
      return BUSFILL_ERR_CUDA;
    tws = tw;  // the up projection's map with SwiGLU, else unused
    if (swiglu && !make_tmap_2d(&tws, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_up, row, (uint64_t)N, row, ub,
                                kTileRows, CU_TENSOR_MAP_SWIZZLE_NONE))
      return BUSFILL_ERR_CUDA;
    // Q6_K: the d plane [S][N], one box of a tile's 128 d per unit
    if (FMT == WFmt::Q6K && !make_tmap_2d(&tws, CU_TENSOR_MAP_DATA_TYPE_UINT16, ws, (uint64_t)N, (uint64_t)S,
                                          (uint64_t)N * 2, kTileRows, 1, CU_TENSOR_MAP_SWIZZLE_NONE))
      return BUSFILL_ERR_CUDA;
  } else {
    if (swiglu) return BUSFILL_ERR_INVALID_ARG;
    if (!make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2, 128,
                      kTileRows, CU_TENSOR_MAP_SWIZZLE_128B))
      return BUSFILL_ERR_CUDA;
    if (!make_tmap_2d(&tws, CU_TENSOR_MAP_DATA_TYPE_UINT16, ws, (uint64_t)K / 32, (uint64_t)N, (uint64_t)K / 16, 8,
                      kTileRows, CU_TENSOR_MAP_SWIZZLE_NONE))
      return BUSFILL_ERR_CUDA;
  }

  // plain GEMMs take up to 64 batch rows a launch (one pass over the weights
  // for M <= 64); the fused SwiGLU and gathered GEMMs 32
  const int step = (swiglu || gather) ? 32 : 64;
  for (int m0 = 0; m0 < M; m0 += step) {
    const int mc = std::min(step, M - m0);
    const int nb = mc <= 16 ? 16 : mc <= 32 ? 32 : 64;
    const DecodeSchedule sch = nb == 16   ? choose_schedule<FMT, 16, OutT>(dev, T, S, di.sm_count, 1 + swiglu)
                               : nb == 32 ? choose_schedule<FMT, 32, OutT>(dev, T, S, di.sm_count, 1 + swiglu)
                                          : choose_schedule<FMT, 64, OutT>(dev, T, S, di.sm_count, 1);
    const uint16_t* a_chunk = a + (size_t)m0 * K;
    if (!make_tmap_act3d(&ta, a_chunk, (uint64_t)mc, (uint64_t)K, (uint32_t)nb, kChunksPerUnit))
      return BUSFILL_ERR_CUDA;
    DecodeParams p;
    p.gather = GatherArgs{};
    if (gather) {
      // rows m0.. of every rank's full output; the first launch waits for the
      // activations' flags, the last one raises this call's flags
      p.gather.npeers = gather->npeers;
      p.gather.col_off = gather->col_off;
      p.gather.ldc = gather->ldc;
      for (int q = 0; q < gather->npeers; ++q) {
        p.gather.out[q] = reinterpret_cast<OutT*>(gather->out[q]) + (size_t)m0 * gather->ldc;
        p.gather.flag[q] = gather->flag[q];
      }
      p.gather.signal = (m0 + step >= M) ? 1 : 0;
      if (m0 == 0 && gather->wait && gather->nwait > 0) {
        p.gather.wait = gather->wait;
        p.gather.wait_gen = gather->wait_gen;
        p.gather.nwait = gather->nwait;
        for (int r = 0; r < gather->nwait; ++r) p.gather.wait_tiles[r] = gather->wait_tiles[r];
      }
    }
    p.c = reinterpret_cast<OutT*>(c) + (size_t)m0 * N;
    p.error = error;
    p.M = mc;
    p.N = N;
    p.K = K;
    p.tiles = T;
    p.units_per_tile = S;
    p.csize = sch.csize;
    p.nclusters = sch.nclusters;
    int st = BUSFILL_ERR_INVALID_ARG;
    if constexpr (FMT == WFmt::Q4K && std::is_same<OutT, __half>::value) {
      // the SwiGLU and gathered entry points are Q4_K
      if (swiglu && gather)
        st = nb == 16 ? launch_decode_nb<FMT, 16, OutT, true, true>(di, tw, tws, ta, p, s)
                      : launch_decode_nb<FMT, 32, OutT, true, true>(di, tw, tws, ta, p, s);
      else if (swiglu)
        st = nb == 16 ? launch_decode_nb<FMT, 16, OutT, true>(di, tw, tws, ta, p, s)
                      : launch_decode_nb<FMT, 32, OutT, true>(di, tw, tws, ta, p, s);
      else if (gather)
        st = nb == 16 ? launch_decode_nb<FMT, 16, OutT, false, true>(di, tw, tws, ta, p, s)
                      : launch_decode_nb<FMT, 32, OutT, false, true>(di, tw, tws, ta, p, s);
    }
    if (!swiglu && !gather)
      st = nb == 16   ? launch_decode_nb<FMT, 16, OutT>(di, tw, tws, ta, p, s)
           : nb == 32 ? launch_decode_nb<FMT, 32, OutT>(di, tw, tws, ta, p, s)
                      : launch_decode_nb<FMT, 64, OutT>(di, tw, tws, ta, p, s);
    if (st != BUSFILL_OK) return st;
  }
  return BUSFILL_OK;
}

// ---------------------------------------------------------------------------
// prefill GEMM launch
// ---------------------------------------------------------------------------
// The items that a stream-K prefill launch of g CTAs over t = items x s units
// splits between CTAs (prefill_gemm.cuh: the CTA ranges and partial slots).
void split_items(long long t, int s, int g, prefill::SplitItems* out) {
  out->n = 0;
  for (int cb = 1; cb < g; ++cb) {
    const long long gb = prefill::first_unit(t, cb, g);
    if (gb % s == 0) continue;                       // a boundary on an item edge splits nothing
    const int it = (int)(gb / s);
    const int c_lo = prefill::cta_of_unit(t, (long long)it * s, g);
    if (c_lo != cb - 1) continue;                    // an earlier boundary of the same item
    const int c_hi = prefill::cta_of_unit(t, (long long)(it + 1) * s - 1, g);
    const int slot_lo = 2 * c_lo + (prefill::first_unit(t, c_lo, g) / s == it ? 0 : 1);
    out->e[out->n++] = make_int4(it, c_lo, c_hi, slot_lo);
  }
}

// `part`: the stream's partial-tile workspace (stream-K), or nullptr for whole
// items round-robin; SwiGLU pairs always take whole items. BT: batch tile.
template <WFmt FMT, typename OutT, int BT>
int run_prefill_bt(const DeviceInfo& di, int dev, const uint8_t* w, const uint16_t* ws, const uint16_t* a, void* c,
                   int M, int N, int K, unsigned* error, cudaStream_t s, const uint8_t* w_up, float* part) {
  constexpr int kItemRows = prefill::Geo<BT>::kItemRows;
  const int S = K / kUnitK;
  const int swiglu = w_up ? 1 : 0;
  if (swiglu && BT != 128) return BUSFILL_ERR_INVALID_ARG;
  CUtensorMap tw, tws, ta;
  std::memset(&tws, 0, sizeof(tws));
  if constexpr (aos_rows<FMT>()) {
    // one box of the item's rows per unit, or with SwiGLU one 128-row box from each matrix
    constexpr int ub = unit_row_bytes<FMT>();
    const uint64_t row = (uint64_t)S * ub;
    const uint32_t box_rows = swiglu ? kTileRows : kItemRows;
    if (!make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, row, (uint64_t)N, row, ub, box_rows,
                      CU_TENSOR_MAP_SWIZZLE_NONE))
      return BUSFILL_ERR_CUDA;
    tws = tw;
    if (swiglu && !make_tmap_2d(&tws, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_up, row, (uint64_t)N, row, ub,
                                box_rows, CU_TENSOR_MAP_SWIZZLE_NONE))
      return BUSFILL_ERR_CUDA;
    if (FMT == WFmt::Q6K && !make_tmap_2d(&tws, CU_TENSOR_MAP_DATA_TYPE_UINT16, ws, (uint64_t)N, (uint64_t)S,
                                          (uint64_t)N * 2, kItemRows, 1, CU_TENSOR_MAP_SWIZZLE_NONE))
      return BUSFILL_ERR_CUDA;
  } else {
    if (swiglu) return BUSFILL_ERR_INVALID_ARG;
    if (!make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2, 128,
                      kItemRows, CU_TENSOR_MAP_SWIZZLE_128B))
      return BUSFILL_ERR_CUDA;
    if (!make_tmap_2d(&tws, CU_TENSOR_MAP_DATA_TYPE_UINT16, ws, (uint64_t)K / 32, (uint64_t)N, (uint64_t)K / 16, 8,
                      kItemRows, CU_TENSOR_MAP_SWIZZLE_NONE))
      return BUSFILL_ERR_CUDA;
  }
  if (!make_tmap_act3d(&ta, a, (uint64_t)M, (uint64_t)K, BT, prefill::Geo<BT>::kXChunks)) return BUSFILL_ERR_CUDA;

  const void* kern = reinterpret_cast<const void*>(prefill_gemm_kernel<FMT, OutT, BT>);
  {
    static std::once_flag once[64];
    static cudaError_t err[64];
    std::call_once(once[dev & 63], [&] {
      err[dev & 63] =
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, prefill::Smem<FMT, BT>::kAlloc);
    });
    if (err[dev & 63] != cudaSuccess) return BUSFILL_ERR_LAUNCH;
  }
  prefill::Params p;
  p.c = c;
  p.error = error;
  p.M = M;
  p.N = N;
  p.K = K;
  p.pairs = swiglu ? (N + kTileRows - 1) / kTileRows : (N + kItemRows - 1) / kItemRows;
  p.swiglu = swiglu;
  p.btiles = (M + BT - 1) / BT;
  p.units = S;
  const long long items = (long long)p.pairs * p.btiles;
  const long long units = items * S;
  if (units > INT32_MAX) return BUSFILL_ERR_SHAPE;   // the kernel counts units in an int
  p.part = swiglu ? nullptr : part;
  p.gate_mul = 0;
  const int grid = p.part ? (int)std::min<long long>(std::min<long long>(units, di.sm_count), prefill::kMaxSplitItems + 1)
                           : (int)std::min<long long>(items, di.sm_count);
  void* args[] = {&tw, &tws, &ta, &p};
  if (launch(kern, dim3(grid), dim3(prefill::kThreads), prefill::Smem<FMT, BT>::kAlloc, s, args,
             g_use_pdl.load() != 0) != cudaSuccess) {
    cudaGetLastError();
    return BUSFILL_ERR_LAUNCH;
  }
  prefill::SplitItems si;
  if (p.part) split_items(units, S, grid, &si);
  if (p.part && si.n > 0) {
    // items split between CTAs: their partial tiles summed in CTA order
    const float* cpart = p.part;
    OutT* cc = reinterpret_cast<OutT*>(c);
    int m = M, n = N, bts = p.btiles;
    void* rargs[] = {&cpart, &cc, &m, &n, &bts, &si};
    const int rows = std::min(M, BT);
    constexpr int kRowsPerBlock = 256 / (kItemRows / 4);
    if (launch(reinterpret_cast<const void*>(prefill_reduce_kernel<OutT, BT>),
               dim3(si.n, (rows + kRowsPerBlock - 1) / kRowsPerBlock), dim3(256), 0, s, rargs,
               g_use_pdl.load() != 0) != cudaSuccess) {
      cudaGetLastError();
      return BUSFILL_ERR_LAUNCH;
    }
  }
  return BUSFILL_OK;
}

// CTA pairs this device runs at once for the pair kernel (one CTA per SM);
// the launch never asks for more, so that no pair waits for a second wave
template <WFmt FMT, typename OutT>
int pair_capacity(int dev, int sm_count) {
  static std::once_flag once[64];
  static int cap[64];
  std::call_once(once[dev & 63], [&] {
    const void* kern = reinterpret_cast<const void*>(prefill_pair_kernel<FMT, OutT>);
    int n = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             prefill_pair::Smem<FMT>::kAlloc) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * (sm_count / 2));
      cfg.blockDim = dim3(prefill_pair::kThreads);
      cfg.dynamicSmemBytes = prefill_pair::Smem<FMT>::kAlloc;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = 2;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();
    cap[dev & 63] = std::min(n, sm_count / 2);
  });
  return cap[dev & 63];
}

// Pairs for whole items: when the item count has a divisor g within 1/8 of
// the pairs that fit (cap), g pairs take items/g whole items each and no item
// is split: no partial tiles, no fix-up launch (at M = 512, N = 17408 the
// fix-up took ~13 us of a ~74 us GEMM under ncu), for at most 1/8 of the SMs.
// 0 when no such divisor exists (stream-K then).
int pair_whole_grid(long long items, int cap) {
  if (items < cap) return 0;
  for (int g = cap; g >= cap - cap / 8 && g > 0; --g)
    if (items % g == 0) return g;
  return 0;
}

// The pair kernel: items of 256 weight rows x 256 batch rows, stream-K over
// the pairs when `part` is given, else whole items round-robin. gate_mul: C
// holds the up projection and receives silu(A W^T) * C (the SwiGLU pair's
// second pass).
template <WFmt FMT, typename OutT>
int run_prefill_pair(const DeviceInfo& di, int dev, const uint8_t* w, const uint16_t* ws, const uint16_t* a, void* c,
                     int M, int N, int K, unsigned* error, cudaStream_t s, float* part, int gate_mul = 0) {
  const int S = K / kUnitK;
  CUtensorMap tw, tws, ta;
  std::memset(&tws, 0, sizeof(tws));
  if constexpr (aos_rows<FMT>()) {
    constexpr int ub = unit_row_bytes<FMT>();
    const uint64_t row = (uint64_t)S * ub;
    if (!make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, row, (uint64_t)N, row, ub, kTileRows,
                      CU_TENSOR_MAP_SWIZZLE_NONE))
      return BUSFILL_ERR_CUDA;
    tws = tw;
    if (FMT == WFmt::Q6K && !make_tmap_2d(&tws, CU_TENSOR_MAP_DATA_TYPE_UINT16, ws, (uint64_t)N, (uint64_t)S,
                                          (uint64_t)N * 2, kTileRows, 1, CU_TENSOR_MAP_SWIZZLE_NONE))
      return BUSFILL_ERR_CUDA;
  } else {
    if (!make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2, 128,
                      kTileRows, CU_TENSOR_MAP_SWIZZLE_128B))
      return BUSFILL_ERR_CUDA;
    if (!make_tmap_2d(&tws, CU_TENSOR_MAP_DATA_TYPE_UINT16, ws, (uint64_t)K / 32, (uint64_t)N, (uint64_t)K / 16, 8,
                      kTileRows, CU_TENSOR_MAP_SWIZZLE_NONE))
      return BUSFILL_ERR_CUDA;
  }
  if (!make_tmap_act3d(&ta, a, (uint64_t)M, (uint64_t)K, 128, 2)) return BUSFILL_ERR_CUDA;
  const int cap = pair_capacity<FMT, OutT>(dev, di.sm_count);
  if (cap < 1) return BUSFILL_ERR_LAUNCH;

  prefill::Params p;
  p.c = c;
  p.error = error;
  p.M = M;
  p.N = N;
  p.K = K;
  p.pairs = (N + prefill_pair::kItemRows - 1) / prefill_pair::kItemRows;
  p.btiles = (M + prefill_pair::kBatchTile - 1) / prefill_pair::kBatchTile;
  p.units = S;
  p.swiglu = 0;
  p.gate_mul = gate_mul;
  const long long items = (long long)p.pairs * p.btiles;
  const long long units = items * S;
  if (units > INT32_MAX) return BUSFILL_ERR_SHAPE;   // the kernel counts units in an int
  const int whole = pair_whole_grid(items, cap);
  if (whole) part = nullptr;
  p.part = part;
  const int pairs = whole ? whole
                    : part ? (int)std::min<long long>(std::min<long long>(units, cap), prefill::kMaxSplitItems + 1)
                           : (int)std::min<long long>(items, cap);
  const void* kern = reinterpret_cast<const void*>(prefill_pair_kernel<FMT, OutT>);
  void* args[] = {&tw, &tws, &ta, &p};
  if (launch(kern, dim3(2 * pairs), dim3(prefill_pair::kThreads), prefill_pair::Smem<FMT>::kAlloc, s, args,
             g_use_pdl.load() != 0, 2) != cudaSuccess) {
    cudaGetLastError();
    return BUSFILL_ERR_LAUNCH;
  }
  prefill::SplitItems si;
  if (part) split_items(units, S, pairs, &si);
  if (part && si.n > 0) {
    // items split between pairs: their partial tiles summed in pair order
    const float* cpart = part;
    OutT* cc = reinterpret_cast<OutT*>(c);
    int m = M, n = N, bts = p.btiles, gm = gate_mul;
    void* rargs[] = {&cpart, &cc, &m, &n, &bts, &gm, &si};
    const int rows = std::min(M, prefill_pair::kBatchTile);
    if (launch(reinterpret_cast<const void*>(prefill_pair_reduce_kernel<OutT>), dim3(si.n, (rows + 15) / 16),
               dim3(256), 0, s, rargs, g_use_pdl.load() != 0) != cudaSuccess) {
      cudaGetLastError();
      return BUSFILL_ERR_LAUNCH;
    }
  }
  return BUSFILL_OK;
}

template <WFmt FMT, typename OutT>
int run_prefill(const DeviceInfo& di, int dev, const uint8_t* w, const uint16_t* ws, const uint16_t* a, void* c,
                int M, int N, int K, unsigned* error, cudaStream_t s, const uint8_t* w_up = nullptr,
                float* part = nullptr) {
  if (prefill_pairs(M, w_up != nullptr))
    return run_prefill_pair<FMT, OutT>(di, dev, w, ws, a, c, M, N, K, error, s, part);
  if (prefill_bt(M, w_up != nullptr) == 256)
    return run_prefill_bt<FMT, OutT, 256>(di, dev, w, ws, a, c, M, N, K, error, s, w_up, part);
  return run_prefill_bt<FMT, OutT, 128>(di, dev, w, ws, a, c, M, N, K, error, s, w_up, part);
}

// Decode (M < prefill threshold) or prefill kernel for one GEMM.
template <WFmt FMT, typename OutT>
int run_gemm(const DeviceInfo& di, int dev, const uint8_t* w, const uint16_t* ws, const uint16_t* a, void* c, int M,
             int N, int K, unsigned* error, cudaStream_t s, const uint8_t* w_up = nullptr, bool may_alloc = true) {
  // SwiGLU pairs of more than 128 rows: two CTA-pair GEMMs, the up
  // projection into C, then the gate with an epilogue that writes silu(gate)
  // * C (the up values rounded to fp16 once); one fused launch takes whole
  // 128-row items and cannot use CTA pairs (the gate and up accumulators of a
  // row would sit in different CTAs). N = 17408, K = 5120, us fused / two
  // passes: M = 128 53.9 / 83.8; 160 99.7 / 85.2; 224 101.8 / 94.7.
  if (w_up && g_prefill_pair.load() != 2 && (g_prefill_pair.load() == 1 || M >= kPairMinM) &&
      use_prefill(M, N, K, true, false)) {
    float* part = may_alloc ? prefill_workspace(dev, s, di.sm_count) : nullptr;
    const int st = run_prefill_pair<FMT, OutT>(di, dev, w_up, ws, a, c, M, N, K, error, s, part, 0);
    if (st != BUSFILL_OK) return st;
    return run_prefill_pair<FMT, OutT>(di, dev, w, ws, a, c, M, N, K, error, s, part, 1);
  }
  // the stream-K workspace is only looked up (and made) for GEMMs that may use it
  const bool want_sk = may_alloc && !w_up && (g_prefill_min_m.load() > 0 || M > 32);
  float* part = want_sk ? prefill_workspace(dev, s, di.sm_count) : nullptr;
  if (use_prefill(M, N, K, w_up != nullptr, part != nullptr))
    return run_prefill<FMT, OutT>(di, dev, w, ws, a, c, M, N, K, error, s, w_up, part);
  return run_decode<FMT, OutT>(di, dev, w, ws, a, c, M, N, K, error, s, w_up);
}

// The gathered GEMM: its arguments checked, always the decode kernel.
template <WFmt FMT>
int gemm_gather_impl(const uint8_t* w, const uint8_t* w_up, bool swiglu, const uint16_t* a, int M, int N, int K,
                     const busfill_gather* g, cudaStream_t s) {
  if (!g) return BUSFILL_ERR_INVALID_ARG;
  if (g->npeers < 1 || g->npeers > kMaxPeers || g->col_off < 0 || N < 0 || g->ldc < g->col_off + N)
    return BUSFILL_ERR_SHAPE;
  if (g->nwait < 0 || g->nwait > kMaxPeers || (g->nwait > 0 && (!g->wait || !g->wait_gen)))
    return BUSFILL_ERR_INVALID_ARG;
  for (int q = 0; q < g->npeers; ++q)
    if (!g->out[q] || !g->flag[q]) return BUSFILL_ERR_INVALID_ARG;
  // A rank that owns no rows of this weight (fewer 128-row tiles than ranks)
  // computes and stores nothing and writes 0 tiles a call, which is what the
  // other ranks' consumers wait for from it: the call is a no-op.
  if (N == 0) return BUSFILL_OK;
  if (swiglu && !w_up) return BUSFILL_ERR_INVALID_ARG;
  int st = check_gemm_args<FMT>(w, nullptr, a, g->out[0], M, N, K);
  if (st != BUSFILL_OK) return st;
  if (w_up && !aligned16(w_up)) return BUSFILL_ERR_ALIGNMENT;
  DeviceInfo di;
  int dev = 0;
  st = current_device(&di, &dev);
  if (st != BUSFILL_OK) return st;
  unsigned* err = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    st = get_error_words(dev, s, &err);
  }
  if (st != BUSFILL_OK) return st;
  return run_decode<FMT, __half>(di, dev, w, nullptr, a, g->out[0], M, N, K, err, s, swiglu ? w_up : nullptr, g);
}

template <WFmt FMT, typename OutT>
int gemm_impl(const uint8_t* w, const uint16_t* ws, const uint16_t* a, void* c, int M, int N, int K,
              cudaStream_t s, const uint8_t* w_up = nullptr, bool swiglu = false) {
  int st = check_gemm_args<FMT>(w, ws, a, c, M, N, K);
  if (st != BUSFILL_OK) return st;
  if (swiglu && !w_up) return BUSFILL_ERR_INVALID_ARG;
  if (w_up && !aligned16(w_up)) return BUSFILL_ERR_ALIGNMENT;
  DeviceInfo di;
  int dev = 0;
  st = current_device(&di, &dev);
  if (st != BUSFILL_OK) return st;
  unsigned* err = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    st = get_error_words(dev, s, &err);
  }
  if (st != BUSFILL_OK) return st;
  return run_gemm<FMT, OutT>(di, dev, w, ws, a, c, M, N, K, err, s, w_up);
}

int grid_for(long long work, int sm_count) {
  const long long g = (work + 255) / 256;
  return (int)std::max<long long>(1, std::min<long long>(g, (long long)sm_count * 8));
}

// ---------------------------------------------------------------------------
// waiting for a gathered output outside a GEMM
// ---------------------------------------------------------------------------
struct WaitTiles {
  int n[kMaxPeers];
};
// One CTA: it is every call's last arrival, so only the call count
// (wait_gen[0]) moves; wait_gen[1] stays 0.
__global__ void __launch_bounds__(32, 1) gather_wait_kernel(const unsigned* wait, unsigned* wait_gen, int nwait,
                                                            WaitTiles tiles, unsigned* error) {
  const unsigned calls = *reinterpret_cast<volatile unsigned*>(wait_gen);
  bool got = true;
  if ((int)threadIdx.x < nwait) got = wait_flag_sys(wait + threadIdx.x, (calls + 1u) * (unsigned)tiles.n[threadIdx.x]);
  got = __all_sync(0xffffffffu, got);
  __syncwarp();
  if (threadIdx.x == 0) {
    if (!got) atomicOr(error, kErrActProducer);
    *wait_gen = calls + 1u;
  }
}

// ---------------------------------------------------------------------------
// statically allocated scratch (busfill_gemm_q4k_noalloc)
// ---------------------------------------------------------------------------
constexpr int kMaxDevices = 64;
uint8_t* g_static_ptr[kMaxDevices] = {};

// Device address of g_static_scratch on `dev`, which must be the current
// device. Looked up once per device; a failed lookup is retried next call.
int static_scratch(int dev, uint8_t** out) {
  if (dev < 0 || dev >= kMaxDevices) return BUSFILL_ERR_UNSUPPORTED_DEVICE;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_static_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p) {
      cudaGetLastError();
      return BUSFILL_ERR_CUDA;
    }
    g_static_ptr[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_static_ptr[dev];
  return BUSFILL_OK;
}

int gemm_q4k_static(const uint8_t* w, const uint16_t* a, uint16_t* c, int M, int N, int K, cudaStream_t s) {
  int st = check_gemm_args<WFmt::Q4K>(w, nullptr, a, c, M, N, K);
  if (st != BUSFILL_OK) return st;
  DeviceInfo di;
  int dev = 0;
  st = current_device(&di, &dev);
  if (st != BUSFILL_OK) return st;
  uint8_t* scratch = nullptr;
  st = static_scratch(dev, &scratch);
  if (st != BUSFILL_OK) return st;
  // the error words must start at zero; a previous call that gave up part way
  // may have left them set
  if (cudaMemsetAsync(scratch, 0, kStaticScratchBytes, s) != cudaSuccess) {
    cudaGetLastError();
    return BUSFILL_ERR_CUDA;
  }
  return run_gemm<WFmt::Q4K, __half>(di, dev, w, nullptr, a, c, M, N, K, reinterpret_cast<unsigned*>(scratch), s,
                                     nullptr, false);
}

// ---------------------------------------------------------------------------
// planar Q4_K: block rows rebuilt per call in a per-(device, stream) buffer
// ---------------------------------------------------------------------------
struct PlanarBuf {
  uint8_t* p = nullptr;
  size_t bytes = 0;
};
std::map<std::pair<int, cudaStream_t>, PlanarBuf> g_planar;

int planar_buffer(int dev, cudaStream_t s, size_t bytes, uint8_t** out) {
  std::lock_guard<std::mutex> lk(g_mu);
  PlanarBuf& b = g_planar[{dev, s}];
  if (b.bytes < bytes) {
    if (capturing(s)) return BUSFILL_ERR_ALLOC;
    if (b.p) {
      cudaFree(b.p);   // synchronizes the device: no kernel still reads the old rows
      b.p = nullptr;
      b.bytes = 0;
    }
    if (cudaMalloc(&b.p, bytes) != cudaSuccess) {
      cudaGetLastError();
      b.p = nullptr;
      return BUSFILL_ERR_ALLOC;
    }
    ++g_internal_allocs;
    b.bytes = bytes;
  }
  *out = b.p;
  return BUSFILL_OK;
}

int repack_q4k_planar_impl(const uint8_t* qs, const uint16_t* d, const uint16_t* dmin, const uint8_t* sc12,
                           uint8_t* blocks, int N, int K, cudaStream_t s) {
  if (!qs || !d || !dmin || !sc12 || !blocks) return BUSFILL_ERR_INVALID_ARG;
  if (N < 1 || K < kUnitK || K % kUnitK != 0) return BUSFILL_ERR_SHAPE;
  if (!aligned16(qs) || !aligned16(blocks) || (reinterpret_cast<uintptr_t>(d) & 1u) ||
      (reinterpret_cast<uintptr_t>(dmin) & 1u) || (reinterpret_cast<uintptr_t>(sc12) & 3u))
    return BUSFILL_ERR_ALIGNMENT;
  DeviceInfo di;
  int dev;
  const int st = current_device(&di, &dev);
  if (st != BUSFILL_OK) return st;
  const long long nb = (long long)N * (K / kUnitK);
  repack_q4k_planar_kernel<<<grid_for(nb * 9, di.sm_count), 256, 0, s>>>(qs, d, dmin, sc12, blocks, nb);
  return cudaGetLastError() == cudaSuccess ? BUSFILL_OK : BUSFILL_ERR_LAUNCH;
}

// ---------------------------------------------------------------------------
// layer sweep: several small-batch Q4_K GEMMs in one launch
// ---------------------------------------------------------------------------
template <int NB>
int launch_sweep(int dev, const sweep::Params& p, cudaStream_t s) {
  const void* kern = reinterpret_cast<const void*>(sweep::sweep_gemm_kernel<NB>);
  constexpr int smem = sweep::Smem<NB>::kAlloc;
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  std::call_once(once[dev & 63], [&] {
    attr_err[dev & 63] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  });
  if (attr_err[dev & 63] != cudaSuccess) return BUSFILL_ERR_LAUNCH;
  void* args[] = {const_cast<sweep::Params*>(&p)};
  if (launch(kern, dim3((unsigned)p.G), dim3(kThreads), smem, s, args, g_use_pdl.load() != 0) != cudaSuccess) {
    cudaGetLastError();
    return BUSFILL_ERR_LAUNCH;
  }
  return BUSFILL_OK;
}

int gemm_sweep_impl(const busfill_sweep_op* ops, int nops, int M, cudaStream_t s) {
  if (!ops) return BUSFILL_ERR_INVALID_ARG;
  if (nops < 1 || nops > sweep::kMaxOps || M < 1 || M > sweep::kMaxNB) return BUSFILL_ERR_SHAPE;
  for (int o = 0; o < nops; ++o) {
    const busfill_sweep_op& op = ops[o];
    if (!op.w || !op.a || !op.c || op.dep < -1 || op.dep >= o) return BUSFILL_ERR_INVALID_ARG;
    if (op.N < 1 || op.N > sweep::kMaxTiles * kTileRows || op.K < kUnitK || op.K % kUnitK != 0 ||
        op.K > (1 << 20))
      return BUSFILL_ERR_SHAPE;
    if (!aligned16(op.w) || !aligned16(op.a) || (op.w_up && !aligned16(op.w_up))) return BUSFILL_ERR_ALIGNMENT;
  }
  DeviceInfo di;
  int dev = 0;
  int st = current_device(&di, &dev);
  if (st != BUSFILL_OK) return st;
  unsigned* err = nullptr;
  unsigned* ws = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    st = get_error_words(dev, s, &err);
    if (st != BUSFILL_OK) return st;
    ws = sweep_workspace(dev, s, di.sm_count);
  }
  if (!ws) return BUSFILL_ERR_ALLOC;
  const int nb = M <= 16 ? 16 : 32;
  sweep::Params p;
  std::memset(&p, 0, sizeof(p));
  unsigned max_units = 0;
  for (int o = 0; o < nops; ++o) {
    const busfill_sweep_op& op = ops[o];
    const int S = op.K / kUnitK;
    const uint64_t row = (uint64_t)S * kQ4KBlockBytes;
    if (!make_tmap_2d(&p.tw[o], CU_TENSOR_MAP_DATA_TYPE_UINT8, op.w, row, (uint64_t)op.N, row, kQ4KBlockBytes,
                      kTileRows, CU_TENSOR_MAP_SWIZZLE_NONE))
      return BUSFILL_ERR_CUDA;
    p.twu[o] = p.tw[o];
    if (op.w_up && !make_tmap_2d(&p.twu[o], CU_TENSOR_MAP_DATA_TYPE_UINT8, op.w_up, row, (uint64_t)op.N, row,
                                 kQ4KBlockBytes, kTileRows, CU_TENSOR_MAP_SWIZZLE_NONE))
      return BUSFILL_ERR_CUDA;
    if (!make_tmap_act3d(&p.ta[o], op.a, (uint64_t)M, (uint64_t)op.K, (uint32_t)nb, kChunksPerUnit))
      return BUSFILL_ERR_CUDA;
    sweep::Op& d = p.op[o];
    d.c = op.c;
    d.N = op.N;
    d.tiles = (op.N + kTileRows - 1) / kTileRows;
    d.S = S;
    d.planes = op.w_up ? 2 : 1;
    d.dep = op.dep;
    d.units = (unsigned)d.tiles * (unsigned)d.planes * (unsigned)S;
    max_units = std::max(max_units, d.units);
  }
  p.nops = nops;
  p.M = M;
  // one CTA per SM (every CTA of the grid must be resident at once: a CTA
  // waits for other CTAs' tiles); BUSFILL_OPT_SWEEP_CTAS may ask for fewer
  const int forced = g_sweep_ctas.load();
  const int cap = forced > 0 ? std::min(forced, di.sm_count) : di.sm_count;
  p.G = (int)std::min<unsigned>((unsigned)cap, max_units);
  // An op whose tiles nearly fill the grid (a multiple of them within 1/8 of
  // the CTAs) takes whole tiles, the same number per CTA, on that many CTAs:
  // no split tiles, so no partial sums through memory (config-3 gate/up:
  // 136 tiles on 148 SMs, 83 us per layer against 85 with all CTAs splitting
  // it); every other op is split over all G CTAs.
  for (int o = 0; o < nops; ++o) {
    sweep::Op& d = p.op[o];
    const int k = (d.tiles + p.G - 1) / p.G;
    const int whole = d.tiles / k;
    d.ctas = (d.tiles % k == 0 && whole <= p.G && whole * 8 >= p.G * 7) ? whole : p.G;
  }
  p.flags = ws;
  p.dep_extra = g_sweep_unmet.load() ? 1u : 0u;
  p.part = reinterpret_cast<float*>(ws + sweep::kFlagWords);
  p.error = err;
  return nb == 16 ? launch_sweep<16>(dev, p, s) : launch_sweep<32>(dev, p, s);
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

int busfill_version(void) { return kVersion; }

unsigned busfill_last_failure_detail(void) { return g_last_detail.load(); }

int busfill_gemm_kernel_for(int M, int N, int K) { return use_prefill(M, N, K, false, true) ? 1 : 0; }

int busfill_gemm_launches(int M, int N, int K, int sm_count) {
  if (M < 1 || N < 1 || K < kUnitK || K % kUnitK != 0) return BUSFILL_ERR_SHAPE;
  if (sm_count <= 0) {
    DeviceInfo di;
    int dev = 0;
    const int st = current_device(&di, &dev);
    if (st != BUSFILL_OK) return st;
    sm_count = di.sm_count;
  }
  if (!use_prefill(M, N, K, false, true)) return (M + 63) / 64;   // the decode kernel, 64 rows a launch
  // the stream-K prefill launch, and the fix-up launch if it splits an item
  const int S = K / kUnitK;
  const long long units = prefill_items(M, N, false) * S;
  // CTAs (or CTA pairs) that split the units: one per SM (pair of SMs); CTA
  // pairs take whole items, with no fix-up, when the item count allows
  if (prefill_pairs(M, false) && pair_whole_grid(prefill_items(M, N, false), sm_count / 2)) return 1;
  const int ctas = prefill_pairs(M, false) ? sm_count / 2 : sm_count;
  const int grid = (int)std::min<long long>(std::min<long long>(units, ctas), prefill::kMaxSplitItems + 1);
  prefill::SplitItems si;
  split_items(units, S, grid, &si);
  return si.n > 0 ? 2 : 1;
}

const char* busfill_status_string(int status) {
  switch (status) {
    case BUSFILL_OK: return "ok";
    case BUSFILL_ERR_INVALID_ARG: return "invalid argument (NULL pointer or unknown option)";
    case BUSFILL_ERR_SHAPE: return "unsupported shape (need M>=1, N>=1, K a positive multiple of 256)";
    case BUSFILL_ERR_ALIGNMENT: return "pointer not 16-byte aligned";
    case BUSFILL_ERR_UNSUPPORTED_DEVICE: return "current device is not sm_100 (B200)";
    case BUSFILL_ERR_LAUNCH: return "kernel launch failed";
    case BUSFILL_ERR_ALLOC: return "workspace allocation failed";
    case BUSFILL_ERR_DEVICE_TIMEOUT: return "a bounded device-side wait expired (kernel gave up)";
    case BUSFILL_ERR_CUDA: return "CUDA runtime error";
    default: return "unknown status";
  }
}

int busfill_set_option(int option, int value) {
  if (option == BUSFILL_OPT_PDL) {
    g_use_pdl.store(value ? 1 : 0);
    return BUSFILL_OK;
  }
  if (option == BUSFILL_OPT_KSPLIT) {
    if (value < 0 || value > 8) return BUSFILL_ERR_INVALID_ARG;
    g_force_ksplit.store(value);
    return BUSFILL_OK;
  }
  if (option == BUSFILL_OPT_PREFILL_MIN_M) {
    if (value < 0) return BUSFILL_ERR_INVALID_ARG;
    g_prefill_min_m.store(value);
    return BUSFILL_OK;
  }
  if (option == BUSFILL_OPT_EXACT_KQUANT) {
    // accepted for compatibility: every K-quant operand is exact
    return value == 0 || value == 1 ? BUSFILL_OK : BUSFILL_ERR_INVALID_ARG;
  }
  if (option == BUSFILL_OPT_PREFILL_BATCH_TILE) {
    if (value != 0 && value != 128 && value != 256) return BUSFILL_ERR_INVALID_ARG;
    g_prefill_bt.store(value);
    return BUSFILL_OK;
  }
  if (option == BUSFILL_OPT_PREFILL_PAIR) {
    if (value < 0 || value > 2) return BUSFILL_ERR_INVALID_ARG;
    g_prefill_pair.store(value);
    return BUSFILL_OK;
  }
  if (option == BUSFILL_OPT_SWEEP_CTAS) {
    if (value < 0 || value > 4096) return BUSFILL_ERR_INVALID_ARG;
    g_sweep_ctas.store(value);
    return BUSFILL_OK;
  }
  if (option == BUSFILL_OPT_SWEEP_UNMET_DEP) {
    if (value < 0 || value > 1) return BUSFILL_ERR_INVALID_ARG;
    g_sweep_unmet.store(value);
    return BUSFILL_OK;
  }
  return BUSFILL_ERR_INVALID_ARG;
}

int busfill_gemm_q4_0(const uint8_t* wq, const uint16_t* ws, const uint16_t* a, uint16_t* c, int M, int N, int K,
                      void* stream) {
  return gemm_impl<WFmt::Q4_0, __half>(wq, ws, a, c, M, N, K, reinterpret_cast<cudaStream_t>(stream));
}

int busfill_gemm_q4k(const uint8_t* blocks, const uint16_t* a, uint16_t* c, int M, int N, int K, void* stream) {
  return gemm_impl<WFmt::Q4K, __half>(blocks, nullptr, a, c, M, N, K, reinterpret_cast<cudaStream_t>(stream));
}

int busfill_gemm_q4k_swiglu(const uint8_t* w_gate, const uint8_t* w_up, const uint16_t* a, uint16_t* h, int M, int N,
                            int K, void* stream) {
  return gemm_impl<WFmt::Q4K, __half>(w_gate, nullptr, a, h, M, N, K, reinterpret_cast<cudaStream_t>(stream), w_up,
                                      true);
}

int busfill_gemm_q4k_sweep(const busfill_sweep_op* ops, int nops, int M, void* stream) {
  return gemm_sweep_impl(ops, nops, M, reinterpret_cast<cudaStream_t>(stream));
}

int busfill_gemm_q5k(const uint8_t* blocks, const uint16_t* a, uint16_t* c, int M, int N, int K, void* stream) {
  return gemm_impl<WFmt::Q5K, __half>(blocks, nullptr, a, c, M, N, K, reinterpret_cast<cudaStream_t>(stream));
}

int busfill_gemm_q6k(const uint8_t* body, const uint16_t* d, const uint16_t* a, uint16_t* c, int M, int N, int K,
                     void* stream) {
  return gemm_impl<WFmt::Q6K, __half>(body, d, a, c, M, N, K, reinterpret_cast<cudaStream_t>(stream));
}

int busfill_repack_q6k(const uint8_t* blocks, uint8_t* body, uint16_t* d, int N, int K, void* stream) {
  if (!blocks || !body || !d) return BUSFILL_ERR_INVALID_ARG;
  if (N < 1 || K < 256 || K % 256 != 0) return BUSFILL_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(blocks) & 1u) || !aligned16(body) || !aligned16(d)) return BUSFILL_ERR_ALIGNMENT;
  DeviceInfo di;
  int dev;
  const int st = current_device(&di, &dev);
  if (st != BUSFILL_OK) return st;
  const long long words = (long long)N * (K / 256) * (kQ6KBodyBytes / 2 + 1);
  repack_q6k_kernel<<<grid_for(words, di.sm_count), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint16_t*>(blocks), reinterpret_cast<uint16_t*>(body), d, N, K / 256);
  return cudaGetLastError() == cudaSuccess ? BUSFILL_OK : BUSFILL_ERR_LAUNCH;
}

int busfill_repack_q4k_planar(const uint8_t* qs, const uint16_t* d, const uint16_t* dmin, const uint8_t* scales12,
                              uint8_t* blocks, int N, int K, void* stream) {
  return repack_q4k_planar_impl(qs, d, dmin, scales12, blocks, N, K, reinterpret_cast<cudaStream_t>(stream));
}

int busfill_gemm_q4k_planar(const uint8_t* qs, const uint16_t* d, const uint16_t* dmin, const uint8_t* scales12,
                            const uint16_t* a, uint16_t* c, int M, int N, int K, void* stream) {
  if (!qs || !d || !dmin || !scales12 || !a || !c) return BUSFILL_ERR_INVALID_ARG;
  if (M < 1 || N < 1 || K < kUnitK || K % kUnitK != 0) return BUSFILL_ERR_SHAPE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  DeviceInfo di;
  int dev = 0;
  int st = current_device(&di, &dev);
  if (st != BUSFILL_OK) return st;
  uint8_t* blocks = nullptr;
  st = planar_buffer(dev, s, (size_t)N * (K / kUnitK) * kQ4KBlockBytes, &blocks);
  if (st != BUSFILL_OK) return st;
  st = repack_q4k_planar_impl(qs, d, dmin, scales12, blocks, N, K, s);
  if (st != BUSFILL_OK) return st;
  return gemm_impl<WFmt::Q4K, __half>(blocks, nullptr, a, c, M, N, K, s);
}

int busfill_mul_mat(const busfill_tensor* src0, const busfill_tensor* src1, busfill_tensor* dst, void* stream) {
  if (!src0 || !src1 || !dst || !src0->data || !src1->data || !dst->data) return BUSFILL_ERR_INVALID_ARG;
  if (src1->type != BUSFILL_TYPE_F16 || dst->type != BUSFILL_TYPE_F16) return BUSFILL_ERR_INVALID_ARG;
  int qk = 0, bs = 0;
  switch (src0->type) {
    case BUSFILL_TYPE_Q4_0: qk = 32; bs = 18; break;
    case BUSFILL_TYPE_Q4_K: qk = 256; bs = kQ4KBlockBytes; break;
    case BUSFILL_TYPE_Q5_K: qk = 256; bs = kQ5KBlockBytes; break;
    default: return BUSFILL_ERR_INVALID_ARG;
  }
  const int64_t K = src0->ne[0], N = src0->ne[1], M = src1->ne[1];
  for (int i = 0; i < 4; ++i)
    if (src0->ne[i] < 1 || src1->ne[i] < 1 || dst->ne[i] < 1) return BUSFILL_ERR_SHAPE;
  if (src1->ne[0] != K || dst->ne[0] != N || dst->ne[1] != M) return BUSFILL_ERR_SHAPE;
  if (dst->ne[2] != src1->ne[2] || dst->ne[3] != src1->ne[3]) return BUSFILL_ERR_SHAPE;
  if (src1->ne[2] % src0->ne[2] != 0 || src1->ne[3] % src0->ne[3] != 0) return BUSFILL_ERR_SHAPE;
  if (K % kUnitK != 0 || K > (1 << 30) || N > (1 << 30) || M > (1 << 30)) return BUSFILL_ERR_SHAPE;
  // rows must be packed: one GEMM runs per batch slice over [rows, K] blocks
  if (src0->nb[0] != (size_t)bs || src0->nb[1] != (size_t)(K / qk) * bs) return BUSFILL_ERR_SHAPE;
  if (src1->nb[0] != 2 || src1->nb[1] != (size_t)K * 2 || dst->nb[0] != 2 || dst->nb[1] != (size_t)N * 2)
    return BUSFILL_ERR_SHAPE;
  const int64_t r2 = src1->ne[2] / src0->ne[2], r3 = src1->ne[3] / src0->ne[3];
  for (int64_t i3 = 0; i3 < src1->ne[3]; ++i3)
    for (int64_t i2 = 0; i2 < src1->ne[2]; ++i2) {
      const uint8_t* w = static_cast<const uint8_t*>(src0->data) + (i2 / r2) * src0->nb[2] + (i3 / r3) * src0->nb[3];
      const uint16_t* a = reinterpret_cast<const uint16_t*>(static_cast<const uint8_t*>(src1->data) +
                                                            i2 * src1->nb[2] + i3 * src1->nb[3]);
      uint16_t* c = reinterpret_cast<uint16_t*>(static_cast<uint8_t*>(dst->data) + i2 * dst->nb[2] + i3 * dst->nb[3]);
      int st;
      if (src0->type == BUSFILL_TYPE_Q4_0)
        st = busfill_gemm_q4_0_ggml(w, a, c, (int)M, (int)N, (int)K, stream);
      else if (src0->type == BUSFILL_TYPE_Q4_K)
        st = busfill_gemm_q4k(w, a, c, (int)M, (int)N, (int)K, stream);
      else
        st = busfill_gemm_q5k(w, a, c, (int)M, (int)N, (int)K, stream);
      if (st != BUSFILL_OK) return st;
    }
  return BUSFILL_OK;
}

int busfill_gemm_q4k_gather(const uint8_t* blocks, const uint16_t* a, int M, int N, int K, const busfill_gather* g,
                            void* stream) {
  return gemm_gather_impl<WFmt::Q4K>(blocks, nullptr, false, a, M, N, K, g, reinterpret_cast<cudaStream_t>(stream));
}

int busfill_gemm_q4k_swiglu_gather(const uint8_t* w_gate, const uint8_t* w_up, const uint16_t* a, int M, int N, int K,
                                   const busfill_gather* g, void* stream) {
  return gemm_gather_impl<WFmt::Q4K>(w_gate, w_up, true, a, M, N, K, g, reinterpret_cast<cudaStream_t>(stream));
}

int busfill_gather_wait(const busfill_gather* g, void* stream) {
  if (!g || !g->wait || !g->wait_gen || g->nwait < 1 || g->nwait > kMaxPeers) return BUSFILL_ERR_INVALID_ARG;
  DeviceInfo di;
  int dev = 0;
  int st = current_device(&di, &dev);
  if (st != BUSFILL_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  unsigned* err = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    st = get_error_words(dev, s, &err);
  }
  if (st != BUSFILL_OK) return st;
  WaitTiles tiles{};
  for (int r = 0; r < g->nwait; ++r) tiles.n[r] = g->wait_tiles[r];
  gather_wait_kernel<<<1, 32, 0, s>>>(g->wait, g->wait_gen, g->nwait, tiles, err);
  if (cudaGetLastError() != cudaSuccess) return BUSFILL_ERR_LAUNCH;
  return BUSFILL_OK;
}

int busfill_ipc_alloc(size_t bytes, void** dev_ptr) {
  if (!dev_ptr || bytes == 0) return BUSFILL_ERR_INVALID_ARG;
  if (cudaMalloc(dev_ptr, bytes) != cudaSuccess) {
    cudaGetLastError();
    return BUSFILL_ERR_ALLOC;
  }
  if (cudaMemset(*dev_ptr, 0, bytes) != cudaSuccess) {
    cudaGetLastError();
    return BUSFILL_ERR_CUDA;
  }
  return BUSFILL_OK;
}

int busfill_ipc_free(void* dev_ptr) {
  if (!dev_ptr) return BUSFILL_ERR_INVALID_ARG;
  return cudaFree(dev_ptr) == cudaSuccess ? BUSFILL_OK : BUSFILL_ERR_CUDA;
}

int busfill_ipc_get_handle(const void* dev_ptr, void* handle64) {
  if (!dev_ptr || !handle64) return BUSFILL_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)) != cudaSuccess) {
    cudaGetLastError();
    return BUSFILL_ERR_CUDA;
  }
  static_assert(sizeof(h) == 64, "IPC handle size");
  std::memcpy(handle64, &h, sizeof(h));
  return BUSFILL_OK;
}

int busfill_ipc_open(const void* handle64, void** dev_ptr) {
  if (!handle64 || !dev_ptr) return BUSFILL_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  if (cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return BUSFILL_ERR_CUDA;
  }
  return BUSFILL_OK;
}

int busfill_ipc_close(void* dev_ptr) {
  if (!dev_ptr) return BUSFILL_ERR_INVALID_ARG;
  if (cudaIpcCloseMemHandle(dev_ptr) != cudaSuccess) {
    cudaGetLastError();
    return BUSFILL_ERR_CUDA;
  }
  return BUSFILL_OK;
}

int busfill_gemm_q4_0_ggml(const uint8_t* blocks, const uint16_t* a, uint16_t* c, int M, int N, int K, void* stream) {
  return gemm_impl<WFmt::Q4_0G, __half>(blocks, nullptr, a, c, M, N, K, reinterpret_cast<cudaStream_t>(stream));
}

int busfill_gemm_q4k_noalloc(const uint8_t* blocks, const uint16_t* a, uint16_t* c, int M, int N, int K,
                             void* stream) {
  return gemm_q4k_static(blocks, a, c, M, N, K, reinterpret_cast<cudaStream_t>(stream));
}

int busfill_noalloc_status(void* stream, unsigned* bits) {
  if (bits) *bits = 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(s) != cudaSuccess) {
    cudaGetLastError();
    return BUSFILL_ERR_CUDA;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return BUSFILL_ERR_CUDA;
  uint8_t* scratch = nullptr;
  const int st = static_scratch(dev, &scratch);
  if (st != BUSFILL_OK) return st;
  unsigned err2[2] = {0, 0};
  if (cudaMemcpy(err2, scratch, sizeof(err2), cudaMemcpyDeviceToHost) != cudaSuccess) {
    cudaGetLastError();
    return BUSFILL_ERR_CUDA;
  }
  if (bits) {
    bits[0] = err2[0];
    g_last_detail = err2[1];
  }
  if (err2[0] == 0) return BUSFILL_OK;
  if (cudaMemset(scratch, 0, kStaticScratchBytes) != cudaSuccess) {
    cudaGetLastError();
    return BUSFILL_ERR_CUDA;
  }
  return BUSFILL_ERR_DEVICE_TIMEOUT;
}

unsigned busfill_internal_allocations(void) { return g_internal_allocs.load(); }

int busfill_q4(const uint16_t* A, const uint8_t* Wq, const uint16_t* Ws, float* C, int Bsz, int K, int N,
               void* stream) {
  return gemm_impl<WFmt::Q4_0, float>(Wq, Ws, A, C, Bsz, N, K, reinterpret_cast<cudaStream_t>(stream));
}

int busfill_dequant_q4_0(const uint8_t* wq, const uint16_t* ws, uint16_t* out, int N, int K, void* stream) {
  if (!wq || !ws || !out) return BUSFILL_ERR_INVALID_ARG;
  if (N < 1 || K < 32 || K % 32 != 0) return BUSFILL_ERR_SHAPE;
  if (!aligned16(wq) || !aligned16(out)) return BUSFILL_ERR_ALIGNMENT;
  DeviceInfo di;
  int dev;
  const int st = current_device(&di, &dev);
  if (st != BUSFILL_OK) return st;
  const long long nb = (long long)N * (K / 32);
  dequant_q4_0_planes_kernel<<<grid_for(nb, di.sm_count), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      wq, reinterpret_cast<const __half*>(ws), reinterpret_cast<__half*>(out), nb);
  return cudaGetLastError() == cudaSuccess ? BUSFILL_OK : BUSFILL_ERR_LAUNCH;
}

int busfill_dequant_q4_0_ggml(const uint8_t* blocks, uint16_t* out, int N, int K, void* stream) {
  if (!blocks || !out) return BUSFILL_ERR_INVALID_ARG;
  if (N < 1 || K < 32 || K % 32 != 0) return BUSFILL_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(blocks) & 1u) || !aligned16(out)) return BUSFILL_ERR_ALIGNMENT;
  DeviceInfo di;
  int dev;
  const int st = current_device(&di, &dev);
  if (st != BUSFILL_OK) return st;
  const long long nb = (long long)N * (K / 32);
  dequant_q4_0_ggml_kernel<<<grid_for(nb, di.sm_count), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      blocks, reinterpret_cast<__half*>(out), nb);
  return cudaGetLastError() == cudaSuccess ? BUSFILL_OK : BUSFILL_ERR_LAUNCH;
}

int busfill_dequant_q4k(const uint8_t* blocks, uint16_t* out, int N, int K, void* stream) {
  if (!blocks || !out) return BUSFILL_ERR_INVALID_ARG;
  if (N < 1 || K < 256 || K % 256 != 0) return BUSFILL_ERR_SHAPE;
  if (!aligned16(blocks) || !aligned16(out)) return BUSFILL_ERR_ALIGNMENT;
  DeviceInfo di;
  int dev;
  const int st = current_device(&di, &dev);
  if (st != BUSFILL_OK) return st;
  const long long nc = (long long)N * (K / 256) * 4;
  dequant_q4k_kernel<<<grid_for(nc, di.sm_count), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      blocks, reinterpret_cast<__half*>(out), nc);
  return cudaGetLastError() == cudaSuccess ? BUSFILL_OK : BUSFILL_ERR_LAUNCH;
}

int busfill_dequant_q5k(const uint8_t* blocks, uint16_t* out, int N, int K, void* stream) {
  if (!blocks || !out) return BUSFILL_ERR_INVALID_ARG;
  if (N < 1 || K < 256 || K % 256 != 0) return BUSFILL_ERR_SHAPE;
  if (!aligned16(blocks) || !aligned16(out)) return BUSFILL_ERR_ALIGNMENT;
  DeviceInfo di;
  int dev;
  const int st = current_device(&di, &dev);
  if (st != BUSFILL_OK) return st;
  const long long nc = (long long)N * (K / 256) * 4;
  dequant_q5k_kernel<<<grid_for(nc, di.sm_count), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      blocks, reinterpret_cast<__half*>(out), nc);
  return cudaGetLastError() == cudaSuccess ? BUSFILL_OK : BUSFILL_ERR_LAUNCH;
}

int busfill_dequant_q6k(const uint8_t* body, const uint16_t* d, uint16_t* out, int N, int K, void* stream) {
  if (!body || !d || !out) return BUSFILL_ERR_INVALID_ARG;
  if (N < 1 || K < 256 || K % 256 != 0) return BUSFILL_ERR_SHAPE;
  if (!aligned16(body) || !aligned16(d) || !aligned16(out)) return BUSFILL_ERR_ALIGNMENT;
  DeviceInfo di;
  int dev;
  const int st = current_device(&di, &dev);
  if (st != BUSFILL_OK) return st;
  const long long nc = (long long)N * (K / 256) * 4;
  dequant_q6k_kernel<<<grid_for(nc, di.sm_count), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      body, reinterpret_cast<const __half*>(d), reinterpret_cast<__half*>(out), N, K / 256);
  return cudaGetLastError() == cudaSuccess ? BUSFILL_OK : BUSFILL_ERR_LAUNCH;
}

int busfill_stream_status(void* stream) { return busfill_stream_status_ex(stream, nullptr); }

int busfill_stream_status_ex(void* stream, unsigned* bits) {
  if (bits) *bits = 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(s) != cudaSuccess) {
    cudaGetLastError();
    return BUSFILL_ERR_CUDA;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return BUSFILL_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_err.find({dev, s});
  if (it == g_err.end() || !it->second) return BUSFILL_OK;
  unsigned err2[2] = {0, 0};
  if (cudaMemcpy(err2, it->second, sizeof(err2), cudaMemcpyDeviceToHost) != cudaSuccess) return BUSFILL_ERR_CUDA;
  const unsigned err = err2[0];
  if (bits) {
    bits[0] = err;
    g_last_detail = err2[1];
  }
  if (err == 0) return BUSFILL_OK;
  // a kernel gave up part way: clear the words for the next call, and the
  // layer-sweep counters (a CTA that gave up may have left some raised)
  if (cudaMemset(it->second, 0, kErrorWordsBytes) != cudaSuccess) return BUSFILL_ERR_CUDA;
  auto sw = g_sweep.find({dev, s});
  if (sw != g_sweep.end() && sw->second && cudaMemset(sw->second, 0, (size_t)sweep::kFlagWords * 4) != cudaSuccess)
    return BUSFILL_ERR_CUDA;
  return BUSFILL_ERR_DEVICE_TIMEOUT;
}

int busfill_probe_umma(const uint16_t* a, const uint16_t* b, float* d, int nb, void* stream) {
  if (!a || !b || !d) return BUSFILL_ERR_INVALID_ARG;
  if (nb != 16 && nb != 32 && nb != 64) return BUSFILL_ERR_SHAPE;
  if (!aligned16(a) || !aligned16(b) || !aligned16(d)) return BUSFILL_ERR_ALIGNMENT;
  DeviceInfo di;
  int dev;
  int st = current_device(&di, &dev);
  if (st != BUSFILL_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  unsigned* err = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    st = get_error_words(dev, s, &err);
  }
  if (st != BUSFILL_OK) return st;
  const __half* ah = reinterpret_cast<const __half*>(a);
  const __half* bh = reinterpret_cast<const __half*>(b);
  if (nb == 16) umma_probe_kernel<16><<<1, 128, 0, s>>>(ah, bh, d, err);
  else if (nb == 32) umma_probe_kernel<32><<<1, 128, 0, s>>>(ah, bh, d, err);
  else umma_probe_kernel<64><<<1, 128, 0, s>>>(ah, bh, d, err);
  return cudaGetLastError() == cudaSuccess ? BUSFILL_OK : BUSFILL_ERR_LAUNCH;
}

}  // extern "C"
