// Batched dequant-fused 4-bit-weight GEMM for small batches (M <= 32 per
// launch) on sm_100a:  C[M, N] = A[M, K] * deq(W)[N, K]^T, fp16 in, fp32
// accumulate.
//
// Replaces the reference kernel `busfill_q4` (kernels/busfill_v1a.cu:41-104,
// launched <<<N/32, 128>>> at kernels/busfill_v1a.cu:151-154), an sm_70
// mma.m8n8k4 loop capped at 32 batch rows.
//
// Shape of the computation. Work is cut into units of 128 weight rows x 256 K
// (one Q4_K super-block, eight Q4_0 blocks), each unit into four 64-value
// chunks. The tensor core runs swap-AB: the 128 weight rows are the MMA M
// dimension, read from tensor memory (TMEM); the batch rows (padded to NB)
// are N, read from shared memory (K-major, 128-byte swizzle).
//
// Synchronisation is per unit, not per chunk: measured on B200, every
// mbarrier probe on the MMA-issuing warp's path costs 40-75 cycles while an
// N=32 MMA issues in ~17, so the MMA warp waits once per unit (`ready`),
// issues the unit's 16 (Q4_K: 17) MMAs back to back and commits once
// (`udone`), which releases the unit's operand and activation slots and
// publishes its accumulator. Three unit slots are kept in flight.
//
// Warp roles (16 warps, one CTA per SM):
//   0      weight TMA producer: one 2D box of 128 rows x one unit (18 KB) per
//          stage into a 6-stage ring. Weights do not depend on earlier kernels,
//          so this runs before griddepcontrol.wait (programmatic dependent
//          launch lets it overlap the previous kernel's tail).
//   1      activation TMA producer: four 64-value x NB-row boxes per unit
//          (128-byte swizzle); TMEM allocator.
//   2      activation stage: waits for a unit's activations, computes (Q4_K)
//          the 32-value sub-block sums Asum, then marks the activations ready.
//   3      MMA issuer (converged warp, one elected thread issues).
//   4-11   dequant: thread (warp%4, lane) owns weight row 32*(warp%4)+lane and
//          writes its fp16 operand into TMEM with tcgen05.st; warp group g =
//          (warp-4)/4 handles chunks {g, g+2} of every unit.
//   12-15  epilogue: row 32*(warp%4)+lane, all NB batch columns; prepares the
//          per-unit scales ahead of time, folds accumulators, flushes.
//
// Numerics.
//   Q4_0: operand fp16_rn((q-8)*d), bit-identical to the reference dequant
//   (kernels/busfill_v0.cu:74-81): the lop3 magic bias 0x6400 gives the exact
//   fp16 1024+q, hsub2 by 1032 is exact, hmul2 by d rounds once.
//   Q4_K: w = d*sc*q - dmin*m. Operand P = sc*q, exact in fp16 from one hfma2
//   ((1024+q)*sc - 1024*sc; high nibbles arrive as 1024+16q and use sc/16 and
//   64*sc, both exact). Per unit the epilogue adds d * X in fp32. The min
//   term sum_k A*dmin*m = sum_j (dmin*m_j) * Asum_j is one K=16 MMA per unit:
//   dmin*m_j (exact in fp32, 17 significant bits) is split into fp16 hi + lo
//   summing to it exactly, and Asum_j is the fp16 pairwise sum of the 32
//   activations of sub-block j (the only rounding the Q4_K path adds beyond
//   fp32 accumulation).
//
// Work split: a tile of 128 weight rows is split along K over the c CTAs of
// a thread-block cluster (rank k takes units [k*S/c, (k+1)*S/c) of every
// tile); cluster g of G takes tiles g, g+G, g+2G, ... The host picks c so
// that the CTAs that stream weights have the most bandwidth each (one SM's
// TMA engine moves ~57 GB/s of these 144-byte rows, so 120 CTAs stream as
// fast as 148 at K = N = 5120). At the end of each tile the non-zero ranks
// write their fp32 partial sums into their own shared memory and signal rank
// 0, which reads them through distributed shared memory, adds them in rank
// order (deterministic) and writes C. No global scratch, no atomics.
//
// Every wait is bounded (ptx.cuh: kWaitTimeoutNs): a kernel that cannot make
// progress records an error bit and winds down instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "ptx.cuh"

namespace busfill {

enum class WFmt : int { Q4_0 = 0, Q4K = 1 };

constexpr int kTileRows = 128;       // weight rows per tile = MMA M
constexpr int kUnitK = 256;          // K per unit
constexpr int kChunkK = 64;          // K per activation box / 32 TMEM operand columns
constexpr int kChunksPerUnit = kUnitK / kChunkK;
constexpr int kQ4KBlockBytes = 144;
constexpr int kWStageBytes = 18432;  // 128 x 144 B (Q4_K) or 128 x 128 B + 128 x 16 B (Q4_0)
constexpr int kQ40ScaleOffset = 16384;
constexpr int kWStages = 6;
constexpr int kSlots = 3;            // units in flight between dequant/activations and the MMA
constexpr int kDStages = 4;          // per-unit row scales prepared ahead by the epilogue
constexpr int kPrepAhead = 2;        // units the epilogue prepares ahead of its fold
constexpr int kThreads = 512;
constexpr int kWarpWProducer = 0;
constexpr int kWarpXProducer = 1;
constexpr int kWarpXStage = 2;
constexpr int kWarpMma = 3;
constexpr int kWarpDequant0 = 4;
constexpr int kWarpEpilogue0 = 12;
constexpr int kEpilogueThreads = 128;
constexpr int kTmemCols = 512;

// device error word bits (OR-ed; 0 = no error)
constexpr unsigned kErrWeightProducer = 1u;
constexpr unsigned kErrActProducer = 2u;
constexpr unsigned kErrMma = 4u;
constexpr unsigned kErrDequant = 8u;
constexpr unsigned kErrEpilogue = 16u;
constexpr unsigned kErrTeardown = 32u;
constexpr unsigned kErrXStage = 64u;

struct DecodeParams {
  void* c;              // [M, N] row-major, OutT
  unsigned* error;      // device error word (+1: first failure record)
  int M, N, K;
  int tiles;            // T = ceil(N / 128)
  int units_per_tile;   // S = K / 256
  int csize;            // CTAs per cluster: the K split of every tile (1..8)
  int nclusters;        // G; cluster g takes tiles g, g + G, ...; G <= T
};

// Units [first, last) of every tile that cluster rank `rank` of `csize` takes.
__host__ __device__ __forceinline__ int ksplit_begin(int rank, int S, int csize) { return rank * S / csize; }

// TMEM column map (512 columns allocated)
template <int NB>
struct DecodeTmem {
  static constexpr int kX = 0;                           // X[b] at b*NB, b = 0, 1
  static constexpr int kY = 2 * NB;                      // Y (Q4_K), one buffer
  static constexpr int kM = kY + NB;                     // (dmin*m) operand, 8 columns per slot
  static constexpr int kA = 128;                         // unit operand slots, 128 columns each
  static_assert(kM + kSlots * 8 <= kA && kA + kSlots * 128 <= kTmemCols, "TMEM budget");
};

template <int NB>
struct DecodeSmem {
  static constexpr int kXChunkBytes = NB * 128;                      // one 64-value activation box
  static constexpr int kXSlotBytes = kChunksPerUnit * kXChunkBytes;  // one unit of activations
  static constexpr int kWOff = 0;
  static constexpr int kXOff = kWOff + kWStages * kWStageBytes;
  static constexpr int kSOff = kXOff + kSlots * kXSlotBytes;         // Asum B tiles, one per slot
  static constexpr int kDOff = kSOff + kSlots * kXChunkBytes;
  static constexpr int kRedOff = kDOff + kDStages * kTileRows * 4;   // [128][NB] fp32 partial (cluster reduction)
  static constexpr int kBarOff = kRedOff + kTileRows * NB * 4;
  // barrier slots
  static constexpr int bWFull = 0, bWEmpty = bWFull + kWStages;
  static constexpr int bXFull = bWEmpty + kWStages;        // activations landed (TMA tx)
  static constexpr int bReady = bXFull + kSlots;           // unit operands + activations ready for the MMA
  static constexpr int bUDone = bReady + kSlots;           // unit's MMAs complete (commit)
  static constexpr int bAccEmpty = bUDone + kSlots;        // X[b] read by the epilogue
  static constexpr int bYEmpty = bAccEmpty + 2;
  static constexpr int bRedFull = bYEmpty + 1;             // rank 0: partials of the other ranks written
  static constexpr int bRedEmpty = bRedFull + 1;           // rank k > 0: rank 0 has read this rank's partial
  static constexpr int bFinal = bRedEmpty + 1;
  static constexpr int kNumBars = bFinal + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kMiscOff + 64;
  static constexpr int kAlloc = kBytes + 1024;  // slack to align the base to 1024 B
};

// ---------------------------------------------------------------------------
// dequant helpers (one weight row per thread)
// ---------------------------------------------------------------------------

// Q4_0, one 32-value block: 16 bytes -> 16 columns of fp16 pairs (k = 2c, 2c+1)
// holding fp16_rn((q-8)*d). Byte j holds elements 2j (low nibble) and 2j+1.
__device__ __forceinline__ void dequant_q4_0_block(const uint4 b, const __half2 d2, uint32_t* out) {
  const __half2 bias = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));  // 1032, 1032
  const uint32_t w[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t lo = w[i];
    const uint32_t hi = w[i] >> 4;
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      // byte0 <- low nibble of byte x, byte2 <- high nibble of byte x
      const uint32_t t = prmt(lo, hi, (uint32_t)(((4 + x) << 8) | x));
      const uint32_t v = lop3_and_or(t, 0x000F000Fu, 0x64006400u);      // {1024+lo, 1024+hi}
      out[4 * i + x] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(v), bias), d2));
    }
  }
}

// Q4_K, one 64-value chunk of a super-block: 32 bytes; byte l holds element l
// of sub-block 2c (low nibble) and of sub-block 2c+1 (high nibble). Writes
// P = sc*q exactly: out[0..15] = sub-block 2c, out[16..31] = sub-block 2c+1.
__device__ __forceinline__ void dequant_q4k_chunk(const uint4 q0, const uint4 q1, const __half2 mlo,
                                                  const __half2 alo, const __half2 mhi, const __half2 ahi,
                                                  uint32_t* out) {
  const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t t0 = prmt(w[i], w[i], 0x0100u);  // byte0 = b0, byte2 = b1
    const uint32_t t1 = prmt(w[i], w[i], 0x0302u);  // byte0 = b2, byte2 = b3
    const uint32_t l01 = lop3_and_or(t0, 0x000F000Fu, 0x64006400u);  // {1024+q, 1024+q}
    const uint32_t l23 = lop3_and_or(t1, 0x000F000Fu, 0x64006400u);
    const uint32_t h01 = lop3_and_or(t0, 0x00F000F0u, 0x64006400u);  // {1024+16q, 1024+16q}
    const uint32_t h23 = lop3_and_or(t1, 0x00F000F0u, 0x64006400u);
    out[2 * i] = h2_as_u32(__hfma2(u32_as_h2(l01), mlo, alo));
    out[2 * i + 1] = h2_as_u32(__hfma2(u32_as_h2(l23), mlo, alo));
    out[16 + 2 * i] = h2_as_u32(__hfma2(u32_as_h2(h01), mhi, ahi));
    out[16 + 2 * i + 1] = h2_as_u32(__hfma2(u32_as_h2(h23), mhi, ahi));
  }
}

// two 6-bit values (bytes 2c' and 2c'+1 of `word`) -> exact fp16 pair
__device__ __forceinline__ __half2 six_bit_pair_to_h2(uint32_t word, int cpair) {
  const uint32_t sel = cpair ? 0x4342u : 0x4140u;  // {b[2c'], 0x64, b[2c'+1], 0x64}
  const uint32_t v = prmt(word, 0x64646464u, sel);
  const __half2 k1024 = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
  return __hsub2(u32_as_h2(v), k1024);
}

// dmin * m (exact in fp32) -> (hi, lo) fp16 with hi + lo == dmin * m exactly
// for normal-range products (hi = fp16_rn(x); x - hi has <= 6 significant bits)
__device__ __forceinline__ void split_hi_lo(float x, __half& hi, __half& lo) {
  hi = __float2half_rn(x);
  lo = __float2half_rn(x - __half2float(hi));
}

// packed fp32 pair FMA (sm_100): d = a*b + c
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(r)
      : "l"(*reinterpret_cast<unsigned long long*>(&a)), "l"(*reinterpret_cast<unsigned long long*>(&b)),
        "l"(*reinterpret_cast<unsigned long long*>(&c)));
  return *reinterpret_cast<float2*>(&r);
}

template <typename OutT>
__device__ __forceinline__ OutT to_out(float v);
template <>
__device__ __forceinline__ __half to_out<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ float to_out<float>(float v) { return v; }

// Per-unit schedule facts every role derives the same way: unit i of this CTA
// is unit sb0 + i % len of its cluster's (i / len)-th tile.
struct UnitInfo {
  int tile, sb, seg;
  bool seg_first, seg_last;   // first / last unit of this CTA's part of the tile
};
__device__ __forceinline__ UnitInfo unit_info(int i, int len, int sb0, int g, int nclusters) {
  UnitInfo r;
  r.seg = i / len;
  const int j = i - r.seg * len;
  r.tile = g + r.seg * nclusters;
  r.sb = sb0 + j;
  r.seg_first = (j == 0);
  r.seg_last = (j == len - 1);
  return r;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <WFmt FMT, int NB, typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
    decode_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_ws,
                       const __grid_constant__ CUtensorMap tmap_a, const DecodeParams p) {
  static_assert(NB == 16 || NB == 32, "batch tile");
  using L = DecodeSmem<NB>;
  using TM = DecodeTmem<NB>;
  constexpr bool kQ4K = (FMT == WFmt::Q4K);
  constexpr uint32_t kIdesc = make_idesc_f16_f32(kTileRows, NB);
  // ready[s] arrivals: 8 dequant warps + the activation-stage warp (+ 4 epilogue warps for Q4_K)
  constexpr uint32_t kReadyCount = kQ4K ? 13u : 9u;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_s + 1023u) & ~1023u) - raw_s);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::kBarOff;
  auto BAR = [&](int slot) { return bar0 + 8u * (uint32_t)slot; };
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);  // [0] tmem base, [1] last-arriver flag
  float* dring = reinterpret_cast<float*>(smem + L::kDOff);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = p.units_per_tile;
  const int csize = p.csize;
  // clusters tile the 1-D grid in blockIdx order: rank = blockIdx.x % csize
  const int crank = (int)(blockIdx.x % (unsigned)csize);
  const int g = (int)(blockIdx.x / (unsigned)csize);
  const int sb0 = ksplit_begin(crank, S, csize);
  const int len = ksplit_begin(crank + 1, S, csize) - sb0;
  const int ntiles = (p.tiles - g + p.nclusters - 1) / p.nclusters;
  const int nunits = ntiles * len;

  // Every role waits with the whole warp; a wait that times out in any lane
  // counts as a failure for the warp, which then stops issuing work.
  bool ok = true;
  int diag_unit = -1;                  // unit being processed, for the failure record
  auto warp_wait = [&](uint32_t bar, uint32_t parity, bool cluster_scope = false) -> bool {
    if (!ok) return false;
    const bool got = cluster_scope ? mbar_wait_cluster(bar, parity) : mbar_wait(bar, parity);
    ok = __all_sync(0xffffffffu, got);
    if (!ok && lane == 0) {
      // first failure in the grid: warp, unit, barrier slot, parity
      const unsigned rec = 0x80000000u | ((unsigned)warp << 24) | ((unsigned)(diag_unit & 0xFFF) << 12) |
                           (((bar - bar0) / 8u) << 1) | parity;
      atomicCAS(p.error + 1, 0u, rec);
    }
    return ok;
  };
  // unit i's slot is free once unit i - kSlots has completed its MMAs
  auto wait_slot_free = [&](int i) -> bool {
    if (i < kSlots) return ok;
    return warp_wait(BAR(L::bUDone + i % kSlots), ((i / kSlots) & 1) ^ 1);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(BAR(L::bWFull + s), 1);
      mbar_init(BAR(L::bWEmpty + s), kQ4K ? 12 : 8);   // dequant warps (+ epilogue warps reading scales)
    }
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(BAR(L::bXFull + s), 1);
      mbar_init(BAR(L::bReady + s), kReadyCount);
      mbar_init(BAR(L::bUDone + s), 1);
    }
    for (int b = 0; b < 2; ++b) mbar_init(BAR(L::bAccEmpty + b), 4);
    mbar_init(BAR(L::bYEmpty), 4);
    mbar_init(BAR(L::bRedFull), csize > 1 ? 4u * (uint32_t)(csize - 1) : 1u);   // 4 epilogue warps per other rank
    mbar_init(BAR(L::bRedEmpty), 4);                                             // rank 0's 4 epilogue warps
    mbar_init(BAR(L::bFinal), 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmap_w);
    if (FMT == WFmt::Q4_0) tma_prefetch_desc(&tmap_ws);
    tma_prefetch_desc(&tmap_a);
  }
  if (warp == kWarpXProducer) {
    tmem_alloc(sbase + L::kMiscOff, kTmemCols);
    tmem_relinquish();
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  // the other CTAs of the cluster arrive on our barriers: they must be initialised first
  if (csize > 1) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = misc[0];
  // Let the next kernel on the stream launch now: its CTAs take SMs as ours
  // retire and begin streaming their weights before our tail completes.
  if (threadIdx.x == 0) pdl_launch_dependents();

  if (warp == kWarpWProducer) {
    // ---------------- weight producer ----------------
    int issued = 0;
    for (int i = 0; i < nunits; ++i) {
      const int s = i % kWStages;
      if (!warp_wait(BAR(L::bWEmpty + s), ((i / kWStages) & 1) ^ 1)) break;
      const UnitInfo ui = unit_info(i, len, sb0, g, p.nclusters);
      const int tile = ui.tile, sb = ui.sb;
      const uint32_t dst = sbase + L::kWOff + s * kWStageBytes;
      if (elect_one()) {
        mbar_arrive_expect_tx(BAR(L::bWFull + s), kWStageBytes);
        if constexpr (kQ4K) {
          tma_load_2d(dst, &tmap_w, sb * kQ4KBlockBytes, tile * kTileRows, BAR(L::bWFull + s), kPolicyEvictFirst);
        } else {
          tma_load_2d(dst, &tmap_w, sb * 128, tile * kTileRows, BAR(L::bWFull + s), kPolicyEvictFirst);
          tma_load_2d(dst + kQ40ScaleOffset, &tmap_ws, sb * 8, tile * kTileRows, BAR(L::bWFull + s),
                      kPolicyEvictFirst);
        }
      }
      __syncwarp();
      issued = i + 1;
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrWeightProducer);
    // never leave the CTA with copies in flight
    ok = true;
    for (int i = issued > kWStages ? issued - kWStages : 0; i < issued; ++i)
      if (!warp_wait(BAR(L::bWFull + i % kWStages), (i / kWStages) & 1)) {
        if (lane == 0) atomicOr(p.error, kErrTeardown);
        break;
      }
  } else if (warp == kWarpXProducer) {
    // ---------------- activation producer ----------------
    pdl_wait_prerequisites();  // activations may be the previous kernel's output
    int issued = 0;
    for (int i = 0; i < nunits; ++i) {
      if (!wait_slot_free(i)) break;
      const int s = i % kSlots;
      const int sb = sb0 + i % len;
      if (elect_one()) {
        mbar_arrive_expect_tx(BAR(L::bXFull + s), L::kXSlotBytes);
#pragma unroll
        for (int cc = 0; cc < kChunksPerUnit; ++cc)
          tma_load_2d(sbase + L::kXOff + s * L::kXSlotBytes + cc * L::kXChunkBytes, &tmap_a,
                      sb * kUnitK + cc * kChunkK, 0, BAR(L::bXFull + s), kPolicyEvictLast);
      }
      __syncwarp();
      issued = i + 1;
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrActProducer);
    ok = true;
    for (int i = issued > kSlots ? issued - kSlots : 0; i < issued; ++i)
      if (!warp_wait(BAR(L::bXFull + i % kSlots), (i / kSlots) & 1)) {
        if (lane == 0) atomicOr(p.error, kErrTeardown);
        break;
      }
  } else if (warp == kWarpXStage) {
    // ---------------- activation stage (+ Q4_K sub-block sums) ----------------
    const int b = lane;                  // batch row (lanes >= NB idle)
    for (int i = 0; i < nunits; ++i) {
      diag_unit = i;
      const int s = i % kSlots;
      if (!warp_wait(BAR(L::bXFull + s), (i / kSlots) & 1)) break;
      if constexpr (kQ4K) {
        // Asum[b][j], j = 0..7: fp16 pairwise sums of 32 activations. The B
        // tile row b holds k 0..7 = Asum[b][0..7] and k 8..15 = the same again.
        uint32_t sums[4];
#pragma unroll
        for (int cc = 0; cc < kChunksPerUnit; ++cc) {
          __half s2[2] = {__float2half(0.f), __float2half(0.f)};
          if (b < NB) {
            const uint8_t* row =
                smem + L::kXOff + s * L::kXSlotBytes + cc * L::kXChunkBytes + (b >> 3) * 1024 + (b & 7) * 128;
#pragma unroll
            for (int h = 0; h < 2; ++h) {   // sub-block 2cc+h = 16-byte chunks 4h..4h+3
              uint4 v[4];
#pragma unroll
              for (int c = 0; c < 4; ++c)
                v[c] = *reinterpret_cast<const uint4*>(row + ((((uint32_t)(4 * h + c)) ^ (uint32_t)(b & 7)) << 4));
              __half2 a0 = __hadd2(u32_as_h2(v[0].x), u32_as_h2(v[0].y));
              __half2 a1 = __hadd2(u32_as_h2(v[0].z), u32_as_h2(v[0].w));
              __half2 a2 = __hadd2(u32_as_h2(v[1].x), u32_as_h2(v[1].y));
              __half2 a3 = __hadd2(u32_as_h2(v[1].z), u32_as_h2(v[1].w));
              __half2 a4 = __hadd2(u32_as_h2(v[2].x), u32_as_h2(v[2].y));
              __half2 a5 = __hadd2(u32_as_h2(v[2].z), u32_as_h2(v[2].w));
              __half2 a6 = __hadd2(u32_as_h2(v[3].x), u32_as_h2(v[3].y));
              __half2 a7 = __hadd2(u32_as_h2(v[3].z), u32_as_h2(v[3].w));
              a0 = __hadd2(a0, a1); a2 = __hadd2(a2, a3); a4 = __hadd2(a4, a5); a6 = __hadd2(a6, a7);
              a0 = __hadd2(a0, a2); a4 = __hadd2(a4, a6);
              a0 = __hadd2(a0, a4);
              s2[h] = __hadd(__low2half(a0), __high2half(a0));
            }
          }
          sums[cc] = h2_as_u32(__halves2half2(s2[0], s2[1]));
        }
        if (b < NB) {
          uint8_t* row = smem + L::kSOff + s * L::kXChunkBytes + (b >> 3) * 1024 + (b & 7) * 128;
          const uint4 v = make_uint4(sums[0], sums[1], sums[2], sums[3]);
          *reinterpret_cast<uint4*>(row + ((0u ^ (uint32_t)(b & 7)) << 4)) = v;
          *reinterpret_cast<uint4*>(row + ((1u ^ (uint32_t)(b & 7)) << 4)) = v;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(L::bReady + s));
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrXStage);
  } else if (warp == kWarpMma) {
    // ---------------- MMA issuer (converged warp, one elected thread issues) ----------------
    int yuses = 0;         // Q4_K segments started (Y buffer uses)
    for (int i = 0; i < nunits; ++i) {
      diag_unit = i;
      const UnitInfo ui = unit_info(i, len, sb0, g, p.nclusters);
      const int s = i % kSlots;
      // every unit accumulates into X[i & 1]; the epilogue folds it into
      // registers, so the MMA is never more than two units ahead of it
      if (!warp_wait(BAR(L::bAccEmpty + (i & 1)), ((i >> 1) & 1) ^ 1)) break;
      if (kQ4K && ui.seg_first) {
        if (!warp_wait(BAR(L::bYEmpty), (yuses & 1) ^ 1)) break;
        ++yuses;
      }
      if (!warp_wait(BAR(L::bReady + s), (i / kSlots) & 1)) break;
      tc_fence_after();
      const uint32_t d_x = tmem + TM::kX + (uint32_t)((i & 1) * NB);
      const uint32_t a_t = tmem + TM::kA + s * 128;
      const uint32_t b_s = sbase + L::kXOff + s * L::kXSlotBytes;
      if (elect_one()) {
#pragma unroll
        for (int cc = 0; cc < kChunksPerUnit; ++cc)
#pragma unroll
          for (int t = 0; t < 4; ++t)
            mma_f16_ts(d_x, a_t + cc * 32 + 8 * t, make_sdesc_sw128(b_s + cc * L::kXChunkBytes + 32 * t), kIdesc,
                       (cc == 0 && t == 0) ? 0u : 1u);
        if constexpr (kQ4K)
          mma_f16_ts(tmem + TM::kY, tmem + TM::kM + s * 8, make_sdesc_sw128(sbase + L::kSOff + s * L::kXChunkBytes),
                     kIdesc, ui.seg_first ? 0u : 1u);
        tc_commit(BAR(L::bUDone + s));  // frees slot s; publishes X (and Y) for this unit
      }
      __syncwarp();
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrMma);
    if (elect_one()) tc_commit(BAR(L::bFinal));  // fires once every MMA issued above has completed
    __syncwarp();
  } else if (warp < kWarpEpilogue0) {
    // ---------------- dequant ----------------
    const int q = warp & 3;                        // TMEM lane quarter this warp may touch
    const int g = (warp - kWarpDequant0) >> 2;     // group: chunks {g, g+2}
    const int r = q * 32 + lane;                   // weight row within the tile
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    for (int i = 0; i < nunits; ++i) {
      diag_unit = i;
      const int ws = i % kWStages;
      if (!warp_wait(BAR(L::bWFull + ws), (i / kWStages) & 1)) break;
      if (!wait_slot_free(i)) break;
      tc_fence_after();
      const uint8_t* stage = smem + L::kWOff + ws * kWStageBytes;
      const uint32_t a_slot = tmem + lane_off + TM::kA + (i % kSlots) * 128;
      uint32_t sc_lo = 0, sc_hi = 0;
      if constexpr (kQ4K) {
        const uint4 hdr = *reinterpret_cast<const uint4*>(stage + r * kQ4KBlockBytes);
        sc_lo = hdr.y & 0x3F3F3F3Fu;
        sc_hi = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
      }
#pragma unroll 1
      for (int k2 = 0; k2 < 2; ++k2) {
        const int cc = g + 2 * k2;
        uint32_t P[32];
        if constexpr (kQ4K) {
          const uint8_t* qs = stage + r * kQ4KBlockBytes + 16 + cc * 32;
          const uint4 q0 = *reinterpret_cast<const uint4*>(qs);
          const uint4 q1 = *reinterpret_cast<const uint4*>(qs + 16);
          const __half2 S2 = six_bit_pair_to_h2(cc < 2 ? sc_lo : sc_hi, cc & 1);  // {sc[2cc], sc[2cc+1]}
          const __half2 mlo = __low2half2(S2);
          const __half2 alo = __hmul2(mlo, __float2half2_rn(-1024.f));
          const __half2 shi = __high2half2(S2);
          const __half2 mhi = __hmul2(shi, __float2half2_rn(0.0625f));
          const __half2 ahi = __hmul2(shi, __float2half2_rn(-64.f));
          dequant_q4k_chunk(q0, q1, mlo, alo, mhi, ahi, P);
        } else {
          const uint8_t* wrow = stage + r * 128;
          const uint32_t sw = (uint32_t)(r & 7);  // TMA 128-byte swizzle: 16-B chunk ^= row % 8
          const uint4 b0 = *reinterpret_cast<const uint4*>(wrow + ((((uint32_t)(2 * cc)) ^ sw) << 4));
          const uint4 b1 = *reinterpret_cast<const uint4*>(wrow + ((((uint32_t)(2 * cc + 1)) ^ sw) << 4));
          const uint32_t dd = *reinterpret_cast<const uint32_t*>(stage + kQ40ScaleOffset + r * 16 + cc * 4);
          const __half2 d01 = u32_as_h2(dd);
          dequant_q4_0_block(b0, __low2half2(d01), P);
          dequant_q4_0_block(b1, __high2half2(d01), P + 16);
        }
        tmem_st_x32(a_slot + cc * 32, P);
      }
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(BAR(L::bReady + i % kSlots));
        mbar_arrive(BAR(L::bWEmpty + ws));
      }
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrDequant);
  } else {
    // ---------------- epilogue ----------------
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    float acc[NB];
#pragma unroll
    for (int t = 0; t < NB; ++t) acc[t] = 0.f;

    // Q4_K: read unit i's scales for this row while its weight stage is
    // resident; keep d for the fold and store dmin*m (split hi + lo) as the
    // min-term operand in TMEM slot i % kSlots.
    auto prep = [&](int i) {
      const int ws = i % kWStages;
      if (!warp_wait(BAR(L::bWFull + ws), (i / kWStages) & 1)) return;
      const uint4 hdr = *reinterpret_cast<const uint4*>(smem + L::kWOff + ws * kWStageBytes + r * kQ4KBlockBytes);
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(L::bWEmpty + ws));
      dring[(i % kDStages) * kTileRows + r] = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xFFFFu)));
      const uint32_t m_lo = hdr.z & 0x3F3F3F3Fu;
      const uint32_t m_hi = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
      const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr.x >> 16)));
      uint32_t mv[8];
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        const uint32_t word = jp < 2 ? m_lo : m_hi;
        const int sh = 16 * (jp & 1);
        __half h0, l0, h1, l1;
        split_hi_lo(dmin * (float)((word >> sh) & 0xFFu), h0, l0);
        split_hi_lo(dmin * (float)((word >> (sh + 8)) & 0xFFu), h1, l1);
        mv[jp] = h2_as_u32(__halves2half2(h0, h1));
        mv[4 + jp] = h2_as_u32(__halves2half2(l0, l1));
      }
      if (!wait_slot_free(i)) return;
      tc_fence_after();
      tmem_st_x8(tmem + lane_off + TM::kM + (i % kSlots) * 8, mv);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(L::bReady + i % kSlots));
    };

    // acc += scale * X[buf]; the unit's MMAs (udone) must have completed
    auto fold_x = [&](int i, int buf, float scale) {
      if (!warp_wait(BAR(L::bUDone + i % kSlots), (i / kSlots) & 1)) return;
      tc_fence_after();
      const float2 sc2 = make_float2(scale, scale);
#pragma unroll
      for (int h = 0; h < NB; h += 16) {
        uint32_t x[16];
        tmem_ld_x16(tmem + lane_off + TM::kX + (uint32_t)(buf * NB + h), x);
        tc_wait_ld();
#pragma unroll
        for (int t = 0; t < 16; t += 2) {
          const float2 v = ffma2(sc2, make_float2(__uint_as_float(x[t]), __uint_as_float(x[t + 1])),
                                 make_float2(acc[h + t], acc[h + t + 1]));
          acc[h + t] = v.x;
          acc[h + t + 1] = v.y;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(L::bAccEmpty + buf));
    };

    // Finish tile `tile` (this CTA's segment `seg`). One CTA per tile: write C.
    // Otherwise ranks k > 0 leave their partial in their own shared memory
    // ([row][NB] fp32, 16-byte chunks swizzled by row) and signal rank 0; rank 0
    // adds them in rank order through distributed shared memory and writes C.
    auto flush = [&](int tile, int seg) {
      const int n = tile * kTileRows + r;
      OutT* C = reinterpret_cast<OutT*>(p.c);
      constexpr int kChunks = NB / 4;
      const uint32_t my_row = sbase + L::kRedOff + (uint32_t)(r * NB * 4);
      const int swz = r & (kChunks - 1);
      if (csize > 1 && crank != 0) {
        // our buffer is free once rank 0 has read the previous segment's partial
        if (seg > 0) warp_wait(BAR(L::bRedEmpty), (uint32_t)((seg - 1) & 1), true);
#pragma unroll
        for (int j = 0; j < kChunks; ++j) {
          const uint32_t a = my_row + (uint32_t)((j ^ swz) << 4);
          asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(acc[4 * j]), "f"(acc[4 * j + 1]),
                       "f"(acc[4 * j + 2]), "f"(acc[4 * j + 3])
                       : "memory");
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(mapa_shared(BAR(L::bRedFull), 0));
        return;
      }
      if (csize > 1) {
        warp_wait(BAR(L::bRedFull), (uint32_t)(seg & 1), true);
        for (int k = 1; k < csize; ++k) {
          const uint32_t src = mapa_shared(my_row, (uint32_t)k);
          float4 v[kChunks];
#pragma unroll
          for (int j = 0; j < kChunks; ++j) v[j] = ld_dsmem_f4(src + (uint32_t)((j ^ swz) << 4));
#pragma unroll
          for (int j = 0; j < kChunks; ++j) {
            acc[4 * j] += v[j].x;
            acc[4 * j + 1] += v[j].y;
            acc[4 * j + 2] += v[j].z;
            acc[4 * j + 3] += v[j].w;
          }
        }
        __syncwarp();
        if (lane == 0)
          for (int k = 1; k < csize; ++k) mbar_arrive_remote(mapa_shared(BAR(L::bRedEmpty), (uint32_t)k));
      }
      pdl_wait_prerequisites();  // C may still be read by the previous kernel
      if (ok && n < p.N) {
#pragma unroll
        for (int t = 0; t < NB; ++t)
          if (t < p.M) C[(size_t)t * p.N + n] = to_out<OutT>(acc[t]);
      }
    };

    if constexpr (kQ4K) {
      for (int i = 0; i < nunits && i < kPrepAhead; ++i) prep(i);
    }
    for (int i = 0; i < nunits; ++i) {
      diag_unit = i;
      const UnitInfo ui = unit_info(i, len, sb0, g, p.nclusters);
      // Every unit is folded, in order: a waiter on a parity barrier must not
      // skip phases (a wait for phase n+1 posted before phase n completed
      // would see the stale parity as complete).
      if constexpr (kQ4K) {
        if (i + kPrepAhead < nunits) prep(i + kPrepAhead);
        fold_x(i, i & 1, dring[(i % kDStages) * kTileRows + r]);
        if (ui.seg_last && ok) {
          // Y of this segment is complete: its last MMA was committed with unit i
#pragma unroll
          for (int h = 0; h < NB; h += 16) {
            uint32_t y[16];
            tmem_ld_x16(tmem + lane_off + TM::kY + h, y);
            tc_wait_ld();
#pragma unroll
            for (int t = 0; t < 16; ++t) acc[h + t] -= __uint_as_float(y[t]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(BAR(L::bYEmpty));
        }
      } else {
        fold_x(i, i & 1, 1.0f);
      }
      if (ui.seg_last) {
        flush(ui.tile, ui.seg);
#pragma unroll
        for (int t = 0; t < NB; ++t) acc[t] = 0.f;
      }
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrEpilogue);
  }

  // ---------------- teardown ----------------
  __syncwarp();
  __syncthreads();
  // no CTA may leave while another CTA of its cluster can still read its
  // shared memory or arrive on its barriers
  if (csize > 1) cluster_sync_all();
  if (warp == kWarpXProducer) {
    bool done = true;
    if (lane == 0) done = mbar_wait(BAR(L::bFinal), 0);
    done = __shfl_sync(0xffffffffu, done ? 1 : 0, 0) != 0;
    if (!done && lane == 0) atomicOr(p.error, kErrTeardown);
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace busfill
