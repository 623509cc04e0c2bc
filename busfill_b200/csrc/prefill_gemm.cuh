// Dequant-fused 4-bit-weight GEMM for large batches (prefill, M >= ~128) on
// sm_100a: C[M, N] = A[M, K] * deq(W)[N, K]^T, fp16 in, fp32 accumulate.
//
// The same contraction as the decode kernel (decode_gemm.cuh), in the regime
// where it turns compute-bound: at M = 2048 the work is 2 M N K flops against
// one pass of 4.5-bit weights, so the tensor pipe, not HBM, sets the time.
// The reference has no such path (its kernel computes batch rows < 32 only,
// kernels/busfill_v1a.cu:41-104); the shapes are BASELINE config 4.
//
// Shape of the computation. A work item is two 128-row weight tiles (256
// weight rows) x 128 batch rows, looped over K in units of 256. The weights
// of a unit are dequantized into tensor memory (the MMA's A operand, one
// 128-lane tile per weight tile) and each tile's accumulator [128 weight rows
// x 128 batch rows] fp32 lives in TMEM next to them:
//   columns   0..127  accumulator of weight tile 0
//   columns 128..255  accumulator of weight tile 1
//   columns 256..511  four half-unit operand slots (t, h) of 64 columns:
//                     tile t, K half h (chunks 2h, 2h+1) of the current unit.
// The MMAs of a unit run (t0,h0) (t1,h0) (t0,h1) (t1,h1), 8 MMAs of
// 128x128x16 each, so a half slot is refilled while the three other MMA
// blocks run. Activations come as one 3-D TMA box per K half (2 chunks x 128
// rows x 64 values, 32 KB) and weights as one box per unit for both tiles
// (256 rows, 36 KB): an SM's TMA unit takes a roughly fixed time per box
// (~0.5 us with every SM loading, measured on B200), so few large boxes. The
// weight ring is three units deep: a weight box lands ~1.7 us after issue
// under load, longer than a unit's MMAs (~1.3 us).
//
// Measured on B200: a 128x128x16 TS MMA (A in TMEM) takes ~74 cycles back to
// back, 92% of the dense fp16 rate; a unit (32 MMAs) ~2400 cycles.
//
// Handoffs: a dequant warp group publishes a half slot with a named-barrier
// arrive that the MMA warp syncs on (no mbarrier round trip on the path of
// every 8 MMAs); the slot comes back through the commit barrier of its MMAs.
// Named barriers have no timeout, so every group arrives, and the MMA warp
// syncs, for every half slot of every unit whatever happens (work is skipped
// after a failed wait, the arrivals are not).
//
// Warp roles (16 warps, one CTA per SM, persistent over work items):
//   0      weight TMA producer (3-stage ring of 36 KB)
//   1      activation TMA producer (3-stage ring of 32 KB); TMEM allocator
//   3      MMA issuer (converged warp, one elected thread issues)
//   4-7    dequant of weight tile 0, 8-11 of weight tile 1: thread (warp%4,
//          lane) owns tile row 32*(warp%4)+lane, both K halves of each unit
//   12-15  epilogue: reads both accumulators once per item, writes C
//   2      idle
//
// Work order: item = pair * B + batch_tile. With a partial-tile workspace
// (stream-K), CTA c of G takes the contiguous range [c T / G, (c+1) T / G) of
// the T = items x S units in item-major order, so every CTA gets the same
// number of units whatever the item count (20 items of K = 17408 fill 148
// SMs): an item that lies wholly inside one CTA's range is written to C by
// that CTA; an item split between CTAs leaves fp32 partial tiles (two slots
// per CTA: its first and its last item), which prefill_reduce_kernel adds in
// CTA order (deterministic) and writes to C. Without a workspace, whole items
// go round-robin (item = c + j G).
//
// Every wait is bounded (ptx.cuh: kWaitTimeoutNs).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "formats.cuh"
#include "ptx.cuh"

namespace busfill {

namespace prefill {

constexpr int kThreads = 512;
constexpr int kBatchTile = 128;                 // batch rows per item = MMA N
constexpr int kPairRows = 2 * kTileRows;        // weight rows per item
constexpr int kXStages = 3;                     // half units (2 chunks each)
constexpr int kXChunk = kBatchTile * 128;       // 64 values x 128 rows, 16 KB
constexpr int kXStage = 2 * kXChunk;            // one K half of a unit, 32 KB
constexpr int kAccCols = kBatchTile;            // per weight tile
constexpr int kSlotCols = 64;                   // half a unit
constexpr int kSlot0 = 2 * kAccCols;
constexpr int kTmemCols = 512;
static_assert(kSlot0 + 4 * kSlotCols == kTmemCols, "TMEM map");
constexpr uint32_t kBarSlot0 = 1;          // named barrier of half slot s: kBarSlot0 + s
constexpr uint32_t kSlotBarThreads = 160;  // the tile's 4 dequant warps + the MMA warp

// shared memory map (the weight stage holds both tiles' unit: 256 rows, then
// the rows' second plane: Q4_0 32 KB of nibbles and 4 KB of scales; Q6_K
// 52 KB of block bodies and 512 B of d)
template <WFmt FMT>
struct Smem {
  static constexpr int kWStage = 2 * wstage_bytes<FMT>();
  static constexpr int kWStages = FMT == WFmt::Q5K || FMT == WFmt::Q6K ? 2 : 3;   // Q5_K / Q6_K: 44 / 52.5 KB
  static constexpr int kWOff = 0;
  static constexpr int kXOff = kWOff + kWStages * kWStage;
  static constexpr int kBarOff = kXOff + kXStages * kXStage;
  static constexpr int bWFull = 0, bWEmpty = bWFull + kWStages;
  static constexpr int bXFull = bWEmpty + kWStages, bXEmpty = bXFull + kXStages;
  static constexpr int bSDone = bXEmpty + kXStages;  // half slot s = 2t + h read by its MMAs (commit)
  static constexpr int bAccFull = bSDone + 4, bAccEmpty = bAccFull + 1, bFinal = bAccEmpty + 1;
  static constexpr int kNumBars = bFinal + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kMiscOff + 64;
  static constexpr int kAlloc = kBytes + 1024;
  static_assert(kXOff % 1024 == 0 && kXStage % 1024 == 0, "swizzled operands need 1 KB alignment");
  static_assert(kAlloc <= 232448, "dynamic shared memory per block on sm_100");
};

struct Params {
  void* c;            // [M, N] row-major, OutT
  unsigned* error;    // device error word (+1: first failure record)
  int M, N, K;
  int pairs;          // P = ceil(N / 256); SwiGLU: ceil(N / 128) (gate tile j, up tile j)
  int btiles;         // B = ceil(M / 128)
  int units;          // S = K / 256
  int swiglu;         // 1: C = silu(A Wg^T) * (A Wu^T); tmap_w gate, tmap_ws up (128-row boxes)
  float* part;        // stream-K partial tiles [2 G][128 batch rows][256 weight rows], or nullptr
};

// Stream-K range of CTA c of g over t units: [first_unit(c), first_unit(c + 1)).
__host__ __device__ __forceinline__ long long first_unit(long long t, int c, int g) { return t * c / g; }
// The CTA whose range holds unit x.
__host__ __device__ __forceinline__ int cta_of_unit(long long t, long long x, int g) {
  return (int)(((x + 1) * g - 1) / t);
}
constexpr int kPartElems = kPairRows * kBatchTile;   // one partial tile, fp32

}  // namespace prefill

template <WFmt FMT, typename OutT>
__global__ void __launch_bounds__(prefill::kThreads, 1)
    prefill_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_ws,
                        const __grid_constant__ CUtensorMap tmap_a, const prefill::Params p) {
  using namespace prefill;
  using SM = Smem<FMT>;
  constexpr int kWStage = SM::kWStage, kWStages = SM::kWStages, kWOff = SM::kWOff, kXOff = SM::kXOff;
  constexpr int kBarOff = SM::kBarOff, kMiscOff = SM::kMiscOff, kNumBars = SM::kNumBars;
  constexpr int bWFull = SM::bWFull, bWEmpty = SM::bWEmpty, bXFull = SM::bXFull, bXEmpty = SM::bXEmpty;
  constexpr int bSDone = SM::bSDone, bAccFull = SM::bAccFull, bAccEmpty = SM::bAccEmpty;
  constexpr int bFinal = SM::bFinal;
  constexpr uint32_t kIdesc = make_idesc_f16_f32(kTileRows, kBatchTile);
  constexpr bool kRows144 = aos_rows<FMT>();
  constexpr int kRowBytes = unit_row_bytes<FMT>();
  constexpr int kAuxOff = kPairRows * kRowBytes;   // second plane of the stage's 256 rows

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_s + 1023u) & ~1023u) - raw_s);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + kBarOff;
  auto BAR = [&](int slot) { return bar0 + 8u * (uint32_t)slot; };
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + kMiscOff);  // [0] tmem base

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = p.units;
  const int items = p.pairs * p.btiles;
  const int G = (int)gridDim.x, bid = (int)blockIdx.x;
  const bool sk = p.part != nullptr;   // stream-K ranges, else whole items round-robin
  const long long T = (long long)items * S;
  const long long g0 = sk ? first_unit(T, bid, G) : 0;
  const int nunits = sk ? (int)(first_unit(T, bid + 1, G) - g0) : ((items - bid + G - 1) / G) * S;
  // item and unit k of this CTA's u-th unit
  auto unit_at = [&](int u, int& it, int& k) {
    if (sk) {
      const long long gu = g0 + u;
      it = (int)(gu / S);
      k = (int)(gu - (long long)it * S);
    } else {
      const int j = u / S;
      k = u - j * S;
      it = bid + j * G;
    }
  };
  // pieces: the (partial) items of this CTA, in order
  const int npieces = nunits == 0 ? 0 : sk ? (int)((g0 + nunits - 1) / S - g0 / S + 1) : nunits / S;
  auto piece_item = [&](int j) { return sk ? (int)(g0 / S) + j : bid + j * G; };

  bool ok = true;
  int diag_unit = -1;
  auto warp_wait = [&](uint32_t bar, uint32_t parity) -> bool {
    if (!ok) return false;
    ok = __all_sync(0xffffffffu, mbar_wait(bar, parity));
    if (!ok && lane == 0) {
      const unsigned rec = 0x80000000u | ((unsigned)warp << 24) | ((unsigned)(diag_unit & 0xFFF) << 12) |
                           (((bar - bar0) / 8u) << 1) | parity;
      atomicCAS(p.error + 1, 0u, rec);
    }
    return ok;
  };
  auto bar_count = [&](int b) -> uint32_t {
    if (b >= bWEmpty && b < bWEmpty + kWStages) return 8;  // both tiles' dequant warps
    if (b == bAccEmpty) return 4;                          // the epilogue warps
    return 1;                                              // TMA expect_tx arrivals, MMA commits
  };

  // weight TMA of this CTA's unit u into stage u % kWStages
  auto issue_w = [&](int u) {
    int it, k;
    unit_at(u, it, k);
    const int pair = it / p.btiles;
    const int s = u % kWStages;
    const uint32_t dst = sbase + kWOff + s * kWStage;
    mbar_arrive_expect_tx(BAR(bWFull + s), kWStage);
    if constexpr (kRows144) {
      if (p.swiglu) {
        tma_load_2d(dst, &tmap_w, k * kRowBytes, pair * kTileRows, BAR(bWFull + s), kPolicyEvictLast);
        tma_load_2d(dst + wstage_bytes<FMT>(), &tmap_ws, k * kRowBytes, pair * kTileRows, BAR(bWFull + s),
                    kPolicyEvictLast);
      } else {
        tma_load_2d(dst, &tmap_w, k * kRowBytes, pair * kPairRows, BAR(bWFull + s), kPolicyEvictLast);
        if constexpr (FMT == WFmt::Q6K)  // the 256 rows' block scales d of unit k ([K/256][N] plane)
          tma_load_2d(dst + kAuxOff, &tmap_ws, pair * kPairRows, k, BAR(bWFull + s), kPolicyEvictLast);
      }
    } else {
      tma_load_2d(dst, &tmap_w, k * 128, pair * kPairRows, BAR(bWFull + s), kPolicyEvictLast);
      tma_load_2d(dst + kAuxOff, &tmap_ws, k * 8, pair * kPairRows, BAR(bWFull + s), kPolicyEvictLast);
    }
  };
  // activations of half unit v = 2u + h (chunks 2h, 2h+1 of unit u) into stage v % kXStages
  auto issue_x = [&](int v) {
    const int u = v >> 1, h = v & 1;
    int it, k;
    unit_at(u, it, k);
    const int bt = it % p.btiles;
    const int s = v % kXStages;
    mbar_arrive_expect_tx(BAR(bXFull + s), kXStage);
    tma_load_3d(sbase + kXOff + s * kXStage, &tmap_a, 0, bt * kBatchTile, k * kChunksPerUnit + 2 * h,
                BAR(bXFull + s), kPolicyEvictLast);
  };

  // set-up: barriers by warp 0's lanes, the first weight stages before the
  // CTA-wide sync (weights never depend on an earlier kernel)
  const int w_early = nunits < kWStages ? nunits : kWStages;
  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmap_w);
      if (FMT == WFmt::Q4_0 || FMT == WFmt::Q6K) tma_prefetch_desc(&tmap_ws);
      tma_prefetch_desc(&tmap_a);
    }
    for (int b = lane; b < kNumBars; b += 32) mbar_init(BAR(b), bar_count(b));
    fence_mbar_init();
    __syncwarp();
    if (lane < w_early) issue_w(lane);
    __syncwarp();
  } else if (warp == 1) {
    tmem_alloc(sbase + kMiscOff, prefill::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];
  if (threadIdx.x == 0) pdl_launch_dependents();

  if (warp == 0) {
    // ---------------- weight producer ----------------
    int issued = w_early;
    for (int u = w_early; u < nunits; ++u) {
      diag_unit = u;
      if (!warp_wait(BAR(bWEmpty + u % kWStages), ((u / kWStages) & 1) ^ 1)) break;
      if (elect_one()) issue_w(u);
      __syncwarp();
      issued = u + 1;
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrWeightProducer);
    ok = true;
    for (int u = issued > kWStages ? issued - kWStages : 0; u < issued; ++u)
      if (!warp_wait(BAR(bWFull + u % kWStages), (u / kWStages) & 1)) {
        if (lane == 0) atomicOr(p.error, kErrTeardown);
        break;
      }
  } else if (warp == 1) {
    // ---------------- activation producer ----------------
    pdl_wait_prerequisites();  // activations may be the previous kernel's output
    int issued = 0;
    for (int v = 0; v < 2 * nunits; ++v) {
      diag_unit = v >> 1;
      if (v >= kXStages && !warp_wait(BAR(bXEmpty + v % kXStages), ((v / kXStages) & 1) ^ 1)) break;
      if (elect_one()) issue_x(v);
      __syncwarp();
      issued = v + 1;
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrActProducer);
    ok = true;
    for (int v = issued > kXStages ? issued - kXStages : 0; v < issued; ++v)
      if (!warp_wait(BAR(bXFull + v % kXStages), (v / kXStages) & 1)) {
        if (lane == 0) atomicOr(p.error, kErrTeardown);
        break;
      }
  } else if (warp == 3) {
    // ---------------- MMA issuer ----------------
    const uint64_t bdesc0 = make_sdesc_sw128(sbase + kXOff);
    int j = 0;   // piece
    for (int u = 0; u < nunits; ++u) {
      diag_unit = u;
      int it, k;
      unit_at(u, it, k);
      const bool first = u == 0 || k == 0, last = u == nunits - 1 || k == S - 1;
      // the accumulators are free once the epilogue has read piece j - 1
      if (first && j >= 1) warp_wait(BAR(bAccEmpty), (uint32_t)((j - 1) & 1));
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const int v = 2 * u + h;
        warp_wait(BAR(bXFull + v % kXStages), (v / kXStages) & 1);
        const uint64_t bx = bdesc0 + (uint64_t)(((v % kXStages) * kXStage) >> 4);
#pragma unroll 1
        for (int t = 0; t < 2; ++t) {
          const int sl = 2 * t + h;
          named_bar_sync(prefill::kBarSlot0 + (uint32_t)sl, prefill::kSlotBarThreads);   // the tile's group published the half
          tc_fence_after();
          if (ok && elect_one()) {
            const uint32_t d_acc = tmem + (uint32_t)(t * kAccCols);
            const uint32_t a_t = tmem + (uint32_t)(kSlot0 + sl * kSlotCols);
#pragma unroll
            for (int cl = 0; cl < 2; ++cl)
#pragma unroll
              for (int ks = 0; ks < 4; ++ks)
                mma_f16_ts(d_acc, a_t + cl * 32 + 8 * ks, bx + (uint64_t)(((cl * kXChunk) + 32 * ks) >> 4), kIdesc,
                           (first && h == 0 && cl == 0 && ks == 0) ? 0u : 1u);
            tc_commit(BAR(bSDone + sl));  // half slot free once these MMAs complete
          }
          __syncwarp();
        }
        if (ok && elect_one()) tc_commit(BAR(bXEmpty + v % kXStages));  // activation stage free
        __syncwarp();
      }
      if (ok && elect_one() && last) tc_commit(BAR(bAccFull));  // piece's accumulators complete
      __syncwarp();
      if (last) ++j;
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrMma);
    if (elect_one()) tc_commit(BAR(bFinal));
    __syncwarp();
  } else if (warp >= 4 && warp < 12) {
    // ---------------- dequant (tile t = group) ----------------
    const int q = warp & 3;
    const int t = (warp - 4) >> 2;
    const int r = q * 32 + lane;
    const int row = t * kTileRows + r;       // row within the 256-row weight stage
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    for (int u = 0; u < nunits; ++u) {
      diag_unit = u;
      const int ws = u % kWStages;
      warp_wait(BAR(bWFull + ws), (u / kWStages) & 1);
      const uint8_t* stage = smem + kWOff + ws * kWStage;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const int sl = 2 * t + h;
        // half slot sl is free once the MMAs of the previous unit read it
        if (u >= 1) warp_wait(BAR(bSDone + sl), (uint32_t)((u - 1) & 1));
        tc_fence_after();
        if (ok) {
          const uint32_t a_col = tmem + lane_off + (uint32_t)(kSlot0 + sl * kSlotCols);
          if (h == 0)
            dequant_unit_row<FMT, 0, 2>(stage, stage + kAuxOff, row, a_col);
          else
            dequant_unit_row<FMT, 2, 4>(stage, stage + kAuxOff, row, a_col);
          tc_wait_st();
        }
        tc_fence_before();
        __syncwarp();
        named_bar_arrive(prefill::kBarSlot0 + (uint32_t)sl, prefill::kSlotBarThreads);   // always: the MMA warp syncs on every half
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(bWEmpty + ws));
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrDequant);
  } else if (warp >= 12) {
    // ---------------- epilogue ----------------
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    OutT* C = reinterpret_cast<OutT*>(p.c);
    bool waited_pdl = false;
    for (int j = 0; j < npieces; ++j) {
      diag_unit = j;
      const int it = piece_item(j);
      const int pair = it / p.btiles, bt = it % p.btiles;
      // stream-K: a piece that is not the whole item goes to the CTA's partial
      // slot (2 bid for its first item, 2 bid + 1 for its last)
      const bool whole = !sk || ((long long)it * S >= g0 && (long long)(it + 1) * S <= g0 + nunits);
      float* part = whole ? nullptr : p.part + (size_t)(2 * bid + (j == 0 ? 0 : 1)) * kPartElems;
      // batch rows of the item that exist: only those are read from TMEM and written
      const int mv = min(kBatchTile, p.M - bt * kBatchTile);
      const bool have = warp_wait(BAR(bAccFull), (uint32_t)(j & 1));
      tc_fence_after();
      if (!waited_pdl) {
        pdl_wait_prerequisites();  // C may still be read by the previous kernel
        waited_pdl = true;
      }
      if (p.swiglu) {
        // accumulator 0 holds the gate tile, 1 the up tile of the same rows
        const int n = pair * kTileRows + r;
#pragma unroll 1
        for (int cb = 0; cb < mv; cb += 16) {
          uint32_t xg[16], xu[16];
          tmem_ld_x16(tmem + lane_off + (uint32_t)cb, xg);
          tmem_ld_x16(tmem + lane_off + (uint32_t)(kAccCols + cb), xu);
          tc_wait_ld();
          if (have && n < p.N) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int b = bt * kBatchTile + cb + i;
              if (b < p.M)
                C[(size_t)b * p.N + n] = to_out<OutT>(silu(__uint_as_float(xg[i])) * __uint_as_float(xu[i]));
            }
          }
        }
      } else {
#pragma unroll 1
        for (int t = 0; t < 2; ++t) {
          const int n = pair * kPairRows + t * kTileRows + r;
#pragma unroll 1
          for (int cb = 0; cb < mv; cb += 32) {
            uint32_t x[32];
            tmem_ld_x16(tmem + lane_off + (uint32_t)(t * kAccCols + cb), x);
            tmem_ld_x16(tmem + lane_off + (uint32_t)(t * kAccCols + cb + 16), x + 16);
            tc_wait_ld();
            if (have && part) {
              // [batch row][weight row] of the pair, the item's existing batch rows
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (cb + i < mv) part[(cb + i) * kPairRows + t * kTileRows + r] = __uint_as_float(x[i]);
            } else if (have && n < p.N) {
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const int b = bt * kBatchTile + cb + i;
                if (b < p.M) C[(size_t)b * p.N + n] = to_out<OutT>(__uint_as_float(x[i]));
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(bAccEmpty));
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrEpilogue);
  }

  // ---------------- teardown ----------------
  __syncwarp();
  __syncthreads();
  if (warp == 1) {
    bool done = true;
    if (lane == 0) done = mbar_wait(BAR(bFinal), 0);
    done = __shfl_sync(0xffffffffu, done ? 1 : 0, 0) != 0;
    if (!done && lane == 0) atomicOr(p.error, kErrTeardown);
    tc_fence_after();
    tmem_dealloc(tmem, prefill::kTmemCols);
  }
}

// The items a stream-K prefill launch splits between CTAs, listed by the host
// (split_items): for each, the item, its first and last CTA and the first
// CTA's partial slot (every later CTA holds the item as its first piece, slot
// 2 c). A launch of G CTAs splits at most G - 1 items.
namespace prefill {
constexpr int kMaxSplitItems = 200;
struct SplitItems {
  int n;
  int4 e[kMaxSplitItems];   // {item, c_lo, c_hi, slot of c_lo}
};
}  // namespace prefill

// Stream-K fix-up: each split item is summed from its CTAs' partial tiles, in
// CTA order, and written to C. Block (x, y): split item x, batch rows 4 y ..
// 4 y + 3 of the item, 64 threads per row, each owning 4 consecutive weight
// rows of the pair (one 16-byte load per partial tile). The loads of up to
// eight partial tiles are issued together and added in CTA order.
template <typename OutT>
__global__ void __launch_bounds__(256) prefill_reduce_kernel(const float* __restrict__ part, OutT* __restrict__ c,
                                                           int M, int N, int btiles,
                                                           const __grid_constant__ prefill::SplitItems si) {
  using namespace prefill;
  pdl_wait_prerequisites();   // the partial tiles are the previous kernel's output
  // the next kernel may start its set-up and weight loads; it reads C, and
  // writes partial tiles, only after its own wait for this grid to finish
  pdl_launch_dependents();
  const int4 e = si.e[blockIdx.x];
  const int it = e.x, c_lo = e.y, c_hi = e.z, slot_lo = e.w;
  const int pair = it / btiles, bt = it - (it / btiles) * btiles;
  const int row = 4 * (int)blockIdx.y + ((int)threadIdx.x >> 6);          // batch row within the item
  const int col = 4 * ((int)threadIdx.x & 63);                            // weight row within the pair
  if (bt * kBatchTile + row >= M) return;
  const size_t off = (size_t)row * kPairRows + col;
  auto slot_ptr = [&](int cc) {
    const int slot = cc == c_lo ? slot_lo : 2 * cc;
    return reinterpret_cast<const float4*>(part + (size_t)slot * kPartElems + off);
  };
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int c0 = c_lo; c0 <= c_hi; c0 += 8) {
    float4 v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (c0 + i <= c_hi) v[i] = *slot_ptr(c0 + i);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (c0 + i <= c_hi) {
        acc.x += v[i].x;
        acc.y += v[i].y;
        acc.z += v[i].z;
        acc.w += v[i].w;
      }
  }
  const int b = bt * kBatchTile + row;
  const int n = pair * kPairRows + col;
  OutT* dst = c + (size_t)b * N + n;
  if (n < N) dst[0] = to_out<OutT>(acc.x);
  if (n + 1 < N) dst[1] = to_out<OutT>(acc.y);
  if (n + 2 < N) dst[2] = to_out<OutT>(acc.z);
  if (n + 3 < N) dst[3] = to_out<OutT>(acc.w);
}

}  // namespace busfill
