// Dequant-fused 4-bit-weight GEMM for large batches (prefill, M >= ~128) on
// sm_100a: C[M, N] = A[M, K] * deq(W)[N, K]^T, fp16 in, fp32 accumulate.
//
// The same contraction as the decode kernel (decode_gemm.cuh), in the regime
// where it turns compute-bound: at M = 2048 the work is 2 M N K flops against
// one pass of 4.5-bit weights, so the tensor pipe, not HBM, sets the time.
// The reference has no such path (its kernel computes batch rows < 32 only,
// kernels/busfill_v1a.cu:41-104); the shapes are BASELINE config 4.
//
// Shape of the computation. A work item is BT batch rows x the weight rows
// of one or two 128-row tiles (Geo below), looped over K in units of 256.
// The weights of a unit are dequantized into tensor memory (the MMA's A
// operand) and the fp32 accumulators live in TMEM next to them:
//   columns   0..255  accumulators: BT = 128, tile 0 then tile 1 [128 weight
//                     rows x 128 batch rows] each; BT = 256, the one tile
//                     [128 weight rows x 256 batch rows]
//   columns 256..511  four half-unit operand slots of 64 columns (one K half,
//                     chunks 2h and 2h+1, of one tile)
// BT = 256 (from M = 256) halves the dequant work per flop and lets two
// units sit in TMEM at once; BT = 128 serves M < 256 and the SwiGLU pairs
// (gate and up accumulators of the same rows). Activations come as 3-D TMA
// boxes of 32 KB (BT = 128: a K half, 2 chunks x 128 rows; BT = 256: one
// chunk x 256 rows, released as soon as its four MMAs complete) and weights
// as one box per unit of the item's rows.
//
// Measured on B200: a 128x128x16 TS MMA (A in TMEM) takes ~74 cycles back to
// back, 92% of the dense fp16 rate; a unit (2 x 128 x 256 x 256 MACs) ~2400
// cycles. A per-unit clock64 trace at M = 512, N = 17408, K = 5120 (BT = 256)
// puts a unit at ~2900-3100 cycles of the MMA warp: ~1600 issuing MMAs (the
// tensor pipe's back-pressure), ~800 waiting for activation boxes (L2 to SM
// traffic: 128 KB of activations per unit) and ~500 of loop overhead. The
// loops step their (item, unit) cursor instead of dividing: a 64-bit
// division per unit had cost each producer and the MMA warp ~400-600 cycles.
//
// Handoffs: a dequant warp group publishes a half slot with a named-barrier
// arrive that the MMA warp syncs on (no mbarrier round trip on the path of
// every 8 MMAs); the slot comes back through the commit barrier of its MMAs.
// Named barriers have no timeout, so every group arrives, and the MMA warp
// syncs, for every half slot of every unit whatever happens (work is skipped
// after a failed wait, the arrivals are not).
//
// Warp roles (16 warps, one CTA per SM, persistent over work items):
//   0      weight TMA producer (ring of 2-3 units)
//   1      activation TMA producer (ring of 32 KB stages); TMEM allocator
//   3      MMA issuer (converged warp, one elected thread issues)
//   4-11   dequant, two groups of four warps (see Geo): thread (warp%4, lane)
//          owns row 32*(warp%4)+lane of its weight tile
//   12-15  epilogue: reads the accumulators once per item, writes C
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
constexpr int kDequantWarp0 = 4, kEpilogueWarp0 = 12;
constexpr int kSlotCols = 64;                   // half a unit of one weight tile
constexpr int kSlot0 = 256;                     // after the accumulators
constexpr int kTmemCols = 512;
static_assert(kSlot0 + 4 * kSlotCols == kTmemCols, "TMEM map");
constexpr uint32_t kBarSlot0 = 1;          // named barrier of half slot s: kBarSlot0 + s
constexpr uint32_t kSlotBarThreads = 160;  // the slot's 4 dequant warps + the MMA warp
constexpr int kXStageBytes = 32768;        // one activation stage

// Item geometry by batch tile BT (= the MMA's N):
//   BT = 128: two 128-row weight tiles x 128 batch rows; an activation stage
//             is a K half of a unit (2 chunks x 128 rows); half slot s = 2t + h
//             holds tile t's K half h of the current unit.
//   BT = 256: one weight tile x 256 batch rows (MMAs of 128x256x16); a stage
//             is one chunk x 256 rows; half slot s = 2 (u % 2) + h holds K half
//             h of unit u, so two units are in TMEM at once. Every dequantized
//             weight feeds twice the batch rows: half the dequant per flop.
// Dequant warp group g (four warps, one per TMEM lane quarter) writes, of
// every unit, BT = 128: both K halves of tile g (half slots 2g, 2g + 1);
// BT = 256: K half g, into half slot 2 (u % 2) + g. Every dequant warp takes
// every unit, so each waits on every phase of the barriers it uses (a warp
// that skipped units could see a barrier two phases back as complete).
template <int BT>
struct Geo {
  static_assert(BT == 128 || BT == 256, "batch tile");
  static constexpr int kTiles = BT == 128 ? 2 : 1;          // weight tiles per item
  static constexpr int kItemRows = kTiles * kTileRows;      // weight rows per item
  static constexpr int kXChunks = BT == 128 ? 2 : 1;        // 64-value chunks per activation stage
  static constexpr int kXPerUnit = kChunksPerUnit / kXChunks;
  static constexpr int kXChunkBytes = BT * 128;             // 64 values x BT rows
  static_assert(kXChunks * kXChunkBytes == kXStageBytes, "activation stage");
  static_assert(kTiles * BT == kSlot0, "accumulators: 256 columns");
};
constexpr int kPartElems = 256 * 128;   // one partial tile, fp32: BT batch rows x item rows

// shared memory map: weight stages of one unit of the item's rows (then the
// rows' second plane: Q4_0 scales, Q6_K d), activation stages, barriers
template <WFmt FMT, int BT>
struct Smem {
  using GE = Geo<BT>;
  static constexpr int kWStage = GE::kTiles * wstage_bytes<FMT>();
  static constexpr int kXStages = BT == 128 ? 3 : 5;
  static constexpr int kWStages =
      kXStages * kXStageBytes + 3 * kWStage + 3072 <= 232448 ? 3 : 2;   // Q5_K / Q6_K: 2
  static constexpr int kWOff = 0;
  static constexpr int kXOff = (kWOff + kWStages * kWStage + 1023) / 1024 * 1024;
  static constexpr int kBarOff = kXOff + kXStages * kXStageBytes;
  static constexpr int bWFull = 0, bWEmpty = bWFull + kWStages;
  static constexpr int bXFull = bWEmpty + kWStages, bXEmpty = bXFull + kXStages;
  static constexpr int bSDone = bXEmpty + kXStages;  // half slot s = 2t + h read by its MMAs (commit)
  static constexpr int bAccFull = bSDone + 4, bAccEmpty = bAccFull + 1, bFinal = bAccEmpty + 1;
  static constexpr int kNumBars = bFinal + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kMiscOff + 64;
  static constexpr int kAlloc = kBytes + 1024;
  static_assert(kXOff % 1024 == 0, "swizzled operands need 1 KB alignment");
  static_assert(kAlloc <= 232448, "dynamic shared memory per block on sm_100");
};

struct Params {
  void* c;            // [M, N] row-major, OutT
  unsigned* error;    // device error word (+1: first failure record)
  int M, N, K;
  int pairs;          // P = ceil(N / item rows); SwiGLU: ceil(N / 128) (gate tile j, up tile j)
  int btiles;         // B = ceil(M / BT)
  int units;          // S = K / 256
  int swiglu;         // 1: C = silu(A Wg^T) * (A Wu^T); tmap_w gate, tmap_ws up (128-row boxes)
  float* part;        // stream-K partial tiles [2 G][BT batch rows][item rows], or nullptr
  int gate_mul;       // CTA-pair kernel: 1 = C holds the up projection (fp16); write silu(A W^T) * C
};

// Stream-K range of CTA c of g over t units: [first_unit(c), first_unit(c + 1)).
__host__ __device__ __forceinline__ long long first_unit(long long t, int c, int g) { return t * c / g; }
// The CTA whose range holds unit x.
__host__ __device__ __forceinline__ int cta_of_unit(long long t, long long x, int g) {
  return (int)(((x + 1) * g - 1) / t);
}
}  // namespace prefill

template <WFmt FMT, typename OutT, int BT>
__global__ void __launch_bounds__(prefill::kThreads, 1)
    prefill_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_ws,
                        const __grid_constant__ CUtensorMap tmap_a, const prefill::Params p) {
  using namespace prefill;
  using SM = Smem<FMT, BT>;
  using GE = Geo<BT>;
  constexpr int kTiles = GE::kTiles, kItemRows = GE::kItemRows, kXPerUnit = GE::kXPerUnit;
  constexpr int kXChunks = GE::kXChunks, kXChunkBytes = GE::kXChunkBytes, kXStages = SM::kXStages;
  constexpr int kWStage = SM::kWStage, kWStages = SM::kWStages, kWOff = SM::kWOff, kXOff = SM::kXOff;
  constexpr int kBarOff = SM::kBarOff, kMiscOff = SM::kMiscOff, kNumBars = SM::kNumBars;
  constexpr int bWFull = SM::bWFull, bWEmpty = SM::bWEmpty, bXFull = SM::bXFull, bXEmpty = SM::bXEmpty;
  constexpr int bSDone = SM::bSDone, bAccFull = SM::bAccFull, bAccEmpty = SM::bAccEmpty;
  constexpr int bFinal = SM::bFinal;
  constexpr uint32_t kIdesc = make_idesc_f16_f32(kTileRows, BT);
  constexpr bool kRows144 = aos_rows<FMT>();
  constexpr int kRowBytes = unit_row_bytes<FMT>();
  constexpr int kAuxOff = kItemRows * kRowBytes;   // second plane of the stage's rows

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
  // item and unit k of this CTA's u-th unit (T < 2^31: items x S units fit
  // an int); the role loops step (it, k) with next_unit instead, a division
  // per unit costing the MMA and producer warps hundreds of cycles each
  auto unit_at = [&](int u, int& it, int& k) {
    if (sk) {
      const int gu = (int)g0 + u;
      it = gu / S;
      k = gu - it * S;
    } else {
      const int j = u / S;
      k = u - j * S;
      it = bid + j * G;
    }
  };
  auto next_unit = [&](int& it, int& k) {
    if (++k == S) {
      k = 0;
      it += sk ? 1 : G;
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
    if (b >= bWEmpty && b < bWEmpty + kWStages) return 8;  // every dequant warp
    if (b == bAccEmpty) return 4;                          // the epilogue warps
    return 1;                                              // TMA expect_tx arrivals, MMA commits
  };

  // weight TMA of this CTA's unit u (item it, K unit k) into stage u % kWStages
  auto issue_w = [&](int u, int it, int k) {
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
        tma_load_2d(dst, &tmap_w, k * kRowBytes, pair * kItemRows, BAR(bWFull + s), kPolicyEvictLast);
        if constexpr (FMT == WFmt::Q6K)  // the item rows' block scales d of unit k ([K/256][N] plane)
          tma_load_2d(dst + kAuxOff, &tmap_ws, pair * kItemRows, k, BAR(bWFull + s), kPolicyEvictLast);
      }
    } else {
      tma_load_2d(dst, &tmap_w, k * 128, pair * kItemRows, BAR(bWFull + s), kPolicyEvictLast);
      tma_load_2d(dst + kAuxOff, &tmap_ws, k * 8, pair * kItemRows, BAR(bWFull + s), kPolicyEvictLast);
    }
  };
  // activation piece v = kXPerUnit u + c (chunks c kXChunks .. of unit u: item
  // it, K unit k) into stage v % kXStages
  auto issue_x = [&](int v, int it, int k, int c) {
    const int bt = it % p.btiles;
    const int s = v % kXStages;
    mbar_arrive_expect_tx(BAR(bXFull + s), kXStageBytes);
    tma_load_3d(sbase + kXOff + s * kXStageBytes, &tmap_a, 0, bt * BT, k * kChunksPerUnit + c * kXChunks,
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
    if (lane < w_early) {
      int it, k;
      unit_at(lane, it, k);
      issue_w(lane, it, k);
    }
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
    int it, k;
    unit_at(w_early, it, k);
    for (int u = w_early; u < nunits; ++u) {
      diag_unit = u;
      if (!warp_wait(BAR(bWEmpty + u % kWStages), ((u / kWStages) & 1) ^ 1)) break;
      if (elect_one()) issue_w(u, it, k);
      __syncwarp();
      issued = u + 1;
      next_unit(it, k);
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
    int it, k, c = 0;
    unit_at(0, it, k);
    for (int v = 0; v < kXPerUnit * nunits; ++v) {
      diag_unit = v / kXPerUnit;
      if (v >= kXStages && !warp_wait(BAR(bXEmpty + v % kXStages), ((v / kXStages) & 1) ^ 1)) break;
      if (elect_one()) issue_x(v, it, k, c);
      __syncwarp();
      issued = v + 1;
      if (++c == kXPerUnit) {
        c = 0;
        next_unit(it, k);
      }
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
    int it, k;
    unit_at(0, it, k);
    for (int u = 0; u < nunits; ++u, next_unit(it, k)) {
      diag_unit = u;
      const bool first = u == 0 || k == 0, last = u == nunits - 1 || k == S - 1;
      // the accumulators are free once the epilogue has read piece j - 1
      if (first && j >= 1) warp_wait(BAR(bAccEmpty), (uint32_t)((j - 1) & 1));
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        // the half's activation stages: pieces v0 .. v0 + 2 / kXChunks - 1; with
        // one chunk a stage (BT = 256) the second is waited for only after the
        // first chunk's MMAs are issued, and each stage is released right after
        // its own MMAs
        const int v0 = (2 * u + h) * (2 / kXChunks);
        warp_wait(BAR(bXFull + v0 % kXStages), (v0 / kXStages) & 1);
#pragma unroll 1
        for (int t = 0; t < kTiles; ++t) {
          const int sl = BT == 128 ? 2 * t + h : 2 * (u & 1) + h;
          named_bar_sync(prefill::kBarSlot0 + (uint32_t)sl, kSlotBarThreads);   // the slot's dequant warps published it
          tc_fence_after();
          const uint32_t d_acc = tmem + (uint32_t)(t * BT);
          const uint32_t a_t = tmem + (uint32_t)(kSlot0 + sl * kSlotCols);
#pragma unroll
          for (int cl = 0; cl < 2; ++cl) {
            // chunk 2h + cl: stage of piece v0 + cl (one chunk a stage) or chunk cl of stage v0
            const int v = kXChunks == 1 ? v0 + cl : v0;
            if (kXChunks == 1 && cl == 1) warp_wait(BAR(bXFull + v % kXStages), (v / kXStages) & 1);
            if (ok && elect_one()) {
              const uint64_t bx =
                  bdesc0 + (uint64_t)(((v % kXStages) * kXStageBytes + (kXChunks == 1 ? 0 : cl * kXChunkBytes)) >> 4);
#pragma unroll
              for (int ks = 0; ks < 4; ++ks)
                mma_f16_ts(d_acc, a_t + cl * 32 + 8 * ks, bx + (uint64_t)((32 * ks) >> 4), kIdesc,
                           (first && h == 0 && cl == 0 && ks == 0) ? 0u : 1u);
              if (kXChunks == 1) tc_commit(BAR(bXEmpty + v % kXStages));   // chunk stage free
              if (cl == 1) tc_commit(BAR(bSDone + sl));   // half slot free once these MMAs complete
            }
            __syncwarp();
          }
        }
        if (kXChunks == 2 && ok && elect_one()) tc_commit(BAR(bXEmpty + v0 % kXStages));  // both tiles read the stage
        __syncwarp();
      }
      if (ok && elect_one() && last) tc_commit(BAR(bAccFull));  // piece's accumulators complete
      __syncwarp();
      if (last) ++j;
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrMma);
    if (elect_one()) tc_commit(BAR(bFinal));
    __syncwarp();
  } else if (warp >= kDequantWarp0 && warp < kEpilogueWarp0) {
    // ---------------- dequant (group g of every unit) ----------------
    const int q = warp & 3;
    const int g = (warp - kDequantWarp0) >> 2;
    const int t = BT == 128 ? g : 0;
    const int r = q * 32 + lane;
    const int row = t * kTileRows + r;       // row within the weight stage
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    for (int u = 0; u < nunits; ++u) {
      diag_unit = u;
      const int ws = u % kWStages;
      warp_wait(BAR(bWFull + ws), (u / kWStages) & 1);
      const uint8_t* stage = smem + kWOff + ws * kWStage;
#pragma unroll 1
      for (int hh = 0; hh < kTiles; ++hh) {   // BT = 128: both halves of tile g; BT = 256: half g
        const int h = BT == 128 ? hh : g;
        const int sl = BT == 128 ? 2 * t + h : 2 * (u & 1) + h;
        // half slot sl is free once the MMAs of its previous use read it
        const int use = BT == 128 ? u : u >> 1;
        if (use >= 1) warp_wait(BAR(bSDone + sl), (uint32_t)((use - 1) & 1));
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
        named_bar_arrive(prefill::kBarSlot0 + (uint32_t)sl, kSlotBarThreads);   // always: the MMA warp syncs on every half
      }
      if (lane == 0) mbar_arrive(BAR(bWEmpty + ws));
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrDequant);
  } else if (warp >= kEpilogueWarp0) {
    // ---------------- epilogue ----------------
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    OutT* C = reinterpret_cast<OutT*>(p.c);
    // fp16 C with rows of a multiple of 8 values on a 16-byte boundary: vector stores
    const bool vec16 = sizeof(OutT) == 2 && (p.N & 7) == 0 && (reinterpret_cast<uintptr_t>(p.c) & 15) == 0;
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
      const int mv = min(BT, p.M - bt * BT);
      const bool have = warp_wait(BAR(bAccFull), (uint32_t)(j & 1));
      tc_fence_after();
      if (!waited_pdl) {
        pdl_wait_prerequisites();  // C may still be read by the previous kernel
        waited_pdl = true;
      }
      if (BT == 128 && p.swiglu) {
        // accumulator 0 holds the gate tile, 1 the up tile of the same rows
        const int n = pair * kTileRows + r;
#pragma unroll 1
        for (int cb = 0; cb < mv; cb += 16) {
          uint32_t xg[16], xu[16];
          tmem_ld_x16(tmem + lane_off + (uint32_t)cb, xg);
          tmem_ld_x16(tmem + lane_off + (uint32_t)(BT + cb), xu);
          tc_wait_ld();
          if (have && n < p.N) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int b = bt * BT + cb + i;
              if (b < p.M)
                C[(size_t)b * p.N + n] = to_out<OutT>(silu(__uint_as_float(xg[i])) * __uint_as_float(xu[i]));
            }
          }
        }
      } else {
#pragma unroll 1
        for (int t = 0; t < kTiles; ++t) {
          const int n = pair * kItemRows + t * kTileRows + r;
#pragma unroll 1
          for (int cb = 0; cb < mv; cb += 32) {
            uint32_t x[32];
            tmem_ld_x16(tmem + lane_off + (uint32_t)(t * BT + cb), x);
            tmem_ld_x16(tmem + lane_off + (uint32_t)(t * BT + cb + 16), x + 16);
            tc_wait_ld();
            if (have && part) {
              // [batch row][weight row] of the item, the item's existing batch rows
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (cb + i < mv) part[(cb + i) * kItemRows + t * kTileRows + r] = __uint_as_float(x[i]);
            } else if (have && vec16) {
              // lane j of each group of 8 then holds batch row 8b + j of the
              // group's 8 consecutive weight rows: one 16-byte store per block
              // (2-byte stores strided by N made the drain of an item ~2.4x
              // longer, and the next item's MMAs wait for it)
              float* v = reinterpret_cast<float*>(x);
              transpose_8x8_blocks<32>(v, lane);
              const int n0 = n - (lane & 7);
#pragma unroll
              for (int b = 0; b < 4; ++b) {
                const int row = bt * BT + cb + 8 * b + (lane & 7);
                if (row < p.M && n0 < p.N) {   // N % 8 == 0: the group's 8 rows are all in range
                  uint4 w;
                  w.x = h2_as_u32(__floats2half2_rn(v[8 * b], v[8 * b + 1]));
                  w.y = h2_as_u32(__floats2half2_rn(v[8 * b + 2], v[8 * b + 3]));
                  w.z = h2_as_u32(__floats2half2_rn(v[8 * b + 4], v[8 * b + 5]));
                  w.w = h2_as_u32(__floats2half2_rn(v[8 * b + 6], v[8 * b + 7]));
                  *reinterpret_cast<uint4*>(C + (size_t)row * p.N + n0) = w;
                }
              }
            } else if (have && n < p.N) {
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const int b = bt * BT + cb + i;
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
// CTA order, and written to C. Block (x, y): split item x, batch rows
// kRowsPerBlock y .. of the item, item rows / 4 threads per batch row, each
// owning 4 consecutive weight rows of the item (one 16-byte load per partial
// tile). The loads of up to eight partial tiles are issued together and added
// in CTA order.
template <typename OutT, int BT>
__global__ void __launch_bounds__(256) prefill_reduce_kernel(const float* __restrict__ part, OutT* __restrict__ c,
                                                           int M, int N, int btiles,
                                                           const __grid_constant__ prefill::SplitItems si) {
  using namespace prefill;
  constexpr int kItemRows = Geo<BT>::kItemRows;
  constexpr int kRowThreads = kItemRows / 4;
  constexpr int kRowsPerBlock = 256 / kRowThreads;
  pdl_wait_prerequisites();   // the partial tiles are the previous kernel's output
  // the next kernel may start its set-up and weight loads; it reads C, and
  // writes partial tiles, only after its own wait for this grid to finish
  pdl_launch_dependents();
  const int4 e = si.e[blockIdx.x];
  const int it = e.x, c_lo = e.y, c_hi = e.z, slot_lo = e.w;
  const int pair = it / btiles, bt = it - (it / btiles) * btiles;
  const int row = kRowsPerBlock * (int)blockIdx.y + (int)threadIdx.x / kRowThreads;   // batch row within the item
  const int col = 4 * ((int)threadIdx.x % kRowThreads);                             // weight row within the item
  if (bt * BT + row >= M) return;
  const size_t off = (size_t)row * kItemRows + col;
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
  const int b = bt * BT + row;
  const int n = pair * kItemRows + col;
  OutT* dst = c + (size_t)b * N + n;
  if (n < N) dst[0] = to_out<OutT>(acc.x);
  if (n + 1 < N) dst[1] = to_out<OutT>(acc.y);
  if (n + 2 < N) dst[2] = to_out<OutT>(acc.z);
  if (n + 3 < N) dst[3] = to_out<OutT>(acc.w);
}

}  // namespace busfill
