// Dequant-fused 4-bit-weight GEMM for large batches on CTA pairs (sm_100a,
// tcgen05 cta_group::2): C[M, N] = A[M, K] * deq(W)[N, K]^T, fp16 in, fp32
// accumulate. The same contraction, stream-K split and numerics as
// prefill_gemm_kernel (prefill_gemm.cuh), with work items of 256 weight rows
// x 256 batch rows computed by the two CTAs of a 2-CTA cluster together.
//
// Why pairs. In the one-CTA kernel with 256-row batch tiles every unit of
// 128 x 256 x 256 MACs pulls 128 KB of activations from L2 into the SM; a
// per-unit trace put ~800 of its ~3000 MMA-warp cycles in waits for those
// boxes. A pair MMA (M = 256: 128 weight rows from each CTA's TMEM; N = 256:
// 128 batch rows from each CTA's shared memory) does the same MACs per SM
// with each CTA loading only its half of the batch rows: 64 KB a unit.
//
// Per CTA (rank r of the pair): weight rows 256 g + 128 r .. + 127 of item
// group g, dequantized into its own TMEM; batch rows 256 b + 128 r .. + 127
// of batch tile b, in its own shared memory; accumulator [its 128 weight rows
// x the item's 256 batch rows] fp32 in its own TMEM (columns 0..255), four
// half-unit operand slots at 256..511 (slot 2 (u % 2) + h: K half h of unit
// u), each with a 32 KB activation stage (chunks 2h, 2h+1 of this CTA's 128
// batch rows). Rank 0 issues every MMA; its commits arrive on the barrier at
// the same offset in both CTAs (half slot and stage free, accumulator full).
// A half slot becomes ready on one barrier of rank 0 that counts both CTAs'
// activation bytes (cta_group::2 copies), both CTAs' dequant warps and rank
// 0's producer, so the MMA warp waits once per 8 MMAs: a per-unit trace had
// six waits per unit (slot, then each chunk's stage, for both halves) costing
// the MMA warp ~1200 cycles even when everything had landed. Rank 1's dequant
// warps arrive remotely without release semantics (their TMEM stores are
// complete by tcgen05.wait::st; a release arrival at cluster scope stalled
// each of them ~1000-1600 cycles per half unit); the epilogue warps arrive on
// rank 0's accumulator barrier with release.
//
// Warp roles (16 warps per CTA, one CTA per SM, persistent over the pair's
// range of units):
//   0      weight TMA producer (this CTA's 128 rows, ring of 3 units)
//   1      activation TMA producer (this CTA's 128 batch rows, a 32 KB
//          stage per half slot); TMEM allocator (collective over the pair)
//   3      MMA issuer (rank 0 only; one elected thread)
//   4-11   dequant: group g = K half g of every unit; thread (warp%4, lane)
//          owns weight row 32*(warp%4)+lane of this CTA's 128
//   12-15  epilogue: this CTA's 128 weight rows of each item
//   2      idle
//
// Every mbarrier wait is bounded (ptx.cuh: kWaitTimeoutNs); the only other
// waits are the two cluster barriers (set-up, teardown), which every thread
// of both CTAs reaches once.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "formats.cuh"
#include "prefill_gemm.cuh"
#include "ptx.cuh"

namespace busfill {

namespace prefill_pair {

constexpr int kThreads = 512;
constexpr int kDequantWarp0 = 4, kEpilogueWarp0 = 12;
constexpr int kItemRows = 256;                  // weight rows per item (128 per CTA)
constexpr int kBatchTile = 256;                 // batch rows per item (128 per CTA)
constexpr int kXChunkBytes = 128 * 128;         // one 64-value chunk x this CTA's 128 batch rows
constexpr int kXStageBytes = 2 * kXChunkBytes;  // a K half of a unit: chunks 2h, 2h + 1
constexpr int kSlot0 = 256, kSlotCols = 64, kTmemCols = 512;
constexpr uint16_t kPairMask = 0x3;             // both CTAs of the pair
static_assert(prefill::kPartElems == 128 * kBatchTile, "a CTA's partial tile fills one workspace slot");

template <WFmt FMT>
struct Smem {
  static constexpr int kWStage = wstage_bytes<FMT>();   // this CTA's 128 rows, one unit
  static constexpr int kWStages = 3;
  static constexpr int kXOff = (kWStages * kWStage + 1023) / 1024 * 1024;
  static constexpr int kBarOff = kXOff + 4 * kXStageBytes;   // one activation stage per half slot
  static constexpr int bWFull = 0, bWEmpty = bWFull + kWStages;
  // half slot s (TMEM operand + activation stage): rank 0's bReady counts both
  // CTAs' dequant warps, rank 0's producer arrival and both CTAs' bytes; each
  // CTA's bFree completes when the slot's MMAs have
  static constexpr int bReady = bWEmpty + kWStages, bFree = bReady + 4;
  static constexpr int bAccFull = bFree + 4, bAccEmpty = bAccFull + 1, bFinal = bAccEmpty + 1;
  static constexpr int kNumBars = bFinal + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kMiscOff + 64;
  static constexpr int kAlloc = kBytes + 1024;
  static_assert(kAlloc <= 232448, "dynamic shared memory per block on sm_100");
};

}  // namespace prefill_pair

template <WFmt FMT, typename OutT>
__global__ void __launch_bounds__(prefill_pair::kThreads, 1)
    prefill_pair_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_ws,
                        const __grid_constant__ CUtensorMap tmap_a, const prefill::Params p) {
  using namespace prefill_pair;
  using SM = Smem<FMT>;
  constexpr int kWStage = SM::kWStage, kWStages = SM::kWStages, kXOff = SM::kXOff;
  constexpr int kBarOff = SM::kBarOff, kMiscOff = SM::kMiscOff, kNumBars = SM::kNumBars;
  constexpr int bWFull = SM::bWFull, bWEmpty = SM::bWEmpty, bReady = SM::bReady, bFree = SM::bFree;
  constexpr int bAccFull = SM::bAccFull, bAccEmpty = SM::bAccEmpty;
  constexpr int bFinal = SM::bFinal;
  constexpr uint32_t kIdesc = make_idesc_f16_f32(2 * kTileRows, kBatchTile);
  constexpr bool kRows144 = aos_rows<FMT>();
  constexpr int kRowBytes = unit_row_bytes<FMT>();
  constexpr int kAuxOff = kTileRows * kRowBytes;   // second plane of the stage's 128 rows

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_s + 1023u) & ~1023u) - raw_s);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + kBarOff;
  auto BAR = [&](int slot) { return bar0 + 8u * (uint32_t)slot; };
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + kMiscOff);  // [0] tmem base

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = (int)cluster_ctarank();         // clusters of 2 tile the grid in blockIdx order
  const int pr = (int)(blockIdx.x >> 1), G = (int)(gridDim.x >> 1);
  const int S = p.units;
  const int items = p.pairs * p.btiles;
  const bool sk = p.part != nullptr;   // stream-K ranges, else whole items round-robin
  const long long T = (long long)items * S;
  const long long g0 = sk ? prefill::first_unit(T, pr, G) : 0;
  const int nunits = sk ? (int)(prefill::first_unit(T, pr + 1, G) - g0) : ((items - pr + G - 1) / G) * S;
  // item and unit k of the pair's u-th unit (T < 2^31); the role loops step a cursor
  auto unit_at = [&](int u, int& it, int& k) {
    if (sk) {
      const int gu = (int)g0 + u;
      it = gu / S;
      k = gu - it * S;
    } else {
      const int j = u / S;
      k = u - j * S;
      it = pr + j * G;
    }
  };
  auto next_unit = [&](int& it, int& k) {
    if (++k == S) {
      k = 0;
      it += sk ? 1 : G;
    }
  };
  const int npieces = nunits == 0 ? 0 : sk ? (int)((g0 + nunits - 1) / S - g0 / S + 1) : nunits / S;
  auto piece_item = [&](int j) { return sk ? (int)(g0 / S) + j : pr + j * G; };

  bool ok = true;
  int diag_unit = -1;
  auto warp_wait = [&](uint32_t bar, uint32_t parity, bool cluster_scope = false) -> bool {
    if (!ok) return false;
    const bool got = cluster_scope ? mbar_wait_cluster(bar, parity) : mbar_wait(bar, parity);
    ok = __all_sync(0xffffffffu, got);
    if (!ok && lane == 0) {
      const unsigned rec = 0x80000000u | ((unsigned)warp << 24) | ((unsigned)(diag_unit & 0xFFF) << 12) |
                           (((bar - bar0) / 8u) << 1) | parity;
      atomicCAS(p.error + 1, 0u, rec);
    }
    return ok;
  };
  auto bar_count = [&](int b) -> uint32_t {
    if (b >= bWEmpty && b < bWEmpty + kWStages) return 8;   // this CTA's dequant warps
    if (b >= bReady && b < bReady + 4) return 9;             // the half's dequant warps of both CTAs + rank 0's producer
    if (b == bAccEmpty) return 8;                            // the epilogue warps of both CTAs
    return 1;   // TMA expect_tx arrivals, MMA commits
  };
  // arrive on rank 0's barrier `b` (local for rank 0, remote for rank 1)
  // for a hand-over whose payload a wait of the arriving warp has completed
  // (tcgen05.wait::st of a TMEM operand, tcgen05.wait::ld of the accumulator
  // it read): no release semantics, which would stall the warp until its
  // earlier global stores were visible at cluster scope (~1000+ cycles)
  auto arrive_rank0 = [&](int b) {
    if (rank == 0)
      mbar_arrive(BAR(b));
    else
      mbar_arrive_remote_relaxed(mapa_shared(BAR(b), 0));
  };

  // weight TMA of the pair's unit u (item it, K unit k): this CTA's 128 rows
  auto issue_w = [&](int u, int it, int k) {
    const int row0 = (it / p.btiles) * kItemRows + rank * kTileRows;
    const int s = u % kWStages;
    const uint32_t dst = sbase + s * kWStage;
    mbar_arrive_expect_tx(BAR(bWFull + s), kWStage);
    if constexpr (kRows144) {
      tma_load_2d(dst, &tmap_w, k * kRowBytes, row0, BAR(bWFull + s), kPolicyEvictLast);
      if constexpr (FMT == WFmt::Q6K)  // the rows' block scales d of unit k ([K/256][N] plane)
        tma_load_2d(dst + kAuxOff, &tmap_ws, row0, k, BAR(bWFull + s), kPolicyEvictLast);
    } else {
      tma_load_2d(dst, &tmap_w, k * 128, row0, BAR(bWFull + s), kPolicyEvictLast);
      tma_load_2d(dst + kAuxOff, &tmap_ws, k * 8, row0, BAR(bWFull + s), kPolicyEvictLast);
    }
  };
  // activations of K half h of unit u (item it, K unit k): this CTA's 128
  // batch rows x chunks 2h, 2h + 1 into the stage of half slot sl, counted on
  // rank 0's ready barrier of the slot (rank 0 also arrives, with both CTAs' bytes)
  auto issue_x = [&](int sl, int it, int k, int h) {
    if (rank == 0) mbar_arrive_expect_tx(BAR(bReady + sl), 2 * kXStageBytes);
    tma_load_3d_pair(sbase + kXOff + sl * kXStageBytes, &tmap_a, 0, (it % p.btiles) * kBatchTile + rank * 128,
                     k * kChunksPerUnit + 2 * h, mapa_shared(BAR(bReady + sl), 0), kPolicyEvictLast);
  };

  // set-up: barriers by warp 0's lanes, then the first weight stages (local
  // copies); the TMEM columns by warp 1 of both CTAs together; a cluster
  // barrier before anything signals the other CTA
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
    tmem_alloc_pair(sbase + kMiscOff, prefill_pair::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
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
    int issued = 0;            // halves
    int it, k;
    unit_at(0, it, k);
    for (int u = 0; u < nunits && ok; ++u, next_unit(it, k)) {
      diag_unit = u;
      for (int h = 0; h < 2; ++h) {
        const int sl = 2 * (u & 1) + h, use = u >> 1;
        // the slot's stage is free once the MMAs of its previous use completed
        if (use >= 1 && !warp_wait(BAR(bFree + sl), (uint32_t)((use - 1) & 1))) break;
        if (elect_one()) issue_x(sl, it, k, h);
        __syncwarp();
        issued = 2 * u + h + 1;
      }
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrActProducer);
    // never leave copies in flight: rank 0's ready barriers count both CTAs'
    // bytes (and the dequant warps, which arrive whatever happens), and rank 1
    // stays until the teardown cluster barrier, after this wait
    ok = true;
    if (rank == 0)
      for (int x = issued > 4 ? issued - 4 : 0; x < issued; ++x)
        if (!warp_wait(BAR(bReady + 2 * ((x >> 1) & 1) + (x & 1)), (uint32_t)((x >> 2) & 1), true)) {
          if (lane == 0) atomicOr(p.error, kErrTeardown);
          break;
        }
  } else if (warp == 3 && rank == 0) {
    // ---------------- MMA issuer (rank 0) ----------------
    const uint64_t bdesc0 = make_sdesc_sw128(sbase + kXOff);
    int j = 0;   // piece
    int it, k;
    unit_at(0, it, k);
    for (int u = 0; u < nunits; ++u, next_unit(it, k)) {
      diag_unit = u;
      const bool first = u == 0 || k == 0, last = u == nunits - 1 || k == S - 1;
      // the accumulators are free once both CTAs' epilogues have read piece j - 1
      if (first && j >= 1) warp_wait(BAR(bAccEmpty), (uint32_t)((j - 1) & 1), true);
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const int sl = 2 * (u & 1) + h;
        // both CTAs' operand halves and activation stages are in place: one wait
        warp_wait(BAR(bReady + sl), (uint32_t)((u >> 1) & 1), true);
        tc_fence_after();
        if (ok && elect_one()) {
          const uint32_t a_t = tmem + (uint32_t)(kSlot0 + sl * kSlotCols);
          const uint64_t bx = bdesc0 + (uint64_t)((sl * kXStageBytes) >> 4);
#pragma unroll
          for (int cl = 0; cl < 2; ++cl)
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              mma_f16_ts_pair(tmem, a_t + cl * 32 + 8 * ks, bx + (uint64_t)((cl * kXChunkBytes + 32 * ks) >> 4),
                              kIdesc, (first && h == 0 && cl == 0 && ks == 0) ? 0u : 1u);
          tc_commit_pair(BAR(bFree + sl), kPairMask);   // both CTAs' half slot and stage free
        }
        __syncwarp();
      }
      if (ok && elect_one() && last) tc_commit_pair(BAR(bAccFull), kPairMask);  // piece complete
      __syncwarp();
      if (last) ++j;
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrMma);
    if (elect_one()) tc_commit_pair(BAR(bFinal), kPairMask);
    __syncwarp();
  } else if (warp >= kDequantWarp0 && warp < kEpilogueWarp0) {
    // ---------------- dequant (K half g of every unit) ----------------
    const int q = warp & 3;
    const int g = (warp - kDequantWarp0) >> 2;
    const int r = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    for (int u = 0; u < nunits; ++u) {
      diag_unit = u;
      const int ws = u % kWStages;
      warp_wait(BAR(bWFull + ws), (u / kWStages) & 1);
      const uint8_t* stage = smem + ws * kWStage;
      const int sl = 2 * (u & 1) + g;
      // half slot sl is free once the MMAs of its previous use completed
      const int use = u >> 1;
      if (use >= 1) warp_wait(BAR(bFree + sl), (uint32_t)((use - 1) & 1));
      tc_fence_after();
      if (ok) {
        const uint32_t a_col = tmem + lane_off + (uint32_t)(kSlot0 + sl * kSlotCols);
        if (g == 0)
          dequant_unit_row<FMT, 0, 2>(stage, stage + kAuxOff, r, a_col);
        else
          dequant_unit_row<FMT, 2, 4>(stage, stage + kAuxOff, r, a_col);
        tc_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        arrive_rank0(bReady + sl);   // the operand is complete (tcgen05.wait::st above)
        mbar_arrive(BAR(bWEmpty + ws));
      }
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrDequant);
  } else if (warp >= kEpilogueWarp0) {
    // ---------------- epilogue (this CTA's 128 weight rows) ----------------
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
      const int grp = it / p.btiles, bt = it % p.btiles;
      // stream-K: a piece that is not the whole item goes to this CTA's
      // partial slot (2 blockIdx for the pair's first item, + 1 for its last)
      const bool whole = !sk || ((long long)it * S >= g0 && (long long)(it + 1) * S <= g0 + nunits);
      float* part = whole ? nullptr : p.part + (size_t)(2 * blockIdx.x + (j == 0 ? 0 : 1)) * prefill::kPartElems;
      const int mv = min(kBatchTile, p.M - bt * kBatchTile);
      const bool have = warp_wait(BAR(bAccFull), (uint32_t)(j & 1));
      tc_fence_after();
      if (!waited_pdl) {
        pdl_wait_prerequisites();  // C may still be read by the previous kernel
        waited_pdl = true;
      }
      const int n = grp * kItemRows + rank * kTileRows + r;
      const int n0 = n - (lane & 7);   // the lane group's first weight row
#pragma unroll 1
      for (int cb = 0; cb < mv; cb += 32) {
        uint32_t x[32];
        tmem_ld_x16(tmem + lane_off + (uint32_t)cb, x);
        tmem_ld_x16(tmem + lane_off + (uint32_t)(cb + 16), x + 16);
        // SwiGLU second pass: the up values this lane will combine after the
        // transpose, loaded before the TMEM wait so their latency overlaps it
        uint4 up[4];
        if (p.gate_mul && have && !part && vec16) {
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const int row = bt * kBatchTile + cb + 8 * b + (lane & 7);
            if (row < p.M && n0 < p.N) up[b] = *reinterpret_cast<const uint4*>(C + (size_t)row * p.N + n0);
          }
        }
        tc_wait_ld();
        if (have && part) {
          // [batch row][this CTA's 128 weight rows], the item's existing batch rows
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (cb + i < mv) part[(cb + i) * kTileRows + r] = __uint_as_float(x[i]);
        } else if (have && vec16) {
          // lane j of each group of 8 then holds batch row 8b + j of the
          // group's 8 consecutive weight rows: one 16-byte store per block
          // (2-byte stores strided by N made the drain of an item ~2.4x longer:
          // 18000 against 7500 cycles at N = 17408, and the next item's MMAs
          // wait for it)
          float* v = reinterpret_cast<float*>(x);
          transpose_8x8_blocks<32>(v, lane);
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const int row = bt * kBatchTile + cb + 8 * b + (lane & 7);
            if (row < p.M && n0 < p.N) {   // N % 8 == 0: the group's 8 rows are all in range
              uint4* dst = reinterpret_cast<uint4*>(C + (size_t)row * p.N + n0);
              if (p.gate_mul) {   // SwiGLU second pass: C holds the up projection
                const __half2* uh = reinterpret_cast<const __half2*>(&up[b]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 uf = __half22float2(uh[e]);
                  v[8 * b + 2 * e] = silu(v[8 * b + 2 * e]) * uf.x;
                  v[8 * b + 2 * e + 1] = silu(v[8 * b + 2 * e + 1]) * uf.y;
                }
              }
              uint4 w;
              w.x = h2_as_u32(__floats2half2_rn(v[8 * b], v[8 * b + 1]));
              w.y = h2_as_u32(__floats2half2_rn(v[8 * b + 2], v[8 * b + 3]));
              w.z = h2_as_u32(__floats2half2_rn(v[8 * b + 4], v[8 * b + 5]));
              w.w = h2_as_u32(__floats2half2_rn(v[8 * b + 6], v[8 * b + 7]));
              *dst = w;
            }
          }
        } else if (have && n < p.N) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int b = bt * kBatchTile + cb + i;
            if (b < p.M) {
              OutT* dst = C + (size_t)b * p.N + n;
              const float g = __uint_as_float(x[i]);
              *dst = to_out<OutT>(p.gate_mul ? silu(g) * out_to_f32(*dst) : g);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive_rank0(bAccEmpty);
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrEpilogue);
  }

  // ---------------- teardown ----------------
  // every MMA of the pair has completed (rank 0's final commit reaches both
  // CTAs), then both CTAs pass a cluster barrier (no remote arrival, copy or
  // MMA operand read is left in flight) before the collective deallocation
  __syncwarp();
  __syncthreads();
  if (warp == 1) {
    bool done = true;
    if (lane == 0) done = mbar_wait(BAR(bFinal), 0);
    done = __shfl_sync(0xffffffffu, done ? 1 : 0, 0) != 0;
    if (!done && lane == 0) atomicOr(p.error, kErrTeardown);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, prefill_pair::kTmemCols);
  }
}

// Stream-K fix-up for the pair kernel: each split item (256 weight rows x up
// to 256 batch rows) is summed from the partial tiles of its pairs, in pair
// order, and written to C. A pair's partial of an item is two tiles, one per
// CTA (its 128 weight rows); CTA 2 c + r of pair c holds slots 2 (2 c + r)
// (first item) and + 1 (last item). Block (x, y): split item x, batch rows
// 16 y .. 16 y + 15; thread t owns 4 consecutive weight rows (4 (t % 64) ..)
// of batch rows 16 y + 4 (t / 64) .. + 3.
template <typename OutT>
__global__ void __launch_bounds__(256) prefill_pair_reduce_kernel(const float* __restrict__ part,
                                                                OutT* __restrict__ c, int M, int N, int btiles,
                                                                int gate_mul,
                                                                const __grid_constant__ prefill::SplitItems si) {
  using namespace prefill_pair;
  pdl_wait_prerequisites();   // the partial tiles are the previous kernel's output
  pdl_launch_dependents();
  const int4 e = si.e[blockIdx.x];
  const int it = e.x, c_lo = e.y, c_hi = e.z, slot_lo = e.w;   // pair indices; slot of c_lo's piece (2 c_lo + which)
  const int grp = it / btiles, bt = it - (it / btiles) * btiles;
  // 4 batch rows per thread: their loads (two pieces at a time) are in
  // flight together, 8 per thread instead of 2 (at M = 512, N = 5120, K =
  // 17408 the fix-up of 40 split items took ~13 us under ncu with one row)
  constexpr int kRowsPerThread = 4;
  const int row0 = 16 * (int)blockIdx.y + kRowsPerThread * ((int)threadIdx.x >> 6);   // batch rows within the item
  const int col = 4 * ((int)threadIdx.x & 63);                                          // weight row within the item
  const int half = col >> 7;                                                           // the CTA of the pair holding it
  const int b0 = bt * kBatchTile + row0;
  if (b0 >= M) return;
  const int nrows = min(kRowsPerThread, M - b0);
  auto slot_ptr = [&](int cc, int rr) {
    const int slot = cc == c_lo ? 2 * (2 * c_lo + half) + (slot_lo & 1) : 2 * (2 * cc + half);
    return reinterpret_cast<const float4*>(part + (size_t)slot * prefill::kPartElems +
                                           (size_t)(row0 + rr) * kTileRows + (col & 127));
  };
  float4 acc[kRowsPerThread];
#pragma unroll
  for (int rr = 0; rr < kRowsPerThread; ++rr) acc[rr] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int c0 = c_lo; c0 <= c_hi; c0 += 2) {   // pieces in pair order, two at a time
    float4 v[kRowsPerThread][2];
#pragma unroll
    for (int rr = 0; rr < kRowsPerThread; ++rr)
#pragma unroll
      for (int i = 0; i < 2; ++i)
        if (rr < nrows && c0 + i <= c_hi) v[rr][i] = *slot_ptr(c0 + i, rr);
#pragma unroll
    for (int rr = 0; rr < kRowsPerThread; ++rr)
#pragma unroll
      for (int i = 0; i < 2; ++i)
        if (rr < nrows && c0 + i <= c_hi) {
          acc[rr].x += v[rr][i].x;
          acc[rr].y += v[rr][i].y;
          acc[rr].z += v[rr][i].z;
          acc[rr].w += v[rr][i].w;
        }
  }
  const int n = grp * kItemRows + col;
#pragma unroll
  for (int rr = 0; rr < kRowsPerThread; ++rr) {
    if (rr >= nrows) break;
    float4 a = acc[rr];
    OutT* dst = c + (size_t)(b0 + rr) * N + n;
    if (gate_mul) {   // SwiGLU second pass: C holds the up projection
      a.x = n < N ? silu(a.x) * out_to_f32(dst[0]) : 0.f;
      a.y = n + 1 < N ? silu(a.y) * out_to_f32(dst[1]) : 0.f;
      a.z = n + 2 < N ? silu(a.z) * out_to_f32(dst[2]) : 0.f;
      a.w = n + 3 < N ? silu(a.w) * out_to_f32(dst[3]) : 0.f;
    }
    if (n < N) dst[0] = to_out<OutT>(a.x);
    if (n + 1 < N) dst[1] = to_out<OutT>(a.y);
    if (n + 2 < N) dst[2] = to_out<OutT>(a.z);
    if (n + 3 < N) dst[3] = to_out<OutT>(a.w);
  }
}

}  // namespace busfill
