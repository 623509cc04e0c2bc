// Batched dequant-fused 4-bit-weight GEMM for small batches (M <= 64 per
// launch for plain GEMMs, 32 for the fused SwiGLU and gathered ones) on
// sm_100a:  C[M, N] = A[M, K] * deq(W)[N, K]^T, fp16 in, fp32
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
// are N, read from shared memory (K-major, 128-byte swizzle). The dequant
// warps write each unit's fp16 weights into one of three TMEM operand slots;
// the MMAs of all units of a tile segment accumulate into one fp32 TMEM
// accumulator, which the epilogue reads once per segment.
//
// The per-unit cost is set by barrier latency, not arithmetic: measured on
// B200, an mbarrier test_wait whose result a warp consumes at once costs it
// ~175 cycles even when the phase has completed, an arrive ~140, and a warp
// serialises them. So each dequant warp handles every other unit (two warp
// groups alternate units, all four chunks each), halving its barrier
// operations per unit, and the MMA warp tests the next unit's barriers right
// after issuing the current unit's MMAs, so that test overlaps the issue and
// it blocks only when the pre-test said "not yet".
//
// Warp roles (16 warps, one CTA per SM):
//   0      weight TMA producer: one 2D box of 128 rows x one unit (18 KB) per
//          stage into a 6- or 8-stage ring; the first stages are issued before
//          the CTA and cluster set-up. Weights do not depend on earlier
//          kernels, so none of this waits for griddepcontrol.wait.
//   1      activation TMA producer: one 3-D box per unit (four 64-value x
//          NB-row chunks, 128-byte swizzle) into a 4- or 6-stage ring of its
//          own, several units ahead of the MMA; the copy completes on the same
//          barrier as the unit's TMEM operands, so the MMA warp waits,
//          pre-tests and commits one barrier per unit; TMEM allocator.
//   3      MMA issuer (converged warp, one elected thread issues).
//   4-11   dequant: thread (warp%4, lane) owns weight row 32*(warp%4)+lane and
//          writes its fp16 operand into TMEM with tcgen05.st; warp group g =
//          (warp-4)/4 handles all four chunks of the units i with i%2 == g.
//   12-15  epilogue: row 32*(warp%4)+lane; once per tile segment it reads the
//          accumulator and finishes the tile (cluster reduction, C store).
//   2      idle.
//
// Numerics: formats.cuh (per format, the fp16 operand each weight becomes).
//
// Work split: a tile of 128 weight rows is split along K over the c CTAs of
// a thread-block cluster (rank k takes units [k*S/c, (k+1)*S/c) of every
// tile); cluster g of G takes tiles g, g+G, g+2G, ... The host picks c from a
// cost model of measured launches. At the end of each tile the non-zero ranks
// move their fp32 partial sums into rank 0's shared memory (staged, then one
// bulk copy each, completing rank 0's barrier), and rank 0 adds them in rank
// order (deterministic) and writes C. No global scratch, no atomics.
//
// Every wait is bounded (ptx.cuh: kWaitTimeoutNs): a kernel that cannot make
// progress records an error bit and winds down instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <type_traits>

#include "formats.cuh"
#include "ptx.cuh"

namespace busfill {

constexpr int kSlots = 3;            // unit operand slots in TMEM between the dequant warps and the MMA
constexpr int kThreads = 512;
constexpr int kWarpWProducer = 0;
constexpr int kWarpXProducer = 1;
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

// Column split over a process group, with the all-gather in the epilogue:
// every rank writes its slice of the output straight into each rank's full
// output (peer memory over NVLink). Each CTA that wrote tiles then adds their
// number to this rank's counter word in every rank's memory with one
// system-scope release reduction (no returning atomic, no last-CTA chain: on
// B200 that chain cost ~4 us per call). A later GEMM that reads the gathered
// output waits until each source rank's word reaches (calls so far + 1) x that
// rank's tiles per call.
constexpr int kMaxPeers = 8;
struct GatherArgs {
  int npeers;                 // ranks receiving the output (this one included); 0 = local C only
  int col_off;                // first column of this rank's slice in the full rows
  int ldc;                    // row length of the full outputs
  int signal;                 // this launch counts its tiles (the last launch of a call)
  void* out[kMaxPeers];       // each rank's full output [rows, ldc], at this launch's first row
  unsigned* flag[kMaxPeers];  // per rank: this rank's tile counter in that rank's memory
  const unsigned* wait;       // nwait local counter words (one per source rank); may be null
  unsigned* wait_gen;         // two words: [0] completed calls of the site, [1] CTAs of the current call through
  int nwait;
  int wait_tiles[kMaxPeers];  // tiles each source rank writes per call
};

struct DecodeParams {
  void* c;              // [M, N] row-major, OutT
  unsigned* error;      // device error word (+1: first failure record)
  int M, N, K;
  int tiles;            // T = ceil(N / 128)
  int units_per_tile;   // S = K / 256
  int csize;            // CTAs per cluster: the K split of every tile (1..8)
  int nclusters;        // G; cluster g takes tiles g, g + G, ...; G <= T
  GatherArgs gather;
};

// Units [first, last) of every tile that cluster rank `rank` of `csize` takes.
__host__ __device__ __forceinline__ int ksplit_begin(int rank, int S, int csize) { return rank * S / csize; }

// TMEM column map (512 columns allocated)
template <int NB>
struct DecodeTmem {
  static constexpr int kAcc = 0;                         // segment accumulators, b * NB for b = 0, 1
  static constexpr int kA = 128;                         // unit operand slots, 128 columns each
  static_assert(2 * NB <= kA && kA + kSlots * 128 <= kTmemCols, "TMEM budget");
};

// Largest cluster (K split) for a batch tile of NB rows: rank 0 receives the
// other ranks' [128][NB] fp32 partials in shared memory.
template <int NB>
constexpr int max_cluster() { return NB == 64 ? 2 : NB == 32 ? 4 : 8; }

// Weight ring depth: what shared memory leaves next to the activation slots
// and rank 0's receive buffer. Even, so that stage s is always filled with
// units of one parity and so waited on by one dequant group in phase order
// (a group that skipped the other group's phase of a stage could see that
// stale phase as complete: mbarrier waits only tell parities apart).
template <int NB, WFmt FMT>
constexpr int w_stages() {
  // Q5_K / Q6_K stages are 22 / 26 KB; 64-row batches take 32 KB activation stages
  return NB == 64 ? (FMT == WFmt::Q6K ? 2 : 4) : FMT == WFmt::Q5K || FMT == WFmt::Q6K ? 4 : 6;
}

// Activation ring depth (one unit per stage), separate from the TMEM operand
// slots so that a unit's activations are requested several units ahead: a
// box waits behind the weight boxes in its SM's TMA queue (~1.2 us from issue
// to landing under load on B200), longer than the three-slot operand cycle.
template <int NB>
constexpr int x_stages() { return NB == 64 ? 3 : NB == 32 ? 4 : 6; }

template <int NB, WFmt FMT>
struct DecodeSmem {
  static constexpr int kXChunkBytes = NB * 128;                      // one 64-value activation box
  static constexpr int kXSlotBytes = kChunksPerUnit * kXChunkBytes;  // one unit of activations
  static constexpr int kWOff = 0;
  static constexpr int kWStage = wstage_bytes<FMT>();               // one unit of 128 weight rows
  static constexpr int kWStages = w_stages<NB, FMT>();
  static_assert(kWStages % 2 == 0, "each weight stage must belong to one dequant group");
  static constexpr int kXStages = x_stages<NB>();
  static_assert(kXStages >= kSlots, "an activation stage per operand slot at least");
  static constexpr int kXOff = (kWOff + kWStages * kWStage + 1023) / 1024 * 1024;   // swizzled stages: 1 KB aligned
  static constexpr int kRedOff = kXOff + kXStages * kXSlotBytes;      // rank 0: [rank-1][128][NB] fp32 partials
  static constexpr int kRedRankBytes = kTileRows * NB * 4;
  static constexpr int kBarOff = kRedOff + (max_cluster<NB>() - 1) * kRedRankBytes;
  // barrier slots
  static constexpr int bWFull = 0, bWEmpty = bWFull + kWStages;
  // unit slot s: operands in TMEM (4 dequant warps) and activations landed
  // (1 producer arrival + TMA bytes)
  static constexpr int bReady = bWEmpty + kWStages;
  static constexpr int bUDone = bReady + kSlots;           // unit's MMAs complete (commit): slot s free
  static constexpr int bAccFull = bUDone + kSlots;         // segment accumulator b complete (commit)
  static constexpr int bAccEmpty = bAccFull + 2;           // segment accumulator b read by the epilogue
  static constexpr int bRedFull = bAccEmpty + 2;           // rank 0: the other ranks' partials landed (tx bytes)
  static constexpr int bRedEmpty = bRedFull + 1;           // rank k > 0: rank 0 has read this rank's partial
  static constexpr int bXFree = bRedEmpty + 1;            // activation stage x free: the MMAs of its unit completed (commit)
  static constexpr int bFinal = bXFree + kXStages;
  static constexpr int kNumBars = bFinal + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kMiscOff + 64;
  static constexpr int kAlloc = kBytes + 1024;  // slack to align the base to 1024 B
  static_assert(kAlloc <= 232448, "dynamic shared memory per block on sm_100");
};

// Per-unit schedule facts every role derives the same way: unit i of this CTA
// is unit sb0 + i % len of its cluster's (i / len)-th segment. A segment is a
// tile; with SwiGLU (sw = 1) segments 2j and 2j+1 are the gate and the up tile
// of the cluster's j-th tile index.
struct UnitInfo {
  int tile, sb, seg;
  bool up;                    // SwiGLU: the up projection's tile
  bool seg_first, seg_last;   // first / last unit of this CTA's part of the tile
};
__device__ __forceinline__ UnitInfo unit_info(int i, int len, int sb0, int g, int nclusters, int sw) {
  UnitInfo r;
  r.seg = i / len;
  const int j = i - r.seg * len;
  r.tile = g + (r.seg >> sw) * nclusters;
  r.up = sw && (r.seg & 1);
  r.sb = sb0 + j;
  r.seg_first = (j == 0);
  r.seg_last = (j == len - 1);
  return r;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// tmap_w: the weight rows; tmap_ws: the second plane (Q4_0 block scales
// [N][K/32], Q6_K block d [K/256][N]) or, with SW, the up projection's rows.
// SW: SwiGLU pair (144-byte formats): tmap_w is the gate, tmap_ws the up
// projection, C = silu(A Wg^T) * (A Wu^T); every tile index of the cluster
// becomes two segments (gate, up).
// GA: the output is gathered over a process group (GatherArgs); else it is
// written to the local C only.
template <WFmt FMT, int NB, typename OutT, bool SW = false, bool GA = false>
__global__ void __launch_bounds__(kThreads, 1)
    decode_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_ws,
                       const __grid_constant__ CUtensorMap tmap_a, const DecodeParams p) {
  static_assert(NB == 16 || NB == 32 || NB == 64, "batch tile");
  static_assert(NB != 64 || (!SW && !GA), "64-row batches: plain GEMMs (the epilogue's registers)");
  using L = DecodeSmem<NB, FMT>;
  using TM = DecodeTmem<NB>;
  constexpr bool kRows144 = aos_rows<FMT>();  // whole block rows per unit (block_q4_K / q5_K, 8 x block_q4_0)
  static_assert(!SW || (kRows144 && FMT != WFmt::Q6K), "SwiGLU pairs take one-plane block-row formats");
  constexpr int kSw = SW ? 1 : 0;
  constexpr uint32_t kIdesc = make_idesc_f16_f32(kTileRows, NB);
  constexpr int kWStages = L::kWStages;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_s + 1023u) & ~1023u) - raw_s);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::kBarOff;
  auto BAR = [&](int slot) { return bar0 + 8u * (uint32_t)slot; };
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);  // [0] tmem base

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = p.units_per_tile;
  const int csize = p.csize;
  // clusters tile the 1-D grid in blockIdx order: rank = blockIdx.x % csize
  const int crank = (int)(blockIdx.x % (unsigned)csize);
  const int g = (int)(blockIdx.x / (unsigned)csize);
  const int sb0 = ksplit_begin(crank, S, csize);
  const int len = ksplit_begin(crank + 1, S, csize) - sb0;
  // segments of this CTA: its cluster's tile indices, two segments each with SwiGLU
  const int ntiles = ((p.tiles - g + p.nclusters - 1) / p.nclusters) << kSw;
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

  // arrivals each barrier expects per phase
  auto bar_count = [&](int b) -> uint32_t {
    if (b >= L::bWEmpty && b < L::bWEmpty + kWStages) return 4;  // the 4 dequant warps of the unit's group
    if (b >= L::bReady && b < L::bReady + kSlots) return 5;       // 4 dequant warps + the activation producer (+ TMA bytes)
    if (b >= L::bAccEmpty && b < L::bAccEmpty + 2) return 4;      // the 4 epilogue warps
    if (b == L::bRedEmpty) return 4;                              // rank 0's 4 epilogue warps
    return 1;  // TMA expect_tx arrivals, MMA commits, rank 0's expect_tx on bRedFull
  };
  // weight TMA for unit i into ring stage i % kWStages (the stage must be free); one thread
  auto issue_w_thread = [&](int i) {
    const int s = i % kWStages;
    const UnitInfo ui = unit_info(i, len, sb0, g, p.nclusters, kSw);
    const uint32_t dst = sbase + L::kWOff + s * L::kWStage;
    mbar_arrive_expect_tx(BAR(L::bWFull + s), L::kWStage);
    if constexpr (kRows144) {
      tma_load_2d(dst, ui.up ? &tmap_ws : &tmap_w, ui.sb * unit_row_bytes<FMT>(), ui.tile * kTileRows, BAR(L::bWFull + s),
                  kPolicyEvictFirst);
      if constexpr (FMT == WFmt::Q6K)  // the tile's 128 block scales d of this unit ([K/256][N] plane)
        tma_load_2d(dst + kTileRows * kQ6KBodyBytes, &tmap_ws, ui.tile * kTileRows, ui.sb, BAR(L::bWFull + s),
                    kPolicyEvictFirst);
    } else {
      tma_load_2d(dst, &tmap_w, ui.sb * 128, ui.tile * kTileRows, BAR(L::bWFull + s), kPolicyEvictFirst);
      tma_load_2d(dst + kQ40ScaleOffset, &tmap_ws, ui.sb * 8, ui.tile * kTileRows, BAR(L::bWFull + s),
                  kPolicyEvictFirst);
    }
  };
  // activations of unit i into stage i % kXStages (the stage must be free);
  // one thread. The copy's bytes and this arrival count towards the slot's ready
  // phase, which the unit's dequant warps complete. One 3-D box brings the
  // unit's four 64-value chunks (dims: 64 values, rows, chunk), landing as
  // [chunk][row][128 B] swizzled, the MMA's B layout: an SM's TMA unit takes
  // about as long per box for 4 KB as for 32 KB (measured on B200), so one
  // box per unit instead of four shortens the activations' path to the MMA.
  auto issue_x_thread = [&](int i) {
    const int s = i % kSlots;
    const int sb = sb0 + i % len;
    mbar_arrive_expect_tx(BAR(L::bReady + s), L::kXSlotBytes);
    tma_load_3d(sbase + L::kXOff + (i % L::kXStages) * L::kXSlotBytes, &tmap_a, 0, 0, sb * kChunksPerUnit,
                BAR(L::bReady + s), kPolicyEvictLast);
  };
  // Set-up is on the critical path of every launch: the CTAs that start last
  // (on the SMs the previous kernel frees last) finish last. So the barriers
  // are initialised by all lanes of warp 0 at once, and the first ring of
  // weight boxes and the first slots of activations are issued one per lane
  // before the CTA-wide sync. Weights do not depend on earlier kernels and
  // never wait for griddepcontrol.wait; activations do.
  // Only the first kWEarly weight stages go out at once; stage i < kWStages
  // follows when stage i - kWEarly has landed. Every SM asking for its whole
  // ring at launch makes each SM's first stage land only at the end of that
  // burst (~2-3 us on B200), which delays the first MMA; the ring still fills
  // well ahead of the dequant.
  constexpr int kWEarly = 2;
  const int w_early = nunits < kWEarly ? nunits : kWEarly;
  const int x_early = nunits < kSlots ? nunits : kSlots;
  if (warp == kWarpWProducer) {
    if (lane == 0) {
      tma_prefetch_desc(&tmap_w);
      if (FMT == WFmt::Q4_0 || FMT == WFmt::Q6K) tma_prefetch_desc(&tmap_ws);
      tma_prefetch_desc(&tmap_a);
    }
    for (int b = lane; b < L::kNumBars; b += 32) mbar_init(BAR(b), bar_count(b));
    fence_mbar_init();
    __syncwarp();
    named_bar_arrive(1, 64);  // barriers ready: release the activation producer
    if (lane < w_early) issue_w_thread(lane);
    __syncwarp();
  } else if (warp == kWarpXProducer) {
    tmem_alloc(sbase + L::kMiscOff, kTmemCols);
    tmem_relinquish();
    named_bar_sync(1, 64);
    pdl_wait_prerequisites();  // activations may be the previous kernel's output
    if (GA && p.gather.nwait > 0) {
      // activations gathered by an earlier GEMM on every rank: wait for each
      // rank's flag, then let this thread's TMA copies see what it acquired.
      // wait_gen[0] counts this site's completed calls and wait_gen[1] the
      // CTAs of the current call that got through: every CTA reads [0] before
      // it arrives on [1], and the last to arrive resets [1] and advances [0],
      // so the count holds whatever grid each call had. The previous call
      // of the site completed before this one started (the stream order, and
      // griddepcontrol.wait above), so [1] starts at 0.
      unsigned calls = 0;
      if (lane == 0) calls = ld_acquire_gpu(p.gather.wait_gen);
      calls = __shfl_sync(0xffffffffu, calls, 0);
      bool got = true;
      if (lane < p.gather.nwait)
        got = wait_flag_sys(p.gather.wait + lane, (calls + 1u) * (unsigned)p.gather.wait_tiles[lane]);
      if (!__all_sync(0xffffffffu, got) && lane == 0) {
        atomicOr(p.error, kErrActProducer);
        atomicCAS(p.error + 1, 0u, 0x80000000u | ((unsigned)warp << 24) | 0xFFFu << 12);
      }
      fence_proxy_async_global();
      if (lane == 0 && atom_add_acq_rel_gpu(p.gather.wait_gen + 1, 1u) == gridDim.x - 1) {
        st_relaxed_gpu(p.gather.wait_gen + 1, 0u);
        red_release_gpu_add(p.gather.wait_gen, 1u);
      }
    }
    if (lane < x_early) issue_x_thread(lane);
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];
  // The other CTAs of the cluster touch our barriers and shared memory only
  // at the end of a tile: arrive now, and wait (for every CTA of the cluster
  // to have initialised its barriers) only before the first such access.
  if (csize > 1) cluster_arrive();
  bool cl_waited = false;    // this thread has waited on the set-up phase
  bool cl_arrived = false;   // this thread has arrived on the teardown phase
  // Let the next kernel on the stream launch now: its CTAs take SMs as ours
  // retire and begin streaming their weights before our tail completes.
  if (threadIdx.x == 0) pdl_launch_dependents();

  if (warp == kWarpWProducer) {
    // ---------------- weight producer ----------------
    int issued = w_early;
    for (int i = w_early; i < nunits; ++i) {
      if (i < kWStages && !warp_wait(BAR(L::bWFull + (i - kWEarly)), 0)) break;
      if (!warp_wait(BAR(L::bWEmpty + i % kWStages), ((i / kWStages) & 1) ^ 1)) break;
      if (elect_one()) issue_w_thread(i);
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
    int issued = x_early;
    for (int i = x_early; i < nunits; ++i) {
      // activation stage i % kXStages is free once the MMAs of unit i - kXStages completed
      if (i >= L::kXStages && !warp_wait(BAR(L::bXFree + i % L::kXStages), ((i / L::kXStages) & 1) ^ 1)) break;
      // the arrival must count towards unit i's phase of its slot barrier: unit
      // i - kSlots's phase must have completed (it cannot complete without
      // this producer, so nothing later can alias it)
      if (!warp_wait(BAR(L::bReady + i % kSlots), ((i / kSlots) & 1) ^ 1)) break;
      if (elect_one()) issue_x_thread(i);
      __syncwarp();
      issued = i + 1;
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrActProducer);
    // never leave the CTA with copies in flight: they complete on bReady (whose
    // phase also needs the unit's dequant warps)
    ok = true;
    for (int i = issued > kSlots ? issued - kSlots : 0; i < issued; ++i)
      if (!warp_wait(BAR(L::bReady + i % kSlots), (i / kSlots) & 1)) {
        if (lane == 0) atomicOr(p.error, kErrTeardown);
        break;
      }
  } else if (warp == kWarpMma) {
    // ---------------- MMA issuer (converged warp, one elected thread issues) ----------------
    // Lean loop: one wait (pre-tested during the previous unit), 16 MMAs, one
    // commit; unit bookkeeping kept incrementally.
    const uint64_t bdesc0 = make_sdesc_sw128(sbase + L::kXOff);  // + (byte offset >> 4) per MMA
    int s = 0, seg = 0, j = 0;
    uint32_t ph = 0;          // parity of unit i's phase on its slot barriers: (i / kSlots) & 1
    bool pre = false;         // unit i's slot already seen ready
    for (int i = 0; i < nunits; ++i) {
      diag_unit = i;
      const int buf = seg & 1;
      // a segment's accumulator is free once the epilogue has read segment seg - 2
      if (j == 0 && seg >= 2 && !warp_wait(BAR(L::bAccEmpty + buf), ((seg >> 1) & 1) ^ 1)) break;
      if (!pre && !warp_wait(BAR(L::bReady + s), ph)) break;
      tc_fence_after();
      if (elect_one()) {
        const uint32_t d_acc = tmem + TM::kAcc + (uint32_t)(buf * NB);
        const uint32_t a_t = tmem + TM::kA + (uint32_t)(s * 128);
        const uint64_t bd = bdesc0 + (uint64_t)(((i % L::kXStages) * L::kXSlotBytes) >> 4);
#pragma unroll
        for (int cc = 0; cc < kChunksPerUnit; ++cc)
#pragma unroll
          for (int t = 0; t < 4; ++t)
            mma_f16_ts(d_acc, a_t + cc * 32 + 8 * t, bd + (uint64_t)((cc * L::kXChunkBytes + 32 * t) >> 4), kIdesc,
                       (j == 0 && cc == 0 && t == 0) ? 0u : 1u);
        tc_commit(BAR(L::bUDone + s));                          // slot s free
        tc_commit(BAR(L::bXFree + i % L::kXStages));            // activation stage free
        if (j == len - 1) tc_commit(BAR(L::bAccFull + buf));    // segment accumulator complete
      }
      __syncwarp();
      // next unit; pre-test its slot while this unit's MMAs run
      if (++s == kSlots) { s = 0; ph ^= 1u; }
      if (++j == len) { j = 0; ++seg; }
      pre = (i + 1 < nunits) && __all_sync(0xffffffffu, mbar_test_wait(BAR(L::bReady + s), ph));
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrMma);
    if (elect_one()) tc_commit(BAR(L::bFinal));  // fires once every MMA issued above has completed
    __syncwarp();
  } else if (warp >= kWarpDequant0 && warp < kWarpEpilogue0) {
    // ---------------- dequant ----------------
    const int q = warp & 3;                        // TMEM lane quarter this warp may touch
    const int grp = (warp - kWarpDequant0) >> 2;   // group: units i with i % 2 == grp
    const int r = q * 32 + lane;                   // weight row within the tile
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    for (int i = grp; i < nunits; i += 2) {
      diag_unit = i;
      const int ws = i % kWStages;
      if (!warp_wait(BAR(L::bWFull + ws), (i / kWStages) & 1)) break;
      // operand slot i % kSlots is free once the MMAs of unit i - kSlots completed
      if (i >= kSlots && !warp_wait(BAR(L::bUDone + i % kSlots), ((i / kSlots) & 1) ^ 1)) break;
      tc_fence_after();
      const uint8_t* stage = smem + L::kWOff + ws * L::kWStage;
      dequant_unit_row<FMT>(stage, stage + kTileRows * unit_row_bytes<FMT>(), r,
                            tmem + lane_off + TM::kA + (i % kSlots) * 128);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(BAR(L::bReady + i % kSlots));
        mbar_arrive(BAR(L::bWEmpty + ws));
      }
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrDequant);
  } else if (warp >= kWarpEpilogue0) {
    // ---------------- epilogue ----------------
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    float acc[NB];
    float gate[SW ? NB : 1];  // SwiGLU: the reduced gate tile, held until its up tile

    // Finish tile `tile` (this CTA's segment `seg`). One CTA per tile: write C.
    // Otherwise ranks k > 0 stage their fp32 partial in their own shared
    // memory and move it into rank 0's with one bulk copy, whose bytes
    // complete rank 0's bRedFull barrier (no separate signal: every release
    // or remote round trip costs ~0.5 us on B200); rank 0 adds the partials
    // in rank order and writes C.
    // Receive layout: [rank-1][row][NB] fp32, 16-byte chunks swizzled by row.
    // After the last tile each CTA arrives on the cluster's teardown barrier
    // as soon as it is done with distributed shared memory (ranks k > 0 once
    // their partials are pushed, rank 0 once it has read them), so rank 0
    // finds the barrier complete when it waits after its C store.
    auto flush = [&](int tile, int seg) {
      const int n = tile * kTileRows + r;
      OutT* C = reinterpret_cast<OutT*>(p.c);
      constexpr int kChunks = NB / 4;
      const int swz = r & (kChunks - 1);
      if (csize > 1 && !cl_waited) {
        __syncwarp();
        cluster_wait();  // every CTA of the cluster has initialised its barriers
        cl_waited = true;
      }
      if (csize > 1 && crank != 0) {
        // rank 0's buffer, and this CTA's staging copy, are free once rank 0
        // has read the previous segment
        if (seg > 0) warp_wait(BAR(L::bRedEmpty), (uint32_t)((seg - 1) & 1), true);
        // Stage the partial in this CTA's own slot of the receive area (ranks
        // k > 0 receive nothing), in the layout rank 0 reads, then move the
        // whole slot with one bulk copy that completes rank 0's barrier: one
        // transfer instead of a 16-byte remote store per thread and chunk.
        const uint32_t slot = sbase + L::kRedOff + (uint32_t)((crank - 1) * L::kRedRankBytes);
        const uint32_t row = slot + (uint32_t)(r * NB * 4);
#pragma unroll
        for (int j = 0; j < kChunks; ++j)
          st_shared_f4(row + (uint32_t)((j ^ swz) << 4), acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
        fence_proxy_async_shared();
        named_bar_sync(2, 128);   // the 4 epilogue warps have staged their rows
        if (warp == kWarpEpilogue0 && lane == 0)
          bulk_copy_to_cluster(mapa_shared(slot, 0), slot, (uint32_t)L::kRedRankBytes, mapa_shared(BAR(L::bRedFull), 0));
        if (seg == ntiles - 1) {
          __syncwarp();
          cluster_arrive();
          cl_arrived = true;
        }
        return;
      }
      if (csize > 1) {
        if (warp == kWarpEpilogue0 && lane == 0)
          mbar_arrive_expect_tx(BAR(L::bRedFull), (uint32_t)((csize - 1) * L::kRedRankBytes));
        warp_wait(BAR(L::bRedFull), (uint32_t)(seg & 1));
        for (int k = 1; k < csize; ++k) {
          const uint8_t* row = smem + L::kRedOff + (k - 1) * L::kRedRankBytes + r * NB * 4;
          float4 v[kChunks];
#pragma unroll
          for (int j = 0; j < kChunks; ++j) v[j] = *reinterpret_cast<const float4*>(row + ((j ^ swz) << 4));
#pragma unroll
          for (int j = 0; j < kChunks; ++j) {
            acc[4 * j] += v[j].x;
            acc[4 * j + 1] += v[j].y;
            acc[4 * j + 2] += v[j].z;
            acc[4 * j + 3] += v[j].w;
          }
        }
        __syncwarp();
        if (seg + 1 < ntiles) {
          // let the other ranks overwrite our buffer with their next partial
          if (lane == 0)
            for (int k = 1; k < csize; ++k) mbar_arrive_remote(mapa_shared(BAR(L::bRedEmpty), (uint32_t)k));
        } else {
          cluster_arrive();
          cl_arrived = true;
        }
      }
      if constexpr (SW) {
        if ((seg & 1) == 0) {
#pragma unroll
          for (int t = 0; t < NB; ++t) gate[t] = acc[t];
          return;
        }
#pragma unroll
        for (int t = 0; t < NB; ++t) acc[t] = silu(gate[t]) * acc[t];
      }
      pdl_wait_prerequisites();  // C may still be read by the previous kernel
      if (GA) {
        // this rank's slice into every rank's full output (peer stores over
        // NVLink), 8 consecutive outputs per 16-byte store where every output
        // row is 16-byte aligned (as for the local store below)
        bool wide = sizeof(OutT) == 2 && ((p.gather.ldc | p.gather.col_off) & 7) == 0;
        for (int q = 0; q < p.gather.npeers; ++q)
          wide = wide && (reinterpret_cast<uintptr_t>(p.gather.out[q]) & 15) == 0;
        if (ok && wide) {
          transpose_8x8_blocks<NB>(acc, lane);
          const int n0 = tile * kTileRows + (warp & 3) * 32 + (lane & ~7);   // the lane group's 8 rows
          uint4 v[NB / 8];
#pragma unroll
          for (int b = 0; b < NB / 8; ++b) {
            v[b].x = h2_as_u32(__floats2half2_rn(acc[8 * b], acc[8 * b + 1]));
            v[b].y = h2_as_u32(__floats2half2_rn(acc[8 * b + 2], acc[8 * b + 3]));
            v[b].z = h2_as_u32(__floats2half2_rn(acc[8 * b + 4], acc[8 * b + 5]));
            v[b].w = h2_as_u32(__floats2half2_rn(acc[8 * b + 6], acc[8 * b + 7]));
          }
          if (n0 < p.N) {   // the local shard width is a multiple of 8 here (ldc and col_off are)
#pragma unroll 1
            for (int q = 0; q < p.gather.npeers; ++q) {
              OutT* Cq = reinterpret_cast<OutT*>(p.gather.out[q]) + p.gather.col_off + n0;
#pragma unroll
              for (int b = 0; b < NB / 8; ++b) {
                const int t = 8 * b + (lane & 7);
                if (t < p.M) *reinterpret_cast<uint4*>(Cq + (size_t)t * p.gather.ldc) = v[b];
              }
            }
          }
        } else if (ok && n < p.N) {
#pragma unroll 1
          for (int q = 0; q < p.gather.npeers; ++q) {
            OutT* Cq = reinterpret_cast<OutT*>(p.gather.out[q]) + p.gather.col_off + n;
#pragma unroll
            for (int t = 0; t < NB; ++t)
              if (t < p.M) Cq[(size_t)t * p.gather.ldc] = to_out<OutT>(acc[t]);
          }
        }
      } else if (ok) {
        if (sizeof(OutT) == 2 && (p.N & 7) == 0 && (reinterpret_cast<uintptr_t>(p.c) & 15) == 0) {
          // one 16-byte store of 8 consecutive outputs per batch row instead of
          // NB 2-byte stores strided by N (the store tail shortens the launch)
          transpose_8x8_blocks<NB>(acc, lane);
          const int n0 = tile * kTileRows + (warp & 3) * 32 + (lane & ~7);   // the lane group's 8 rows
#pragma unroll
          for (int b = 0; b < NB / 8; ++b) {
            const int t = 8 * b + (lane & 7);
            if (t < p.M && n0 < p.N) {   // N % 8 == 0: the group's 8 rows are all in range
              uint4 v;
              v.x = h2_as_u32(__floats2half2_rn(acc[8 * b], acc[8 * b + 1]));
              v.y = h2_as_u32(__floats2half2_rn(acc[8 * b + 2], acc[8 * b + 3]));
              v.z = h2_as_u32(__floats2half2_rn(acc[8 * b + 4], acc[8 * b + 5]));
              v.w = h2_as_u32(__floats2half2_rn(acc[8 * b + 6], acc[8 * b + 7]));
              *reinterpret_cast<uint4*>(C + (size_t)t * p.N + n0) = v;
            }
          }
        } else if (n < p.N) {
#pragma unroll
          for (int t = 0; t < NB; ++t)
            if (t < p.M) C[(size_t)t * p.N + n] = to_out<OutT>(acc[t]);
        }
      }
    };

    for (int seg = 0; seg < ntiles; ++seg) {
      diag_unit = seg * len + len - 1;
      const int buf = seg & 1;
      if (warp_wait(BAR(L::bAccFull + buf), (uint32_t)((seg >> 1) & 1))) {
        tc_fence_after();
#pragma unroll
        for (int h = 0; h < NB; h += 16) {
          uint32_t x[16];
          tmem_ld_x16(tmem + lane_off + TM::kAcc + (uint32_t)(buf * NB + h), x);
          tc_wait_ld();
#pragma unroll
          for (int t = 0; t < 16; ++t) acc[h + t] = __uint_as_float(x[t]);
        }
      } else {
#pragma unroll
        for (int t = 0; t < NB; ++t) acc[t] = 0.f;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(L::bAccEmpty + buf));
      flush(g + (seg >> kSw) * p.nclusters, seg);
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrEpilogue);
  }

  // ---------------- teardown ----------------
  // Every thread of the cluster arrives once and waits once on each of the two
  // cluster barrier phases: set-up (barriers initialised) and teardown (done
  // with distributed shared memory); the epilogue warps took their turns above.
  __syncwarp();
  if (csize > 1) {
    if (!cl_waited) cluster_wait();
    if (!cl_arrived) cluster_arrive();
  }
  __syncthreads();
  if (warp == kWarpXProducer) {
    bool done = true;
    if (lane == 0) done = mbar_wait(BAR(L::bFinal), 0);
    done = __shfl_sync(0xffffffffu, done ? 1 : 0, 0) != 0;
    if (!done && lane == 0) atomicOr(p.error, kErrTeardown);
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  // no CTA may leave while another CTA of its cluster can still read its
  // shared memory or arrive on its barriers
  if (csize > 1) cluster_wait();
  // Gathered output: a CTA that wrote tiles (rank 0 of its cluster) adds
  // their number to this rank's counter in every rank's memory. The CTA
  // barrier above orders the epilogue warps' peer stores before warp 0; lane
  // q then makes them visible at system scope (one fence for the warp) and
  // adds to peer q's counter with a relaxed reduction, all peers at once, so
  // a consumer that acquires the counter sees the data (a data-then-flag
  // protocol over NVLink). One release reduction per peer in turn instead
  // made every reduction wait for the previous one to be performed.
  if (GA && p.gather.signal && crank == 0 && warp == 0 && lane < p.gather.npeers) {
    fence_acq_rel_sys();
    red_relaxed_sys_add(p.gather.flag[lane], (unsigned)(ntiles >> kSw));
  }
}

}  // namespace busfill
