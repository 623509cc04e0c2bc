// One launch for a list of up to eight small-batch Q4_K GEMMs (one or two
// decoder layers' projections: O, QKV, gate/up SwiGLU pair, down), M <= 32,
// on sm_100a.
//
// Why: a decode-sized GEMM (M <= 32) is too short to amortise a launch. Each
// launch of the one-GEMM decode kernel (decode_gemm.cuh) pays a fixed ~7 us on
// B200: its CTAs can start only when the previous kernel's CTA on that SM has
// left (one CTA fills an SM), then they wait for their first weight boxes,
// dequantize the first unit, and finish with a reduction and the C stores. A
// layer is four such launches. Here one resident grid walks the layer's
// whole list of GEMMs ("ops"): a CTA that finishes its share of one op goes
// straight on to the next op's weight boxes and dequant, which depend on
// nothing, and only the MMAs of an op that reads an earlier op's output wait
// for that output (a device-side count of the tiles stored, acquired by the
// activation producer before its first activation box of the op).
//
// Work split (stream-K per op): op o is T tiles of 128 weight rows, each
// P planes (P = 2 for a SwiGLU pair: gate then up) of S = K / 256 units; its
// U = T P S units are cut into G contiguous ranges, CTA b taking units
// [U b / G, U (b + 1) / G). Every CTA thus takes an equal share of every op,
// so all CTAs reach an op's end together and a dependent op waits little.
// An op whose tiles nearly fill the grid takes whole tiles on fewer CTAs
// instead (Op::ctas, chosen by the host), so that none of its tiles is split.
// A tile that lies inside one CTA's range is finished by that CTA (C stored;
// a SwiGLU pair's gate tile waits in TMEM for its up tile). A tile split
// between CTAs: each contributor
// stores its fp32 sums of the tile's planes into its own partial slots, makes
// them visible and adds 1 to the tile's counter; the contributor that brings
// the counter to the number of contributors (the last to arrive) adds all
// contributors' partials in CTA order (deterministic, whichever CTA is last),
// applies silu(gate) * up for a SwiGLU pair, stores C, and resets the counter.
// No CTA waits for another inside an op; counters are zero between launches.
//
// Per CTA and unit the pipeline is the decode kernel's (weight TMA ring ->
// dequant warps -> TMEM operand slots -> swap-AB tcgen05.mma into one of
// three TMEM accumulators -> epilogue), see decode_gemm.cuh: the same
// warp roles, barriers and numerics, with the unit list spanning all ops.
//
// Every wait is bounded (kWaitTimeoutNs); a CTA that gives up records an error
// bit in the stream's error word and winds down.
//
// The reference has no counterpart: its kernel (kernels/busfill_v1a.cu:41-104)
// is one GEMM per launch; this is the layer-sweep form of the same GEMM.
#pragma once

#include "decode_gemm.cuh"

namespace busfill {
namespace sweep {

constexpr int kMaxOps = 8;   // two decoder layers
constexpr int kMaxTiles = 1024;    // tiles per op: N <= 131072
constexpr int kSlotsPerCta = 4;    // partial tiles per CTA and op: {first, last tile} x {plane 0, 1}
constexpr int kMaxNB = 32;
// TMEM accumulators: three segment buffers, so that the MMAs can run two
// segments ahead of the epilogue (whose split-tile hand-offs take microseconds
// of global-memory round trips), then the SwiGLU gate tile; the operand slots
// start at column 128
constexpr int kAccBufs = 3;
// counter words ahead of the partial slots in a workspace: per op and tile
// the contributions, then per op the tiles stored, then the CTAs finished
constexpr int kCntWords = kMaxOps * kMaxTiles;
constexpr int kDoneOff = kCntWords;
constexpr int kFinOff = kDoneOff + kMaxOps;
constexpr int kFlagWords = 16384;   // 64 KB, keeps the partial slots 256-byte aligned
static_assert(kFinOff < kFlagWords, "flag region");

struct Op {
  void* c;          // [M, N] fp16
  int N;
  int tiles;        // T = ceil(N / 128)
  int S;            // units per plane = K / 256
  int planes;       // 1, or 2 for a SwiGLU pair (tw = gate, twu = up)
  int dep;          // index of an earlier op whose output this op's activations are, or -1
  unsigned units;   // T * planes * S
  int ctas;         // CTAs 0 .. ctas-1 share the op (<= G; the others have no units of it)
};

struct Params {
  CUtensorMap tw[kMaxOps];    // weight rows (the gate with planes == 2)
  CUtensorMap twu[kMaxOps];   // the up projection's rows (planes == 2)
  CUtensorMap ta[kMaxOps];    // activations [M, K] as (64 values, rows, K / 64)
  Op op[kMaxOps];
  int nops;
  int M;
  int G;                      // CTAs in the grid
  unsigned* flags;            // kFlagWords counter words (zero between launches)
  unsigned dep_extra;         // 0; failure-detection tests: 1 makes every dependency wait run out
  float* part;                // [nops][G][kSlotsPerCta][128 * NB] fp32 partial tiles
  unsigned* error;            // device error word (+1: first failure record)
};

// first unit of CTA b's range of an op of U units over G CTAs
__host__ __device__ __forceinline__ unsigned range_begin(unsigned U, int b, int G) {
  return (unsigned)(((unsigned long long)U * (unsigned)b) / (unsigned)G);
}
// the CTA whose range holds unit u: the largest b with range_begin(U, b, G) <= u
__host__ __device__ __forceinline__ int owner(unsigned U, unsigned u, int G) {
  return (int)((((unsigned long long)u + 1ull) * (unsigned)G - 1ull) / U);
}
// first unit of CTA b's range when CTAs [0, Go) share the op (b >= Go: none)
__host__ __device__ __forceinline__ unsigned op_begin(unsigned U, int b, int Go) {
  return b >= Go ? U : range_begin(U, b, Go);
}
// partial slot of a CTA whose range starts at unit rs, for tile `tile` and plane pl
__host__ __device__ __forceinline__ int slot_of(unsigned rs, unsigned Q, int tile, int pl) {
  return ((int)(rs / Q) == tile ? 0 : 2) + pl;
}

template <int NB>
struct Smem {
  static constexpr int kXChunkBytes = NB * 128;                      // one 64-value activation box
  static constexpr int kXSlotBytes = kChunksPerUnit * kXChunkBytes;  // one unit of activations
  static constexpr int kWStage = wstage_bytes<WFmt::Q4K>();
  static constexpr int kWStages = 8;   // even: every stage belongs to one dequant group
  static constexpr int kXStages = x_stages<NB>();
  static constexpr int kXOff = (kWStages * kWStage + 1023) / 1024 * 1024;
  static constexpr int kBarOff = kXOff + kXStages * kXSlotBytes;
  static constexpr int bWFull = 0, bWEmpty = bWFull + kWStages;
  static constexpr int bReady = bWEmpty + kWStages;   // 4 dequant warps + the activation producer (+ TMA bytes)
  static constexpr int bUDone = bReady + kSlots;      // unit's MMAs complete: operand slot free
  static constexpr int bAccFull = bUDone + kSlots;    // segment accumulator b complete
  static constexpr int bAccEmpty = bAccFull + kAccBufs;   // segment accumulator b read by the epilogue
  static constexpr int bXFree = bAccEmpty + kAccBufs;     // activation stage free
  static constexpr int bFinal = bXFree + kXStages;
  static constexpr int kNumBars = bFinal + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kMiscOff + 64;
  static constexpr int kAlloc = kBytes + 1024;
  static_assert(kAlloc <= 232448, "dynamic shared memory per block on sm_100");
};

// Position in this CTA's unit list: op, unit within the op, and what it is.
// The op's shape is copied in when the cursor enters it, so that stepping
// from unit to unit reads registers only (the op table is a kernel parameter
// indexed at run time: every read of it is a memory load).
struct Cursor {
  int op;            // p.nops when past the end
  unsigned u, end;   // unit within the op; end of this CTA's range in it
  unsigned rs;       // start of this CTA's range in the op
  int S, P;          // the op's units per plane and planes
  unsigned U;        // the op's units
  int Go;            // CTAs sharing the op (Op::ctas)
  int tile, plane, sb;
  bool first;        // first unit of a segment (a run of one plane of one tile)
};

__device__ __forceinline__ void seek_op(const Params& p, int b, Cursor& c, int o) {
  for (; o < p.nops; ++o) {
    const unsigned U = p.op[o].units;
    const int Go = p.op[o].ctas;
    const unsigned u0 = op_begin(U, b, Go), u1 = op_begin(U, b + 1, Go);
    if (u0 < u1) {
      const unsigned S = (unsigned)p.op[o].S, Q = S * (unsigned)p.op[o].planes;
      c.S = (int)S;
      c.P = p.op[o].planes;
      c.U = U;
      c.Go = Go;
      c.op = o;
      c.u = u0;
      c.rs = u0;
      c.end = u1;
      c.tile = (int)(u0 / Q);
      const unsigned w = u0 - (unsigned)c.tile * Q;
      c.plane = (int)(w / S);
      c.sb = (int)(w - (unsigned)c.plane * S);
      c.first = true;
      return;
    }
  }
  c.op = p.nops;
}

__device__ __forceinline__ void step(const Params& p, int b, Cursor& c) {
  if (++c.u == c.end) {
    seek_op(p, b, c, c.op + 1);
    return;
  }
  c.first = false;
  if (++c.sb == c.S) {
    c.sb = 0;
    c.first = true;
    if (++c.plane == c.P) {
      c.plane = 0;
      ++c.tile;
    }
  }
}

// last unit of its segment
__device__ __forceinline__ bool seg_last(const Params& p, const Cursor& c) {
  return c.u + 1 == c.end || c.sb == c.S - 1;
}

// Bounded wait (kWaitTimeoutNs) until *addr >= target, acquiring at GPU scope.
__device__ __forceinline__ bool wait_count_gpu(const unsigned* addr, unsigned target) {
  if (ld_acquire_gpu(addr) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 16; ++i) {
      if (ld_acquire_gpu(addr) >= target) return true;
      __nanosleep(128);
    }
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) return false;
  }
}

template <int NB>
__global__ void __launch_bounds__(kThreads, 1) sweep_gemm_kernel(const __grid_constant__ Params p) {
  static_assert(NB == 16 || NB == 32, "batch tile");
  using L = Smem<NB>;
  using TM = DecodeTmem<NB>;
  constexpr uint32_t kIdesc = make_idesc_f16_f32(kTileRows, NB);
  constexpr int kWStages = L::kWStages;
  constexpr int kSlotFloats = kTileRows * NB;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_s + 1023u) & ~1023u) - raw_s);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::kBarOff;
  auto BAR = [&](int slot) { return bar0 + 8u * (uint32_t)slot; };
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(smem + L::kMiscOff);  // [0] tmem base, [1] last arriver

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int b = (int)blockIdx.x;
  const int G = p.G;
  int nunits = 0;
  for (int o = 0; o < p.nops; ++o)
    nunits += (int)(op_begin(p.op[o].units, b + 1, p.op[o].ctas) - op_begin(p.op[o].units, b, p.op[o].ctas));

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
  auto bar_count = [&](int bb) -> uint32_t {
    if (bb >= L::bWEmpty && bb < L::bWEmpty + kWStages) return 4;
    if (bb >= L::bReady && bb < L::bReady + kSlots) return 5;
    if (bb >= L::bAccEmpty && bb < L::bAccEmpty + kAccBufs) return 4;
    return 1;
  };
  // weight TMA for unit i (cursor c) into ring stage i % kWStages; one thread
  auto issue_w = [&](const Cursor& c, int i) {
    const int s = i % kWStages;
    mbar_arrive_expect_tx(BAR(L::bWFull + s), L::kWStage);
    tma_load_2d(sbase + s * L::kWStage, c.plane ? &p.twu[c.op] : &p.tw[c.op], c.sb * kQ4KBlockBytes,
                c.tile * kTileRows, BAR(L::bWFull + s), kPolicyEvictFirst);
  };

  // set-up: barriers (warp 0), TMEM (warp 1), the first weight boxes
  constexpr int kWEarly = 2;
  const int w_early = nunits < kWEarly ? nunits : kWEarly;
  if (warp == kWarpWProducer) {
    for (int bb = lane; bb < L::kNumBars; bb += 32) mbar_init(BAR(bb), bar_count(bb));
    fence_mbar_init();
    __syncwarp();
    if (lane < w_early) {
      Cursor c;
      seek_op(p, b, c, 0);
      for (int k = 0; k < lane; ++k) step(p, b, c);
      issue_w(c, lane);
    }
    __syncwarp();
  } else if (warp == kWarpXProducer) {
    tmem_alloc(sbase + L::kMiscOff, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];
  if (threadIdx.x == 0) pdl_launch_dependents();

  if (warp == kWarpWProducer) {
    // ---------------- weight producer ----------------
    Cursor c;
    seek_op(p, b, c, 0);
    for (int k = 0; k < w_early; ++k) step(p, b, c);
    int issued = w_early;
    for (int i = w_early; i < nunits; ++i, step(p, b, c)) {
      diag_unit = i;
      if (i < kWStages && !warp_wait(BAR(L::bWFull + (i - kWEarly)), 0)) break;
      if (!warp_wait(BAR(L::bWEmpty + i % kWStages), ((i / kWStages) & 1) ^ 1)) break;
      if (lane == 0) issue_w(c, i);
      __syncwarp();
      issued = i + 1;
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrWeightProducer);
    ok = true;   // never leave with copies in flight
    for (int i = issued > kWStages ? issued - kWStages : 0; i < issued; ++i)
      if (!warp_wait(BAR(L::bWFull + i % kWStages), (i / kWStages) & 1)) {
        if (lane == 0) atomicOr(p.error, kErrTeardown);
        break;
      }
  } else if (warp == kWarpXProducer) {
    // ---------------- activation producer ----------------
    // Lane 0 alone acquires the dependency counts and issues the copies, so
    // that its async-proxy fence orders what it acquired before its TMA reads.
    pdl_wait_prerequisites();   // the first op's activations may be the previous kernel's output
    Cursor c;
    seek_op(p, b, c, 0);
    int issued = 0, waited_op = -1;
    for (int i = 0; i < nunits; ++i, step(p, b, c)) {
      diag_unit = i;
      if (i >= L::kXStages && !warp_wait(BAR(L::bXFree + i % L::kXStages), ((i / L::kXStages) & 1) ^ 1)) break;
      if (i >= kSlots && !warp_wait(BAR(L::bReady + i % kSlots), ((i / kSlots) & 1) ^ 1)) break;
      if (c.op != waited_op) {
        waited_op = c.op;
        const int d = p.op[c.op].dep;
        if (d >= 0) {
          // every tile of op d stored (by whichever CTA finished it)
          bool got = true;
          if (lane == 0) {
            got = wait_count_gpu(p.flags + kDoneOff + d, (unsigned)p.op[d].tiles + p.dep_extra);
            fence_proxy_async_global();
          }
          if (!__shfl_sync(0xffffffffu, got ? 1 : 0, 0)) {
            ok = false;
            if (lane == 0) atomicCAS(p.error + 1, 0u, 0x80000000u | ((unsigned)warp << 24) | ((unsigned)(i & 0xFFF) << 12));
            break;
          }
        }
      }
      if (lane == 0) {
        const int s = i % kSlots;
        mbar_arrive_expect_tx(BAR(L::bReady + s), L::kXSlotBytes);
        tma_load_3d(sbase + L::kXOff + (i % L::kXStages) * L::kXSlotBytes, &p.ta[c.op], 0, 0, c.sb * kChunksPerUnit,
                    BAR(L::bReady + s), kPolicyEvictLast);
      }
      __syncwarp();
      issued = i + 1;
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrActProducer);
    ok = true;
    for (int i = issued > kSlots ? issued - kSlots : 0; i < issued; ++i)
      if (!warp_wait(BAR(L::bReady + i % kSlots), (i / kSlots) & 1)) {
        if (lane == 0) atomicOr(p.error, kErrTeardown);
        break;
      }
  } else if (warp == kWarpMma) {
    // ---------------- MMA issuer ----------------
    const uint64_t bdesc0 = make_sdesc_sw128(sbase + L::kXOff);
    Cursor c;
    seek_op(p, b, c, 0);
    int s = 0, seg = 0, abuf = 0;
    uint32_t ph = 0, aph = 0;   // aph: parity of this use of accumulator abuf (seg / kAccBufs)
    bool pre = false;
    for (int i = 0; i < nunits; ++i) {
      diag_unit = i;
      const bool first = c.first, last = seg_last(p, c);
      // accumulator abuf is free once the epilogue has read segment seg - kAccBufs
      if (first && seg >= kAccBufs && !warp_wait(BAR(L::bAccEmpty + abuf), aph ^ 1u)) break;
      if (!pre && !warp_wait(BAR(L::bReady + s), ph)) break;
      tc_fence_after();
      if (elect_one()) {
        const uint32_t d_acc = tmem + (uint32_t)(abuf * NB);
        const uint32_t a_t = tmem + TM::kA + (uint32_t)(s * 128);
        const uint64_t bd = bdesc0 + (uint64_t)(((i % L::kXStages) * L::kXSlotBytes) >> 4);
#pragma unroll
        for (int cc = 0; cc < kChunksPerUnit; ++cc)
#pragma unroll
          for (int t = 0; t < 4; ++t)
            mma_f16_ts(d_acc, a_t + cc * 32 + 8 * t, bd + (uint64_t)((cc * L::kXChunkBytes + 32 * t) >> 4), kIdesc,
                       (first && cc == 0 && t == 0) ? 0u : 1u);
        tc_commit(BAR(L::bUDone + s));
        tc_commit(BAR(L::bXFree + i % L::kXStages));
        if (last) tc_commit(BAR(L::bAccFull + abuf));
      }
      __syncwarp();
      if (++s == kSlots) {
        s = 0;
        ph ^= 1u;
      }
      if (last) {
        ++seg;
        if (++abuf == kAccBufs) {
          abuf = 0;
          aph ^= 1u;
        }
      }
      step(p, b, c);
      pre = (i + 1 < nunits) && __all_sync(0xffffffffu, mbar_test_wait(BAR(L::bReady + s), ph));
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrMma);
    if (elect_one()) tc_commit(BAR(L::bFinal));
    __syncwarp();
  } else if (warp >= kWarpDequant0 && warp < kWarpEpilogue0) {
    // ---------------- dequant ----------------
    const int q = warp & 3;
    const int grp = (warp - kWarpDequant0) >> 2;
    const int r = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    for (int i = grp; i < nunits; i += 2) {
      diag_unit = i;
      const int ws = i % kWStages;
      if (!warp_wait(BAR(L::bWFull + ws), (i / kWStages) & 1)) break;
      if (i >= kSlots && !warp_wait(BAR(L::bUDone + i % kSlots), ((i / kSlots) & 1) ^ 1)) break;
      tc_fence_after();
      const uint8_t* stage = smem + ws * L::kWStage;
      dequant_unit_row<WFmt::Q4K>(stage, stage + kTileRows * unit_row_bytes<WFmt::Q4K>(), r,
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
    const bool leader = (warp == kWarpEpilogue0 && lane == 0);
    float acc[NB];
    // SwiGLU: the finished gate tile waits for its up tile in TMEM columns
    // [2 NB, 3 NB) (free: the accumulators take [0, 2 NB), the operand slots
    // start at 128), not in registers
    const uint32_t gate_t = tmem + lane_off + (uint32_t)(kAccBufs * NB);
    static_assert((kAccBufs + 1) * NB <= DecodeTmem<NB>::kA, "accumulator and gate columns");
    auto save_gate = [&]() {
#pragma unroll
      for (int h = 0; h < NB; h += 16) tmem_st_x16(gate_t + (uint32_t)h, reinterpret_cast<const uint32_t*>(acc + h));
      tc_wait_st();
    };
    auto apply_gate = [&]() {
#pragma unroll
      for (int h = 0; h < NB; h += 16) {
        uint32_t x[16];
        tmem_ld_x16(gate_t + (uint32_t)h, x);
        tc_wait_ld();
#pragma unroll
        for (int t = 0; t < 16; ++t) acc[h + t] = silu(__uint_as_float(x[t])) * acc[h + t];
      }
    };

    // C rows of tile `tile` from acc (fp16; 16-byte stores of 8 outputs
    // where every row of C is 16-byte aligned)
    auto store_tile = [&](const Op& op, int tile) {
      __half* C = reinterpret_cast<__half*>(op.c);
      if ((op.N & 7) == 0 && (reinterpret_cast<uintptr_t>(C) & 15) == 0) {
        transpose_8x8_blocks<NB>(acc, lane);
        const int n0 = tile * kTileRows + q * 32 + (lane & ~7);
#pragma unroll
        for (int bb = 0; bb < NB / 8; ++bb) {
          const int t = 8 * bb + (lane & 7);
          if (t < p.M && n0 < op.N) {
            uint4 v;
            v.x = h2_as_u32(__floats2half2_rn(acc[8 * bb], acc[8 * bb + 1]));
            v.y = h2_as_u32(__floats2half2_rn(acc[8 * bb + 2], acc[8 * bb + 3]));
            v.z = h2_as_u32(__floats2half2_rn(acc[8 * bb + 4], acc[8 * bb + 5]));
            v.w = h2_as_u32(__floats2half2_rn(acc[8 * bb + 6], acc[8 * bb + 7]));
            *reinterpret_cast<uint4*>(C + (size_t)t * op.N + n0) = v;
          }
        }
      } else {
        const int n = tile * kTileRows + r;
        if (n < op.N) {
#pragma unroll
          for (int t = 0; t < NB; ++t)
            if (t < p.M) C[(size_t)t * op.N + n] = __float2half_rn(acc[t]);
        }
      }
    };

    pdl_wait_prerequisites();   // partial slots, counters and C may still be in use by the previous kernel
    Cursor c;
    seek_op(p, b, c, 0);
    int seg = 0, abuf = 0;
    uint32_t aph = 0;
    unsigned stored = 0;   // tiles of the current op this CTA stored
    while (c.op < p.nops) {
      const Op& op = p.op[c.op];
      const unsigned S = (unsigned)c.S, P = (unsigned)c.P, Q = S * P, U = c.U;
      const unsigned len = min(S - (unsigned)c.sb, c.end - c.u);
      const unsigned t_lo = (unsigned)c.tile * Q, t_hi = t_lo + Q;
      const bool whole = c.rs <= t_lo && t_hi <= c.end;
      const bool tile_end = c.u + len == min(t_hi, c.end);
      const bool op_end = c.u + len == c.end;
      diag_unit = seg;
      if (warp_wait(BAR(L::bAccFull + abuf), aph)) {
        tc_fence_after();
#pragma unroll
        for (int h = 0; h < NB; h += 16) {
          uint32_t x[16];
          tmem_ld_x16(tmem + lane_off + (uint32_t)(abuf * NB + h), x);
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
      if (lane == 0) mbar_arrive(BAR(L::bAccEmpty + abuf));
      if (++abuf == kAccBufs) {
        abuf = 0;
        aph ^= 1u;
      }

      if (whole) {
        if (P == 2 && c.plane == 0) {
          save_gate();
        } else {
          if (P == 2) apply_gate();
          if (ok) store_tile(op, c.tile);
          ++stored;
        }
      } else {
        // this CTA's part of a split tile: into its partial slot, chunk-major
        // ([NB / 4][128 rows] of float4) so that a warp's stores are contiguous
        float4* slot = reinterpret_cast<float4*>(
            p.part + ((size_t)(c.op * G + b) * kSlotsPerCta + slot_of(c.rs, Q, c.tile, c.plane)) * kSlotFloats);
#pragma unroll
        for (int j = 0; j < NB / 4; ++j)
          __stcg(slot + j * kTileRows + r, make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]));
        if (tile_end) {
          // Publish: the epilogue threads' stores, then one release by the
          // leader after the CTA barrier (a fence per thread instead cost
          // ~4 us per tile on B200 while the TMA streams ran); the leader's
          // acquire half makes the other contributors' partials visible to
          // the loads below, which the second barrier orders after it.
          const int Go = c.Go;
          const int c_lo = owner(U, t_lo, Go), c_hi = owner(U, t_hi - 1, Go);
          named_bar_sync(2, kEpilogueThreads);
          if (leader) {
            // contributors: the CTAs in [c_lo, c_hi] with units in this op
            // (all of them unless the op has fewer units than CTAs)
            unsigned n = (unsigned)(c_hi - c_lo + 1);
            if (U < (unsigned)Go) {
              n = 0;
              for (int cc = c_lo; cc <= c_hi; ++cc)
                n += range_begin(U, cc, Go) < range_begin(U, cc + 1, Go) ? 1u : 0u;
            }
            unsigned* cnt = p.flags + c.op * kMaxTiles + c.tile;
            misc[1] = (atom_add_acq_rel_gpu(cnt, 1u) == n - 1u) ? 1u : 0u;
          }
          named_bar_sync(2, kEpilogueThreads);
          if (misc[1]) {
            // the last contributor: every partial of the tile is visible
            for (unsigned pl = 0; pl < P; ++pl) {
#pragma unroll
              for (int t = 0; t < NB; ++t) acc[t] = 0.f;
              const unsigned p_lo = t_lo + pl * S, p_hi = p_lo + S;
              unsigned a1 = range_begin(U, c_lo, Go);
              for (int cc = c_lo; cc <= c_hi; ++cc) {
                const unsigned a0 = a1;
                a1 = range_begin(U, cc + 1, Go);
                if (max(a0, p_lo) >= min(a1, p_hi)) continue;   // no units of this plane
                const float4* src = reinterpret_cast<const float4*>(
                    p.part + ((size_t)(c.op * G + cc) * kSlotsPerCta + slot_of(a0, Q, c.tile, (int)pl)) * kSlotFloats);
                float4 v[NB / 4];
#pragma unroll
                for (int j = 0; j < NB / 4; ++j) v[j] = __ldcg(src + j * kTileRows + r);
#pragma unroll
                for (int j = 0; j < NB / 4; ++j) {
                  acc[4 * j] += v[j].x;
                  acc[4 * j + 1] += v[j].y;
                  acc[4 * j + 2] += v[j].z;
                  acc[4 * j + 3] += v[j].w;
                }
              }
              if (P == 2 && pl == 0) save_gate();
            }
            if (P == 2) apply_gate();
            if (ok) store_tile(op, c.tile);
            ++stored;
            if (leader) st_relaxed_gpu(p.flags + c.op * kMaxTiles + c.tile, 0u);   // for the next launch
          }
        }
      }
      if (op_end) {
        // this CTA's tiles of the op are stored: count them for the ops that read its output
        if (stored) {
          named_bar_sync(2, kEpilogueThreads);
          if (leader) red_release_gpu_add(p.flags + kDoneOff + c.op, stored);   // after the CTA barrier: covers every thread's C stores
        }
        stored = 0;
      }
      ++seg;
      // next segment
      if (op_end) {
        seek_op(p, b, c, c.op + 1);
      } else {
        c.u += len;
        c.sb = 0;
        c.first = true;
        if (++c.plane == (int)P) {
          c.plane = 0;
          ++c.tile;
        }
      }
    }
    if (!ok && lane == 0) atomicOr(p.error, kErrEpilogue);
    tc_fence_before();   // this role's TMEM accesses before the dealloc
  }

  // ---------------- teardown ----------------
  __syncwarp();
  __syncthreads();
  if (warp == kWarpXProducer) {
    bool done = true;
    if (lane == 0) done = mbar_wait(BAR(L::bFinal), 0);
    done = __shfl_sync(0xffffffffu, done ? 1 : 0, 0) != 0;
    if (!done && lane == 0) atomicOr(p.error, kErrTeardown);
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  // The last CTA to finish zeroes the op counts for the next launch: every
  // CTA has passed all its waits on them by the time it arrives here.
  if (threadIdx.x == 0) {
    pdl_wait_prerequisites();
    if (atom_add_acq_rel_gpu(p.flags + kFinOff, 1u) == (unsigned)(G - 1)) {
      for (int o = 0; o < p.nops; ++o) st_relaxed_gpu(p.flags + kDoneOff + o, 0u);
      st_relaxed_gpu(p.flags + kFinOff, 0u);
    }
  }
}

}  // namespace sweep
}  // namespace busfill
