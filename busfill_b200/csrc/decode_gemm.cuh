// Batched dequant-fused 4-bit-weight GEMM for small batches (M <= 64) on
// sm_100a:  C[M, N] = A[M, K] * deq(W)[N, K]^T, fp16 in, fp32 accumulate.
//
// Replaces the reference kernel `busfill_q4` (kernels/busfill_v1a.cu:41-104,
// launched <<<N/32, 128>>> at kernels/busfill_v1a.cu:151-154), which is an
// sm_70 mma.m8n8k4 loop capped at 32 batch rows.
//
// Design (one persistent CTA per SM, 12 warps):
//   warp 0      TMA producer for the weight stream: one 2D box of 128 weight
//               rows x one 256-value unit per stage (18 KB) into a 6-stage
//               shared-memory ring. Weights do not depend on earlier kernels,
//               so this starts before griddepcontrol.wait (PDL overlap).
//   warp 2      TMA producer for activations: one 64-value x NB-row box per
//               chunk, 128-byte swizzled (the UMMA K-major SW128 layout).
//   warps 4-11  dequant: thread (warp%4, lane) owns weight row 32*(warp%4)+lane
//               and writes its fp16 operand straight into TMEM with
//               tcgen05.st (the tensor core reads A from TMEM); the same warps
//               run the per-unit epilogue from TMEM.
//   warp 1      TMEM allocator + the single MMA-issuing thread:
//               tcgen05.mma.cta_group::1.kind::f16, M=128 weight rows, N=NB
//               batch rows (swap-AB), K=16 per instruction.
//
// Work split: the GEMM is cut into units of (128 weight rows) x (256 K).
// CTA c of G takes units [floor(c*U/G), floor((c+1)*U/G)) in tile-major
// order ("stream-K"), so every SM streams the same number of weight bytes.
// A tile split across CTAs is reduced deterministically: each contributor
// stores its fp32 partial in its slot, the last arriver (by an atomic
// counter) sums the slots in slot order and writes C, then resets the counter.
//
// Numerics.
//   Q4_0: the operand is fp16_rn((q-8)*d), bit-identical to the reference
//   dequant (kernels/busfill_v0.cu:74-81): lop3 magic bias 0x6400 gives the
//   exact fp16 1024+q, hsub2 by 1032 is exact, hmul2 by d rounds once.
//   Q4_K: w = d*sc*q - dmin*m. The operand is P = sc*q, made exactly in fp16
//   by one hfma2 ((1024+q)*sc - 1024*sc; the high nibble arrives as 1024+16q
//   and uses sc/16 and 64*sc, both exact). A second operand holds m broadcast
//   over its 32-value sub-block. Per unit the tensor core accumulates
//   X = sum A*P and Y = sum A*m in fp32; the epilogue adds d*X - dmin*Y in
//   fp32. All products are exact, so the result equals an fp32-accumulated
//   matmul of the exact dequantized weights up to summation order.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "ptx.cuh"

namespace busfill {

enum class WFmt : int { Q4_0 = 0, Q4K = 1 };

constexpr int kTileRows = 128;       // weight rows per tile = MMA M
constexpr int kUnitK = 256;          // K per unit: one Q4_K super-block / eight Q4_0 blocks
constexpr int kChunkK = 64;          // K per TMEM operand stage and per activation box
constexpr int kChunksPerUnit = kUnitK / kChunkK;
constexpr int kQ4KBlockBytes = 144;
constexpr int kWStageBytes = 18432;  // 128 x 144 B (Q4_K) or 128 x 128 B + 128 x 16 B (Q4_0)
constexpr int kQ40ScaleOffset = 16384;
constexpr int kWStages = 6;
constexpr int kXStages = 8;
constexpr int kAStages = 4;          // TMEM operand stages, 64 columns each
constexpr int kThreads = 384;
constexpr int kFirstDequantWarp = 4;
constexpr int kDequantThreads = 256;
constexpr int kTmemCols = 512;

// device error word bits (OR-ed; 0 = no error)
constexpr unsigned kErrWeightProducer = 1u;
constexpr unsigned kErrActProducer = 2u;
constexpr unsigned kErrMma = 4u;
constexpr unsigned kErrDequant = 8u;
constexpr unsigned kErrEpilogue = 16u;
constexpr unsigned kErrTeardown = 32u;

struct DecodeParams {
  void* c;              // [M, N] row-major, OutT
  float* partials;      // [tiles][max_slots][128][NB] fp32 split-K partials
  unsigned* counters;   // [tiles] arrival counters, zero between calls
  unsigned* error;      // device error word
  int M, N, K;
  int tiles;            // T = ceil(N / 128)
  int units_per_tile;   // S = K / 256
  int units;            // U = T * S
  int max_slots;        // max CTAs contributing to one tile
};

__host__ __device__ __forceinline__ int streamk_first_unit(long long cta, long long units, long long grid) {
  return (int)((cta * units) / grid);
}
// CTA whose unit range contains unit u: max{c : floor(c*U/G) <= u}.
__host__ __device__ __forceinline__ int streamk_cta_of(long long u, long long units, long long grid) {
  return (int)(((u + 1) * grid + units - 1) / units - 1);
}

template <int NB>
struct DecodeSmem {
  static constexpr int kXStageBytes = NB * 128;
  static constexpr int kWOff = 0;
  static constexpr int kXOff = kWOff + kWStages * kWStageBytes;
  static constexpr int kBarOff = kXOff + kXStages * kXStageBytes;
  // barriers: wfull, wempty, xfull, xempty, afull, aempty, accfull[2], accempty[2], final
  static constexpr int kNumBars = 2 * kWStages + 2 * kXStages + 2 * kAStages + 4 + 1;
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

__device__ __forceinline__ void named_bar_sync_dequant() {
  asm volatile("bar.sync 1, %0;" ::"n"(kDequantThreads) : "memory");
}

template <typename OutT>
__device__ __forceinline__ OutT to_out(float v);
template <>
__device__ __forceinline__ __half to_out<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ float to_out<float>(float v) { return v; }

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <WFmt FMT, int NB, typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
    decode_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_ws,
                       const __grid_constant__ CUtensorMap tmap_a, const DecodeParams p) {
  static_assert(NB == 16 || NB == 32 || NB == 64, "batch tile");
  using L = DecodeSmem<NB>;
  constexpr int HALF = NB / 2;  // batch columns per epilogue group
  constexpr uint32_t kIdesc = make_idesc_f16_f32(kTileRows, NB);
  constexpr int kAccCols = 2 * NB;            // X (and Y for Q4_K) per accumulator buffer
  constexpr int kAOff = 2 * kAccCols;         // operand stages start after 2 accumulators
  static_assert(kAOff + kAStages * 64 <= kTmemCols, "TMEM budget");

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_s + 1023u) & ~1023u) - raw_s);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::kBarOff;
  auto BAR_WFULL = [&](int s) { return bar0 + 8u * s; };
  auto BAR_WEMPTY = [&](int s) { return bar0 + 8u * (kWStages + s); };
  auto BAR_XFULL = [&](int s) { return bar0 + 8u * (2 * kWStages + s); };
  auto BAR_XEMPTY = [&](int s) { return bar0 + 8u * (2 * kWStages + kXStages + s); };
  auto BAR_AFULL = [&](int s) { return bar0 + 8u * (2 * kWStages + 2 * kXStages + s); };
  auto BAR_AEMPTY = [&](int s) { return bar0 + 8u * (2 * kWStages + 2 * kXStages + kAStages + s); };
  auto BAR_ACCFULL = [&](int b) { return bar0 + 8u * (2 * kWStages + 2 * kXStages + 2 * kAStages + b); };
  auto BAR_ACCEMPTY = [&](int b) { return bar0 + 8u * (2 * kWStages + 2 * kXStages + 2 * kAStages + 2 + b); };
  const uint32_t BAR_FINAL = bar0 + 8u * (2 * kWStages + 2 * kXStages + 2 * kAStages + 4);
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);  // [0] tmem base, [1] last-arriver flag

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = p.units_per_tile;
  const int u0 = streamk_first_unit(blockIdx.x, p.units, gridDim.x);
  const int u1 = streamk_first_unit(blockIdx.x + 1, p.units, gridDim.x);
  const int nunits = u1 - u0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kWStages; ++s) { mbar_init(BAR_WFULL(s), 1); mbar_init(BAR_WEMPTY(s), 8); }
    for (int s = 0; s < kXStages; ++s) { mbar_init(BAR_XFULL(s), 1); mbar_init(BAR_XEMPTY(s), 1); }
    for (int s = 0; s < kAStages; ++s) { mbar_init(BAR_AFULL(s), 4); mbar_init(BAR_AEMPTY(s), 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(BAR_ACCFULL(b), 1); mbar_init(BAR_ACCEMPTY(b), 8); }
    mbar_init(BAR_FINAL, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmap_w);
    if (FMT == WFmt::Q4_0) tma_prefetch_desc(&tmap_ws);
    tma_prefetch_desc(&tmap_a);
  }
  if (warp == 1) {
    tmem_alloc(sbase + L::kMiscOff, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];
  // Let the next kernel on the stream launch now: its CTAs take SMs as ours
  // retire and begin streaming their weights before our tail completes.
  if (threadIdx.x == 0) pdl_launch_dependents();

  if (warp == 0) {
    // ---------------- weight producer ----------------
    if (lane == 0) {
      bool ok = true;
      int issued = 0;
      for (int i = 0; i < nunits; ++i) {
        const int s = i % kWStages;
        if (!mbar_wait(BAR_WEMPTY(s), ((i / kWStages) & 1) ^ 1)) { ok = false; break; }
        const int u = u0 + i;
        const int tile = u / S, sb = u - tile * S;
        const uint32_t dst = sbase + L::kWOff + s * kWStageBytes;
        mbar_arrive_expect_tx(BAR_WFULL(s), kWStageBytes);
        if constexpr (FMT == WFmt::Q4K) {
          tma_load_2d(dst, &tmap_w, sb * kQ4KBlockBytes, tile * kTileRows, BAR_WFULL(s), kPolicyEvictFirst);
        } else {
          tma_load_2d(dst, &tmap_w, sb * 128, tile * kTileRows, BAR_WFULL(s), kPolicyEvictFirst);
          tma_load_2d(dst + kQ40ScaleOffset, &tmap_ws, sb * 8, tile * kTileRows, BAR_WFULL(s), kPolicyEvictFirst);
        }
        issued = i + 1;
      }
      if (!ok) atomicOr(p.error, kErrWeightProducer);
      // never leave the CTA with copies in flight
      for (int i = issued > kWStages ? issued - kWStages : 0; i < issued; ++i)
        if (!mbar_wait(BAR_WFULL(i % kWStages), (i / kWStages) & 1)) atomicOr(p.error, kErrTeardown);
    }
  } else if (warp == 2) {
    // ---------------- activation producer ----------------
    if (lane == 0) {
      pdl_wait_prerequisites();  // activations may be the previous kernel's output
      bool ok = true;
      int issued = 0;
      const int total = nunits * kChunksPerUnit;
      for (int j = 0; j < total; ++j) {
        const int s = j % kXStages;
        if (!mbar_wait(BAR_XEMPTY(s), ((j / kXStages) & 1) ^ 1)) { ok = false; break; }
        const int u = u0 + j / kChunksPerUnit;
        const int sb = u % S;
        mbar_arrive_expect_tx(BAR_XFULL(s), L::kXStageBytes);
        tma_load_2d(sbase + L::kXOff + s * L::kXStageBytes, &tmap_a, sb * kUnitK + (j % kChunksPerUnit) * kChunkK, 0,
                    BAR_XFULL(s), kPolicyEvictLast);
        issued = j + 1;
      }
      if (!ok) atomicOr(p.error, kErrActProducer);
      for (int j = issued > kXStages ? issued - kXStages : 0; j < issued; ++j)
        if (!mbar_wait(BAR_XFULL(j % kXStages), (j / kXStages) & 1)) atomicOr(p.error, kErrTeardown);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      bool ok = true;
      int accq = 0;        // accumulator buffers handed out so far
      int prev_tile = -1;
      int acc = 0;
      for (int i = 0; i < nunits && ok; ++i) {
        const int u = u0 + i;
        const int tile = u / S;
        const bool fresh = (FMT == WFmt::Q4K) || (tile != prev_tile);
        const bool closes = (FMT == WFmt::Q4K) || (i == nunits - 1) || ((u + 1) / S != tile);
        prev_tile = tile;
        if (fresh) {
          acc = accq & 1;
          if (!mbar_wait(BAR_ACCEMPTY(acc), ((accq >> 1) & 1) ^ 1)) { ok = false; break; }
          tc_fence_after();
        }
        const uint32_t d_x = tmem + acc * kAccCols;
        const uint32_t d_y = d_x + NB;
        for (int cc = 0; cc < kChunksPerUnit; ++cc) {
          const int j = i * kChunksPerUnit + cc;
          const int as = j % kAStages, xs = j % kXStages;
          if (!mbar_wait(BAR_AFULL(as), (j / kAStages) & 1)) { ok = false; break; }
          if (!mbar_wait(BAR_XFULL(xs), (j / kXStages) & 1)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_t = tmem + kAOff + as * 64;
          const uint32_t b_s = sbase + L::kXOff + xs * L::kXStageBytes;
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const uint64_t bdesc = make_sdesc_sw128(b_s + 32 * t);
            const uint32_t accum = (fresh && cc == 0 && t == 0) ? 0u : 1u;
            mma_f16_ts(d_x, a_t + 8 * t, bdesc, kIdesc, accum);
            if constexpr (FMT == WFmt::Q4K) mma_f16_ts(d_y, a_t + 32 + 8 * t, bdesc, kIdesc, accum);
          }
          tc_commit(BAR_AEMPTY(as));
          tc_commit(BAR_XEMPTY(xs));
        }
        if (!ok) break;
        if (closes) {
          tc_commit(BAR_ACCFULL(acc));
          ++accq;
        }
      }
      if (!ok) atomicOr(p.error, kErrMma);
      tc_commit(BAR_FINAL);  // fires once every MMA issued above has completed
    }
  } else if (warp >= kFirstDequantWarp) {
    // ---------------- dequant + epilogue ----------------
    const int q = warp & 3;                          // TMEM lane quarter this warp may touch
    const int g = (warp - kFirstDequantWarp) >> 2;   // group: chunks {g, g+2}, batch half g
    const int r = q * 32 + lane;                     // weight row within the tile
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    bool ok = true;
    float accv[HALF];
#pragma unroll
    for (int t = 0; t < HALF; ++t) accv[t] = 0.f;
    float pend_d = 0.f, pend_dmin = 0.f;  // Q4_K scales of the unit awaiting its epilogue
    int accq = 0;                          // Q4_0: accumulator buffers consumed

    auto warp_wait = [&](uint32_t bar, uint32_t parity) -> bool {
      if (!ok) return false;
      const bool got = mbar_wait(bar, parity);
      ok = __all_sync(0xffffffffu, got);
      return ok;
    };

    // write this thread's finished segment (tile) result
    auto flush = [&](int tile) {
      pdl_wait_prerequisites();  // C / workspace may still be in use by the previous kernel
      const int tfirst = tile * S, tlast = tile * S + S - 1;
      const int first_cta = streamk_cta_of(tfirst, p.units, gridDim.x);
      const int last_cta = streamk_cta_of(tlast, p.units, gridDim.x);
      const int n = tile * kTileRows + r;
      OutT* C = reinterpret_cast<OutT*>(p.c);
      if (first_cta == last_cta) {
        if (ok && n < p.N) {
#pragma unroll
          for (int t = 0; t < HALF; ++t) {
            const int b = g * HALF + t;
            if (b < p.M) C[(size_t)b * p.N + n] = to_out<OutT>(accv[t]);
          }
        }
        return;
      }
      const int slot = (int)blockIdx.x - first_cta;
      const int ncontrib = last_cta - first_cta + 1;
      float* mine = p.partials + (((size_t)tile * p.max_slots + slot) * kTileRows + r) * NB + g * HALF;
#pragma unroll
      for (int t = 0; t < HALF; t += 4)
        *reinterpret_cast<float4*>(mine + t) = make_float4(accv[t], accv[t + 1], accv[t + 2], accv[t + 3]);
      __threadfence();
      named_bar_sync_dequant();
      if (threadIdx.x == kFirstDequantWarp * 32) {
        const unsigned old = atomicAdd(&p.counters[tile], 1u);
        misc[1] = (old == (unsigned)(ncontrib - 1)) ? 1u : 0u;
      }
      named_bar_sync_dequant();
      if (misc[1] != 0u) {
        __threadfence();
        float sum[HALF];
#pragma unroll
        for (int t = 0; t < HALF; ++t) sum[t] = 0.f;
        for (int s = 0; s < ncontrib; ++s) {
          if (s == slot) {
#pragma unroll
            for (int t = 0; t < HALF; ++t) sum[t] += accv[t];
          } else {
            const float* other = p.partials + (((size_t)tile * p.max_slots + s) * kTileRows + r) * NB + g * HALF;
#pragma unroll
            for (int t = 0; t < HALF; t += 4) {
              const float4 v = __ldcg(reinterpret_cast<const float4*>(other + t));
              sum[t] += v.x; sum[t + 1] += v.y; sum[t + 2] += v.z; sum[t + 3] += v.w;
            }
          }
        }
        if (ok && n < p.N) {
#pragma unroll
          for (int t = 0; t < HALF; ++t) {
            const int b = g * HALF + t;
            if (b < p.M) C[(size_t)b * p.N + n] = to_out<OutT>(sum[t]);
          }
        }
        if (threadIdx.x == kFirstDequantWarp * 32) p.counters[tile] = 0u;  // ready for the next call
      }
    };

    // epilogue for unit i (runs one unit behind the dequant)
    auto finish = [&](int i) {
      const int u = u0 + i;
      const int tile = u / S;
      const bool closes = (i == nunits - 1) || ((u + 1) / S != tile);
      if constexpr (FMT == WFmt::Q4K) {
        const int acc = i & 1;
        if (warp_wait(BAR_ACCFULL(acc), (i >> 1) & 1)) {
          tc_fence_after();
          const uint32_t cx = tmem + lane_off + acc * kAccCols + g * HALF;
          constexpr int CH = HALF < 16 ? HALF : 16;
#pragma unroll
          for (int c0 = 0; c0 < HALF; c0 += CH) {
            uint32_t xr[CH], yr[CH];
            tmem_ld_cols<CH>(cx + c0, xr);
            tmem_ld_cols<CH>(cx + NB + c0, yr);
            tc_wait_ld();
#pragma unroll
            for (int t = 0; t < CH; ++t) {
              accv[c0 + t] = fmaf(pend_d, __uint_as_float(xr[t]), accv[c0 + t]);
              accv[c0 + t] = fmaf(-pend_dmin, __uint_as_float(yr[t]), accv[c0 + t]);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(BAR_ACCEMPTY(acc));
        }
      } else {
        if (closes) {
          const int acc = accq & 1;
          if (warp_wait(BAR_ACCFULL(acc), (accq >> 1) & 1)) {
            tc_fence_after();
            const uint32_t cx = tmem + lane_off + acc * kAccCols + g * HALF;
            constexpr int CH = HALF < 16 ? HALF : 16;
#pragma unroll
            for (int c0 = 0; c0 < HALF; c0 += CH) {
              uint32_t xr[CH];
              tmem_ld_cols<CH>(cx + c0, xr);
              tc_wait_ld();
#pragma unroll
              for (int t = 0; t < CH; ++t) accv[c0 + t] = __uint_as_float(xr[t]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(BAR_ACCEMPTY(acc));
          }
          ++accq;
        }
      }
      if (closes) {
        flush(tile);
#pragma unroll
        for (int t = 0; t < HALF; ++t) accv[t] = 0.f;
      }
    };

    for (int i = 0; i < nunits; ++i) {
      const int ws = i % kWStages;
      const bool have_w = warp_wait(BAR_WFULL(ws), (i / kWStages) & 1);
      const uint8_t* stage = smem + L::kWOff + ws * kWStageBytes;
      float cur_d = 0.f, cur_dmin = 0.f;
      uint32_t sc_lo = 0, sc_hi = 0, m_lo = 0, m_hi = 0;
      if constexpr (FMT == WFmt::Q4K) {
        if (have_w) {
          const uint4 hdr = *reinterpret_cast<const uint4*>(stage + r * kQ4KBlockBytes);
          cur_d = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xFFFFu)));
          cur_dmin = __half2float(__ushort_as_half((unsigned short)(hdr.x >> 16)));
          sc_lo = hdr.y & 0x3F3F3F3Fu;
          m_lo = hdr.z & 0x3F3F3F3Fu;
          sc_hi = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
          m_hi = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
        }
      }
#pragma unroll 1
      for (int k2 = 0; k2 < 2; ++k2) {
        const int cc = g + 2 * k2;
        const int j = i * kChunksPerUnit + cc;
        const int as = j % kAStages;
        if (!have_w || !warp_wait(BAR_AEMPTY(as), ((j / kAStages) & 1) ^ 1)) continue;
        tc_fence_after();
        uint32_t P[32];
        const uint32_t a_t = tmem + lane_off + kAOff + as * 64;
        if constexpr (FMT == WFmt::Q4K) {
          const uint8_t* qs = stage + r * kQ4KBlockBytes + 16 + cc * 32;
          const uint4 q0 = *reinterpret_cast<const uint4*>(qs);
          const uint4 q1 = *reinterpret_cast<const uint4*>(qs + 16);
          const uint32_t scw = (cc < 2) ? sc_lo : sc_hi;
          const uint32_t mw = (cc < 2) ? m_lo : m_hi;
          const __half2 S2 = six_bit_pair_to_h2(scw, cc & 1);  // {sc[2cc], sc[2cc+1]}
          const __half2 M2 = six_bit_pair_to_h2(mw, cc & 1);   // {m[2cc],  m[2cc+1]}
          const __half2 mlo = __low2half2(S2);
          const __half2 alo = __hmul2(mlo, __float2half2_rn(-1024.f));
          const __half2 shi = __high2half2(S2);
          const __half2 mhi = __hmul2(shi, __float2half2_rn(0.0625f));
          const __half2 ahi = __hmul2(shi, __float2half2_rn(-64.f));
          dequant_q4k_chunk(q0, q1, mlo, alo, mhi, ahi, P);
          tmem_st_x32(a_t, P);
          tmem_st_x16_bcast(a_t + 32, h2_as_u32(__low2half2(M2)));
          tmem_st_x16_bcast(a_t + 48, h2_as_u32(__high2half2(M2)));
        } else {
          const uint8_t* wrow = stage + r * 128;
          const uint32_t sw = (uint32_t)(r & 7);  // TMA 128-byte swizzle: 16-B chunk ^= row % 8
          const uint4 b0 = *reinterpret_cast<const uint4*>(wrow + ((((uint32_t)(2 * cc)) ^ sw) << 4));
          const uint4 b1 = *reinterpret_cast<const uint4*>(wrow + ((((uint32_t)(2 * cc + 1)) ^ sw) << 4));
          const uint32_t dd = *reinterpret_cast<const uint32_t*>(stage + kQ40ScaleOffset + r * 16 + cc * 4);
          const __half2 d01 = u32_as_h2(dd);
          dequant_q4_0_block(b0, __low2half2(d01), P);
          dequant_q4_0_block(b1, __high2half2(d01), P + 16);
          tmem_st_x32(a_t, P);
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(BAR_AFULL(as));
      }
      __syncwarp();
      if (have_w && lane == 0) mbar_arrive(BAR_WEMPTY(ws));
      if (i > 0) finish(i - 1);
      pend_d = cur_d;
      pend_dmin = cur_dmin;
    }
    if (nunits > 0) finish(nunits - 1);
    if (!ok && lane == 0) atomicOr(p.error, kErrDequant);
  }

  // ---------------- teardown ----------------
  __syncthreads();
  if (warp == 1) {
    bool done = true;
    if (lane == 0) done = mbar_wait(BAR_FINAL, 0);
    done = __shfl_sync(0xffffffffu, done ? 1 : 0, 0) != 0;
    if (!done && lane == 0) atomicOr(p.error, kErrTeardown);
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace busfill
