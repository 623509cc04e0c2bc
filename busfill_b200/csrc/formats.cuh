// Weight formats of the quantized GEMMs and the per-row dequant of one unit
// (128 weight rows x 256 K) into a tcgen05 A operand in tensor memory.
//
// Numerics (fp32 accumulation of fp16 products in every format). The fp16
// operand of every format is bit-identical to the CPU dequant (the oracle):
//   Q4_0: fp16_rn((q-8)*d), the reference dequant (kernels/busfill_v0.cu:
//   74-81): the lop3 magic bias 0x6400 gives the exact fp16 1024+q, hsub2 by
//   1032 is exact, hmul2 by d rounds once.
//   Q4_0G (llama.cpp block_q4_0 rows): the same rule; high nibbles go
//   through the bias 0x5400 (64 + q) and hsub2 by 72.
//   Q4_K / Q5_K: fp16_rn(w32) with w32 = fp32(d*sc*q - dmin*m), the
//   llama.cpp CPU order (d1 = d*sc and m1 = dmin*m exact in fp32, d1*q exact,
//   one rounding of the subtraction). Steps, all exact but the last two:
//   the byte-permute / lop3 magic bias gives fp16 B + q (B = 1024, or 64 for
//   high nibbles, whose mantissa step is 1/16); hfma2(B + q, sc, -B*sc) =
//   q*sc, an integer below 2048 and so exact in fp16 (q <= 31, sc <= 63);
//   the sm_100 mixed-precision fma.rn.f32.f16(q*sc, d, -m1) multiplies two
//   fp16 values exactly and rounds q*sc*d - m1 once to fp32 (= w32, since
//   q*sc*d = d1*q); cvt.rn.f16x2.f32 rounds the pair to fp16.
//   Q6_K: fp16_rn(fp32(d*sc) * (q-32)). fma.rn.f32.f16(1024 + q, d, -1056*d)
//   = (q-32)*d exactly (16 significant bits), times sc in fp32 is exact too
//   (at most 23 bits, the oracle's product is exact as well), then one
//   rounding to fp16.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>
#include <type_traits>

#include "ptx.cuh"

namespace busfill {

// Q4_0: the reference's split planes; Q4K: llama.cpp block_q4_K rows;
// Q4_0G: llama.cpp block_q4_0 rows (18-byte blocks: fp16 d, 16 nibble bytes);
// Q5K: llama.cpp block_q5_K rows (176 bytes per 256 values);
// Q6K: llama.cpp block_q6_K rows repacked by busfill_repack_q6k into 208-byte
// block bodies (ql, qh, scales) per row and a plane of the blocks' fp16 d,
// block-major [K/256][N] (210-byte rows have no 16-byte row stride, which the
// tensor-memory-access copies need, unless K is a multiple of 2048).
enum class WFmt : int { Q4_0 = 0, Q4K = 1, Q4_0G = 2, Q5K = 3, Q6K = 4 };

constexpr int kTileRows = 128;       // weight rows per tile = MMA M
constexpr int kUnitK = 256;          // K per unit
constexpr int kChunkK = 64;          // K per activation box / 32 TMEM operand columns
constexpr int kChunksPerUnit = kUnitK / kChunkK;
constexpr int kQ4KBlockBytes = 144;
constexpr int kQ5KBlockBytes = 176;
constexpr int kQ6KBodyBytes = 208;   // block_q6_K without its trailing fp16 d
constexpr int kWStageBytes = 18432;  // 128 x 144 B (Q4_K) or 128 x 128 B + 128 x 16 B (Q4_0)

// Formats stored as whole block rows (one TMA box per unit of 128 rows).
template <WFmt F>
constexpr bool aos_rows() { return F != WFmt::Q4_0; }
// Bytes of one 256-value unit of a weight row as stored (Q4_0: its nibble
// plane; Q6_K: its block body).
template <WFmt F>
constexpr int unit_row_bytes() {
  return F == WFmt::Q5K ? kQ5KBlockBytes : F == WFmt::Q6K ? kQ6KBodyBytes : F == WFmt::Q4_0 ? 128 : kQ4KBlockBytes;
}
// Bytes per row and unit of the format's second plane, which a weight stage
// holds after the rows of the unit (Q4_0: 8 fp16 block scales; Q6_K: fp16 d).
template <WFmt F>
constexpr int aux_row_bytes() { return F == WFmt::Q4_0 ? 16 : F == WFmt::Q6K ? 2 : 0; }
// One unit of 128 weight rows in shared memory: the rows, then their second plane.
template <WFmt F>
constexpr int wstage_bytes() { return kTileRows * (unit_row_bytes<F>() + aux_row_bytes<F>()); }
static_assert(wstage_bytes<WFmt::Q4_0>() == kWStageBytes && wstage_bytes<WFmt::Q4K>() == kWStageBytes, "stages");
constexpr int kQ40ScaleOffset = 16384;
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

// Per-sub-block constants of the exact Q4_K / Q5_K operand: sc2 = {sc, sc}
// and nbsc2 = {-B*sc, -B*sc} in fp16 (exact: sc <= 63, B*sc <= 64512) for the
// magic bias B of the value words, nm1 = -fp32(dmin)*m (exact in fp32).
struct KSub {
  __half2 sc2, nbsc2;
  float nm1;
};
__device__ __forceinline__ KSub ksub(uint32_t sc, uint32_t m, float dmin, float bias) {
  KSub k;
  k.sc2 = __float2half2_rn((float)sc);
  k.nbsc2 = __float2half2_rn(-bias * (float)sc);
  k.nm1 = -dmin * (float)m;
  return k;
}

// One operand pair of an exact K-quant sub-block from the fp16 pair {B + q0,
// B + q1}: hfma2 gives q*sc exactly (an integer below 2048), the mixed fma
// rounds q*sc*d - m1 once to fp32 (= w32), the pack rounds to fp16.
__device__ __forceinline__ uint32_t k_exact_pair(uint32_t biased, const KSub& k, uint16_t d16) {
  const uint32_t qs = h2_as_u32(__hfma2(u32_as_h2(biased), k.sc2, k.nbsc2));
  float lo, hi;
  fma_f16x2_f32(qs, d16, k.nm1, lo, hi);
  return h2_as_u32(__floats2half2_rn(lo, hi));
}

// Q4_K, one 64-value chunk of a super-block: 32 bytes; byte l holds element l
// of sub-block 2c (low nibble) and of sub-block 2c+1 (high nibble). Writes
// fp16_rn(w32): out[0..15] = sub-block 2c (lo: bias 1024), out[16..31] =
// sub-block 2c+1 (hi: bias 64); d16 = the block's fp16 d bits.
__device__ __forceinline__ void dequant_q4k_chunk(const uint4 q0, const uint4 q1, uint16_t d16, const KSub& lo,
                                                  const KSub& hi, uint32_t* out) {
  const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t t0 = prmt(w[i], w[i], 0x0100u);  // byte0 = b0, byte2 = b1
    const uint32_t t1 = prmt(w[i], w[i], 0x0302u);  // byte0 = b2, byte2 = b3
    const uint32_t l01 = lop3_and_or(t0, 0x000F000Fu, 0x64006400u);  // {1024 + q}: mantissa step 1
    const uint32_t l23 = lop3_and_or(t1, 0x000F000Fu, 0x64006400u);
    const uint32_t h01 = lop3_and_or(t0, 0x00F000F0u, 0x54005400u);  // {64 + q}: mantissa step 1/16
    const uint32_t h23 = lop3_and_or(t1, 0x00F000F0u, 0x54005400u);
    out[2 * i] = k_exact_pair(l01, lo, d16);
    out[2 * i + 1] = k_exact_pair(l23, lo, d16);
    out[16 + 2 * i] = k_exact_pair(h01, hi, d16);
    out[16 + 2 * i + 1] = k_exact_pair(h23, hi, d16);
  }
}

// llama.cpp block_q4_0 rows, one 64-value chunk cc (blocks 2cc and 2cc+1 of
// the unit's eight 18-byte blocks). A unit is 144 bytes of the row; the chunk
// is its bytes [36cc, 36cc+36), i.e. words cc..cc+8 of the three 16-byte
// loads w[0..11] that cover bytes [16*floor(36cc/16), +48). Block 2cc starts
// on a 4-byte boundary (d in the low half of its first word, nibbles 2 bytes
// further on), block 2cc+1 two bytes later (d in the high half of word 4,
// nibbles word-aligned from word 5). Element e < 16 of a block is the low
// nibble of its byte e, element e >= 16 the high nibble of byte e - 16.
// Writes fp16_rn((q-8)*d): out[0..15] block 2cc, out[16..31] block 2cc+1.
template <int CC>
__device__ __forceinline__ void dequant_q4_0g_chunk(const uint32_t* w, uint32_t* out) {
  constexpr int o = CC;  // first word of the chunk within w
  const __half2 b1032 = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));  // 1032
  const __half2 b72 = __halves2half2(__ushort_as_half(0x5480), __ushort_as_half(0x5480));    // 72
  uint32_t q[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] = prmt(w[o + i], w[o + i + 1], 0x5432u);  // bytes 2.. of the first block
#pragma unroll
  for (int i = 0; i < 4; ++i) q[4 + i] = w[o + 5 + i];
  const uint32_t d0 = w[o] & 0xFFFFu, d1 = w[o + 4] >> 16;
  const __half2 dd[2] = {u32_as_h2(d0 | (d0 << 16)), u32_as_h2(d1 | (d1 << 16))};
#pragma unroll
  for (int b = 0; b < 2; ++b) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t t0 = prmt(q[4 * b + i], q[4 * b + i], 0x0100u);  // byte0 = byte 4i, byte2 = byte 4i+1
      const uint32_t t1 = prmt(q[4 * b + i], q[4 * b + i], 0x0302u);  // bytes 4i+2, 4i+3
      const uint32_t l01 = lop3_and_or(t0, 0x000F000Fu, 0x64006400u);  // {1024 + q}
      const uint32_t l23 = lop3_and_or(t1, 0x000F000Fu, 0x64006400u);
      const uint32_t h01 = lop3_and_or(t0, 0x00F000F0u, 0x54005400u);  // {64 + q}
      const uint32_t h23 = lop3_and_or(t1, 0x00F000F0u, 0x54005400u);
      out[16 * b + 2 * i] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(l01), b1032), dd[b]));
      out[16 * b + 2 * i + 1] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(l23), b1032), dd[b]));
      out[16 * b + 8 + 2 * i] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(h01), b72), dd[b]));
      out[16 * b + 8 + 2 * i + 1] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(h23), b72), dd[b]));
    }
  }
}

// silu(x) = x * sigmoid(x), in fp32 (one exp and one fast division through
// the CUDA intrinsics); the SwiGLU epilogues write fp16_rn(silu(gate) * up) of
// the fp32 accumulators. The IEEE division took its slow path whenever exp(-x)
// overflowed (x < -88, common for unnormalised gates) and cost the prefill
// SwiGLU ~40 us at M = 512; the fast division returns 0 for such divisors
// (silu -> -0), the limit of x / (1 + exp(-x)).
__device__ __forceinline__ float silu(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
__device__ __forceinline__ float out_to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float out_to_f32(float v) { return v; }

// Q5_K, one 64-value chunk cc of a super-block: q0/q1 are the chunk's 32 qs
// bytes (byte l: low nibble element l of sub-block 2cc, high nibble element l
// of sub-block 2cc+1), h0/h1 the 32 qh bytes (bit G of byte l: the fifth bit
// of element l of sub-block G). Each byte of a word is first made the whole
// 5-bit value (nibble | fifth bit << 4); a byte-permute then sets each value
// under the fp16 exponent byte 0x64, giving the exact fp16 1024 + q, and
// k_exact_pair makes fp16_rn(w32) of it (both sub-blocks with bias 1024).
template <int CC>
__device__ __forceinline__ void dequant_q5k_chunk(const uint4 q0, const uint4 q1, const uint4 h0, const uint4 h1,
                                                  uint16_t d16, const KSub& lo, const KSub& hi, uint32_t* out) {
  const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
  constexpr int bl = 2 * CC, bh = 2 * CC + 1;   // the fifth bits' positions in the qh bytes
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    // move bit b of every qh byte to bit 4 of the same byte (bits pushed into
    // a neighbouring byte never land on bit 4 and are masked off)
    const uint32_t fl = (bl <= 4 ? hw[i] << (4 - bl) : hw[i] >> (bl - 4)) & 0x10101010u;
    const uint32_t fh = (bh <= 4 ? hw[i] << (4 - bh) : hw[i] >> (bh - 4)) & 0x10101010u;
    const uint32_t ql = lop3_and_or(w[i], 0x0F0F0F0Fu, fl);        // four 5-bit values, sub-block 2cc
    const uint32_t qh = lop3_and_or(w[i] >> 4, 0x0F0F0F0Fu, fh);   // sub-block 2cc+1
    out[2 * i] = k_exact_pair(prmt(ql, 0x64u, 0x4140u), lo, d16);   // {1024 + q}
    out[2 * i + 1] = k_exact_pair(prmt(ql, 0x64u, 0x4342u), lo, d16);
    out[16 + 2 * i] = k_exact_pair(prmt(qh, 0x64u, 0x4140u), hi, d16);
    out[16 + 2 * i + 1] = k_exact_pair(prmt(qh, 0x64u, 0x4342u), hi, d16);
  }
}

// Q6_K, one 64-value chunk cc of a block (half h = cc / 2; odd = cc % 2):
// qlp points at the half's 64 ql bytes (shared memory, 16-byte aligned),
// qh[0..7] are its 32 qh bytes. Element l
// of group jj (elements 32 jj + l of the chunk) has its low 4 bits in ql byte
// 32 jj + l (low nibble for even chunks, high nibble for odd ones) and its
// top 2 bits at bit 4 odd + 2 jj of qh byte l. scf[t]: the int8 scale of the
// chunk's 16-value group t as fp32; d16 / nd1056 = the block's fp16 d bits
// and -1056*d (exact in fp32). Writes fp16_rn(fp32(d*sc) * (q-32)):
// out[16 jj + i] = elements 32 jj + 2i, +1.
template <int ODD>
__device__ __forceinline__ void dequant_q6k_chunk(const uint8_t* qlp, const uint32_t* qh, uint16_t d16,
                                                  float nd1056, const float* scf, uint32_t* out) {
#pragma unroll
  for (int jj = 0; jj < 2; ++jj) {
    constexpr int kLoSh = 4 * ODD;  // nibble of the ql bytes
    const uint4 x0 = *reinterpret_cast<const uint4*>(qlp + 32 * jj);
    const uint4 x1 = *reinterpret_cast<const uint4*>(qlp + 32 * jj + 16);
    const uint32_t ql[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      // the top 2 bits sit at bit s = 4 ODD + 2 jj of each qh byte; move them
      // to bits 4-5 (bits that cross into a neighbouring byte are masked off)
      const int s = 4 * ODD + 2 * jj;
      const uint32_t hq = s <= 4 ? qh[i] << (4 - s) : qh[i] >> (s - 4);
      // four 6-bit values (bytes) of elements 4i .. 4i+3 of the group
      const uint32_t q4 = lop3_and_or(ql[i] >> kLoSh, 0x0F0F0F0Fu, hq & 0x30303030u);
      const float sc = scf[2 * jj + (i >> 2)];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        // {0x64 q, 0x64 q'}: fp16 1024 + q; (1024 + q) d - 1056 d = (q - 32) d exactly
        float lo, hi;
        fma_f16x2_f32(prmt(q4, 0x64u, h ? 0x4342u : 0x4140u), d16, nd1056, lo, hi);
        mul_f32x2(lo, hi, sc);   // exact: at most 23 significant bits
        out[16 * jj + 2 * i + h] = h2_as_u32(__floats2half2_rn(lo, hi));
      }
    }
  }
}

template <typename OutT>
__device__ __forceinline__ OutT to_out(float v);
template <>
__device__ __forceinline__ __half to_out<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ float to_out<float>(float v) { return v; }

// Dequantize chunks [C0, C1) of this thread's weight row r of one unit held
// in a weight stage (the TMA box of the unit: Q4_K / Q4_0G rows of 144 B;
// Q5_K rows of 176 B; Q6_K rows of 208 B and the rows' fp16 d at `aux` + 2 r;
// Q4_0 rows of 128 B of nibbles with the 128-byte swizzle, and 8 fp16 scales
// per row at `aux` + 16 r) and store them as TMEM operand columns from
// `a_slot` (this warp's lane quarter already in the address): chunk cc goes
// to columns 32 (cc - C0) .. +31, column c of a chunk holding k = 64 cc + 2c,
// 2c+1 as an fp16 pair. The caller waits for the stores (tcgen05.wait::st)
// before publishing the slot.
template <WFmt FMT, int C0 = 0, int C1 = kChunksPerUnit>
__device__ __forceinline__ void dequant_unit_row(const uint8_t* stage, const uint8_t* aux, int r,
                                                 uint32_t a_slot) {
  static_assert(0 <= C0 && C0 < C1 && C1 <= kChunksPerUnit, "chunk range");
  if constexpr (FMT == WFmt::Q4K || FMT == WFmt::Q5K) {
    // this row's block header: d, dmin and the 6-bit scales/mins of its
    // sub-blocks (llama.cpp get_scale_min_k4 packing): *_lo holds
    // sub-blocks 0-3 in bytes 0-3, *_hi sub-blocks 4-7. Q5_K: qh at 16,
    // qs at 48; Q4_K: qs at 16.
    constexpr int kRow = unit_row_bytes<FMT>();
    const uint8_t* row = stage + r * kRow;
    const uint4 hdr = *reinterpret_cast<const uint4*>(row);
    const uint16_t d16 = (uint16_t)(hdr.x & 0xFFFFu);
    const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr.x >> 16)));
    const uint32_t sc_lo = hdr.y & 0x3F3F3F3Fu;
    const uint32_t m_lo = hdr.z & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
    const uint32_t m_hi = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
    auto chunk = [&](auto cc_tag) {
      constexpr int cc = decltype(cc_tag)::value;
      // chunk cc covers sub-blocks 2cc, 2cc+1: bytes 2(cc&1), 2(cc&1)+1 of the
      // _lo words (cc < 2) or of the _hi words (cc >= 2)
      const uint32_t scw = cc < 2 ? sc_lo : sc_hi;
      const uint32_t mw = cc < 2 ? m_lo : m_hi;
      constexpr int sh = 16 * (cc & 1);
      // value-word biases: Q4_K low nibbles 1024, high nibbles 64; Q5_K 1024
      constexpr float kBiasHi = FMT == WFmt::Q4K ? 64.f : 1024.f;
      const KSub lo = ksub((scw >> sh) & 0xFFu, (mw >> sh) & 0xFFu, dmin, 1024.f);
      const KSub hi = ksub((scw >> (sh + 8)) & 0xFFu, (mw >> (sh + 8)) & 0xFFu, dmin, kBiasHi);
      uint32_t P[32];
      if constexpr (FMT == WFmt::Q4K) {
        const uint4 q0 = *reinterpret_cast<const uint4*>(row + 16 + cc * 32);
        const uint4 q1 = *reinterpret_cast<const uint4*>(row + 32 + cc * 32);
        dequant_q4k_chunk(q0, q1, d16, lo, hi, P);
      } else {
        const uint4 q0 = *reinterpret_cast<const uint4*>(row + 48 + cc * 32);
        const uint4 q1 = *reinterpret_cast<const uint4*>(row + 64 + cc * 32);
        const uint4 h0 = *reinterpret_cast<const uint4*>(row + 16);
        const uint4 h1 = *reinterpret_cast<const uint4*>(row + 32);
        dequant_q5k_chunk<cc>(q0, q1, h0, h1, d16, lo, hi, P);
      }
      tmem_st_x32(a_slot + (cc - C0) * 32, P);
    };
    if constexpr (C0 <= 0 && 0 < C1) chunk(std::integral_constant<int, 0>{});
    if constexpr (C0 <= 1 && 1 < C1) chunk(std::integral_constant<int, 1>{});
    if constexpr (C0 <= 2 && 2 < C1) chunk(std::integral_constant<int, 2>{});
    if constexpr (C0 <= 3 && 3 < C1) chunk(std::integral_constant<int, 3>{});
  } else if constexpr (FMT == WFmt::Q6K) {
    const uint8_t* row = stage + r * kQ6KBodyBytes;   // ql at 0, qh at 128, int8 scales at 192
    const uint16_t d16 = *reinterpret_cast<const uint16_t*>(aux + 2 * r);
    const float nd1056 = -1056.f * __half2float(__ushort_as_half(d16));
    const uint4 scv = *reinterpret_cast<const uint4*>(row + 192);
    const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
    auto chunk = [&](auto cc_tag) {
      constexpr int cc = decltype(cc_tag)::value;
      constexpr int h = cc >> 1;
      uint32_t qh[8];
#pragma unroll
      for (int v = 0; v < 2; ++v) {
        const uint4 x = *reinterpret_cast<const uint4*>(row + 128 + 32 * h + 16 * v);
        qh[4 * v] = x.x; qh[4 * v + 1] = x.y; qh[4 * v + 2] = x.z; qh[4 * v + 3] = x.w;
      }
      float scf[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) scf[t] = (float)(int)(int8_t)((scw[cc] >> (8 * t)) & 0xFFu);
      uint32_t P[32];
      dequant_q6k_chunk<cc & 1>(row + 64 * h, qh, d16, nd1056, scf, P);
      tmem_st_x32(a_slot + (cc - C0) * 32, P);
    };
    if constexpr (C0 <= 0 && 0 < C1) chunk(std::integral_constant<int, 0>{});
    if constexpr (C0 <= 1 && 1 < C1) chunk(std::integral_constant<int, 1>{});
    if constexpr (C0 <= 2 && 2 < C1) chunk(std::integral_constant<int, 2>{});
    if constexpr (C0 <= 3 && 3 < C1) chunk(std::integral_constant<int, 3>{});
  } else if constexpr (FMT == WFmt::Q4_0G) {
    const uint8_t* urow = stage + r * unit_row_bytes<FMT>();
    uint32_t P[32];
    auto chunk = [&](auto cc_tag) {
      constexpr int cc = decltype(cc_tag)::value;
      constexpr int v0 = (36 * cc) / 16;  // first 16-byte load covering the chunk
      uint32_t w[12];
#pragma unroll
      for (int v = 0; v < 3; ++v) {
        const uint4 x = *reinterpret_cast<const uint4*>(urow + 16 * (v0 + v));
        w[4 * v] = x.x; w[4 * v + 1] = x.y; w[4 * v + 2] = x.z; w[4 * v + 3] = x.w;
      }
      dequant_q4_0g_chunk<(36 * cc % 16) / 4>(w, P);
      tmem_st_x32(a_slot + (cc - C0) * 32, P);
    };
    if constexpr (C0 <= 0 && 0 < C1) chunk(std::integral_constant<int, 0>{});
    if constexpr (C0 <= 1 && 1 < C1) chunk(std::integral_constant<int, 1>{});
    if constexpr (C0 <= 2 && 2 < C1) chunk(std::integral_constant<int, 2>{});
    if constexpr (C0 <= 3 && 3 < C1) chunk(std::integral_constant<int, 3>{});
  } else {
    const uint8_t* wrow = stage + r * 128;
    const uint32_t sw = (uint32_t)(r & 7);  // TMA 128-byte swizzle: 16-B chunk ^= row % 8
    const uint4 dd = *reinterpret_cast<const uint4*>(aux + r * 16);  // 8 block scales
    auto chunk = [&](auto cc_tag) {
      constexpr int cc = decltype(cc_tag)::value;
      uint32_t P[32];
      const uint4 b0 = *reinterpret_cast<const uint4*>(wrow + ((((uint32_t)(2 * cc)) ^ sw) << 4));
      const uint4 b1 = *reinterpret_cast<const uint4*>(wrow + ((((uint32_t)(2 * cc + 1)) ^ sw) << 4));
      const __half2 d01 = u32_as_h2(cc == 0 ? dd.x : cc == 1 ? dd.y : cc == 2 ? dd.z : dd.w);
      dequant_q4_0_block(b0, __low2half2(d01), P);
      dequant_q4_0_block(b1, __high2half2(d01), P + 16);
      tmem_st_x32(a_slot + (cc - C0) * 32, P);
    };
    if constexpr (C0 <= 0 && 0 < C1) chunk(std::integral_constant<int, 0>{});
    if constexpr (C0 <= 1 && 1 < C1) chunk(std::integral_constant<int, 1>{});
    if constexpr (C0 <= 2 && 2 < C1) chunk(std::integral_constant<int, 2>{});
    if constexpr (C0 <= 3 && 3 < C1) chunk(std::integral_constant<int, 3>{});
  }
}

}  // namespace busfill
