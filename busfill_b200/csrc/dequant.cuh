// Bit-exact dequantization to fp16 [N, K] row-major. These serve the
// "dequant is bit-exact" gate and the cuBLAS fp16 comparator, and they run the
// same in-register instruction chains as the GEMM's operand producers.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

#include "decode_gemm.cuh"
#include "ptx.cuh"

namespace busfill {

// Q4_0 split planes (kernels/busfill_v1a.cu:43-45): one thread per 32-value
// block; output fp16_rn((q-8)*d) (kernels/busfill_v0.cu:74-81).
__global__ void dequant_q4_0_planes_kernel(const uint8_t* __restrict__ wq, const __half* __restrict__ ws,
                                           __half* __restrict__ out, long long nblocks) {
  for (long long b = blockIdx.x * (long long)blockDim.x + threadIdx.x; b < nblocks;
       b += (long long)gridDim.x * blockDim.x) {
    const uint4 q = *reinterpret_cast<const uint4*>(wq + b * 16);
    const __half2 d2 = __half2half2(ws[b]);
    uint32_t v[16];
    dequant_q4_0_block(q, d2, v);
    uint4* o = reinterpret_cast<uint4*>(out + b * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  }
}

// llama.cpp block_q4_0 (18 bytes: fp16 d, 16 bytes; byte j = element j (low
// nibble) and element j+16 (high nibble)). The blocks are only 2-byte
// aligned, so bytes are read with 16-bit loads.
__global__ void dequant_q4_0_ggml_kernel(const uint8_t* __restrict__ blocks, __half* __restrict__ out,
                                         long long nblocks) {
  for (long long b = blockIdx.x * (long long)blockDim.x + threadIdx.x; b < nblocks;
       b += (long long)gridDim.x * blockDim.x) {
    const uint16_t* blk = reinterpret_cast<const uint16_t*>(blocks + b * 18);
    const __half d = __ushort_as_half(blk[0]);
    const float df = __half2float(d);
    __half lo[16], hi[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t two = blk[1 + i];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t byte = (two >> (8 * h)) & 0xFFu;
        lo[2 * i + h] = __float2half_rn((float)((int)(byte & 0xFu) - 8) * df);
        hi[2 * i + h] = __float2half_rn((float)((int)(byte >> 4) - 8) * df);
      }
    }
    __half* o = out + b * 32;
#pragma unroll
    for (int i = 0; i < 16; ++i) { o[i] = lo[i]; o[16 + i] = hi[i]; }
  }
}

// Q4_K block_q4_K rows: one thread per 64-value chunk of a super-block.
// w32 = fp32(d)*sc * q - fp32(dmin)*m (one fp32 rounding), out = fp16_rn(w32).
__global__ void dequant_q4k_kernel(const uint8_t* __restrict__ blocks, __half* __restrict__ out,
                                   long long nchunks) {
  for (long long c = blockIdx.x * (long long)blockDim.x + threadIdx.x; c < nchunks;
       c += (long long)gridDim.x * blockDim.x) {
    const long long sb = c >> 2;
    const int cc = (int)(c & 3);
    const uint8_t* blk = blocks + sb * kQ4KBlockBytes;
    const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
    const float d = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xFFFFu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr.x >> 16)));
    const uint32_t sc_lo = hdr.y & 0x3F3F3F3Fu;
    const uint32_t m_lo = hdr.z & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
    const uint32_t m_hi = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
    const uint32_t scw = cc < 2 ? sc_lo : sc_hi;
    const uint32_t mw = cc < 2 ? m_lo : m_hi;
    const int sh = 16 * (cc & 1);
    const float d1a = d * (float)((scw >> sh) & 0xFFu);
    const float m1a = dmin * (float)((mw >> sh) & 0xFFu);
    const float d1b = d * (float)((scw >> (sh + 8)) & 0xFFu);
    const float m1b = dmin * (float)((mw >> (sh + 8)) & 0xFFu);
    const uint4 q0 = *reinterpret_cast<const uint4*>(blk + 16 + cc * 32);
    const uint4 q1 = *reinterpret_cast<const uint4*>(blk + 16 + cc * 32 + 16);
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    __half* o = out + sb * 256 + cc * 64;
    uint32_t lo[16], hi[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t b0 = (w[i] >> (16 * h)) & 0xFFu;
        const uint32_t b1 = (w[i] >> (16 * h + 8)) & 0xFFu;
        const __half l0 = __float2half_rn(fmaf(d1a, (float)(b0 & 0xFu), -m1a));
        const __half l1 = __float2half_rn(fmaf(d1a, (float)(b1 & 0xFu), -m1a));
        const __half h0 = __float2half_rn(fmaf(d1b, (float)(b0 >> 4), -m1b));
        const __half h1 = __float2half_rn(fmaf(d1b, (float)(b1 >> 4), -m1b));
        lo[2 * i + h] = h2_as_u32(__halves2half2(l0, l1));
        hi[2 * i + h] = h2_as_u32(__halves2half2(h0, h1));
      }
    }
    uint4* o4 = reinterpret_cast<uint4*>(o);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      o4[i] = make_uint4(lo[4 * i], lo[4 * i + 1], lo[4 * i + 2], lo[4 * i + 3]);
      o4[4 + i] = make_uint4(hi[4 * i], hi[4 * i + 1], hi[4 * i + 2], hi[4 * i + 3]);
    }
  }
}

// ---------------------------------------------------------------------------
// tcgen05 layout probe (the sm_100a counterpart of kernels/frag_probe.cu):
// D[128, NB] = A[128, 64] * B[NB, 64]^T with A written to TMEM by tcgen05.st
// (row r -> lane r, column c -> k = 2c, 2c+1) and B stored in shared memory
// in the K-major 128-byte-swizzled layout, then four K=16 MMAs exactly as the
// GEMM issues them. A wrong layout assumption shows up as wrong numbers.
// ---------------------------------------------------------------------------
template <int NB>
__global__ void __launch_bounds__(128, 1)
    umma_probe_kernel(const __half* __restrict__ a, const __half* __restrict__ b, float* __restrict__ d,
                      unsigned* __restrict__ error) {
  __shared__ __align__(1024) uint8_t bs[NB * 128];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_slot;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr uint32_t kIdesc = make_idesc_f16_f32(128, NB);
  if (tid == 0) {
    mbar_init(smem_u32(&bar), 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&tmem_slot), 128);
    tmem_relinquish();
  }
  // B -> smem, SW128: 16-B chunk j of row n at (n/8)*1024 + (n%8)*128 + ((j ^ n%8) * 16)
  for (int e = tid; e < NB * 8; e += 128) {
    const int n = e >> 3, j = e & 7;
    const uint4 v = *reinterpret_cast<const uint4*>(b + n * 64 + j * 8);
    *reinterpret_cast<uint4*>(bs + (n >> 3) * 1024 + (n & 7) * 128 + ((j ^ (n & 7)) << 4)) = v;
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  {
    uint32_t r[32];
    const uint32_t* src = reinterpret_cast<const uint32_t*>(a + tid * 64);
#pragma unroll
    for (int c = 0; c < 32; ++c) r[c] = src[c];
    tmem_st_x32(tmem + lane_off + 64, r);  // operand at columns 64..95
    tc_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  if (tid == 0) {
    tc_fence_after();
#pragma unroll
    for (int t = 0; t < 4; ++t)
      mma_f16_ts(tmem, tmem + 64 + 8 * t, make_sdesc_sw128(smem_u32(bs) + 32 * t), kIdesc, t > 0 ? 1u : 0u);
    tc_commit(smem_u32(&bar));
  }
  __syncwarp();
  const bool got = mbar_wait(smem_u32(&bar), 0);
  if (!got && lane == 0) atomicOr(error, kErrMma);
  tc_fence_after();
  if (__all_sync(0xffffffffu, got)) {
    uint32_t r[NB];
    tmem_ld_cols<(NB < 32 ? NB : 32)>(tmem + lane_off, r);
    if constexpr (NB > 32) tmem_ld_cols<32>(tmem + lane_off + 32, r + 32);
    tc_wait_ld();
#pragma unroll
    for (int n = 0; n < NB; ++n) d[tid * NB + n] = __uint_as_float(r[n]);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// block_q5_K rows: one thread per 64-value chunk (sub-blocks 2cc, 2cc+1);
// fp16_rn(fp32(d)*sc*q - fp32(dmin)*m) with q = nibble | (qh bit << 4), the
// gguf-py 0.19.0 Q5_K dequant rounded once to fp16 (products exact in fp32).
__global__ void dequant_q5k_kernel(const uint8_t* __restrict__ blocks, __half* __restrict__ out,
                                   long long nchunks) {
  for (long long c = blockIdx.x * (long long)blockDim.x + threadIdx.x; c < nchunks;
       c += (long long)gridDim.x * blockDim.x) {
    const long long sb = c >> 2;
    const int cc = (int)(c & 3);
    const uint8_t* blk = blocks + sb * kQ5KBlockBytes;
    const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
    const float d = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xFFFFu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr.x >> 16)));
    const uint32_t sc_lo = hdr.y & 0x3F3F3F3Fu;
    const uint32_t m_lo = hdr.z & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
    const uint32_t m_hi = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
    const uint32_t scw = cc < 2 ? sc_lo : sc_hi;
    const uint32_t mw = cc < 2 ? m_lo : m_hi;
    const int sh = 16 * (cc & 1);
    const float d1a = d * (float)((scw >> sh) & 0xFFu);
    const float m1a = dmin * (float)((mw >> sh) & 0xFFu);
    const float d1b = d * (float)((scw >> (sh + 8)) & 0xFFu);
    const float m1b = dmin * (float)((mw >> (sh + 8)) & 0xFFu);
    const uint8_t* qh = blk + 16;
    const uint8_t* qs = blk + 48 + cc * 32;
    __half* o = out + sb * 256 + cc * 64;
    for (int l = 0; l < 32; ++l) {
      const uint32_t b = qs[l], h = qh[l];
      const float qa = (float)((b & 0xFu) | (((h >> (2 * cc)) & 1u) << 4));
      const float qb = (float)((b >> 4) | (((h >> (2 * cc + 1)) & 1u) << 4));
      o[l] = __float2half_rn(fmaf(d1a, qa, -m1a));
      o[32 + l] = __float2half_rn(fmaf(d1b, qb, -m1b));
    }
  }
}

// block_q6_K rows [N][S x 210 B] -> the GEMM's Q6_K layout: block bodies
// (ql, qh, scales: the first 208 bytes of each block) [N][S x 208 B] and the
// blocks' fp16 d as a plane [S][N]. One thread per 2-byte word of the source
// (210-byte blocks are 2-byte aligned), so loads and stores are coalesced.
__global__ void repack_q6k_kernel(const uint16_t* __restrict__ src, uint16_t* __restrict__ body,
                                  uint16_t* __restrict__ dplane, int n, int s) {
  constexpr int kWords = kQ6KBodyBytes / 2 + 1;  // 105 words per block, d last
  const long long row_words = (long long)s * kWords;
  const long long total = (long long)n * row_words;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / row_words;
    const long long rem = i - row * row_words;
    const int b = (int)(rem / kWords);
    const int w = (int)(rem - (long long)b * kWords);
    const uint16_t v = src[i];
    if (w < kWords - 1)
      body[(row * s + b) * (kWords - 1) + w] = v;
    else
      dplane[(long long)b * n + row] = v;
  }
}

// Q6_K (repacked) -> fp16 [N, K]: one thread per 64-value chunk of a block;
// fp16_rn((fp32(d) * sc) * (q - 32)), the gguf-py 0.19.0 Q6_K dequant rounded
// once to fp16 (d * sc is exact in fp32; the second product rounds once).
__global__ void dequant_q6k_kernel(const uint8_t* __restrict__ body, const __half* __restrict__ dplane,
                                   __half* __restrict__ out, int n, int s) {
  const long long nchunks = (long long)n * s * 4;
  for (long long c = blockIdx.x * (long long)blockDim.x + threadIdx.x; c < nchunks;
       c += (long long)gridDim.x * blockDim.x) {
    const long long blk_i = c >> 2;        // row * s + block
    const int cc = (int)(c & 3);
    const long long row = blk_i / s;
    const int b = (int)(blk_i - row * s);
    const uint8_t* blk = body + blk_i * kQ6KBodyBytes;
    const float d = __half2float(dplane[(long long)b * n + row]);
    const int h = cc >> 1, odd = cc & 1;
    __half* o = out + blk_i * 256 + cc * 64;
    for (int jj = 0; jj < 2; ++jj) {
      for (int l = 0; l < 32; ++l) {
        const int e = 64 * cc + 32 * jj + l;   // element within the block
        const uint32_t qlb = blk[64 * h + 32 * jj + l];
        const uint32_t qhb = blk[128 + 32 * h + l];
        const int q = (int)(((odd ? qlb >> 4 : qlb) & 0xFu) | (((qhb >> (4 * odd + 2 * jj)) & 3u) << 4));
        const float ds = d * (float)(int)(int8_t)blk[192 + e / 16];
        o[32 * jj + l] = __float2half_rn(ds * (float)(q - 32));
      }
    }
  }
}

// Q4_K planes -> llama.cpp block_q4_K rows: one thread per 16-byte word of
// an output block (9 per 144-byte block). Word 0 is the header (fp16 d,
// fp16 dmin, the 12 packed scale/min bytes), words 1..8 the block's 128
// nibble bytes. Planes: qs [N][S][128], d and dmin [N][S] fp16, scales
// [N][S][12]; the bytes are moved, never changed.
__global__ void repack_q4k_planar_kernel(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ d,
                                         const uint16_t* __restrict__ dmin, const uint8_t* __restrict__ sc12,
                                         uint8_t* __restrict__ blocks, long long nblocks) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nblocks * 9;
       i += (long long)gridDim.x * blockDim.x) {
    const long long b = i / 9;
    const int w = (int)(i - b * 9);
    uint4 v;
    if (w == 0) {
      const uint32_t* s4 = reinterpret_cast<const uint32_t*>(sc12 + b * 12);   // 4-byte aligned
      v.x = (uint32_t)d[b] | ((uint32_t)dmin[b] << 16);
      v.y = s4[0];
      v.z = s4[1];
      v.w = s4[2];
    } else {
      v = reinterpret_cast<const uint4*>(qs + b * 128)[w - 1];
    }
    reinterpret_cast<uint4*>(blocks + b * 144)[w] = v;
  }
}

}  // namespace busfill
