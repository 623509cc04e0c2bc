// Thin inline-PTX wrappers for the sm_100a features the kernels use:
// mbarriers (with bounded waits), TMA tensor loads, tcgen05 (TMEM alloc,
// MMA with A in TMEM, commit, ld/st, fences), programmatic dependent launch.
// Everything here is a single PTX instruction or a short bounded loop.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace busfill {

// ----------------------------------------------------------------------------
// misc
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// (a & b) | c
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// lo = fp16(a2.lo) * fp16(b) + c and hi = fp16(a2.hi) * fp16(b) + c in fp32,
// each with one rounding: the sm_100 mixed-precision fma.rn.f32.f16 forms
// the product of two fp16 values exactly (at most 22 significant bits).
__device__ __forceinline__ void fma_f16x2_f32(uint32_t a2, uint16_t b, float c, float& lo, float& hi) {
  asm("{\n\t.reg .b16 l, h;\n\t"
      "mov.b32 {l, h}, %2;\n\t"
      "fma.rn.f32.f16 %0, l, %3, %4;\n\t"
      "fma.rn.f32.f16 %1, h, %3, %4;\n\t}"
      : "=f"(lo), "=f"(hi)
      : "r"(a2), "h"(b), "f"(c));
}

// (a, b) *= s as one packed fp32 multiply (sm_100 mul.rn.f32x2).
__device__ __forceinline__ void mul_f32x2(float& a, float& b, float s) {
  asm("{\n\t.reg .b64 x, y;\n\t"
      "mov.b64 x, {%0, %1};\n\t"
      "mov.b64 y, {%2, %2};\n\t"
      "mul.rn.f32x2 x, x, y;\n\t"
      "mov.b64 {%0, %1}, x;\n\t}"
      : "+f"(a), "+f"(b)
      : "f"(s));
}

// One thread of the (converged) warp is elected; returns true in that thread.
// Issuing tcgen05.mma / TMA from a converged warp through elect.sync keeps the
// operands warp-uniform (measured on B200: ~21 cycles per N=32 MMA this way
// versus ~46 from a loop that only lane 0 executes).
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 %%rx;\n\t.reg .pred %%px;\n\t"
      "elect.sync %%rx|%%px, %1;\n\t"
      "@%%px mov.s32 %0, 1;\n\t}"
      : "+r"(pred)
      : "r"(0xffffffffu));
  return pred != 0;
}

// ----------------------------------------------------------------------------
// programmatic dependent launch
// ----------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait_prerequisites() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ----------------------------------------------------------------------------
// mbarrier
// ----------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// Suspend-time hint of the blocking tests below: a waiting thread may sleep
// up to this long (it wakes when the phase completes), instead of spinning
// and taking issue slots from the warps that do the work.
constexpr uint32_t kSuspendHintNs = 1000000;   // 1 ms

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

// Every wait in the kernels is bounded: after `timeout_ns` of wall time the
// wait gives up and returns false, the caller records an error code in global
// memory and winds down, so a logic error can never hang the GPU.
constexpr uint64_t kWaitTimeoutNs = 1000ull * 1000ull * 1000ull;  // 1 s

// non-blocking probe of a phase (cheaper than try_wait when already complete)
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) return false;
  }
}

// ----------------------------------------------------------------------------
// thread-block clusters and distributed shared memory
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the local shared::cta address `saddr` in CTA `rank`
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
  return d;
}
// arrive on an mbarrier of another CTA of the cluster; releases this thread's
// prior memory operations at cluster scope
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// arrive on an mbarrier of another CTA of the cluster without release
// semantics: for a signal whose payload was completed by a wait of its own
// (tcgen05.wait::st before a TMEM operand is handed over). A release arrival
// at cluster scope costs the arriving warp ~1000-1600 cycles on B200.
__device__ __forceinline__ void mbar_arrive_remote_relaxed(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// wait that acquires at cluster scope (pairs with mbar_arrive_remote)
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i) {
      uint32_t ok;
      asm volatile(
          "{\n\t.reg .pred p;\n\t"
          "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
          "selp.u32 %0, 1, 0, p;\n\t}"
          : "=r"(ok)
          : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
          : "memory");
      if (ok) return true;
    }
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) return false;
  }
}
// Asynchronous 16-byte store into another CTA's shared memory that counts its
// bytes against that CTA's mbarrier (complete_tx): the receiver's wait on the
// barrier phase makes the data visible, with no fence on the sender.
__device__ __forceinline__ void st_async_f4(uint32_t cluster_addr, float a, float b, float c, float d,
                                            uint32_t cluster_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   cluster_addr),
               "f"(a), "f"(b), "f"(c), "f"(d), "r"(cluster_bar)
               : "memory");
}
// Bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from
// this CTA's shared memory into another CTA's of the cluster (no multicast);
// the bytes complete that CTA's mbarrier (complete_tx), which is also the only
// completion: the source stays untouched until the receiver says it has read it.
__device__ __forceinline__ void bulk_copy_to_cluster(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes,
                                                     uint32_t bar_cluster) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst_cluster),
               "r"(src_cta), "r"(bytes), "r"(bar_cluster)
               : "memory");
}
// Make this thread's generic-proxy shared-memory writes visible to later
// asynchronous-proxy operations (bulk copies) of the CTA.
__device__ __forceinline__ void fence_proxy_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void st_shared_f4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}
// all threads of all CTAs of the cluster (converged warps)
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The two halves of cluster_sync_all, for a split barrier: every thread of the
// cluster arrives once and later waits once per phase (converged warps); the
// wait returns when every thread of the cluster has arrived.
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// ----------------------------------------------------------------------------
// flags between GPUs (peer memory mapped over NVLink)
// ----------------------------------------------------------------------------
// add to a (possibly peer) word without a result, relaxed at system scope; a
// fence_acq_rel_sys before it in the same thread makes the pair a release of
// this thread's prior writes (and those ordered before them)
__device__ __forceinline__ void red_relaxed_sys_add(unsigned* addr, unsigned v) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* addr) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}
// returns the old value; acquire and release at GPU scope
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* addr, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void st_relaxed_gpu(unsigned* addr, unsigned v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_gpu_add(unsigned* addr, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* addr) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}
// Wait (bounded, kWaitTimeoutNs) until *addr has reached `epoch` (wrap-safe);
// acquires at system scope. Returns false on timeout.
__device__ __forceinline__ bool wait_flag_sys(const unsigned* addr, unsigned epoch) {
  if ((int)(ld_acquire_sys(addr) - epoch) >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if ((int)(ld_acquire_sys(addr) - epoch) >= 0) return true;
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) return false;
  }
}
// order this thread's generic-proxy view of global memory before its later
// async-proxy (TMA) reads of it
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// CTA named barriers (ids 1..15; id 0 is __syncthreads): `count` threads, a
// multiple of 32, take part; arrive does not wait.
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(uint32_t id, uint32_t count) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ----------------------------------------------------------------------------
// TMA: plain tensor loads into this CTA's own shared memory only
// ----------------------------------------------------------------------------
constexpr uint64_t kPolicyEvictFirst = 0x12F0000000000000ull;
constexpr uint64_t kPolicyEvictLast = 0x14F0000000000000ull;

__device__ __forceinline__ void tma_prefetch_desc(const void* desc) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(desc)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* desc, int32_t x, int32_t y, uint32_t bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(bar), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* desc, int32_t x, int32_t y, int32_t z,
                                            uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(bar), "r"(x), "r"(y), "r"(z), "l"(policy)
      : "memory");
}

// Transposes, in each group of 8 lanes, the 8x8 blocks of the NB values the
// lanes hold: before, lane j of a group holds batch rows 0..NB-1 of weight
// row n0 + j; after, acc[8b + i] of lane j holds batch row 8b + j of weight
// row n0 + i. Three butterfly stages (lane distance 4, 2, 1); in each, the
// lanes of a pair swap the halves the other needs. All 32 lanes take part.
template <int NB>
__device__ __forceinline__ void transpose_8x8_blocks(float* acc, int lane) {
  const int j = lane & 7;
#pragma unroll
  for (int b = 0; b < NB / 8; ++b) {
    float* v = acc + 8 * b;
#pragma unroll
    for (int m = 4; m >= 1; m >>= 1) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (i & m) continue;
        const bool hi = (j & m) != 0;
        const float y = __shfl_xor_sync(0xffffffffu, hi ? v[i] : v[i | m], m);
        if (hi)
          v[i] = y;
        else
          v[i | m] = y;
      }
    }
  }
}

// ----------------------------------------------------------------------------
// tcgen05
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Arrive on `bar` once every tcgen05 operation this thread issued so far has
// completed (the MMAs reading a stage, or writing an accumulator).
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16 (fp16 inputs, fp32 accumulate).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// --- CTA pairs (cta_group::2): one MMA over both SMs of a 2-CTA cluster ---
// TMEM allocation of the same columns in both CTAs: a collective of one warp
// with the same warp index in each CTA of the pair, same destination offset.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D (+)= A * B^T over the pair, issued by the pair's rank-0 CTA: A [256 x 16]
// from TMEM (rows 0-127 in rank 0's lanes, 128-255 in rank 1's), B [N x 16]
// from shared memory at the same offset in both CTAs (rank 0 holds rows
// 0..N/2-1, rank 1 the rest), D [256 x N] fp32 split like A.
__device__ __forceinline__ void mma_f16_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the mbarrier at offset `bar` in each CTA of `cta_mask` once every
// tcgen05 operation this thread issued has completed (pair MMAs).
__device__ __forceinline__ void tc_commit_pair(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(cta_mask)
      : "memory");
}
// 3-D tensor copy into this CTA's shared memory whose completion is counted
// on an mbarrier of either CTA of the pair (`bar_cluster`, a shared::cluster
// address): both CTAs' halves of an operand complete on rank 0's barrier.
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const void* desc, int32_t x, int32_t y, int32_t z,
                                                 uint32_t bar_cluster, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z), "l"(policy)
      : "memory");
}

// Instruction descriptor for kind::f16: fp16 A/B, fp32 D, both K-major,
// M = m (128; 256 for a CTA pair), N = n (multiple of 16, 16..256).
__host__ __device__ constexpr uint32_t make_idesc_f16_f32(int m, int n) {
  return (1u << 4)                                 // D format: f32
         | (0u << 7) | (0u << 10)                  // A, B format: f16
         | (0u << 15) | (0u << 16)                 // A, B K-major
         | ((uint32_t)(n >> 3) << 17)              // N >> 3
         | ((uint32_t)(m >> 4) << 24);             // M >> 4
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows of 128 B
// (64 fp16), 8-row atoms of 1024 B stacked along M/N (SBO = 1024). The start
// address may step by 32 B inside an atom to select a K=16 slice.
__device__ __forceinline__ uint64_t make_sdesc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);     // start address >> 4, bits 0-13
  d |= (uint64_t)(16 >> 4) << 16;              // leading byte offset (unused for SW128 K-major)
  d |= (uint64_t)(1024 >> 4) << 32;            // stride byte offset = 1024
  d |= (uint64_t)1 << 46;                      // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                      // layout: SWIZZLE_128B
  return d;
}

// --- tcgen05.st / tcgen05.ld, 32 lanes x 32 bit, x8 / x16 / x32 columns ---
__device__ __forceinline__ void tmem_st_x8(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
// the same 32-bit value into 16 consecutive columns
__device__ __forceinline__ void tmem_st_x16_bcast(uint32_t taddr, uint32_t v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
      "r"(v)
      : "memory");
}
__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// Load `N` consecutive fp32 columns (N a multiple of 8, <= 32) of this warp's
// 32 lanes, 16 columns at a time.
template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t* r) {
  static_assert(N % 8 == 0 && N <= 32, "column count");
  if constexpr (N % 16 == 0) {
#pragma unroll
    for (int i = 0; i < N / 16; ++i) tmem_ld_x16(taddr + 16 * i, r + 16 * i);
  } else {
#pragma unroll
    for (int i = 0; i < N / 8; ++i) tmem_ld_x8(taddr + 8 * i, r + 8 * i);
  }
}

}  // namespace busfill
