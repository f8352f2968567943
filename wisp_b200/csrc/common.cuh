// common.cuh -- device helpers shared by the wisp_b200 kernels (sm_100a only).
//
// Inline-PTX wrappers for the Blackwell pieces the kernels use: mbarriers,
// TMA tensor loads (no TMA or bulk load with cluster multicast anywhere in
// this library; only tcgen05.commit signals both CTAs of a pair), tcgen05
// tensor-memory allocation / load / store / MMA / commit, cp.async, plus the
// int4 -> fp16 conversion used by every int4 kernel.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define WB_DEV __device__ __forceinline__

namespace wb {

// Programmatic dependent launch (router -> decode planner): a kernel
// launched with launch_k_pdl waits here before its first read of anything
// the kernels before it write; pdl_trigger lets the next kernel's CTAs start
// (both are no-ops for kernels launched in plain stream order).
WB_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
WB_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// int4 nibble -> fp16 conversion.
//
// Packed format (reference: wisp/converter/quantizer.py:1-17): two nibbles
// per byte, the low nibble holds the even flattened index; value =
// (nibble - 8) * scale + zero. A 32-bit word therefore holds K offsets
// 8w+0 .. 8w+7 at bit positions 0,4,...,28.
//
// OR-ing a nibble into the mantissa of fp16 1024.0 (0x6400) gives 1024 + n
// exactly (the ulp of 1024 is 1). Masking the word with 0x000F000F yields
// nibbles 0 and 4 in the two halves; 0x00F000F0 yields nibbles 1 and 5
// pre-multiplied by 16 (1024 + 16n, still exact). Shifting the word right
// by 8 exposes nibbles 2,6 and 3,7 the same way. The four half2 values are
// therefore the K pairs (0,4) (1,5) (2,6) (3,7) -- the "interleaved" K
// order that every fp16 activation operand in this library is stored in
// (within each group of 8 K: 0,4,1,5,2,6,3,7).
// ---------------------------------------------------------------------------
WB_DEV uint32_t lop_or_and(uint32_t a, uint32_t mask, uint32_t orv) {
  uint32_t r;
  // (a & mask) | orv in one LOP3 (immediate LUT 0xEA = (a & b) | c).
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));
  return r;
}

WB_DEV __half2 u2h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
WB_DEV uint32_t h22u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Exact (n - 8) for the eight nibbles of `q`, as four half2 in interleaved
// K order: out[0] = (k0,k4), out[1] = (k1,k5), out[2] = (k2,k6), out[3] = (k3,k7).
WB_DEV void nib8_centered(uint32_t q, __half2 out[4]) {
  const uint32_t MAGIC = 0x64006400u;
  uint32_t q8 = q >> 8;
  __half2 h0 = u2h2(lop_or_and(q, 0x000F000Fu, MAGIC));
  __half2 h1 = u2h2(lop_or_and(q, 0x00F000F0u, MAGIC));
  __half2 h2 = u2h2(lop_or_and(q8, 0x000F000Fu, MAGIC));
  __half2 h3 = u2h2(lop_or_and(q8, 0x00F000F0u, MAGIC));
  // fp16 bit patterns, so the constants are immediates rather than
  // conversions: -1032 = 0xE408, 1/16 = 0x2C00, -72 = 0xD480.
  const __half2 c1032 = u2h2(0xE408E408u);
  const __half2 inv16 = u2h2(0x2C002C00u);
  const __half2 c72 = u2h2(0xD480D480u);
  out[0] = __hadd2(h0, c1032);          // (1024+n) - 1032
  out[1] = __hfma2(h1, inv16, c72);     // (1024+16n)/16 - 72
  out[2] = __hadd2(h2, c1032);
  out[3] = __hfma2(h3, inv16, c72);
}

// (n - 8) * s + z for the eight nibbles of q, one rounding per value.
WB_DEV void nib8_dequant(uint32_t q, __half2 s2, __half2 z2, uint32_t out[4]) {
  __half2 c[4];
  nib8_centered(q, c);
#pragma unroll
  for (int j = 0; j < 4; j++) out[j] = h22u(__hfma2(c[j], s2, z2));
}

// Interleaved position of K offset k within its group of 8, and back.
// Logical slot j holds physical offset kPhys[j] = {0,4,1,5,2,6,3,7}[j].
WB_DEV int k_interleave_slot(int k) {  // physical k -> logical slot
  const int r = k & 7;
  return (k & ~7) | ((r & 3) << 1) | (r >> 2);
}

// ---------------------------------------------------------------------------
// Shared-memory addresses, mbarriers (bounded waits), fences.
// ---------------------------------------------------------------------------
WB_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

WB_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

WB_DEV void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

WB_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}"
               ::"r"(smem_u32(bar)) : "memory");
}

WB_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
      ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// try_wait with a suspend-time hint: the warp may sleep (without taking
// issue slots) until the phase completes or ~20 us pass.
WB_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(20000u) : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete. Gives up after
// `limit_cycles` SM clocks: sets *abort and returns false, so a lost
// arrival turns into an error status instead of a hung GPU.
WB_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                      long long limit_cycles = 4000000000LL) {
  if (mbar_try_wait(bar, parity)) return true;
  long long t0 = clock64();
  for (int it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63) == 63) {
      if (*abort) return false;
      if (clock64() - t0 > limit_cycles) {
        *abort = 1;
        return false;
      }
    }
  }
}

// The same wait with cluster-scope acquire: for barriers that threads of the
// other CTA of a cluster arrive on.
WB_DEV bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(20000u) : "memory");
  return ok != 0;
}

WB_DEV bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort,
                              long long limit_cycles = 4000000000LL) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  long long t0 = clock64();
  for (int it = 0;; ++it) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((it & 63) == 63) {
      if (*abort) return false;
      if (clock64() - t0 > limit_cycles) {
        *abort = 1;
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Thread-block clusters.
// ---------------------------------------------------------------------------
WB_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the same shared-memory location in CTA `rank`.
WB_DEV uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

// Arrive on an mbarrier of another CTA of this cluster (the default
// semantics of the instruction; what the waiting side reads is tensor memory
// and shared memory that the tcgen05 and TMA fences already order).
WB_DEV void mbar_arrive_remote(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

// All threads of every CTA of the cluster.
WB_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}

// ---------------------------------------------------------------------------
// TMA (tensor map loads into shared memory, completion on an mbarrier).
// ---------------------------------------------------------------------------
WB_DEV void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

WB_DEV void tma_load_2d(void* smem_dst, const CUtensorMap* m, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)),
        "r"(x), "r"(y)
      : "memory");
}

WB_DEV void tma_load_3d(void* smem_dst, const CUtensorMap* m, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)),
        "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Untiled bulk copy global -> shared (no multicast), completion on an
// mbarrier. Both addresses 16-byte aligned, size a multiple of 16.
WB_DEV void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(smem_dst)), "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// cp.async (per-thread async copies into shared memory).
// ---------------------------------------------------------------------------
WB_DEV void cp_async_16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc)
               : "memory");
}
WB_DEV void cp_async_4(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gsrc)
               : "memory");
}
WB_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
WB_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
WB_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ---------------------------------------------------------------------------
// tcgen05: tensor memory and the 5th-generation MMA.
// TMEM address = (lane << 16) | column. A warp may touch only the 32 lanes
// of its sub-partition: lanes 32*(warp_id % 4) .. +31.
// ---------------------------------------------------------------------------
WB_DEV void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               ::"r"(smem_u32(smem_result)), "r"(ncols) : "memory");
}
WB_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
WB_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// The same for a CTA pair (cta_group::2): issued by the same warp of both
// CTAs, which get the same columns.
WB_DEV void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
               ::"r"(smem_u32(smem_result)), "r"(ncols) : "memory");
}
WB_DEV void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
WB_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
WB_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
WB_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
WB_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
WB_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Store 32 consecutive 32-bit columns of this thread's lane.
WB_DEV void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {"
      "%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]),
        "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]),
        "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]),
        "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]),
        "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// Store 16 consecutive 32-bit columns of this thread's lane.
WB_DEV void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {"
      "%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]),
        "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]),
        "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

// Load 16 consecutive 32-bit columns of this thread's lane.
WB_DEV void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {"
      "%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
        "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16 (fp16 inputs, fp32 accumulate),
// cta_group::1. A: M=128 lanes x 16 K (8 columns), K-major.
WB_DEV void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same, with the accumulate flag a compile-time constant.
template <int ACC>
WB_DEV void mma_f16_ts_c(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "n"(ACC)
      : "memory");
}

// Pair MMA (cta_group::2, issued by the even CTA of the pair): D[tmem] (+)=
// A[tmem] * B[smem]^T with M = 256, rows 0-127 in the even CTA's tensor
// memory and 128-255 in the odd one's (A and D at the same addresses in
// both); B's N rows are split in halves, the first in the even CTA's shared
// memory at the descriptor's address, the second at the same address in the
// odd CTA.
template <int ACC>
WB_DEV void mma_f16_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "n"(ACC)
      : "memory");
}

// Arrive on the mbarrier at this shared-memory offset in both CTAs of the
// pair once all pair MMAs issued by this thread have completed.
WB_DEV void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)), "h"((uint16_t)3) : "memory");
}

// Instruction descriptor for a pair MMA: as below with M = 256.
WB_DEV uint32_t idesc_f16_m256(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}

// Arrive on an mbarrier once all tcgen05.mma previously issued by this
// thread have completed.
WB_DEV void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
      ::"r"(smem_u32(bar)) : "memory");
}

// Instruction descriptor for kind::f16: fp16 A and B, fp32 D, both K-major,
// M = 128, N = n (multiple of 16, 16..256).
WB_DEV uint32_t idesc_f16_m128(int n) {
  return (1u << 4)                              // D format: f32
         | (0u << 7) | (0u << 10)               // A, B format: f16
         | (0u << 15) | (0u << 16)              // A, B K-major
         | ((uint32_t)(n >> 3) << 17)           // N >> 3
         | ((uint32_t)(128 >> 4) << 24);        // M >> 4
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, rows of 128 B,
// 8-row core groups 1024 B apart (SBO). Start address in 16-byte units.
WB_DEV uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);      // start address
  d |= (uint64_t)1u << 16;                      // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;            // SBO
  d |= (uint64_t)1u << 46;                      // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;                      // layout: SWIZZLE_128B
  return d;
}

WB_DEV float silu(float g) { return g / (1.0f + __expf(-g)); }

WB_DEV void red_add_f32(float* addr, float v) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(addr), "f"(v) : "memory");
}

WB_DEV bool elect_one() { return (threadIdx.x & 31) == 0; }

}  // namespace wb
