// Thin inline-PTX wrappers for sm_100a: mbarriers with bounded waits, TMA tile loads, tcgen05 (TMEM
// allocation, MMA, commit, loads) and the shared-memory matrix descriptor of a K-major 128-byte-swizzled tile.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace dcx {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------------ mbarrier

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase of parity `parity` to complete. Gives up after `limit_ns` of wall time (globaltimer):
// sets *abort and ORs `code` into the device error word, and returns false. Nothing waits forever.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort, uint32_t *err,
                                          uint32_t code, uint64_t limit_ns = 2000000000ull) {
  if (mbar_try(bar, parity)) return true;
  uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; i++) {
    if (mbar_try(bar, parity)) return true;
    if ((i & 255) == 0) {
      if (*abort) return false;
      if (globaltimer() - t0 > limit_ns) {
        *abort = 1;
        atomicOr(err, code);
        return false;
      }
    }
  }
}

// ------------------------------------------------------------------ TMA

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// 4-byte global -> shared copy (cp.async); src_bytes 0 writes zeros without reading.
// TMA store of a 2D box from this CTA's shared memory (same swizzled layout a load of the box would write), in a
// bulk group; bulk_store_read_wait waits until the stores of the thread's groups have read their shared memory
// (the writes complete by themselves before the grid does, and are visible to the kernels after it).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, int x, int y, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(x),
               "r"(y), "r"(src)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_store_read_wait() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

__device__ __forceinline__ void cp_async_4(uint32_t dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
// 8-byte global -> shared copy (cp.async); src_bytes 0 writes zeros without reading.
__device__ __forceinline__ void cp_async_8(uint32_t dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
// One arrival on `bar` once this thread's earlier cp.async copies have landed (counted in the barrier's
// expected arrivals).
__device__ __forceinline__ void cp_async_mbar_arrive(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Makes this thread's generic-proxy shared-memory writes visible to the async proxy (TMA, tcgen05.mma).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------ tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] . B[smem desc]^T, f16 inputs, f32 accumulation (kind::f16, one CTA).
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// ------------------------------------------------------------------ CTA pair (tcgen05 cta_group::2)
// Two CTAs of a cluster share one MMA of M = 256: each holds 128 rows of A and half of B (N/2 rows) in its own
// shared memory at the same offsets, and its 128 rows of the f32 accumulator in its own tensor memory. One
// thread of the even CTA issues the MMAs. Every tcgen05 instruction of such a kernel uses cta_group::2.

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// One arrival on an mbarrier of another CTA of the cluster (shared::cluster address), with the default release
// semantics (this thread's earlier writes, e.g. shared memory already fenced for the async proxy).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
// One arrival on an mbarrier of another CTA of the cluster, with no ordering of this thread's memory operations
// (a pure signal, e.g. "I am done reading").
__device__ __forceinline__ void mbar_arrive_remote_relaxed(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
// try_wait with acquire at cluster scope: for barriers that other CTAs of the cluster arrive on.
__device__ __forceinline__ bool mbar_try_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, volatile int *abort, uint32_t *err,
                                                  uint32_t code, uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_cluster(bar, parity)) return true;
  uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; i++) {
    if (mbar_try_cluster(bar, parity)) return true;
    if ((i & 255) == 0) {
      if (*abort) return false;
      if (globaltimer() - t0 > limit_ns) {
        *abort = 1;
        atomicOr(err, code);
        return false;
      }
    }
  }
}
// TMA tile load into this CTA's shared memory whose completion is counted on the pair's mbarrier `bar_cluster`
// (which may be in the peer CTA).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap *map, int x, int y,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives once on `bar_cluster` (this CTA's or the peer's) when every pair MMA this thread issued has completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
               : "memory");
}

// Instruction descriptor of kind::f16 with f16 A and B (both K-major) and an f32 accumulator, M x N.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4)                          // D format: f32
         | (0u << 7) | (0u << 10)           // A, B format: f16
         | (0u << 15) | (0u << 16)          // A, B K-major
         | ((uint32_t)(N >> 3) << 17)       // N / 8
         | ((uint32_t)(M >> 4) << 24);      // M / 16
}

// Shared-memory descriptor of a K-major tile stored as the TMA writes it with 128-byte swizzling: rows of
// 64 f16 (128 bytes), 8-row atoms of 1024 bytes (stride byte offset), 16-byte chunk c of row r at c ^ (r % 8).
// The tile base must be 1024-byte aligned; a K offset inside the atom is added to the start address.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset
  d |= (uint64_t)1 << 46;             // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}

// 32 lanes x 32 consecutive 32-bit TMEM columns -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%"
      "19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 16 consecutive columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Waits for this thread's tcgen05.ld and ties the loaded registers to the wait: the compiler sees no dependency
// between a load's output registers and the wait, and could otherwise schedule a use of them before it.
template <int N>
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[N]) {
  tmem_ld_wait();
#pragma unroll
  for (int i = 0; i < N; i++) asm volatile("" : "+r"(r[i]));
}

// 32 lanes x 16 consecutive 32-bit TMEM columns <- 16 registers per thread (the thread's own lane).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[tmem] . B[smem desc]^T: the A operand (M = 128 rows, K-major) read from tensor memory, row m in
// lane m, two f16 per 32-bit column (the even k in the low half).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 2^x by the hardware approximation (PTX ex2.approx, relative error about 2^-22): the softmax weights it feeds
// are rounded to f16 right after, so the approximation is invisible in the result.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ------------------------------------------------------------------ dequantisation
// Exact f16 dequantisation without conversions: 0x6400 | b is the f16 1024 + b for a byte b < 256, so
// (1024 + b) - (1024 + Z) = b - Z exactly, and one f16 multiply by the scale rounds once: the result is
// f16((code - Z) * scale), bit for bit.

// Four q8 codes (one little-endian word) -> two half2 {c0, c1}, {c2, c3}.
__device__ __forceinline__ void deq_q8_word(uint32_t w, __half2 s2, __half2 &o01, __half2 &o23) {
  const uint32_t magic = 0x64646464u;
  uint32_t a, b;
  asm("prmt.b32 %0, %1, %2, 0x5150;" : "=r"(a) : "r"(w), "r"(magic));
  asm("prmt.b32 %0, %1, %2, 0x5352;" : "=r"(b) : "r"(w), "r"(magic));
  const __half2 z = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
  o01 = __hmul2(__hsub2(*reinterpret_cast<__half2 *>(&a), z), s2);
  o23 = __hmul2(__hsub2(*reinterpret_cast<__half2 *>(&b), z), s2);
}

// Eight q4 codes (one word, low nibble first) -> four half2 {c0,c1}, {c2,c3}, {c4,c5}, {c6,c7}.
__device__ __forceinline__ void deq_q4_word(uint32_t w, __half2 s2, __half2 (&o)[4]) {
  const uint32_t lo = w & 0x0F0F0F0Fu;         // c0 c2 c4 c6
  const uint32_t hi = (w >> 4) & 0x0F0F0F0Fu;  // c1 c3 c5 c7
  const __half2 z = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));  // 1032
#pragma unroll
  for (int j = 0; j < 4; j++) {
    // byte 0 <- lo.j, byte 2 <- hi.j; bytes 1 and 3 <- the sign of lo.j replicated, 0 (a nibble's top bit is clear);
    // then 0x64 into the high bytes: the halves 1024 + c
    const uint32_t sel = (uint32_t)j | ((8u | j) << 4) | ((4u + j) << 8) | ((8u | j) << 12);
    uint32_t p;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(p) : "r"(lo), "r"(hi), "r"(sel));
    p |= 0x64006400u;
    o[j] = __hmul2(__hsub2(*reinterpret_cast<__half2 *>(&p), z), s2);
  }
}

}  // namespace dcx
