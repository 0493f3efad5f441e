// af2_device.cuh -- sm_100a building blocks shared by every kernel of
// libaf2cuda: mbarriers with bounded waits, TMA tile loads, and the tcgen05
// (TMEM allocation, MMA issue, commit, TMEM loads) instructions, written as
// inline PTX.
//
// Every wait is bounded: a wait that sees no progress for kWaitLimitNs (by
// %globaltimer) or that sees another role of the CTA give up, records a
// code in the context's error word, raises the CTA's abort flag and returns
// false.  Callers then leave their loops, drain what they have in flight
// (again with bounded waits) and free TMEM, so a kernel never spins forever.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace af2 {

// Error word bits (the host reads them in af2_sync).
constexpr unsigned int kErrWaitProducer = 1u << 0;
constexpr unsigned int kErrWaitMma = 1u << 1;
constexpr unsigned int kErrWaitEpilogue = 1u << 2;
constexpr unsigned int kErrWaitNormalizer = 1u << 3;
constexpr unsigned int kErrWaitDrain = 1u << 4;

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s without progress

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier -------------------------------------------------------------

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

__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes or `hint_ns` passes, instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_test_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return done != 0;
}

constexpr uint32_t kSleepHintNs = 200000;  // 0.2 ms per try; the overall bound is kWaitLimitNs

// Waits until the phase of parity `parity` of `bar` has completed.  Returns
// false (and sets the abort flag and the error word) when the wait runs out
// or another role has aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                       unsigned int *err, unsigned int code) {
  if (mbar_test(bar, parity)) return true;
  const unsigned long long start = globaltimer();
  for (uint32_t tries = 0; tries < 0x7fffffffu; ++tries) {
    if (mbar_test_sleep(bar, parity, kSleepHintNs)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - start > kWaitLimitNs) break;
  }
  *abort_flag = 1;
  atomicOr(err, code);
  return false;
}

// Drain-time wait: bounded, never raises the abort flag (it is already up).
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity, unsigned int *err) {
  const unsigned long long start = globaltimer();
  for (uint32_t tries = 0; tries < 0x7fffffffu; ++tries) {
    if (mbar_test_sleep(bar, parity, kSleepHintNs)) return true;
    if (globaltimer() - start > kWaitLimitNs) break;
  }
  atomicOr(err, kErrWaitDrain);
  return false;
}

// 4-byte asynchronous copy global -> shared (zero-filled when `valid` is false;
// the source is then not read), and the arrive-on of `bar` that fires once all
// of this thread's earlier such copies have landed (counted against the
// barrier's expected arrivals).
__device__ __forceinline__ void cp_async_4(uint32_t dst, const void *src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(valid ? 4 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ---- proxy fences / named barriers -----------------------------------------

// Makes this thread's generic-proxy shared-memory writes visible to the async
// proxy (TMA, tensor cores).
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---- TMA -------------------------------------------------------------------

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 3-D tiled load into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// 4-D tiled load into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// 4-D tiled store from this CTA's shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_4d(const CUtensorMap *map, uint32_t src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

// 3-D tiled store from this CTA's shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, uint32_t src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}

// 3-D tiled element-wise add of shared memory into global memory (done in L2).
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap *map, uint32_t src, int c0, int c1, int c2) {
  asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until every committed bulk store has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Every committed bulk group but the most recent one has finished reading its shared memory.
__device__ __forceinline__ void bulk_wait_read_but_one() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
// Waits until every committed bulk store has completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ---- tcgen05 ---------------------------------------------------------------

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

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---- warp-wide MMA issue ----------------------------------------------------
// The whole issuing warp runs the MMA loop with warp-uniform control flow and
// operands, and one lane elected inside each instruction issues it.  With the
// loop in a single lane (a divergent branch) the descriptors cannot live in
// uniform registers and every MMA pays for moving them there: measured on B200,
// M=128 MMAs issue at 100-180 clk each that way, against 48 / 64 / 128 clk (the
// tensor core's own rate at N = 64 / 128 / 256) from a uniform warp.

// This thread's warp index, provably warp-uniform to the compiler.
__device__ __forceinline__ int warp_index_uniform() { return __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0); }

// D[tmem] (+)= A[smem] B[smem]^T from one elected lane of a converged warp.
__device__ __forceinline__ void umma_first(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, 0;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc)
      : "memory");
}
__device__ __forceinline__ void umma_acc(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, 1;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc)
      : "memory");
}
// The same with A in TMEM (128 lanes x 16 f16, packed pairs, K-major).
__device__ __forceinline__ void umma_ts_first(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, 0;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc)
      : "memory");
}
__device__ __forceinline__ void umma_ts_acc(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, 1;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc)
      : "memory");
}
// tcgen05.commit from one elected lane: one arrival on `bar` when every MMA this warp issued has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\t"
      "@p tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar)
      : "memory");
}

// ---- CTA pairs (tcgen05 cta_group::2) -----------------------------------------
// A cluster of two CTAs computes one M = 256 tile: each CTA holds its 128 rows
// of A and half of the rows of B in shared memory at the same offsets, the
// even CTA (the leader) issues the MMAs, and each CTA's TMEM receives its own
// 128 rows of D.  The shared::cta address of a cluster CTA carries its rank in
// bit 24, so clearing that bit names the same offset in the leader.

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of both CTAs.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t leader_addr(uint32_t smem_addr) { return smem_addr & 0xFEFFFFFFu; }
// One arrival on the leader's barrier at this barrier's offset (the leader itself included).
__device__ __forceinline__ void mbar_arrive_leader(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(leader_addr(bar)) : "memory");
}
// 4-D tiled load into this CTA's shared memory, completing on the leader's barrier.
__device__ __forceinline__ void tma_load_4d_pair(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c0, int c1,
                                                 int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_addr(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
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
// D[tmem] (+)= A B^T over the CTA pair, from one elected lane of the leader's issuing warp.
__device__ __forceinline__ void umma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, a;\n\tsetp.ne.u32 a, %4, 0;\n\telect.sync _|p, 0xffffffff;\n\t"
      "@p tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, a;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// One arrival on `bar` in both CTAs once the pair's MMAs issued so far have completed.
__device__ __forceinline__ void umma_commit_pair_both(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\t"
      "@p tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}" ::"r"(
          bar),
      "h"((uint16_t)0x3)
      : "memory");
}
// One arrival on this CTA's `bar` once the pair's MMAs issued so far have completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\t"
      "@p tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar)
      : "memory");
}

// A shared-memory descriptor moved by `bytes` (a multiple of 16): the start
// address field is address >> 4 in the low 14 bits, and every shared address
// is below 2^18, so the add never carries out of the field.
__host__ __device__ constexpr uint64_t desc_add(uint64_t desc, uint32_t bytes) { return desc + (bytes >> 4); }


// 32 lanes x 32 consecutive 32-bit columns; thread t of the warp gets lane
// (base lane + t), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
      " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// 32 lanes x 8 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

// 16 lanes x 64 consecutive 32-bit columns in the 16x256b shape, repeated 8 times along the
// columns: thread t gets, for k = 0..7, r[4k], r[4k + 1] = lane (base + t / 4), columns
// 8k + 2 (t % 4) and + 1, and r[4k + 2], r[4k + 3] = the same columns of lane (base + 8 + t / 4).
__device__ __forceinline__ void tmem_ld_16x256b_x8(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x8.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
      " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// The 16x256b shape once (8 columns): r[0], r[1] = lane (base + t / 4), columns 2 (t % 4) and
// + 1; r[2], r[3] = the same columns of lane (base + 8 + t / 4).
__device__ __forceinline__ void tmem_ld_16x256b_x1(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x1.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}

// 16 lanes x 32 consecutive 32-bit columns stored in the 16x128b shape, repeated 8 times:
// thread t writes, for k = 0..7, r[2k] to lane (base + t / 4), column 4k + t % 4, and r[2k + 1]
// to lane (base + 8 + t / 4), the same column.
__device__ __forceinline__ void tmem_st_16x128b_x8(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x128b.x8.b32 [%0],"
      " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns stored: thread t writes lane (base lane + t).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0],"
      " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16,"
      " %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns stored.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t *r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0],"
      " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand tile in the 128-byte
// swizzled layout: rows of 64 16-bit elements (128 B), groups of 8 rows 1024 B
// apart.  The tile base must be 1024-byte aligned; stepping K by 16 elements
// inside the 128-byte row adds 32 bytes to the start address.
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);  // start address
  d |= static_cast<uint64_t>(1) << 16;                   // leading byte offset (unused when swizzled)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;           // stride byte offset: 8 rows
  d |= static_cast<uint64_t>(1) << 46;                   // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                   // SWIZZLE_128B
  return d;
}

// The same for the 64-byte swizzled layout: rows of 32 16-bit elements (64 B),
// groups of 8 rows 512 B apart; the tile base must be 512-byte aligned.
__device__ __forceinline__ uint64_t sdesc_k_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);  // start address
  d |= static_cast<uint64_t>(1) << 16;                   // leading byte offset (unused when swizzled)
  d |= static_cast<uint64_t>(512 >> 4) << 32;            // stride byte offset: 8 rows
  d |= static_cast<uint64_t>(1) << 46;                   // descriptor version (sm_100)
  d |= static_cast<uint64_t>(4) << 61;                   // SWIZZLE_64B
  return d;
}

// Shared-memory matrix descriptor for an MN-major operand tile in the 128-byte
// swizzled layout: K-rows of 64 16-bit MN-elements (128 B), 8 K-rows per
// 1024-byte atom.  `lbo` is the byte distance between consecutive 64-element
// MN blocks, `sbo` between consecutive groups of 8 K-rows.  Stepping K by 16
// adds 2 * sbo to the start address.
__device__ __forceinline__ uint64_t sdesc_mn_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor, kind::f16: f16 A and B, f32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n) {
  return (1u << 4)                                   // D format f32
         | (0u << 7) | (0u << 10)                    // A, B format f16
         | (static_cast<uint32_t>(n >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);    // M / 16
}

// The same with A MN-major (transpose-A bit).
__host__ __device__ constexpr uint32_t idesc_f16_f32_amn(int m, int n) { return idesc_f16_f32(m, n) | (1u << 15); }

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` in a 128B-swizzled tile.
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

// ---- warp-level helpers ------------------------------------------------------

constexpr unsigned kFull = 0xffffffffu;

// Rounds the dynamic shared-memory base up to 1024 bytes (the 128-byte
// swizzle atom).  The offset is added to the __shared__ pointer itself so the
// compiler still knows every access through it is a shared-memory access
// (LDS/STS); rounding through an integer would turn them into generic loads.
__device__ __forceinline__ uint8_t *align1024(uint8_t *p) {
  const uint32_t a = smem_u32(p);
  return p + (((a + 1023u) & ~1023u) - a);
}

__device__ __forceinline__ float reduce16(float v) {
  v += __shfl_xor_sync(kFull, v, 8);
  v += __shfl_xor_sync(kFull, v, 4);
  v += __shfl_xor_sync(kFull, v, 2);
  v += __shfl_xor_sync(kFull, v, 1);
  return v;
}

// Warp-uniform bounded wait: every lane waits, and the warp proceeds only if
// every lane saw the phase complete.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                          unsigned int *err, unsigned int code) {
  const bool ok = mbar_wait(bar, parity, abort_flag, err, code);
  return __all_sync(kFull, ok);
}


// ---- small conversions -------------------------------------------------------

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ float from_f32<float>(float v) {
  return v;
}

// Eight 16-bit values packed in a uint4 -> f32.
template <typename T>
__device__ __forceinline__ void unpack8(const uint4 &v, float (&x)[8]) {
  const T *e = reinterpret_cast<const T *>(&v);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = to_f32<T>(e[i]);
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&h);
}

// Logistic function from the hardware base-2 exponential and reciprocal
// (ex2.approx and rcp.approx, both within 2 ulp of f32): 1 / (1 + 2^(-v log2 e)).
// Saturates cleanly: a large negative v gives 1/inf = 0, a large positive one 1/1.
__device__ __forceinline__ float sigmoidf(float v) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(v * -1.4426950408889634f));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
  return r;
}

// Logistic function from one hardware tanh: sigmoid(v) = 0.5 + 0.5 tanh(v / 2).
// tanh.approx has a relative error below 2^-10.98, so the result is within
// about 2.5e-4 absolute -- used where the multi-function unit, not memory,
// would otherwise bound the kernel (the gated projections).
__device__ __forceinline__ float tanhf_approx(float v) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(v));
  return t;
}

// Packed f32x2 arithmetic (two lanes of f32 per instruction on sm_100).
__device__ __forceinline__ float2 f2fma(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 f2add(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 f2mul(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

// Two 16-bit values of a 32-bit word -> f32 (low half first).
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t w);
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2 *>(&w));
}
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// Two f32 values rounded to a packed pair of 16-bit outputs (low half first).
template <typename OT>
__device__ __forceinline__ uint32_t pack2_t(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2_t<__half>(float lo, float hi) {
  return pack_half2(lo, hi);
}
template <>
__device__ __forceinline__ uint32_t pack2_t<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}
// f32 outputs never take a packed 16-bit path; this only lets shared kernel
// code that branches on the output type compile for f32.
template <>
__device__ __forceinline__ uint32_t pack2_t<float>(float, float) {
  return 0;
}

// Writes y into columns [c0, c0 + 32) of an output row, or with `residual`
// adds y to what is there (in f32, rounded once).  Whole 32-column chunks of
// 16-byte aligned rows (`vector`) use 16-byte accesses; otherwise elements
// past `cols` are left alone.
template <typename OT>
__device__ __forceinline__ void store_out32(OT *orow, int c0, int cols, const float (&y)[32], bool vector,
                                            bool residual) {
  if (vector && c0 + 32 <= cols) {
    if constexpr (sizeof(OT) == 4) {
      float4 *o4 = reinterpret_cast<float4 *>(orow + c0);
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        float4 val = make_float4(y[4 * w], y[4 * w + 1], y[4 * w + 2], y[4 * w + 3]);
        if (residual) {
          const float4 r = o4[w];
          val.x += r.x;
          val.y += r.y;
          val.z += r.z;
          val.w += r.w;
        }
        o4[w] = val;
      }
    } else {
      uint4 *o4 = reinterpret_cast<uint4 *>(orow + c0);
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        float v8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v8[i] = y[8 * w + i];
        if (residual) {
          const uint4 r = o4[w];
          const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = unpack2<OT>(rw[i]);
            v8[2 * i] += f.x;
            v8[2 * i + 1] += f.y;
          }
        }
        o4[w] = make_uint4(pack2_t<OT>(v8[0], v8[1]), pack2_t<OT>(v8[2], v8[3]), pack2_t<OT>(v8[4], v8[5]),
                           pack2_t<OT>(v8[6], v8[7]));
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int col = c0 + i;
      if (col < cols) orow[col] = from_f32<OT>(residual ? to_f32<OT>(orow[col]) + y[i] : y[i]);
    }
  }
}

}  // namespace af2
