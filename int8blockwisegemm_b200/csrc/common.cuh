// Shared device/host helpers for the sm_100a kernels of libi8moe.
//
// Inline-PTX wrappers for mbarrier, TMA (cp.async.bulk.tensor), bulk
// shared->global copies and the tcgen05 (5th-generation tensor core + TMEM)
// instructions, plus bounded waits: every spin in these kernels gives up
// after kWaitTimeoutNs of %globaltimer time, records an error code in a
// device word and lets the kernel exit instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "i8moe.h"

namespace i8moe {

// ---------------------------------------------------------------------------
// host-side status plumbing (capi.cu)
// ---------------------------------------------------------------------------
int set_error(int code, const std::string& msg);
// quant.cu: Q/F factorisation of raw block scales (shared by the fused w13
// epilogue's entry point)
int launch_scales_to_qf(const float* scale, int64_t rows_upper, const int32_t* rows_dev,
                        int64_t kb, int64_t q_max, int64_t sg, int32_t* Q, float* F,
                        cudaStream_t st);
int check_launch(const char* what);
int num_sms(int device);
int current_device();

#define I8_REQUIRE(cond, ...)                                                   \
  do {                                                                          \
    if (!(cond)) {                                                              \
      char _buf[512];                                                           \
      snprintf(_buf, sizeof(_buf), __VA_ARGS__);                                \
      return ::i8moe::set_error(I8MOE_ERR_INVALID, _buf);                       \
    }                                                                           \
  } while (0)

#define I8_CUDA(call)                                                           \
  do {                                                                          \
    cudaError_t _e = (call);                                                    \
    if (_e != cudaSuccess) {                                                    \
      return ::i8moe::set_error(I8MOE_ERR_CUDA,                                 \
                                std::string(#call ": ") + cudaGetErrorString(_e)); \
    }                                                                           \
  } while (0)

// ---------------------------------------------------------------------------
// device error word bits
// ---------------------------------------------------------------------------
enum : unsigned {
  kErrProducerTimeout = 1u << 0,
  kErrMmaTimeout = 1u << 1,
  kErrEpilogueTimeout = 1u << 2,
  kErrDrainTimeout = 1u << 3,
  kErrBadProblem = 1u << 4,
  kErrBadIndex = 1u << 5,
};

#ifndef I8MOE_WAIT_TIMEOUT_NS
#define I8MOE_WAIT_TIMEOUT_NS 4000000000ull  // 4 s; every kernel here runs for ms
#endif

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the warp sleeps in hardware until the
// phase completes (or the hint elapses) instead of spinning on the issue
// slots that the MMA / TMA warps need.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity,
                                                    uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Gives up after
// `timeout_ns` (or as soon as *abort is set by another warp), records `code`
// in *err and returns false.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort,
                                          unsigned* err, unsigned code,
                                          uint64_t timeout_ns = I8MOE_WAIT_TIMEOUT_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 1000000u)) return true;
    if (*abort) return false;
    if (globaltimer() - t0 > timeout_ns) {
      *abort = 1;
      atomicOr(err, code);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// TMA
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const void* desc) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(desc)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* desc, uint32_t bar, int x,
                                            int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* desc, uint32_t bar, int x,
                                            int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// L2 prefetch of one tensor box (no shared memory, no completion tracking).
__device__ __forceinline__ void tma_prefetch_l2_2d(const void* desc, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(desc)),
               "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void tma_prefetch_l2_3d(const void* desc, int x, int y, int z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(desc)),
               "r"(x), "r"(y), "r"(z)
               : "memory");
}

// Four rows (row0..row3, any order) x box-width columns of a 2-D tensor whose
// tensor map has a one-row box; the rows land consecutively in shared memory.
__device__ __forceinline__ void tma_gather4(uint32_t dst, const void* desc, uint32_t bar, int col,
                                            int r0, int r1, int r2, int r3) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(bar), "r"(col), "r"(r0), "r"(r1), "r"(r2), "r"(r3)
      : "memory");
}

// Tiled shared -> global tensor store (bulk group); the coordinates must be
// non-negative and x * element size a multiple of 16 bytes.
__device__ __forceinline__ void tma_store_2d(const void* desc, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(desc)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}

// Bulk (non-tensor) shared -> global copy; both addresses 16-B aligned,
// size a multiple of 16.
__device__ __forceinline__ void bulk_store(void* gdst, uint32_t ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst),
               "r"(ssrc), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait0() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 4-byte global -> shared asynchronous copy (no register destination), and
// the wait for all of this thread's outstanding ones.
__device__ __forceinline__ void cp_async4(uint32_t sdst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(sdst), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32.
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when all previously issued tcgen05 ops of this thread
// have completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// ---------------------------------------------------------------------------
// CTA pairs: a cluster of two CTAs sharing one tcgen05.mma.cta_group::2
// (M = 256: each CTA holds 128 rows of A, half of the B columns and its
// 128 accumulator rows in its own TMEM).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// shared::cluster address of this CTA's shared-memory offset `addr` in CTA
// `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// every thread of both CTAs; orders prior shared-memory work (barrier
// initialisation included) before anything after it in the other CTA
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// arrive on an mbarrier of either CTA (shared::cluster address); the
// default .release.cta semantics suffice to hand a TMEM accumulator back
// after tcgen05.wait::ld and tcgen05.fence::before_thread_sync
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}
// TMA tile loads into this CTA's shared memory whose completion is counted
// on the mbarrier `bar` of either CTA of the pair (shared::cluster address)
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void* desc, uint32_t bar,
                                                 int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const void* desc, uint32_t bar,
                                                 int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}
// TMEM allocation shared by the pair: one warp of each CTA, same warp id
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// issued by one thread of the pair's first CTA; the descriptors' shared
// memory offsets are read in both CTAs
__device__ __forceinline__ void umma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive once on the mbarrier `bar` (shared::cluster address, either CTA)
// when the issuing thread's previous pair MMAs have completed in both CTAs
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// lane (taddr.lane + t), columns [taddr.col, taddr.col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 32 lanes x 8 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7])
               :
               : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
        "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
        "+r"(r[14]), "+r"(r[15])
      :
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit TMEM columns, multiplied by q and added to
// (tmem_mad16) or written into (tmem_mul16) sixteen int32 sums of this thread:
// the load, its wait and the sixteen integer multiplies in one asm block, so
// the loaded values live only in block-local registers.
__device__ __forceinline__ void tmem_mad16(
    uint32_t taddr, int q,
    int32_t& w0, int32_t& w1, int32_t& w2, int32_t& w3,
    int32_t& w4, int32_t& w5, int32_t& w6, int32_t& w7,
    int32_t& w8, int32_t& w9, int32_t& w10, int32_t& w11,
    int32_t& w12, int32_t& w13, int32_t& w14, int32_t& w15) {
  asm volatile(
      "{\n\t.reg .b32 t0, t1, t2, t3, t4, t5, t6, t7, t8, t9, t10, t11, t12, t13, t14, t15;\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {t0, t1, t2, t3, t4, t5, t6, t7, t8, t9, t10, t11, t12, t13, t14, t15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n\t"
      "mad.lo.s32 %0, t0, %17, %0;\n\t"
      "mad.lo.s32 %1, t1, %17, %1;\n\t"
      "mad.lo.s32 %2, t2, %17, %2;\n\t"
      "mad.lo.s32 %3, t3, %17, %3;\n\t"
      "mad.lo.s32 %4, t4, %17, %4;\n\t"
      "mad.lo.s32 %5, t5, %17, %5;\n\t"
      "mad.lo.s32 %6, t6, %17, %6;\n\t"
      "mad.lo.s32 %7, t7, %17, %7;\n\t"
      "mad.lo.s32 %8, t8, %17, %8;\n\t"
      "mad.lo.s32 %9, t9, %17, %9;\n\t"
      "mad.lo.s32 %10, t10, %17, %10;\n\t"
      "mad.lo.s32 %11, t11, %17, %11;\n\t"
      "mad.lo.s32 %12, t12, %17, %12;\n\t"
      "mad.lo.s32 %13, t13, %17, %13;\n\t"
      "mad.lo.s32 %14, t14, %17, %14;\n\t"
      "mad.lo.s32 %15, t15, %17, %15;\n\t"
      "}"
      : "+r"(w0), "+r"(w1), "+r"(w2), "+r"(w3),
        "+r"(w4), "+r"(w5), "+r"(w6), "+r"(w7),
        "+r"(w8), "+r"(w9), "+r"(w10), "+r"(w11),
        "+r"(w12), "+r"(w13), "+r"(w14), "+r"(w15)
      : "r"(taddr), "r"(q)
      : "memory");
}

__device__ __forceinline__ void tmem_mul16(
    uint32_t taddr, int q,
    int32_t& w0, int32_t& w1, int32_t& w2, int32_t& w3,
    int32_t& w4, int32_t& w5, int32_t& w6, int32_t& w7,
    int32_t& w8, int32_t& w9, int32_t& w10, int32_t& w11,
    int32_t& w12, int32_t& w13, int32_t& w14, int32_t& w15) {
  asm volatile(
      "{\n\t.reg .b32 t0, t1, t2, t3, t4, t5, t6, t7, t8, t9, t10, t11, t12, t13, t14, t15;\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {t0, t1, t2, t3, t4, t5, t6, t7, t8, t9, t10, t11, t12, t13, t14, t15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n\t"
      "mul.lo.s32 %0, t0, %17;\n\t"
      "mul.lo.s32 %1, t1, %17;\n\t"
      "mul.lo.s32 %2, t2, %17;\n\t"
      "mul.lo.s32 %3, t3, %17;\n\t"
      "mul.lo.s32 %4, t4, %17;\n\t"
      "mul.lo.s32 %5, t5, %17;\n\t"
      "mul.lo.s32 %6, t6, %17;\n\t"
      "mul.lo.s32 %7, t7, %17;\n\t"
      "mul.lo.s32 %8, t8, %17;\n\t"
      "mul.lo.s32 %9, t9, %17;\n\t"
      "mul.lo.s32 %10, t10, %17;\n\t"
      "mul.lo.s32 %11, t11, %17;\n\t"
      "mul.lo.s32 %12, t12, %17;\n\t"
      "mul.lo.s32 %13, t13, %17;\n\t"
      "mul.lo.s32 %14, t14, %17;\n\t"
      "mul.lo.s32 %15, t15, %17;\n\t"
      "}"
      : "=r"(w0), "=r"(w1), "=r"(w2), "=r"(w3),
        "=r"(w4), "=r"(w5), "=r"(w6), "=r"(w7),
        "=r"(w8), "=r"(w9), "=r"(w10), "=r"(w11),
        "=r"(w12), "=r"(w13), "=r"(w14), "=r"(w15)
      : "r"(taddr), "r"(q)
      : "memory");
}

// 32 lanes x 32 consecutive TMEM columns multiplied by q and added to
// (mad) or written into (mul) 32 int32 sums w[0..31] (indices that resolve
// to registers after inlining).  The _release forms then hand the
// accumulator back: tcgen05.fence::before_thread_sync and an arrive of this
// thread on the mbarrier `bar` (shared::cta), right after the load has
// landed, before the multiplies.  `bar` is ignored by the other forms.
__device__ __forceinline__ void tmem_mad32(uint32_t taddr, int q, uint32_t bar, int32_t* w) {
  asm volatile(
      "{\n\t.reg .b32 t0, t1, t2, t3, t4, t5, t6, t7, t8, t9, t10, t11, t12, t13, t14, t15, t16, t17, t18, t19, t20, t21, t22, t23, t24, t25, t26, t27, t28, t29, t30, t31;\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {t0, t1, t2, t3, t4, t5, t6, t7, t8, t9, t10, t11, t12, t13, t14, t15, t16, t17, t18, t19, t20, t21, t22, t23, t24, t25, t26, t27, t28, t29, t30, t31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n\t"
      "mad.lo.s32 %0, t0, %33, %0;\n\t"
      "mad.lo.s32 %1, t1, %33, %1;\n\t"
      "mad.lo.s32 %2, t2, %33, %2;\n\t"
      "mad.lo.s32 %3, t3, %33, %3;\n\t"
      "mad.lo.s32 %4, t4, %33, %4;\n\t"
      "mad.lo.s32 %5, t5, %33, %5;\n\t"
      "mad.lo.s32 %6, t6, %33, %6;\n\t"
      "mad.lo.s32 %7, t7, %33, %7;\n\t"
      "mad.lo.s32 %8, t8, %33, %8;\n\t"
      "mad.lo.s32 %9, t9, %33, %9;\n\t"
      "mad.lo.s32 %10, t10, %33, %10;\n\t"
      "mad.lo.s32 %11, t11, %33, %11;\n\t"
      "mad.lo.s32 %12, t12, %33, %12;\n\t"
      "mad.lo.s32 %13, t13, %33, %13;\n\t"
      "mad.lo.s32 %14, t14, %33, %14;\n\t"
      "mad.lo.s32 %15, t15, %33, %15;\n\t"
      "mad.lo.s32 %16, t16, %33, %16;\n\t"
      "mad.lo.s32 %17, t17, %33, %17;\n\t"
      "mad.lo.s32 %18, t18, %33, %18;\n\t"
      "mad.lo.s32 %19, t19, %33, %19;\n\t"
      "mad.lo.s32 %20, t20, %33, %20;\n\t"
      "mad.lo.s32 %21, t21, %33, %21;\n\t"
      "mad.lo.s32 %22, t22, %33, %22;\n\t"
      "mad.lo.s32 %23, t23, %33, %23;\n\t"
      "mad.lo.s32 %24, t24, %33, %24;\n\t"
      "mad.lo.s32 %25, t25, %33, %25;\n\t"
      "mad.lo.s32 %26, t26, %33, %26;\n\t"
      "mad.lo.s32 %27, t27, %33, %27;\n\t"
      "mad.lo.s32 %28, t28, %33, %28;\n\t"
      "mad.lo.s32 %29, t29, %33, %29;\n\t"
      "mad.lo.s32 %30, t30, %33, %30;\n\t"
      "mad.lo.s32 %31, t31, %33, %31;\n\t"
      "}"
      : "+r"(w[0]), "+r"(w[1]), "+r"(w[2]), "+r"(w[3]),
        "+r"(w[4]), "+r"(w[5]), "+r"(w[6]), "+r"(w[7]),
        "+r"(w[8]), "+r"(w[9]), "+r"(w[10]), "+r"(w[11]),
        "+r"(w[12]), "+r"(w[13]), "+r"(w[14]), "+r"(w[15]),
        "+r"(w[16]), "+r"(w[17]), "+r"(w[18]), "+r"(w[19]),
        "+r"(w[20]), "+r"(w[21]), "+r"(w[22]), "+r"(w[23]),
        "+r"(w[24]), "+r"(w[25]), "+r"(w[26]), "+r"(w[27]),
        "+r"(w[28]), "+r"(w[29]), "+r"(w[30]), "+r"(w[31])
      : "r"(taddr), "r"(q), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tmem_mul32(uint32_t taddr, int q, uint32_t bar, int32_t* w) {
  asm volatile(
      "{\n\t.reg .b32 t0, t1, t2, t3, t4, t5, t6, t7, t8, t9, t10, t11, t12, t13, t14, t15, t16, t17, t18, t19, t20, t21, t22, t23, t24, t25, t26, t27, t28, t29, t30, t31;\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {t0, t1, t2, t3, t4, t5, t6, t7, t8, t9, t10, t11, t12, t13, t14, t15, t16, t17, t18, t19, t20, t21, t22, t23, t24, t25, t26, t27, t28, t29, t30, t31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n\t"
      "mul.lo.s32 %0, t0, %33;\n\t"
      "mul.lo.s32 %1, t1, %33;\n\t"
      "mul.lo.s32 %2, t2, %33;\n\t"
      "mul.lo.s32 %3, t3, %33;\n\t"
      "mul.lo.s32 %4, t4, %33;\n\t"
      "mul.lo.s32 %5, t5, %33;\n\t"
      "mul.lo.s32 %6, t6, %33;\n\t"
      "mul.lo.s32 %7, t7, %33;\n\t"
      "mul.lo.s32 %8, t8, %33;\n\t"
      "mul.lo.s32 %9, t9, %33;\n\t"
      "mul.lo.s32 %10, t10, %33;\n\t"
      "mul.lo.s32 %11, t11, %33;\n\t"
      "mul.lo.s32 %12, t12, %33;\n\t"
      "mul.lo.s32 %13, t13, %33;\n\t"
      "mul.lo.s32 %14, t14, %33;\n\t"
      "mul.lo.s32 %15, t15, %33;\n\t"
      "mul.lo.s32 %16, t16, %33;\n\t"
      "mul.lo.s32 %17, t17, %33;\n\t"
      "mul.lo.s32 %18, t18, %33;\n\t"
      "mul.lo.s32 %19, t19, %33;\n\t"
      "mul.lo.s32 %20, t20, %33;\n\t"
      "mul.lo.s32 %21, t21, %33;\n\t"
      "mul.lo.s32 %22, t22, %33;\n\t"
      "mul.lo.s32 %23, t23, %33;\n\t"
      "mul.lo.s32 %24, t24, %33;\n\t"
      "mul.lo.s32 %25, t25, %33;\n\t"
      "mul.lo.s32 %26, t26, %33;\n\t"
      "mul.lo.s32 %27, t27, %33;\n\t"
      "mul.lo.s32 %28, t28, %33;\n\t"
      "mul.lo.s32 %29, t29, %33;\n\t"
      "mul.lo.s32 %30, t30, %33;\n\t"
      "mul.lo.s32 %31, t31, %33;\n\t"
      "}"
      : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]),
        "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7]),
        "=r"(w[8]), "=r"(w[9]), "=r"(w[10]), "=r"(w[11]),
        "=r"(w[12]), "=r"(w[13]), "=r"(w[14]), "=r"(w[15]),
        "=r"(w[16]), "=r"(w[17]), "=r"(w[18]), "=r"(w[19]),
        "=r"(w[20]), "=r"(w[21]), "=r"(w[22]), "=r"(w[23]),
        "=r"(w[24]), "=r"(w[25]), "=r"(w[26]), "=r"(w[27]),
        "=r"(w[28]), "=r"(w[29]), "=r"(w[30]), "=r"(w[31])
      : "r"(taddr), "r"(q), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tmem_mad32_release(uint32_t taddr, int q, uint32_t bar, int32_t* w) {
  asm volatile(
      "{\n\t.reg .b32 t0, t1, t2, t3, t4, t5, t6, t7, t8, t9, t10, t11, t12, t13, t14, t15, t16, t17, t18, t19, t20, t21, t22, t23, t24, t25, t26, t27, t28, t29, t30, t31;\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {t0, t1, t2, t3, t4, t5, t6, t7, t8, t9, t10, t11, t12, t13, t14, t15, t16, t17, t18, t19, t20, t21, t22, t23, t24, t25, t26, t27, t28, t29, t30, t31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n\t"
      "tcgen05.fence::before_thread_sync;\n\t"
      "mbarrier.arrive.shared::cta.b64 _, [%34];\n\t"
      "mad.lo.s32 %0, t0, %33, %0;\n\t"
      "mad.lo.s32 %1, t1, %33, %1;\n\t"
      "mad.lo.s32 %2, t2, %33, %2;\n\t"
      "mad.lo.s32 %3, t3, %33, %3;\n\t"
      "mad.lo.s32 %4, t4, %33, %4;\n\t"
      "mad.lo.s32 %5, t5, %33, %5;\n\t"
      "mad.lo.s32 %6, t6, %33, %6;\n\t"
      "mad.lo.s32 %7, t7, %33, %7;\n\t"
      "mad.lo.s32 %8, t8, %33, %8;\n\t"
      "mad.lo.s32 %9, t9, %33, %9;\n\t"
      "mad.lo.s32 %10, t10, %33, %10;\n\t"
      "mad.lo.s32 %11, t11, %33, %11;\n\t"
      "mad.lo.s32 %12, t12, %33, %12;\n\t"
      "mad.lo.s32 %13, t13, %33, %13;\n\t"
      "mad.lo.s32 %14, t14, %33, %14;\n\t"
      "mad.lo.s32 %15, t15, %33, %15;\n\t"
      "mad.lo.s32 %16, t16, %33, %16;\n\t"
      "mad.lo.s32 %17, t17, %33, %17;\n\t"
      "mad.lo.s32 %18, t18, %33, %18;\n\t"
      "mad.lo.s32 %19, t19, %33, %19;\n\t"
      "mad.lo.s32 %20, t20, %33, %20;\n\t"
      "mad.lo.s32 %21, t21, %33, %21;\n\t"
      "mad.lo.s32 %22, t22, %33, %22;\n\t"
      "mad.lo.s32 %23, t23, %33, %23;\n\t"
      "mad.lo.s32 %24, t24, %33, %24;\n\t"
      "mad.lo.s32 %25, t25, %33, %25;\n\t"
      "mad.lo.s32 %26, t26, %33, %26;\n\t"
      "mad.lo.s32 %27, t27, %33, %27;\n\t"
      "mad.lo.s32 %28, t28, %33, %28;\n\t"
      "mad.lo.s32 %29, t29, %33, %29;\n\t"
      "mad.lo.s32 %30, t30, %33, %30;\n\t"
      "mad.lo.s32 %31, t31, %33, %31;\n\t"
      "}"
      : "+r"(w[0]), "+r"(w[1]), "+r"(w[2]), "+r"(w[3]),
        "+r"(w[4]), "+r"(w[5]), "+r"(w[6]), "+r"(w[7]),
        "+r"(w[8]), "+r"(w[9]), "+r"(w[10]), "+r"(w[11]),
        "+r"(w[12]), "+r"(w[13]), "+r"(w[14]), "+r"(w[15]),
        "+r"(w[16]), "+r"(w[17]), "+r"(w[18]), "+r"(w[19]),
        "+r"(w[20]), "+r"(w[21]), "+r"(w[22]), "+r"(w[23]),
        "+r"(w[24]), "+r"(w[25]), "+r"(w[26]), "+r"(w[27]),
        "+r"(w[28]), "+r"(w[29]), "+r"(w[30]), "+r"(w[31])
      : "r"(taddr), "r"(q), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tmem_mul32_release(uint32_t taddr, int q, uint32_t bar, int32_t* w) {
  asm volatile(
      "{\n\t.reg .b32 t0, t1, t2, t3, t4, t5, t6, t7, t8, t9, t10, t11, t12, t13, t14, t15, t16, t17, t18, t19, t20, t21, t22, t23, t24, t25, t26, t27, t28, t29, t30, t31;\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {t0, t1, t2, t3, t4, t5, t6, t7, t8, t9, t10, t11, t12, t13, t14, t15, t16, t17, t18, t19, t20, t21, t22, t23, t24, t25, t26, t27, t28, t29, t30, t31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n\t"
      "tcgen05.fence::before_thread_sync;\n\t"
      "mbarrier.arrive.shared::cta.b64 _, [%34];\n\t"
      "mul.lo.s32 %0, t0, %33;\n\t"
      "mul.lo.s32 %1, t1, %33;\n\t"
      "mul.lo.s32 %2, t2, %33;\n\t"
      "mul.lo.s32 %3, t3, %33;\n\t"
      "mul.lo.s32 %4, t4, %33;\n\t"
      "mul.lo.s32 %5, t5, %33;\n\t"
      "mul.lo.s32 %6, t6, %33;\n\t"
      "mul.lo.s32 %7, t7, %33;\n\t"
      "mul.lo.s32 %8, t8, %33;\n\t"
      "mul.lo.s32 %9, t9, %33;\n\t"
      "mul.lo.s32 %10, t10, %33;\n\t"
      "mul.lo.s32 %11, t11, %33;\n\t"
      "mul.lo.s32 %12, t12, %33;\n\t"
      "mul.lo.s32 %13, t13, %33;\n\t"
      "mul.lo.s32 %14, t14, %33;\n\t"
      "mul.lo.s32 %15, t15, %33;\n\t"
      "mul.lo.s32 %16, t16, %33;\n\t"
      "mul.lo.s32 %17, t17, %33;\n\t"
      "mul.lo.s32 %18, t18, %33;\n\t"
      "mul.lo.s32 %19, t19, %33;\n\t"
      "mul.lo.s32 %20, t20, %33;\n\t"
      "mul.lo.s32 %21, t21, %33;\n\t"
      "mul.lo.s32 %22, t22, %33;\n\t"
      "mul.lo.s32 %23, t23, %33;\n\t"
      "mul.lo.s32 %24, t24, %33;\n\t"
      "mul.lo.s32 %25, t25, %33;\n\t"
      "mul.lo.s32 %26, t26, %33;\n\t"
      "mul.lo.s32 %27, t27, %33;\n\t"
      "mul.lo.s32 %28, t28, %33;\n\t"
      "mul.lo.s32 %29, t29, %33;\n\t"
      "mul.lo.s32 %30, t30, %33;\n\t"
      "mul.lo.s32 %31, t31, %33;\n\t"
      "}"
      : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]),
        "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7]),
        "=r"(w[8]), "=r"(w[9]), "=r"(w[10]), "=r"(w[11]),
        "=r"(w[12]), "=r"(w[13]), "=r"(w[14]), "=r"(w[15]),
        "=r"(w[16]), "=r"(w[17]), "=r"(w[18]), "=r"(w[19]),
        "=r"(w[20]), "=r"(w[21]), "=r"(w[22]), "=r"(w[23]),
        "=r"(w[24]), "=r"(w[25]), "=r"(w[26]), "=r"(w[27]),
        "=r"(w[28]), "=r"(w[29]), "=r"(w[30]), "=r"(w[31])
      : "r"(taddr), "r"(q), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// tcgen05.wait::ld that also ties the 32 destination registers of the
// preceding tcgen05.ld, so no use of them can be scheduled above the wait.
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
        "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
        "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]),
        "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),
        "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}

// Shared-memory matrix descriptor for a K-major operand stored with the
// 128-byte swizzle: rows of 128 bytes, 8-row (1024-byte) swizzle atoms
// stacked along M/N.  Start address must lie in a 1024-byte aligned atom;
// advancing along K inside the atom adds the byte offset to the start
// address.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);  // start address
  d |= static_cast<uint64_t>(1) << 16;                       // LBO (unused for SW128 K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;               // SBO: 8 rows x 128 B
  d |= static_cast<uint64_t>(1) << 46;                       // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                       // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::i8: D s32, A/B signed int8, both K-major.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// ---------------------------------------------------------------------------
// small numeric helpers
// ---------------------------------------------------------------------------
template <typename T>
struct Num;
template <>
struct Num<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <>
struct Num<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};
template <>
struct Num<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};

__device__ __forceinline__ int warp_max_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace i8moe
