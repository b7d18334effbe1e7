// Thin inline-PTX layer for sm_100a: mbarriers, TMA (no multicast anywhere),
// tcgen05 (TMEM alloc, UMMA issue/commit, TMEM load/store) and the shared-memory
// matrix descriptors the UMMA reads its operands through.
//
// Every wait here is bounded: a wait that does not complete within
// kWaitLimitNs sets the CTA's abort flag (and the kernel's device error word),
// after which every other wait in the CTA returns false at once and the kernel
// unwinds to its teardown (TMEM dealloc) instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace va {

// Device error codes (written with atomicCAS into the context's error word; the
// first error wins).
enum DevError : int {
  kDevOk = 0,
  kDevTimeoutProducer = 1,  // TMA producer gave up waiting for a free stage
  kDevTimeoutMma = 2,       // MMA issuer gave up waiting for operands / P
  kDevTimeoutConsumer = 3,  // softmax / epilogue gave up waiting for the accumulator
  kDevBadShape = 4,         // a kernel saw a shape its host checks should have rejected
  kDevTimeoutPeer = 5,      // the K'/V exchange barrier gave up waiting for a peer GPU
};

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s per wait

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void report_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
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

// try_wait with a suspend-time hint: the thread may sleep (up to hint_ns) until the
// phase completes instead of spinning, so waiting warps leave their issue slots
// to the warps that compute.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
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
constexpr uint32_t kWaitSleepHintNs = 20000;

// Waits for the phase with the given parity to complete.  Returns false when the
// wait timed out (the abort flag and the device error word are then set) or when
// another thread of the CTA already aborted.
__device__ __forceinline__ bool mbar_wait_for(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                              int* err, int code, unsigned long long limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, kWaitSleepHintNs)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > limit_ns) {
      *abort_flag = 1;
      report_error(err, code);
      return false;
    }
  }
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int* err, int code) {
  return mbar_wait_for(bar, parity, abort_flag, err, code, kWaitLimitNs);
}

// ---------------------------------------------------------------------------
// TMA (tiled, no multicast).  The innermost coordinate is always a multiple of
// 64 bf16 elements (128 B) in this library.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// System-scope flag access (another GPU writes or reads the flag over NVLink).
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// Named barrier `id` (1..15) over `count` threads (a multiple of 32).
__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Shared -> global TMA store of one box (bulk-group completion), no multicast.
// The box lands at coordinates (x, y); parts outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y), "r"(z)
               : "memory");
}
// Shared -> global TMA reduction of one box (bulk-group completion), no multicast:
// every element of the box is added to the global tensor's element (F32 add,
// performed at L2); parts outside the tensor are not touched.
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until every committed bulk store of this thread has completed.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Waits until every committed bulk store of this thread has finished reading its
// shared-memory source (the writes to global memory may still be in flight).
__device__ __forceinline__ void bulk_wait_all_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
// Byte offset of 16-byte chunk c of row r in a SWIZZLE_128B tile of 128-byte rows
// (the tile base 1024-byte aligned): the chunk index is XORed with r mod 8.
__device__ __forceinline__ uint32_t sw128_offset(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (UMMA / TMA) reads of them.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: tensor memory and UMMA
// ---------------------------------------------------------------------------
// TMEM address = (lane << 16) | column.
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
// Arrives once on `bar` when every tcgen05 op issued so far by this thread is done.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]  (kind::f16: bf16 in, f32 accumulate)
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]; A is M lanes x (K/2) columns of packed bf16x2.
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Four SS UMMAs stepping K by 16 elements (32 B) in both K-major SW128 operands:
// D (+)= A[:, 0:64] * B[:, 0:64].  Only the descriptors' 14-bit start field moves
// (by 2 per step, in 16-byte units), and shared memory stays below 256 KB, so a
// 32-bit add on the low word is exact.  `accumulate` applies to the first step;
// the other three always accumulate.
__device__ __forceinline__ void umma_ss_k64(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t.reg .b32 alo, ahi, blo, bhi, t0, t1;\n\t.reg .b64 a, b;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "setp.eq.b32 q, %4, %4;\n\t"
      "mov.b64 {alo, ahi}, %1;\n\t"
      "mov.b64 {blo, bhi}, %2;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t"
      "add.u32 t0, alo, 2;\n\tadd.u32 t1, blo, 2;\n\t"
      "mov.b64 a, {t0, ahi};\n\tmov.b64 b, {t1, bhi};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, q;\n\t"
      "add.u32 t0, alo, 4;\n\tadd.u32 t1, blo, 4;\n\t"
      "mov.b64 a, {t0, ahi};\n\tmov.b64 b, {t1, bhi};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, q;\n\t"
      "add.u32 t0, alo, 6;\n\tadd.u32 t1, blo, 6;\n\t"
      "mov.b64 a, {t0, ahi};\n\tmov.b64 b, {t1, bhi};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, q;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Eight TS UMMAs stepping K by 16: A from TMEM (8 columns of packed pairs per step),
// B an MN-major SW128 operand whose 16-row K step is 2048 B (128 in the start
// field).  `accumulate` applies to the first step; the others always accumulate.
__device__ __forceinline__ void umma_ts_k128_mn(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t.reg .b32 blo, bhi, ta, tb;\n\t.reg .b64 b;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "setp.eq.b32 q, %4, %4;\n\t"
      "mov.b64 {blo, bhi}, %2;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t"
      "add.u32 ta, %1, 8;\n\tadd.u32 tb, blo, 128;\n\tmov.b64 b, {tb, bhi};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, q;\n\t"
      "add.u32 ta, %1, 16;\n\tadd.u32 tb, blo, 256;\n\tmov.b64 b, {tb, bhi};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, q;\n\t"
      "add.u32 ta, %1, 24;\n\tadd.u32 tb, blo, 384;\n\tmov.b64 b, {tb, bhi};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, q;\n\t"
      "add.u32 ta, %1, 32;\n\tadd.u32 tb, blo, 512;\n\tmov.b64 b, {tb, bhi};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, q;\n\t"
      "add.u32 ta, %1, 40;\n\tadd.u32 tb, blo, 640;\n\tmov.b64 b, {tb, bhi};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, q;\n\t"
      "add.u32 ta, %1, 48;\n\tadd.u32 tb, blo, 768;\n\tmov.b64 b, {tb, bhi};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, q;\n\t"
      "add.u32 ta, %1, 56;\n\tadd.u32 tb, blo, 896;\n\tmov.b64 b, {tb, bhi};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, q;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Half of the above: 4 UMMAs over 64 keys (P columns [a_tmem, a_tmem + 32), B rows of
// the descriptor's first 64 keys).  `accumulate` applies to the first UMMA only.
__device__ __forceinline__ void umma_ts_k64_mn(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t.reg .b32 blo, bhi, ta, tb;\n\t.reg .b64 b;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "setp.eq.b32 q, %4, %4;\n\t"
      "mov.b64 {blo, bhi}, %2;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t"
      "add.u32 ta, %1, 8;\n\tadd.u32 tb, blo, 128;\n\tmov.b64 b, {tb, bhi};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, q;\n\t"
      "add.u32 ta, %1, 16;\n\tadd.u32 tb, blo, 256;\n\tmov.b64 b, {tb, bhi};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, q;\n\t"
      "add.u32 ta, %1, 24;\n\tadd.u32 tb, blo, 384;\n\tmov.b64 b, {tb, bhi};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, q;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor, kind::f16 with bf16 A/B and f32 D.
//   [4,6) D fmt (1 = f32)  [7,10) A fmt (1 = bf16)  [10,13) B fmt (1 = bf16)
//   [15] A MN-major  [16] B MN-major  [17,23) N>>3  [24,29) M>>4
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n, bool a_mn_major,
                                                      bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(a_mn_major) << 15) |
         (static_cast<uint32_t>(b_mn_major) << 16) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

// Same with f16 A/B (format 0).
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n, bool a_mn_major,
                                                     bool b_mn_major) {
  return (1u << 4) | (static_cast<uint32_t>(a_mn_major) << 15) |
         (static_cast<uint32_t>(b_mn_major) << 16) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

// Shared-memory matrix descriptor, SWIZZLE_128B (layout type 2), sm100 version 1.
//   [0,14) start >> 4   [16,30) LBO >> 4   [32,46) SBO >> 4   [46,48) version=1
//   [49,52) base offset (0: every tile is 1024-B aligned)   [61,64) layout type
// K-major operand: rows of 128 B (64 bf16 of K), 8-row groups SBO = 1024 B apart;
//   the K step inside the 128-B row is taken by advancing the start address.
// MN-major operand: rows of 128 B hold 64 MN elements, one row per K index,
//   8-K groups SBO = 1024 B apart, LBO = distance between 64-element MN blocks.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// TMEM -> registers, 32 lanes x 32 columns of 32 bit (thread i of the warp gets
// lane (warp%4)*32+i, columns [col, col+32)).  The wait is inside the same asm
// statement so no use of the registers can be scheduled before it.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Registers -> TMEM, 32 lanes x 16 columns of 32 bit.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// TMEM -> registers, 32 lanes x 128 columns in one instruction, then wait.
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, float* v) {
  uint32_t r[128];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64, %65, %66, %67, %68, %69, %70, %71, %72, %73, %74, %75, %76, %77, %78, %79, %80, %81, %82, %83, %84, %85, %86, %87, %88, %89, %90, %91, %92, %93, %94, %95, %96, %97, %98, %99, %100, %101, %102, %103, %104, %105, %106, %107, %108, %109, %110, %111, %112, %113, %114, %115, %116, %117, %118, %119, %120, %121, %122, %123, %124, %125, %126, %127}, [%128];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]), "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]), "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]), "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]), "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]), "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]), "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]), "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]), "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 128; ++i) v[i] = __uint_as_float(r[i]);
}

// Registers -> TMEM, 32 lanes x 64 columns in one instruction.
__device__ __forceinline__ void tmem_st64(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64};"
      :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]), "r"(r[32]), "r"(r[33]), "r"(r[34]), "r"(r[35]), "r"(r[36]), "r"(r[37]), "r"(r[38]), "r"(r[39]), "r"(r[40]), "r"(r[41]), "r"(r[42]), "r"(r[43]), "r"(r[44]), "r"(r[45]), "r"(r[46]), "r"(r[47]), "r"(r[48]), "r"(r[49]), "r"(r[50]), "r"(r[51]), "r"(r[52]), "r"(r[53]), "r"(r[54]), "r"(r[55]), "r"(r[56]), "r"(r[57]), "r"(r[58]), "r"(r[59]), "r"(r[60]), "r"(r[61]), "r"(r[62]), "r"(r[63])
      : "memory");
}

// Packed arithmetic of sm_100: two F32 per 64-bit register (f32x2) and two F16
// per 32-bit register (f16x2).  For a pair (lo, hi), lo is the lower half.
__device__ __forceinline__ uint64_t f32x2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint64_t f32x2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ void f32x2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f32x2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f32x2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f32x2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// 2^x for a pair of F32 on the FMA pipe (no MUFU), for x <= 2^22.
// Method: Cody-Waite style split x = n + f with n = round(x) obtained by adding
// 1.5*2^23 (the sum's low mantissa bits then hold n), f in [-0.5, 0.5]; 2^f by a
// cubic whose coefficients were fitted here (Lawson-reweighted least squares on
// 4001 Chebyshev nodes of [-0.5, 0.5], relative error < 7.5e-5 over the range);
// 2^n applied by adding n to the exponent field.  x is clamped at -125 so the
// exponent never underflows (2^-125 ~ 2.4e-38 stands in for smaller values).
constexpr float kExp2C0 = 0x1.fff692p-1f;
constexpr float kExp2C1 = 0x1.62f31ap-1f;
constexpr float kExp2C2 = 0x1.f0de1ap-3f;
constexpr float kExp2C3 = 0x1.c3f75ep-5f;
__device__ __forceinline__ void exp2_fma_x2(float x0, float x1, float& y0, float& y1) {
  x0 = fmaxf(x0, -125.0f);
  x1 = fmaxf(x1, -125.0f);
  const uint64_t magic = f32x2_pack(12582912.0f, 12582912.0f);
  const uint64_t x = f32x2_pack(x0, x1);
  const uint64_t t = f32x2_add(x, magic);
  const uint64_t f = f32x2_sub(x, f32x2_sub(t, magic));
  uint64_t p = f32x2_fma(f32x2_pack(kExp2C3, kExp2C3), f, f32x2_pack(kExp2C2, kExp2C2));
  p = f32x2_fma(p, f, f32x2_pack(kExp2C1, kExp2C1));
  p = f32x2_fma(p, f, f32x2_pack(kExp2C0, kExp2C0));
  float p0, p1, t0, t1;
  f32x2_unpack(p, p0, p1);
  f32x2_unpack(t, t0, t1);
  y0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  y1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}
// (lo, hi) F32 -> f16x2, round to nearest even.
__device__ __forceinline__ uint32_t f16x2_from_f32(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// 2^x on both halves (MUFU, approximate).
__device__ __forceinline__ uint32_t f16x2_ex2(uint32_t x) {
  uint32_t r;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}
__device__ __forceinline__ uint32_t f16x2_add(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ float f16x2_sum_to_f32(uint32_t v) {
  __half2 h = *reinterpret_cast<__half2*>(&v);
  const float2 f = __half22float2(h);
  return f.x + f.y;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// (lo, hi) F32 -> bf16x2 with integer ops only: add half a bf16 ulp to each bit
// pattern (round half up; differs from round-to-nearest-even only on exact ties),
// then one byte permute takes the upper halves.  Finite inputs below 2^127 only.
__device__ __forceinline__ uint32_t pack_bf16x2_round_prmt(float lo, float hi) {
  const uint32_t a = __float_as_uint(lo) + 0x8000u;
  const uint32_t b = __float_as_uint(hi) + 0x8000u;
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);  // .x = lo (low 16 bits), .y = hi
  return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace va
