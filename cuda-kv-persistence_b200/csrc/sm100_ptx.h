// Device primitives shared by the sm_100a kernels (attn_sm100.cu,
// qkv_sm100.cu): mbarriers, TMA loads, tcgen05 MMA / commit / fences, TMEM
// loads and stores, the 128B-swizzle UMMA descriptor.  Inline PTX only.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>

#include "kvp_common.h"

namespace kvp {
namespace ptx {

constexpr unsigned long long kWaitNs = 1000000000ull;  // bounded waits: ~1 s
constexpr uint32_t kSuspendNs = 200000;                 // longest single hardware suspend in a wait

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)),
                 "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(
                     smem_u32(b)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
            smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(b)), "r"(parity) : "memory");
    return ok != 0;
}
// Non-blocking check of a phase (never suspends the thread).
__device__ __forceinline__ bool mbar_test(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(b)), "r"(parity) : "memory");
    return ok != 0;
}
// try_wait that lets the hardware suspend the thread until the phase
// completes (or kSuspendNs passes), so a waiting warp takes no issue slots
// from the softmax warps that share its SM sub-partition.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(b)), "r"(parity), "r"(kSuspendNs) : "memory");
    return ok != 0;
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 16-byte global -> shared copy (L2 only), zero-filling the bytes past
// src_bytes (0 or 16).
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"((unsigned long long)map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
// TMA gather: rows y0..y3 (any order, any rows) of a 2D tensor whose map has
// a one-row box, columns [x, x + box width), into four consecutive rows of
// shared memory at dst (128-byte aligned; the map's swizzle applies by
// address, as for a four-row box stored there).
__device__ __forceinline__ void tma_gather4(void* dst, const CUtensorMap* map, int x, int y0, int y1,
                                            int y2, int y3, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];"
        ::"r"(smem_u32(dst)), "l"((unsigned long long)map), "r"(x), "r"(y0), "r"(y1), "r"(y2), "r"(y3),
          "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(b)) : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

// O_tmem (+)= A_tmem * B_smem: A read from tensor memory (K-major, two bf16
// per 32-bit column, row i in lane i), B described in shared memory.
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate));
}

#define KVP_TMEM_LD32(taddr, r)                                                                  \
    asm volatile(                                                                                \
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15," \
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                 \
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),      \
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),  \
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),            \
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),            \
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])             \
        : "r"(taddr))

#define KVP_TMEM_ST32(taddr, r)                                                                  \
    asm volatile(                                                                                \
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14," \
        "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),   \
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),    \
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),         \
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),        \
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),        \
        "r"(r[29]), "r"(r[30]), "r"(r[31]) : "memory")

// tcgen05.wait::ld that also names the 32 destination registers of the
// load in flight as in/out operands, so no use of them can be scheduled
// before the wait (the load writes them asynchronously).
#define KVP_TMEM_WAIT_LD_DEP(r)                                                                   \
    asm volatile("tcgen05.wait::ld.sync.aligned;"                                                \
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),        \
                   "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),      \
                   "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),  \
                   "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),  \
                   "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),  \
                   "+r"(r[30]), "+r"(r[31])                                                       \
                 :                                                                                \
                 : "memory")

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// UMMA shared-memory descriptor, 128B swizzle (layout type 2), version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Byte offset of (row, 16-byte chunk) inside a 128B-swizzled [rows][64 bf16] panel.
__device__ __forceinline__ uint32_t sw128_off(int row, int chunk) {
    return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}


// Bounded wait (S: the kernel's shared-memory struct, with an int
// abort_flag).  Returns false (and raises the CTA abort flag and the global
// status) when the phase did not complete within kWaitNs, or when another
// role already aborted.
template <class S>
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, S& sm, int* status) {
    if (mbar_try_wait(b, parity)) return true;
    const unsigned long long t0 = globaltimer();
    for (;;) {
        if (mbar_try_wait_sleep(b, parity)) return true;
        if (*(volatile int*)&sm.abort_flag) return false;
        if (globaltimer() - t0 > kWaitNs) {
            *(volatile int*)&sm.abort_flag = 1;
            atomicOr(status, KVP_STATUS_TIMEOUT);
            return false;
        }
    }
}
// Warp-uniform bounded wait: every lane polls and the verdicts are combined
// (a completed phase stays completed until this warp itself moves the
// protocol on), so the warp stays converged for the .sync.aligned tcgen05
// and shuffle instructions that follow.
template <class S>
__device__ __forceinline__ bool warp_wait(uint64_t* b, uint32_t parity, S& sm, int* status) {
    if (__any_sync(0xffffffffu, mbar_try_wait(b, parity))) return true;
    const unsigned long long t0 = globaltimer();
    for (;;) {
        if (__any_sync(0xffffffffu, mbar_try_wait_sleep(b, parity))) return true;
        if (__any_sync(0xffffffffu, *(volatile int*)&sm.abort_flag != 0)) return false;
        if (__any_sync(0xffffffffu, globaltimer() - t0 > kWaitNs)) {
            if ((threadIdx.x & 31) == 0) {
                *(volatile int*)&sm.abort_flag = 1;
                atomicOr(status, KVP_STATUS_TIMEOUT);
            }
            __syncwarp();
            return false;
        }
    }
}

}  // namespace ptx
}  // namespace kvp
