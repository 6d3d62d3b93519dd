// BF16 remapped multi-head attention on SM pairs (sm_100a, tcgen05
// cta_group::2).  Same semantics, inputs and outputs as attn_sm100.cu's
// kernel (the reference's attn_forward_kernel,
// src/gated_attention_kernel.cu:34-139, in bf16 with fp32 accumulation; key
// row j read from arena row KVMap[j] when KVMap[j] >= 0), organised for a
// longer softmax window.
//
// A cluster of two CTAs (one per SM) handles 256 query rows of one head,
// 128 per CTA.  The leader CTA issues every MMA for both SMs with
// cta_group::2 (M = 256): each SM holds its own 128 query rows of Q, S, P
// and O, and supplies half of each K tile (64 keys, all 128 dims) and half
// of each V tile (all 128 keys, 64 dims), so every byte of K/V is staged
// once per pair and each SM reads 6 KB of shared memory per K16 step of the
// S GEMM instead of 8 KB.
//
// Tensor memory per SM: three S buffers [0,128), [128,256), [256,384) and
// O [384,512).  P of key tile j is written as packed bf16 into the first 64
// columns of S buffer j%3 and stays there until PV(j) has read it, so the
// MMA order is S(j), PV(j-2), S(j+1), PV(j-1), ...: between S(j) landing and
// PV(j) being issued the tensor cores run four other GEMMs (about 2,000
// cycles), which is the softmax's window for tile j.  (A one-SM kernel with
// two query tiles has two GEMMs, which is shorter than the exponential work
// of a 128 x 128 tile on the SM's MUFU units.)
//
// Warp roles (384 threads per CTA):
//   warp 0   Q and the K producer (this CTA's 64 keys of each tile)
//   warp 1   TMEM allocation (both CTAs); MMA issuer (leader CTA, one thread)
//   warp 2   the V producer (this CTA's 64 dims of each tile)
//   warp 3   peer CTA only: relays the completion of its Q, K and V loads to
//            the leader's barriers (each CTA's TMA signals its own barrier)
//   warps 4-11 softmax and epilogue, two threads per query row: warps 4-7
//            take columns 0-63 of each S tile and warps 8-11 columns 64-127
//            of the same rows (TMEM lanes 32*(warp%4) ..).  The two halves of
//            a row share its running max through shared memory (a flag per
//            tile, the tile max only when a row's max moves) and keep
//            separate partial sums; each writes the P of its 64 keys and
//            scales its 64 columns of O.  Splitting the row halves the
//            latency of a tile's exponentials, which bounds the step.
// Producers stage each K/V tile through the KVMap exactly as the one-SM
// kernel does: whole-tile TMA boxes when no row is remapped, power-of-two
// boxes per ascending arena run, TMA gathers for scattered arena groups,
// 16-byte cp.async for mixed groups and padding.
//
// Every wait is bounded (about one second of %globaltimer); a CTA that gives
// up raises KVP_STATUS_TIMEOUT and its own and its peer's abort flags, and
// both CTAs unwind.  The two CTAs leave together (a bounded handshake), so
// neither exits while the other may still read its shared memory.
#include <cuda.h>
#include <cuda_bf16.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "attn_pair_sm100.h"
#include "attn_softmax_sm100.cuh"
#include "kvp_common.h"
#include "sm100_ptx.h"

namespace kvp {

namespace {

using namespace ptx;
using namespace attn_dev;

constexpr int kBM = 128;            // query rows per CTA (256 per pair)
constexpr int kBN = 128;            // keys per tile
constexpr int kDH = 128;            // head dim
constexpr int kSBufs = 3;           // S buffers in TMEM
constexpr int kKStages = 6;         // K ring depth (16 KB stages)
constexpr int kVStages = 6;         // V ring depth (16 KB stages)
constexpr int kThreads = 384;
constexpr uint32_t kGroupPanel = 8 * 128;          // 8 rows x 64 bf16, 128B swizzle
constexpr uint32_t kQPanel = 128 * 128;            // [128 rows][64 bf16]
constexpr uint32_t kKPanel = 64 * 128;             // [64 rows][64 bf16]
constexpr uint32_t kKStageBytes = 2 * kKPanel;     // this CTA's 64 keys x 128 dims
constexpr uint32_t kVStageBytes = 128 * 128;       // 128 keys x this CTA's 64 dims
constexpr int kRegsLow = 96;        // warps 0-3
constexpr int kRegsHigh = 200;      // warps 4-11 (softmax)
static_assert(kRegsLow * 128 + kRegsHigh * 256 <= 65536, "register split exceeds the SM");
constexpr float kRedoSum = 256.f;   // a tile row sum above this recomputes with the new max
constexpr int kBoxKinds = 5;        // TMA box heights 8, 16, 32, 64, 128 rows

struct __align__(1024) PairSmem {
    uint8_t q[2 * kQPanel];
    uint8_t k[kKStages][kKStageBytes];
    uint8_t v[kVStages][kVStageBytes];
    uint64_t bar_q;                 // leader: own Q + the peer's relay (2 arrivals)
    uint64_t bar_kfull[kKStages];   // leader: 2 arrivals (own producer, peer relay); peer: 1
    uint64_t bar_kempty[kKStages];  // this CTA's softmax saw S(j) land
    uint64_t bar_vfull[kVStages];
    uint64_t bar_vempty[kVStages];  // PV(j) landed (commit from the leader, both CTAs)
    uint64_t bar_s_full[kSBufs];    // S(j) landed (commit from the leader, both CTAs)
    uint64_t bar_p_full[kSBufs];    // leader: P(j) in both CTAs' TMEM (one arrival per softmax warp)
    uint64_t bar_xch[4];            // the two softmax warps of row quarter q exchanged a value
    uint64_t bar_mma_done;          // leader: every issued MMA landed
    uint64_t bar_exit;              // the peer is done with this CTA's memory
    float xch[2][2][kBM];           // [exchange parity][column half][row]
    uint32_t tmem_base;
    int abort_flag;
};

struct PairMaps {
    CUtensorMap q8;                 // Q [q_rows][D], box 64 x 8
    CUtensorMap kv[2][kBoxKinds];   // K / V [kv_rows][D], box 64 x (8 << i)
    CUtensorMap a[kBoxKinds];       // arena [arena_rows][2D], box 64 x (8 << i)
    CUtensorMap a1;                 // arena, box 64 x 1 (TMA gather)
};

struct PairParams {
    const __nv_bfloat16* k;
    const __nv_bfloat16* v;
    const __nv_bfloat16* arena;
    const long long* kvmap;
    __nv_bfloat16* out;
    int* status;
    long long q_rows, kv_rows, arena_rows;
    int D, T, frames, q_frame0, mode, window, head0, nheads, flat, items_per_head, n_blk;
    int base_boxes, arena_boxes, arena_gather;
    float scale_log2;
};

// ------------------------------------------------------------ cluster PTX
__device__ __forceinline__ uint32_t cta_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// The shared::cluster address of `p` (a shared::cta pointer of this CTA) in CTA `rank`.
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
// Arrival on a barrier of either CTA of the pair (default release.cta
// semantics).  What it publishes is ordered by its own completion
// mechanism: TMA loads by their completed transaction count (observed
// through a local barrier first), P stores by tcgen05.wait::st and
// tcgen05.fence::before_thread_sync.  A cluster-scope release costs about
// 1,500 cycles per arrival here, on the softmax's critical path.
__device__ __forceinline__ void arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool try_wait_cluster(uint64_t* b, uint32_t parity) {
    return mbar_try_wait_sleep(b, parity);
}
__device__ __forceinline__ bool test_wait_cluster(uint64_t* b, uint32_t parity) {
    return mbar_test(b, parity);
}
__device__ __forceinline__ void store_cluster_u32(uint32_t cluster_addr, int v) {
    asm volatile("st.relaxed.cluster.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}
// Commit of every MMA issued so far by this thread, arriving once on the
// barrier at the same offset in both CTAs of the pair.
__device__ __forceinline__ void tc_commit_pair(uint64_t* b) {
    asm volatile(
        "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}"
        ::"r"(smem_u32(b)) : "memory");
}

// Raises this CTA's and the peer's abort flags and the global status.
__device__ __forceinline__ void abort_pair(PairSmem& sm, int* status) {
    *(volatile int*)&sm.abort_flag = 1;
    store_cluster_u32(peer_addr(&sm.abort_flag, cta_rank() ^ 1u), 1);
    atomicOr(status, KVP_STATUS_TIMEOUT);
}

// Bounded wait of one thread (acquire at cluster scope: the barrier may be
// arrived on by the peer CTA or by the leader's commits).
__device__ __forceinline__ bool pair_wait(uint64_t* b, uint32_t parity, PairSmem& sm, int* status) {
    if (test_wait_cluster(b, parity)) return true;
    const unsigned long long t0 = globaltimer();
    for (;;) {
        if (try_wait_cluster(b, parity)) return true;
        if (*(volatile int*)&sm.abort_flag) return false;
        if (globaltimer() - t0 > kWaitNs) {
            abort_pair(sm, status);
            return false;
        }
    }
}
// Warp-uniform bounded wait.
__device__ __forceinline__ bool pair_warp_wait(uint64_t* b, uint32_t parity, PairSmem& sm, int* status) {
    if (__any_sync(0xffffffffu, test_wait_cluster(b, parity))) return true;
    const unsigned long long t0 = globaltimer();
    for (;;) {
        if (__any_sync(0xffffffffu, try_wait_cluster(b, parity))) return true;
        if (__any_sync(0xffffffffu, *(volatile int*)&sm.abort_flag != 0)) return false;
        if (__any_sync(0xffffffffu, globaltimer() - t0 > kWaitNs)) {
            if ((threadIdx.x & 31) == 0) abort_pair(sm, status);
            __syncwarp();
            return false;
        }
    }
}

// ------------------------------------------------------------ pair GEMMs
// S = Q K^T, M = 256 (cta_group::2), N = 128, K = 128: eight K16 MMAs.  A
// (Q, [128 rows][128] per SM, two 16 KB panels) and B (K, [64 keys][128]
// per SM, two 8 KB panels), both K-major 128B swizzle: step ks starts
// (ks>>2) panels + (ks&3)*32 bytes in.
__device__ __forceinline__ void pair_gemm_s(uint32_t d_tmem, uint64_t a0, uint64_t b0, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred pf, pt;\n\t.reg .b64 a, b;\n\t"
        "setp.ne.b32 pf, 0, 0;\n\tsetp.eq.b32 pt, 0, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, pf;\n\t"
        "add.s64 a, %1, 2;\n\tadd.s64 b, %2, 2;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], a, b, %3, pt;\n\t"
        "add.s64 a, %1, 4;\n\tadd.s64 b, %2, 4;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], a, b, %3, pt;\n\t"
        "add.s64 a, %1, 6;\n\tadd.s64 b, %2, 6;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], a, b, %3, pt;\n\t"
        "add.s64 a, %1, 1024;\n\tadd.s64 b, %2, 512;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], a, b, %3, pt;\n\t"
        "add.s64 a, %1, 1026;\n\tadd.s64 b, %2, 514;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], a, b, %3, pt;\n\t"
        "add.s64 a, %1, 1028;\n\tadd.s64 b, %2, 516;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], a, b, %3, pt;\n\t"
        "add.s64 a, %1, 1030;\n\tadd.s64 b, %2, 518;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], a, b, %3, pt;\n\t}"
        ::"r"(d_tmem), "l"(a0), "l"(b0), "r"(idesc));
}
// O (+)= P V, M = 256, N = 128 (64 dims per SM), K = 128 keys: P from TMEM
// (keys 0-63 at columns +0..31 and keys 64-127 at +64..95 of the S buffer,
// as the two softmax halves write them: step ks at column 8*ks + 32*(ks>=4)),
// V MN-major with step ks 16 keys = 2048 bytes further (+128 in the address
// field).
__device__ __forceinline__ void pair_gemm_pv(uint32_t d_tmem, uint32_t a_tmem, uint64_t b0, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred pf, pt;\n\t.reg .b64 b;\n\t.reg .b32 a;\n\t"
        "setp.ne.b32 pf, %4, 0;\n\tsetp.eq.b32 pt, 0, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, pf;\n\t"
        "add.s32 a, %1, 8;\n\tadd.s64 b, %2, 128;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a], b, %3, pt;\n\t"
        "add.s32 a, %1, 16;\n\tadd.s64 b, %2, 256;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a], b, %3, pt;\n\t"
        "add.s32 a, %1, 24;\n\tadd.s64 b, %2, 384;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a], b, %3, pt;\n\t"
        "add.s32 a, %1, 64;\n\tadd.s64 b, %2, 512;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a], b, %3, pt;\n\t"
        "add.s32 a, %1, 72;\n\tadd.s64 b, %2, 640;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a], b, %3, pt;\n\t"
        "add.s32 a, %1, 80;\n\tadd.s64 b, %2, 768;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a], b, %3, pt;\n\t"
        "add.s32 a, %1, 88;\n\tadd.s64 b, %2, 896;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a], b, %3, pt;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b0), "r"(idesc), "r"(accumulate));
}

// kind::f16 instruction descriptor: bf16 x bf16 -> f32, M = 256, N = 128.
constexpr uint32_t idesc_pair(bool b_mn_major) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
           ((uint32_t)(128 >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}

// ------------------------------------------------------------ work item
struct PairWork {
    int head;
    long long klo;       // first key row (both CTAs)
    long long khi;       // end of the staged key rows (max over both CTAs' rows)
    int n_tiles;         // 128-key tiles (both CTAs)
    long long row0;      // this CTA's first query row
    int nq;              // this CTA's valid query rows (0..128)
    long long my_khi;    // key limit of this CTA's rows >= split
    long long my_khi_lo; // key limit of rows < split
    int split;
};

// Rows [row0, row0 + n) of a launch ending at R1: valid rows and key limits.
__device__ __forceinline__ void flat_rows(long long row0, long long R1, long long T, int& nq, long long& khi,
                                          long long& khi_lo, int& split) {
    if (row0 >= R1) {
        nq = 0; khi = khi_lo = 0; split = 0;
        return;
    }
    const long long last = (row0 + kBM < R1 ? row0 + kBM : R1) - 1;
    nq = (int)(last - row0 + 1);
    const long long fl = last / T, ff = row0 / T;
    khi = (fl + 1) * T;
    split = ff != fl ? (int)(fl * T - row0) : 0;
    khi_lo = (ff + 1) * T;
}

__device__ __forceinline__ PairWork decode_pair(const PairParams& P, uint32_t rank) {
    PairWork w;
    const int cluster = blockIdx.x >> 1;
    const int h_local = cluster / P.items_per_head;
    const int i = cluster % P.items_per_head;
    w.head = P.head0 + h_local;
    const long long T = P.T;
    long long khi0, khi1;
    if (P.flat) {
        const long long R0 = (long long)P.q_frame0 * T;
        const long long R1 = (long long)(P.q_frame0 + P.frames) * T;
        const long long b = (long long)(P.items_per_head - 1 - i);   // longest first
        const long long pair0 = R0 + b * 2 * kBM;
        w.klo = 0;
        int nq0, nq1, s0, s1;
        long long lo0, lo1;
        flat_rows(pair0, R1, T, nq0, khi0, lo0, s0);
        flat_rows(pair0 + kBM, R1, T, nq1, khi1, lo1, s1);
        w.row0 = pair0 + (long long)rank * kBM;
        w.nq = rank ? nq1 : nq0;
        w.my_khi = rank ? khi1 : khi0;
        w.my_khi_lo = rank ? lo1 : lo0;
        w.split = rank ? s1 : s0;
        if (nq1 == 0) khi1 = khi0;
    } else {
        // item = (frame, 256-row block), longest key span first
        const int fr = i / P.n_blk, blk = i % P.n_blk;
        const int f = P.q_frame0 + P.frames - 1 - fr;
        if (P.mode == 0) {
            w.klo = (long long)f * T;
        } else {
            const int base = P.window > 0 ? (f - P.window + 1 > 0 ? f - P.window + 1 : 0) : 0;
            w.klo = (long long)base * T;
        }
        const long long in0 = (long long)blk * 2 * kBM + (long long)rank * kBM;   // row within the frame
        w.row0 = (long long)f * T + in0;
        const long long left = T - in0;
        w.nq = left <= 0 ? 0 : (int)(left < kBM ? left : kBM);
        khi0 = khi1 = (long long)(f + 1) * T;
        w.my_khi = w.my_khi_lo = khi0;
        w.split = 0;
    }
    w.khi = khi0 > khi1 ? khi0 : khi1;
    w.n_tiles = w.khi > w.klo ? (int)((w.khi - w.klo + kBN - 1) / kBN) : 0;
    return w;
}

// ------------------------------------------------------------ producer
// Stages rows [r0, r0 + kRows) of the key range (rows >= khi are padding,
// zero-filled) of one operand into a kPanels x [kRows][64] swizzled tile:
// panel p holds columns col + 64p of the base tensor (arena: acol + 64p).
// Lane l classifies rows 4l..4l+3 (lanes past kRows/4 take no part); lanes
// 2g and 2g+1 form 8-row group g.  The caller has waited for the stage to be
// free; this arms `full` with the tile's TMA bytes and arrives on it once.
template <int kRows, int kPanels>
__device__ __forceinline__ void stage_tile(const PairParams& P, const PairMaps& maps, const CUtensorMap* base_maps,
                                           const __nv_bfloat16* base, int col, int acol, long long r0,
                                           long long khi, const long long (&m_in)[4], uint8_t* dst_tile,
                                           uint64_t* full, int lane) {
    constexpr int kGroups = kRows / 8;
    constexpr uint32_t kPanelBytes = (uint32_t)kRows * 128;
    constexpr unsigned kActive = kRows >= 128 ? 0xffffffffu : ((1u << (kRows / 4)) - 1u);
    constexpr int kWholeKind = kRows == 128 ? 4 : kRows == 64 ? 3 : kRows == 32 ? 2 : kRows == 16 ? 1 : 0;
    const bool active = ((kActive >> lane) & 1u) != 0;
    long long m[4] = {m_in[0], m_in[1], m_in[2], m_in[3]};
    bool pad[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        pad[i] = !active || r0 + 4 * lane + i >= khi;
        if (m[i] >= P.arena_rows || (m[i] >= 0 && !P.arena)) {
            atomicOr(P.status, KVP_STATUS_MAP);
            m[i] = -1;   // out-of-range entry: read the base row
        }
        if (!active) m[i] = -1;
    }
    const bool all_neg = m[0] < 0 && m[1] < 0 && m[2] < 0 && m[3] < 0;
    const bool asc = !pad[3] && m[0] >= 0 && m[1] == m[0] + 1 && m[2] == m[0] + 2 && m[3] == m[0] + 3;
    const bool p_neg = __shfl_xor_sync(0xffffffffu, all_neg, 1);
    const bool p_asc = __shfl_xor_sync(0xffffffffu, asc, 1);
    const long long p_m0 = __shfl_xor_sync(0xffffffffu, m[0], 1);
    const bool even = (lane & 1) == 0;
    const bool p_pad0 = __shfl_xor_sync(0xffffffffu, pad[0], 1);
    const bool group_pad = even ? pad[0] : p_pad0;
    const bool g_base = active && all_neg && p_neg && !group_pad;
    const bool g_arena = active && P.arena_boxes > 0 && asc && p_asc &&
                         (even ? p_m0 == m[0] + 4 : m[0] == p_m0 + 4);
    const bool all_arena = !pad[3] && m[0] >= 0 && m[1] >= 0 && m[2] >= 0 && m[3] >= 0;
    const bool p_all_arena = __shfl_xor_sync(0xffffffffu, all_arena, 1);
    const bool g_gather = active && P.arena_gather && all_arena && p_all_arena && !g_arena;
    const unsigned base_mask = __ballot_sync(0xffffffffu, g_base);
    const unsigned arena_mask = __ballot_sync(0xffffffffu, g_arena);
    const unsigned gather_mask = __ballot_sync(0xffffffffu, g_gather);
    const unsigned mixed_mask = ~(base_mask | arena_mask | gather_mask) & kActive;
    const bool whole_base = (__ballot_sync(0xffffffffu, all_neg) & kActive) == kActive &&
                            P.base_boxes > kWholeKind;
    const long long prev_m0 = __shfl_up_sync(0xffffffffu, m[0], 2);
    const bool cont = even && lane >= 2 &&
        ((g_base && ((base_mask >> (lane - 2)) & 1u)) ||
         (g_arena && ((arena_mask >> (lane - 2)) & 1u) && m[0] == prev_m0 + 8));
    const unsigned cont_mask = __ballot_sync(0xffffffffu, cont);
    if (lane == 0) {
        uint32_t bytes = 0;
        if (whole_base) {
            bytes = kPanels * kPanelBytes;
        } else {
            for (int g = 0; g < kGroups; ++g)
                if (((base_mask | arena_mask | gather_mask) >> (2 * g)) & 1u) bytes += kPanels * kGroupPanel;
        }
        mbar_expect_tx(full, bytes);
        if (whole_base)
            for (int p = 0; p < kPanels; ++p)
                tma_load_2d(dst_tile + p * kPanelBytes, &base_maps[kWholeKind], col + 64 * p, (int)r0, full);
    }
    __syncwarp();  // expect_tx is registered before any lane issues a group load
    if (!whole_base) {
        if (even && (g_base || g_arena) && !cont) {
            const int g = lane >> 1;
            int len = 1;
            while (g + len < kGroups && ((cont_mask >> (2 * (g + len))) & 1u)) ++len;
            const CUtensorMap* mp = g_base ? base_maps : maps.a;
            const int kinds = g_base ? P.base_boxes : P.arena_boxes;
            for (int off = 0; off < len;) {
                int kind = 0;
                while (kind + 1 < kinds && (2 << kind) <= len - off) ++kind;
                const int row = g_base ? (int)(r0 + 8 * (g + off)) : (int)(m[0] + 8 * off);
                const int c = g_base ? col : acol;
                for (int p = 0; p < kPanels; ++p)
                    tma_load_2d(dst_tile + p * kPanelBytes + (g + off) * kGroupPanel, &mp[kind], c + 64 * p, row,
                                full);
                off += 1 << kind;
            }
        }
        if (g_gather) {
            const int g = lane >> 1;
            const uint32_t half = (lane & 1) ? 4u * 128u : 0u;
            for (int p = 0; p < kPanels; ++p)
                tma_gather4(dst_tile + p * kPanelBytes + g * kGroupPanel + half, &maps.a1, acol + 64 * p,
                            (int)m[0], (int)m[1], (int)m[2], (int)m[3], full);
        }
        // Mixed / padding groups: 16-byte cp.async per (panel, row, chunk),
        // every group in flight at once, then one wait.
        unsigned mm = mixed_mask & 0x55555555u;
        const unsigned any_mixed = mm;
        while (mm) {
            const int g = __ffs(mm) >> 1;
            mm &= mm - 1;
            const long long e[4] = {
                __shfl_sync(0xffffffffu, m[0], 2 * g), __shfl_sync(0xffffffffu, m[1], 2 * g),
                __shfl_sync(0xffffffffu, m[2], 2 * g), __shfl_sync(0xffffffffu, m[3], 2 * g)};
            const long long f4[4] = {
                __shfl_sync(0xffffffffu, m[0], 2 * g + 1), __shfl_sync(0xffffffffu, m[1], 2 * g + 1),
                __shfl_sync(0xffffffffu, m[2], 2 * g + 1), __shfl_sync(0xffffffffu, m[3], 2 * g + 1)};
#pragma unroll
            for (int c = lane; c < 64 * kPanels; c += 32) {
                const int pnl = c >> 6, rr = (c >> 3) & 7, chunk = c & 7;
                const long long m_row = rr < 4 ? e[rr] : f4[rr - 4];
                const int row_in_tile = 8 * g + rr;
                const long long key = r0 + row_in_tile;
                const bool is_pad = key >= khi;
                const __nv_bfloat16* src = is_pad ? base
                    : m_row >= 0 ? P.arena + (size_t)m_row * 2 * P.D + acol + 64 * pnl
                                 : base + (size_t)key * P.D + col + 64 * pnl;
                cp_async16(dst_tile + pnl * kPanelBytes + sw128_off(row_in_tile, chunk),
                           reinterpret_cast<const uint4*>(src) + (is_pad ? 0 : chunk), is_pad ? 0u : 16u);
            }
        }
        if (any_mixed) {
            cp_async_wait_all();
            fence_proxy_async_smem();
        }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(full);
}

// ------------------------------------------------------------------ kernel
__global__ void __launch_bounds__(kThreads, 1)
attn_pair_sm100_kernel(const __grid_constant__ PairMaps maps, const __grid_constant__ PairParams P) {
    extern __shared__ uint8_t smem_raw[];
    // Same layout in both CTAs (the MMA reads the peer's tiles at the same
    // offsets), so both take this exit together.
    if (reinterpret_cast<uintptr_t>(smem_raw) & 1023) {
        if (threadIdx.x == 0) atomicOr(P.status, KVP_STATUS_ALIGN);
        return;
    }
    PairSmem& sm = *reinterpret_cast<PairSmem*>(smem_raw);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cta_rank();
    const bool leader = rank == 0;
    const PairWork w = decode_pair(P, rank);
    const int n_tiles = w.n_tiles;

    if (threadIdx.x == 0) {
        mbar_init(&sm.bar_q, leader ? 2 : 1);
        for (int s = 0; s < kKStages; ++s) {
            mbar_init(&sm.bar_kfull[s], leader ? 2 : 1);
            mbar_init(&sm.bar_kempty[s], 1);
        }
        for (int s = 0; s < kVStages; ++s) {
            mbar_init(&sm.bar_vfull[s], leader ? 2 : 1);
            mbar_init(&sm.bar_vempty[s], 1);
        }
        for (int b = 0; b < kSBufs; ++b) {
            mbar_init(&sm.bar_s_full[b], 1);
            mbar_init(&sm.bar_p_full[b], 16);   // eight softmax warps in each CTA
        }
        for (int q = 0; q < 4; ++q) mbar_init(&sm.bar_xch[q], 2);
        mbar_init(&sm.bar_mma_done, 1);
        mbar_init(&sm.bar_exit, 1);
        sm.abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_proxy_async_smem();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&sm.tmem_base)), "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    // Both CTAs' barriers are initialised before any remote arrival.
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    const int D = P.D;
    const int hcol = w.head * kDH;

    if (warp < 4) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsLow));
        if (warp == 0 || warp == 2) {
            // ============================ producers ===========================
            const int op = warp == 0 ? 0 : 1;
            if (op == 0 && lane == 0 && n_tiles > 0) {
                // Q: this CTA's 128 rows, 8-row groups that start inside the tensor.
                uint32_t qbytes = 0;
                for (int g = 0; g < kBM / 8; ++g)
                    if (w.row0 + 8 * g < P.q_rows) qbytes += 2 * kGroupPanel;
                mbar_arrive_expect_tx(&sm.bar_q, qbytes);
                for (int g = 0; g < kBM / 8; ++g) {
                    if (w.row0 + 8 * g >= P.q_rows) break;
                    for (int p = 0; p < 2; ++p)
                        tma_load_2d(sm.q + p * kQPanel + g * kGroupPanel, &maps.q8, hcol + 64 * p,
                                    (int)(w.row0 + 8 * g), &sm.bar_q);
                }
            }
            const int n_st = op == 0 ? kKStages : kVStages;
            uint64_t* bar_full = op == 0 ? sm.bar_kfull : sm.bar_vfull;
            uint64_t* bar_empty = op == 0 ? sm.bar_kempty : sm.bar_vempty;
            const CUtensorMap* base_maps = maps.kv[op];
            const __nv_bfloat16* base = op == 0 ? P.k : P.v;
            // K: this CTA's 64 keys of the tile, all 128 dims (two panels);
            // V: all 128 keys, this CTA's 64 dims (one panel).
            const int col = op == 0 ? hcol : hcol + 64 * (int)rank;
            const int acol = op == 0 ? hcol : D + hcol + 64 * (int)rank;
            const long long key_off = op == 0 ? 64LL * rank : 0;
            const int rows = op == 0 ? 64 : 128;
            int last_armed = -1;
            auto map_rows = [&](int jj, long long (&mm)[4]) {
                const long long rr0 = w.klo + (long long)jj * kBN + key_off;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const long long row = rr0 + 4 * lane + i;
                    mm[i] = (jj < n_tiles && 4 * lane < rows && row < w.khi && P.kvmap) ? __ldg(P.kvmap + row) : -1;
                }
            };
            long long m_next[4];
            map_rows(0, m_next);
            for (int j = 0; j < n_tiles; ++j) {
                long long m[4] = {m_next[0], m_next[1], m_next[2], m_next[3]};
                map_rows(j + 1, m_next);
                const int s = j % n_st;
                const uint32_t ph = (uint32_t)(j / n_st) & 1u;
                if (!pair_warp_wait(&bar_empty[s], ph ^ 1u, sm, P.status)) break;
                const long long r0 = w.klo + (long long)j * kBN + key_off;
                if (op == 0)
                    stage_tile<64, 2>(P, maps, base_maps, base, col, acol, r0, w.khi, m,
                                      sm.k[s], &bar_full[s], lane);
                else
                    stage_tile<128, 1>(P, maps, base_maps, base, col, acol, r0, w.khi, m,
                                       sm.v[s], &bar_full[s], lane);
                last_armed = j;
            }
            // Drain: never leave TMA writes in flight into a CTA that is exiting.
            if (lane == 0 && sm.abort_flag) {
                for (int j = last_armed - n_st + 1; j <= last_armed; ++j) {
                    if (j < 0) continue;
                    const unsigned long long t0 = globaltimer();
                    while (!mbar_try_wait(&bar_full[j % n_st], (uint32_t)(j / n_st) & 1u) &&
                           globaltimer() - t0 < kWaitNs) {
                    }
                }
                if (op == 0 && n_tiles > 0) {
                    const unsigned long long t0 = globaltimer();
                    while (!mbar_try_wait(&sm.bar_q, 0) && globaltimer() - t0 < kWaitNs) {
                    }
                }
            }
        } else if (warp == 3) {
            // ========================= relay (peer CTA) =======================
            // The leader's MMAs read this CTA's Q, K and V halves: forward the
            // completion of each local load to the leader's barrier.
            if (!leader && lane == 0 && n_tiles > 0) {
                bool ok = pair_wait(&sm.bar_q, 0, sm, P.status);
                if (ok) arrive_cluster(peer_addr(&sm.bar_q, 0));
                for (int j = 0; ok && j < n_tiles; ++j) {
                    const int ks = j % kKStages, vs = j % kVStages;
                    ok = pair_wait(&sm.bar_kfull[ks], (uint32_t)(j / kKStages) & 1u, sm, P.status);
                    if (!ok) break;
                    arrive_cluster(peer_addr(&sm.bar_kfull[ks], 0));
                    ok = pair_wait(&sm.bar_vfull[vs], (uint32_t)(j / kVStages) & 1u, sm, P.status);
                    if (!ok) break;
                    arrive_cluster(peer_addr(&sm.bar_vfull[vs], 0));
                }
            }
            __syncwarp();
        } else if (warp == 1 && leader) {
            // ============================ MMA issuer ==========================
            // S(j) into buffer j%3, then PV(j-2): P(j) is read four GEMMs
            // after S(j) was issued.  S(j) overwrites the buffer of P(j-3),
            // whose PV was issued one step earlier (MMAs run in issue order).
            if (lane == 0) {
                constexpr uint32_t idS = idesc_pair(false);
                constexpr uint32_t idO = idesc_pair(true);
                const uint64_t dq = sw128_desc(smem_u32(sm.q), 16, 1024);
                const uint64_t dk = sw128_desc(smem_u32(sm.k[0]), 16, 1024);
                const uint64_t dv = sw128_desc(smem_u32(sm.v[0]), kVStageBytes, 1024);
                const uint32_t o_tm = tmem + 384u;
                bool ok = n_tiles == 0 || pair_wait(&sm.bar_q, 0, sm, P.status);
                for (int j = 0; ok && j < n_tiles + 2; ++j) {
                    if (j < n_tiles) {
                        const int ks = j % kKStages;
                        if (!pair_wait(&sm.bar_kfull[ks], (uint32_t)(j / kKStages) & 1u, sm, P.status)) { ok = false; break; }
                        tc_fence_after();
                        pair_gemm_s(tmem + 128u * (uint32_t)(j % kSBufs), dq, dk + (uint64_t)ks * (kKStageBytes >> 4),
                                    idS);
                        tc_commit_pair(&sm.bar_s_full[j % kSBufs]);
                    }
                    const int jj = j - 2;
                    if (jj >= 0) {
                        const int vs = jj % kVStages;
                        if (!pair_wait(&sm.bar_vfull[vs], (uint32_t)(jj / kVStages) & 1u, sm, P.status)) { ok = false; break; }
                        if (!pair_wait(&sm.bar_p_full[jj % kSBufs], (uint32_t)(jj / kSBufs) & 1u, sm, P.status)) { ok = false; break; }
                        tc_fence_after();
                        pair_gemm_pv(o_tm, tmem + 128u * (uint32_t)(jj % kSBufs),
                                     dv + (uint64_t)vs * (kVStageBytes >> 4), idO, jj > 0 ? 1u : 0u);
                        tc_commit_pair(&sm.bar_vempty[vs]);
                    }
                }
                // Every issued MMA lands before TMEM is freed.
                asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 smem_u32(&sm.bar_mma_done)) : "memory");
                const unsigned long long t0 = globaltimer();
                while (!mbar_try_wait(&sm.bar_mma_done, 0) && globaltimer() - t0 < kWaitNs) {
                }
            }
            __syncwarp();
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsHigh));
        // ========================== softmax + epilogue ========================
        const int half = (warp - 4) >> 2;               // column half of each S tile
        const int quarter = warp & 3;                   // row quarter (TMEM lanes)
        const int row = quarter * 32 + lane;
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        const uint32_t o_tm = tmem + lane_base + 384u + 64u * (uint32_t)half;
        const long long my_khi = row < w.split ? w.my_khi_lo : w.my_khi;
        const float sl2 = P.scale_log2;
        float m_run = -INFINITY, l_run = 0.f;           // l over this half's columns
        uint32_t n_xch = 0;
        bool ok = true;
        // Swaps one value per row with the other half's warp of this row
        // quarter (double-buffered by exchange parity: a warp runs at most one
        // exchange ahead of its partner).
        auto exchange = [&](float mine, float& other) -> bool {
            const uint32_t par = n_xch & 1u;
            sm.xch[par][half][row] = mine;
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.bar_xch[quarter]);
            if (!pair_warp_wait(&sm.bar_xch[quarter], par, sm, P.status)) return false;
            other = sm.xch[par][half ^ 1][row];
            ++n_xch;
            return true;
        };
        for (int j = 0; j < n_tiles; ++j) {
            const int buf = j % kSBufs;
            const uint32_t s_tm = tmem + lane_base + 128u * (uint32_t)buf + 64u * (uint32_t)half;
            if (!pair_warp_wait(&sm.bar_s_full[buf], (uint32_t)(j / kSBufs) & 1u, sm, P.status)) { ok = false; break; }
            tc_fence_after();
            // S(j) landed: both halves of K(j) are read (in both CTAs).
            if (warp == 4 && lane == 0) mbar_arrive(&sm.bar_kempty[j % kKStages]);
            const long long left_ll = my_khi - (w.klo + (long long)j * kBN) - 64LL * half;
            const int left = left_ll >= 64 ? 64 : (left_ll < 0 ? 0 : (int)left_ll);
            const bool masked = !__all_sync(0xffffffffu, left == 64);
            uint32_t pk[32];
            float rsum = 0.f, m_new = m_run, other = 0.f;
            if (j > 0) {
                rsum = masked ? exp_row<true, 2>(s_tm, m_run, sl2, left, pk)
                              : exp_row<false, 2>(s_tm, m_run, sl2, left, pk);
                // A half whose sum overgrows (the row max rose by more than 8
                // in log2 units) makes both halves of the row start again
                // from the new max.
                const float flag = rsum <= kRedoSum ? 0.f : 1.f;
                if (!exchange(flag, other)) { ok = false; break; }
                const bool redo = flag != 0.f || other != 0.f;
                if (__any_sync(0xffffffffu, redo)) {
                    const float tmax = masked ? max_row<true, 2>(s_tm, left) : max_row<false, 2>(s_tm, left);
                    if (!exchange(tmax, other)) { ok = false; break; }
                    const float t01 = half == 0 ? fmaxf(tmax, other) : fmaxf(other, tmax);
                    if (redo) m_new = fmaxf(m_run, t01 * sl2);
                    rsum = masked ? exp_row<true, 2>(s_tm, m_new, sl2, left, pk)
                                  : exp_row<false, 2>(s_tm, m_new, sl2, left, pk);
                }
            } else {
                const float tmax = masked ? max_row<true, 2>(s_tm, left) : max_row<false, 2>(s_tm, left);
                if (!exchange(tmax, other)) { ok = false; break; }
                const float t01 = half == 0 ? fmaxf(tmax, other) : fmaxf(other, tmax);
                m_new = fmaxf(m_run, t01 * sl2);
                rsum = masked ? exp_row<true, 2>(s_tm, m_new, sl2, left, pk)
                              : exp_row<false, 2>(s_tm, m_new, sl2, left, pk);
            }
            const float alpha = m_new == m_run ? 1.f : ex2_approx(m_run - m_new);
            l_run = l_run * alpha + rsum;
            m_run = m_new;
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
                // O must hold PV(j-1) complete before it is rescaled.
                const int pj = j - 1;
                if (!pair_warp_wait(&sm.bar_vempty[pj % kVStages], (uint32_t)(pj / kVStages) & 1u, sm, P.status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c2 = 0; c2 < 2; ++c2) {
                    uint32_t o[32];
                    KVP_TMEM_LD32(o_tm + 32 * c2, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 32; ++c)
                        o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
                    KVP_TMEM_ST32(o_tm + 32 * c2, o);
                }
            }
            // P of this half's 64 keys -> the first 32 columns of its half of S
            KVP_TMEM_ST32(s_tm, pk);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) arrive_cluster(peer_addr(&sm.bar_p_full[buf], 0));
        }
        // Epilogue: O / (l_0 + l_1) -> bf16 once PV(n-1) (and with it every PV) landed.
        float l_other = 0.f;
        if (ok && n_tiles > 0 && exchange(l_run, l_other)) {
            const int pj = n_tiles - 1;
            if (pair_warp_wait(&sm.bar_vempty[pj % kVStages], (uint32_t)(pj / kVStages) & 1u, sm, P.status)) {
                tc_fence_after();
                const float inv = 1.f / (half == 0 ? l_run + l_other : l_other + l_run);
                __nv_bfloat16* dst = P.out + (size_t)(w.row0 + row) * D + hcol + 64 * half;
#pragma unroll
                for (int c2 = 0; c2 < 2; ++c2) {
                    uint32_t o[32];
                    KVP_TMEM_LD32(o_tm + 32 * c2, o);
                    tmem_wait_ld();
                    if (row < w.nq) {
#pragma unroll
                        for (int c = 0; c < 32; c += 8) {
                            uint4 pkt;
                            pkt.x = pack_bf16(__uint_as_float(o[c]) * inv, __uint_as_float(o[c + 1]) * inv);
                            pkt.y = pack_bf16(__uint_as_float(o[c + 2]) * inv, __uint_as_float(o[c + 3]) * inv);
                            pkt.z = pack_bf16(__uint_as_float(o[c + 4]) * inv, __uint_as_float(o[c + 5]) * inv);
                            pkt.w = pack_bf16(__uint_as_float(o[c + 6]) * inv, __uint_as_float(o[c + 7]) * inv);
                            *reinterpret_cast<uint4*>(dst + 32 * c2 + c) = pkt;
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    // Leave together: each CTA tells the peer it no longer touches the
    // peer's memory, then waits (bounded) for the same word from the peer.
    if (threadIdx.x == 0) {
        arrive_cluster(peer_addr(&sm.bar_exit, rank ^ 1u));
        const unsigned long long t0 = globaltimer();
        bool done = false;
        while (!(done = try_wait_cluster(&sm.bar_exit, 0)) && globaltimer() - t0 < kWaitNs) {
        }
        if (!done) atomicOr(P.status, KVP_STATUS_TIMEOUT);
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}

}  // namespace

bool attn_pair_supported(const AttnDesc& d) {
    return d.head_dim == kDH;
}

int launch_attn_bf16_pair(const LayerIO& io, const AttnDesc& d, int* d_status, cudaStream_t stream) {
    const long long T = d.tokens;
    const int D = d.heads * kDH;
    const int rc_check = check_attn_bf16(io, d);
    if (rc_check != KVP_OK) return rc_check;
    if (!d_status) {
        set_error("attn_bf16_pair: no status word");
        return KVP_ERR_ARG;
    }
    PairMaps maps;
    std::memset(&maps, 0, sizeof maps);
    int base_boxes = 0, arena_boxes = 0;
    while (base_boxes < kBoxKinds && (8LL << base_boxes) <= io.kv_rows) ++base_boxes;
    if (io.arena)
        while (arena_boxes < kBoxKinds && (8LL << arena_boxes) <= io.arena_rows) ++arena_boxes;
    int rc = make_bf16_tensor_map(&maps.q8, io.q, io.q_rows, D, D, 8);
    for (int i = 0; !rc && i < kBoxKinds; ++i) {
        const uint32_t h = 8u << (i < base_boxes ? i : 0);
        rc = make_bf16_tensor_map(&maps.kv[0][i], io.k, io.kv_rows, D, D, h);
        if (!rc) rc = make_bf16_tensor_map(&maps.kv[1][i], io.v, io.kv_rows, D, D, h);
        if (!rc && arena_boxes)
            rc = make_bf16_tensor_map(&maps.a[i], io.arena, io.arena_rows, 2 * D, 2 * D,
                                      8u << (i < arena_boxes ? i : 0));
    }
    if (!rc && arena_boxes) rc = make_bf16_tensor_map(&maps.a1, io.arena, io.arena_rows, 2 * D, 2 * D, 1);
    if (rc) return rc;
    if (base_boxes == 0 || io.q_rows < 8) {
        set_error("attn_bf16_pair: Q and K/V need at least 8 rows");
        return KVP_ERR_ARG;
    }
    PairParams P;
    std::memset(&P, 0, sizeof P);
    P.k = (const __nv_bfloat16*)io.k;
    P.v = (const __nv_bfloat16*)io.v;
    P.arena = (const __nv_bfloat16*)io.arena;
    P.kvmap = io.kvmap;
    P.out = (__nv_bfloat16*)io.out;
    P.status = d_status;
    P.q_rows = io.q_rows;
    P.kv_rows = io.kv_rows;
    P.arena_rows = io.arena ? io.arena_rows : 0;
    P.D = D;
    P.T = (int)T;
    P.frames = d.frames;
    P.q_frame0 = d.q_frame0;
    P.mode = d.mode;
    P.window = d.window;
    P.head0 = d.head0;
    P.nheads = d.nheads;
    P.flat = d.flat;
    P.n_blk = (int)((T + 2 * kBM - 1) / (2 * kBM));
    P.items_per_head = d.flat ? (int)(((long long)d.frames * T + 2 * kBM - 1) / (2 * kBM))
                              : d.frames * P.n_blk;
    P.base_boxes = base_boxes;
    P.arena_boxes = arena_boxes;
    P.arena_gather = arena_boxes > 0 ? 1 : 0;
    P.scale_log2 = 1.4426950408889634f / sqrtf((float)kDH);

    const int smem = (int)sizeof(PairSmem);
    static PerDeviceOnce setup;
    const int rc_setup = setup([&](int dev) -> int {
        int optin = 0;
        KVP_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        if (smem > optin) {
            set_error("attn_bf16_pair: needs %d B of shared memory per block, device allows %d", smem, optin);
            return KVP_ERR_UNSUPPORTED;
        }
        cudaFuncAttributes fa;
        KVP_CUDA(cudaFuncGetAttributes(&fa, attn_pair_sm100_kernel));
        if ((long long)fa.numRegs * kThreads < (long long)kRegsLow * 128 + (long long)kRegsHigh * 128) {
            set_error("attn_bf16_pair: kernel built with %d registers per thread, the register split needs %d",
                      fa.numRegs, (kRegsLow * 128 + kRegsHigh * 128 + kThreads - 1) / kThreads);
            return KVP_ERR_UNSUPPORTED;
        }
        KVP_CUDA(cudaFuncSetAttribute(attn_pair_sm100_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        return KVP_OK;
    });
    if (rc_setup != KVP_OK) return rc_setup;
    const long long clusters = (long long)d.nheads * P.items_per_head;
    if (clusters <= 0 || 2 * clusters > 0x7fffffffLL) return KVP_ERR_ARG;
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof cfg);
    cfg.gridDim = dim3((unsigned)(2 * clusters), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t le = cudaLaunchKernelEx(&cfg, attn_pair_sm100_kernel, maps, P);
    if (le != cudaSuccess) return cuda_status(le, "attn_bf16_pair launch");
    return KVP_OK;
}

}  // namespace kvp
