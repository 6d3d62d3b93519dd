// BF16 remapped multi-head attention for B200 (sm_100a): tcgen05 tensor
// cores with TMEM accumulators, TMA-staged K/V resolved through the KVMap.
//
// Semantics: those of the reference's attn_forward_kernel
// (src/gated_attention_kernel.cu:34-139) in bf16 with fp32 accumulation:
// per (query row, head) softmax(q.K^T / sqrt(128)) . V over the row's key
// span, key row j read from arena row KVMap[j] (K at column h*128, V at
// column D + h*128 of a 2*D-element row) when KVMap[j] >= 0, else from the
// base K/V.  Arena rows are copies of base rows and the arithmetic below
// never depends on where a row came from, so outputs are bitwise identical
// across policies.
//
// CTA = two 128-row query tiles (Q0, Q1) x one head; both tiles consume the
// same stream of 128-key K/V tiles, so every staged K/V tile feeds four
// 128x128x128 GEMMs.  Warp roles (384 threads):
//   warp 0      Q loads and the K producer, warp 2 the V producer: each reads
//               the KVMap for its 128-key tile, classifies every 8-row group
//               (all base / one ascending arena run / all arena in any slot
//               order / mixed) and stages the tile with TMA: one 128-row box
//               per panel when the whole tile is base rows, power-of-two
//               boxes per run otherwise, two four-row TMA gathers per panel
//               for scattered arena groups; mixed groups and padding are
//               copied with 16-byte cp.async into the same 128B-swizzled
//               layout
//   warp 1      TMEM allocation and the single-thread MMA issuer, in the
//               order S0_j, PV1_{j-1}, S1_j, PV0_j: while one tile's softmax
//               runs, the tensor cores work on the other tile.  Each GEMM is
//               one asm block of eight MMAs.
//   warp 3      idle (its warpgroup gives registers to the softmax:
//               setmaxnreg 104 / 200)
//   warps 4-7   softmax of Q0, warps 8-11 softmax of Q1: thread i owns query
//               row i (TMEM lane i) and all 128 columns of each S tile.
//               Exponentials are computed with the running max first; only a
//               row whose tile sum exceeds 256 (its max grew by more than 8 in
//               log2 units) recomputes with the new max and rescales O.  P is
//               written back into the first 64 columns of its own S
//               accumulator as packed bf16 and read from there by the PV MMA.
//               The warpgroup of the tile with the full key span also
//               releases the K/V stages once its S tile lands.  The same
//               warps run the epilogue O / l -> bf16 -> global.
// TMEM columns: S0 [0,128), S1 [128,256), O0 [256,384), O1 [384,512).
// Shared memory: Q0, Q1 (32 KB each), a K ring of two and a V ring of three
// 32 KB stages.  Every mbarrier wait is bounded (about one second of
// %globaltimer); on expiry the CTA records KVP_STATUS_TIMEOUT in the status
// word and unwinds without hanging.
#include <cuda.h>
#include <cuda_bf16.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "attn_pair_sm100.h"
#include "attn_sm100.h"
#include "kvp_common.h"
#include "attn_softmax_sm100.cuh"
#include "sm100_ptx.h"

namespace kvp {

namespace {

using namespace ptx;
using namespace attn_dev;

constexpr int kBM = 128;           // query rows per query tile
constexpr int kQTiles = 2;         // query tiles per CTA
constexpr int kBN = 128;           // keys per tile
constexpr int kDH = 128;           // head dim
constexpr int kKStages = 2;        // depth of the K ring
constexpr int kVStages = 3;        // depth of the V ring (V_j stays until PV1_j, one tile later)
constexpr int kThreads = 384;      // producers, MMA, 1 idle, 2 x 4 softmax warps
constexpr uint32_t kPanel = 128 * 128;        // one [128 rows][64 bf16] swizzled panel
constexpr uint32_t kTileBytes = 2 * kPanel;   // [128][128] bf16
constexpr uint32_t kGroupPanel = 8 * 128;     // one 8-row group of a panel
constexpr int kRegsLow = 104;      // registers per thread, warps 0-3 (producers, MMA)
constexpr int kRegsHigh = 200;     // registers per thread, warps 4-11 (softmax)
static_assert(kRegsLow * 128 + 2 * kRegsHigh * 128 <= 65536, "register split exceeds the SM");
constexpr float kRedoSum = 256.f;  // a tile row sum above this recomputes with the new max

struct __align__(1024) Smem {
    uint8_t q[kQTiles][kTileBytes];
    uint8_t k[kKStages][kTileBytes];
    uint8_t v[kVStages][kTileBytes];
    uint64_t bar_q[kQTiles];
    uint64_t bar_kfull[kKStages];
    uint64_t bar_kempty[kKStages];
    uint64_t bar_vfull[kVStages];
    uint64_t bar_vempty[kVStages];
    uint64_t bar_s_full[kQTiles];   // S_q(j) landed (and, by issue order, PV_q(j-1) too)
    uint64_t bar_p_full[kQTiles];   // P_q(j) in TMEM, S_q(j) read, O_q rescaled
    uint64_t bar_o_done[kQTiles];   // last PV_q landed
    uint64_t bar_mma_done;          // every issued MMA landed (TMEM may be freed)
    uint32_t tmem_base;
    int abort_flag;
};

constexpr int kBoxKinds = 5;       // TMA box heights 8, 16, 32, 64, 128 rows

struct TmaMaps {
    CUtensorMap q8;                 // Q [q_rows][D], box 64 x 8
    CUtensorMap kv[2][kBoxKinds];   // K / V [kv_rows][D], box 64 x (8 << i)
    CUtensorMap a[kBoxKinds];       // arena [arena_rows][2D], box 64 x (8 << i)
    CUtensorMap a1;                 // arena, box 64 x 1 (TMA gather of scattered slots)
};

// One layer's tensors (a launch covers one or several of them: a segment
// table).  Segment i owns CTAs [cta0, cta0 + nheads * items_per_head).
struct Seg {
    TmaMaps maps;
    const __nv_bfloat16* k;      // base rows, for mixed groups
    const __nv_bfloat16* v;
    const __nv_bfloat16* arena;
    const long long* kvmap;
    __nv_bfloat16* out;
    long long q_rows, kv_rows, arena_rows;
    int D, head0, nheads, cta0, q_frame0;
    int base_boxes, arena_boxes;   // box kinds usable (heights <= tensor rows); 0 = no arena TMA
    int arena_gather;              // 1 = maps.a1 is encoded (scattered arena groups by TMA gather)
};

// A segment's scalars, copied into registers at the start of the kernel: a
// launch over several segments indexes its table with the CTA's segment, and
// reads through that runtime address would otherwise repeat in the loops.
struct SegHot {
    const __nv_bfloat16* k;
    const __nv_bfloat16* v;
    const __nv_bfloat16* arena;
    const long long* kvmap;
    __nv_bfloat16* out;
    long long q_rows, kv_rows, arena_rows;
    int D, head0, nheads, cta0, q_frame0, base_boxes, arena_boxes, arena_gather;
};

__device__ __forceinline__ SegHot seg_hot(const Seg& g) {
    return SegHot{g.k, g.v, g.arena, g.kvmap, g.out, g.q_rows, g.kv_rows, g.arena_rows,
                  g.D, g.head0, g.nheads, g.cta0, g.q_frame0, g.base_boxes, g.arena_boxes,
                  g.arena_gather};
}

// Segments per launch: 1 for kvp_attn_bf16, up to kMaxSegs for
// kvp_attn_bf16_multi (the table is a kernel parameter, 2.3 KB a segment).
constexpr int kMaxSegs = kAttnSegsPerLaunch;

template <int kSegs>
struct SegTable {
    Seg seg[kSegs];
};

// What every segment of a launch shares: the frames and masking, the
// split workspace, the status word.
struct Params {
    int* status;
    int T, frames, mode, window, flat, items_per_head, n_qt, n_pairs, n_segs;
    float scale_log2;
    // Key-range split (per-frame tiling only): splits > 1 writes fp32 partial
    // (O, m, l) to ws instead of bf16 output; combine_splits_kernel merges.
    int splits;
    float* ws;
    long long ws_rows;             // query rows of the launch (frames * T)
};

// ------------------------------------------------------------- primitives
// (mbarriers, TMA, tcgen05, bounded waits: sm100_ptx.h)
// One 128x128x128 GEMM as eight back-to-back K16 MMAs, issued in two asm
// blocks (steps 0-5, then 6-7) so the issuer can test the next GEMM's
// barriers while the first six are queued.  The descriptors of steps 1..7
// are immediate offsets of step 0's: nothing but an add sits between two MMA
// issues, and the tensor core's shallow instruction queue never runs dry
// inside a GEMM.
//   S = Q K^T: A and B K-major, 128B swizzle, two 64-column panels 16 KB
//   apart: step ks starts (ks>>2)*16384 + (ks&3)*32 bytes in, i.e. adds
//   (ks>>2)*1024 + (ks&3)*2 to the 16-byte address field.
__device__ __forceinline__ void tc_gemm_ss_head(uint32_t d_tmem, uint64_t a0, uint64_t b0, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred pf, pt;\n\t.reg .b64 a, b;\n\t"
        "setp.ne.b32 pf, 0, 0;\n\tsetp.eq.b32 pt, 0, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, pf;\n\t"
        "add.s64 a, %1, 2;\n\tadd.s64 b, %2, 2;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, pt;\n\t"
        "add.s64 a, %1, 4;\n\tadd.s64 b, %2, 4;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, pt;\n\t"
        "add.s64 a, %1, 6;\n\tadd.s64 b, %2, 6;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, pt;\n\t"
        "add.s64 a, %1, 1024;\n\tadd.s64 b, %2, 1024;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, pt;\n\t"
        "add.s64 a, %1, 1026;\n\tadd.s64 b, %2, 1026;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, pt;\n\t}"
        ::"r"(d_tmem), "l"(a0), "l"(b0), "r"(idesc));
}
__device__ __forceinline__ void tc_gemm_ss_tail(uint32_t d_tmem, uint64_t a0, uint64_t b0, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred pt;\n\t.reg .b64 a, b;\n\t"
        "setp.eq.b32 pt, 0, 0;\n\t"
        "add.s64 a, %1, 1028;\n\tadd.s64 b, %2, 1028;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, pt;\n\t"
        "add.s64 a, %1, 1030;\n\tadd.s64 b, %2, 1030;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, pt;\n\t}"
        ::"r"(d_tmem), "l"(a0), "l"(b0), "r"(idesc));
}
//   O (+)= P V: P from TMEM (step ks at column +8*ks), V MN-major with step
//   ks 16 rows = 2048 bytes further (+128 in the address field).
__device__ __forceinline__ void tc_gemm_ts_head(uint32_t d_tmem, uint32_t a_tmem, uint64_t b0, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred pf, pt;\n\t.reg .b64 b;\n\t.reg .b32 a;\n\t"
        "setp.ne.b32 pf, %4, 0;\n\tsetp.eq.b32 pt, 0, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, pf;\n\t"
        "add.s32 a, %1, 8;\n\tadd.s64 b, %2, 128;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, pt;\n\t"
        "add.s32 a, %1, 16;\n\tadd.s64 b, %2, 256;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, pt;\n\t"
        "add.s32 a, %1, 24;\n\tadd.s64 b, %2, 384;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, pt;\n\t"
        "add.s32 a, %1, 32;\n\tadd.s64 b, %2, 512;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, pt;\n\t"
        "add.s32 a, %1, 40;\n\tadd.s64 b, %2, 640;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, pt;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b0), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void tc_gemm_ts_tail(uint32_t d_tmem, uint32_t a_tmem, uint64_t b0, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred pt;\n\t.reg .b64 b;\n\t.reg .b32 a;\n\t"
        "setp.eq.b32 pt, 0, 0;\n\t"
        "add.s32 a, %1, 48;\n\tadd.s64 b, %2, 768;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, pt;\n\t"
        "add.s32 a, %1, 56;\n\tadd.s64 b, %2, 896;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, pt;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b0), "r"(idesc));
}

// kind::f16 instruction descriptor: bf16 x bf16 -> f32, M=128, N=128.
constexpr uint32_t idesc_bf16(bool b_mn_major) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
           ((uint32_t)(128 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// --------------------------------------------------------------- work item
struct QTile {
    long long row0;      // first query row (absolute in Q/out)
    int nq;              // valid query rows (<= 128); 0 = empty tile
    int n_tiles;         // 128-key tiles this query tile consumes
    long long khi;       // key rows [klo, khi) for rows >= split
    long long khi_lo;    // key limit of rows < split (flat tiles crossing a frame)
    int split;
};

struct Work {
    int head;
    long long klo;       // first key row, shared by both query tiles
    long long khi;       // end of the staged key rows (max over the tiles)
    int n_tiles;         // K/V tiles staged (max over the tiles)
    int chunk;           // key-range chunk of this CTA (0 without a split)
    QTile t[kQTiles];
};

__device__ __forceinline__ Work decode_work(const Params& P, const SegHot& S) {
    Work w;
    const int blk = (int)blockIdx.x - S.cta0;
    const int h_local = blk / P.items_per_head;
    const int i = blk % P.items_per_head;
    w.head = S.head0 + h_local;
    w.chunk = 0;
    const long long T = P.T;
    if (P.flat) {
        const long long R0 = (long long)S.q_frame0 * T;
        const long long R1 = (long long)(S.q_frame0 + P.frames) * T;
        const long long t = (long long)(P.items_per_head - 1 - i);  // longest first
        w.klo = 0;
#pragma unroll
        for (int q = 0; q < kQTiles; ++q) {
            QTile& x = w.t[q];
            x.row0 = R0 + (t * kQTiles + q) * kBM;
            if (x.row0 >= R1) {
                x.nq = 0; x.n_tiles = 0; x.khi = x.khi_lo = 0; x.split = 0;
                continue;
            }
            const long long last = (x.row0 + kBM < R1 ? x.row0 + kBM : R1) - 1;
            x.nq = (int)(last - x.row0 + 1);
            const long long fl = last / T, ff = x.row0 / T;
            x.khi = (fl + 1) * T;
            x.split = ff != fl ? (int)(fl * T - x.row0) : 0;
            x.khi_lo = (ff + 1) * T;
        }
    } else {
        // item = (frame, query tile pair, key chunk), chunk fastest
        w.chunk = i % P.splits;
        const int ip = i / P.splits;
        const int fr = ip / P.n_pairs, pr = ip % P.n_pairs;
        const int f = S.q_frame0 + P.frames - 1 - fr;  // longest key span first
        if (P.mode == 0) {
            w.klo = (long long)f * T;
        } else {
            const int base = P.window > 0 ? (f - P.window + 1 > 0 ? f - P.window + 1 : 0) : 0;
            w.klo = (long long)base * T;
        }
#pragma unroll
        for (int q = 0; q < kQTiles; ++q) {
            QTile& x = w.t[q];
            const int qt = pr * kQTiles + q;
            x.row0 = (long long)f * T + (long long)qt * kBM;
            const long long left = T - (long long)qt * kBM;
            x.nq = qt < P.n_qt ? (int)(left < kBM ? left : kBM) : 0;
            x.khi = x.khi_lo = (long long)(f + 1) * T;
            x.split = 0;
        }
    }
    w.khi = w.klo;
    w.n_tiles = 0;
#pragma unroll
    for (int q = 0; q < kQTiles; ++q) {
        QTile& x = w.t[q];
        if (x.nq > 0) {
            x.n_tiles = (int)((x.khi - w.klo + kBN - 1) / kBN);
            if (x.khi > w.khi) w.khi = x.khi;
        } else {
            x.n_tiles = 0;
        }
        if (x.n_tiles > w.n_tiles) w.n_tiles = x.n_tiles;
    }
    if (!P.flat && P.splits > 1) {
        // Both tiles of a per-frame pair share one key span: chunk c takes
        // whole 128-key tiles [c*per, (c+1)*per).  Rows keep their own key
        // limit (x.khi) for masking; the staged range ends at the chunk.
        const int total = w.n_tiles;
        const int per = (total + P.splits - 1) / P.splits;
        const int t0 = w.chunk * per;
        const int t1 = t0 + per < total ? t0 + per : total;
        const int nt = t1 > t0 ? t1 - t0 : 0;
        const long long klo0 = w.klo;
        w.klo = klo0 + (long long)t0 * kBN;
        const long long kend = klo0 + (long long)t1 * kBN;
        w.khi = nt > 0 ? (kend < w.khi ? kend : w.khi) : w.klo;
        w.n_tiles = nt;
#pragma unroll
        for (int q = 0; q < kQTiles; ++q)
            if (w.t[q].nq > 0) w.t[q].n_tiles = nt;
    }
    return w;
}

// Stage release by the softmax: valid when the tile issuing
// the last S GEMM of every K/V step also issues the PV GEMMs of the step
// before it -- Q1 when it has the full key span (n1 == max), or Q0 alone.
// The only other case, 0 < n1 < n0, does not arise from decode_work (flat
// tiles have n1 >= n0, per-frame tiles n1 in {0, n0}); the MMA issuer then
// releases the stages itself.
__device__ __forceinline__ bool soft_release(int n0, int n1) { return !(n1 > 0 && n1 < n0); }

// ------------------------------------------------------------------ kernel
template <int kSegs>
__global__ void __launch_bounds__(kThreads, 1)
attn_bf16_sm100_kernel(const __grid_constant__ SegTable<kSegs> tab, const __grid_constant__ Params P) {
    extern __shared__ uint8_t smem_raw[];
    // The layout needs a 1024-byte aligned base (128B-swizzle atoms) and uses
    // nearly all of the 227 KB, so there is no room to realign: refuse instead.
    if (reinterpret_cast<uintptr_t>(smem_raw) & 1023) {
        if (threadIdx.x == 0) atomicOr(P.status, KVP_STATUS_ALIGN);
        return;
    }
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    int si = 0;
#pragma unroll
    for (int i = 1; i < kSegs; ++i)
        if (i < P.n_segs && (int)blockIdx.x >= tab.seg[i].cta0) si = i;
    const TmaMaps& maps = tab.seg[si].maps;
    const SegHot S = seg_hot(tab.seg[si]);
    const Work w = decode_work(P, S);
    const int n_tiles = w.n_tiles;

    if (threadIdx.x == 0) {
        for (int q = 0; q < kQTiles; ++q) {
            mbar_init(&sm.bar_q[q], 1);
            mbar_init(&sm.bar_s_full[q], 1);
            mbar_init(&sm.bar_p_full[q], 128);
            mbar_init(&sm.bar_o_done[q], 1);
        }
        for (int s = 0; s < kKStages; ++s) {
            mbar_init(&sm.bar_kfull[s], 1);
            mbar_init(&sm.bar_kempty[s], 1);
        }
        for (int s = 0; s < kVStages; ++s) {
            mbar_init(&sm.bar_vfull[s], 1);
            mbar_init(&sm.bar_vempty[s], 1);
        }
        mbar_init(&sm.bar_mma_done, 1);
        sm.abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_proxy_async_smem();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&sm.tmem_base)), "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    const int D = S.D;
    const int hcol = w.head * kDH;
    // Register split: the producer / MMA warpgroup hands registers to the two
    // softmax warpgroups.  The host checks before launch that the kernel's
    // register pool covers kRegsLow * 128 + 2 * kRegsHigh * 128, so the
    // increase never waits on registers that do not exist.
    // (Each role branch sets its own limit, so no code is compiled for both.)
    if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsLow));
    if (warp == 0 || warp == 2) {
        // ============================ producers ===============================
        // Warp 0 stages Q and the K ring, warp 2 the V ring; each reads the
        // KVMap rows of its tile itself, so K of tile j+2 can load as soon as
        // S1_j = Q1 K_j^T is done, independently of the V ring.
        const int op = warp == 0 ? 0 : 1;
        if (op == 0 && lane == 0) {
            // Q: 8-row groups that start inside the tensor come by TMA (a group
            // running past the end is zero-filled by TMA); groups wholly past
            // q_rows are not loaded -- their rows only feed output rows that are
            // never stored (S, P and O are row-independent).
#pragma unroll
            for (int q = 0; q < kQTiles; ++q) {
                if (w.t[q].n_tiles == 0) continue;
                const long long qr0 = w.t[q].row0;
                uint32_t qbytes = 0;
                for (int g = 0; g < kBM / 8; ++g)
                    if (qr0 + 8 * g < S.q_rows) qbytes += 2 * kGroupPanel;
                mbar_arrive_expect_tx(&sm.bar_q[q], qbytes);
                for (int g = 0; g < kBM / 8; ++g) {
                    if (qr0 + 8 * g >= S.q_rows) break;
                    for (int p = 0; p < 2; ++p)
                        tma_load_2d(sm.q[q] + p * kPanel + g * kGroupPanel, &maps.q8, hcol + 64 * p,
                                    (int)(qr0 + 8 * g), &sm.bar_q[q]);
                }
            }
        }
        const int n_st = op == 0 ? kKStages : kVStages;
        uint64_t* bar_full = op == 0 ? sm.bar_kfull : sm.bar_vfull;
        uint64_t* bar_empty = op == 0 ? sm.bar_kempty : sm.bar_vempty;
        uint8_t* ring = op == 0 ? sm.k[0] : sm.v[0];
        const CUtensorMap* base_maps = maps.kv[op];
        const __nv_bfloat16* base = op == 0 ? S.k : S.v;
        const int acol = (op == 0 ? 0 : D) + hcol;     // column of this operand in an arena row
        int last_armed = -1;
        // KVMap rows of a tile are read one tile ahead, so their L2 latency
        // overlaps the wait for a free stage instead of delaying the TMA issue.
        auto map_rows = [&](int jj, long long (&mm)[4]) {
            const long long rr0 = w.klo + (long long)jj * kBN;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const long long row = rr0 + 4 * lane + i;
                mm[i] = (jj < n_tiles && row < w.khi && S.kvmap) ? __ldg(S.kvmap + row) : -1;
            }
        };
        long long m_next[4];
        map_rows(0, m_next);
        for (int j = 0; j < n_tiles; ++j) {
            long long m[4] = {m_next[0], m_next[1], m_next[2], m_next[3]};
            map_rows(j + 1, m_next);
            const int s = j % n_st;
            const uint32_t ph = (uint32_t)(j / n_st) & 1u;
            if (!warp_wait(&bar_empty[s], ph ^ 1u, sm, P.status)) break;
            const long long r0 = w.klo + (long long)j * kBN;
            // Lane l classifies rows 4l..4l+3; lanes 2g, 2g+1 form 8-row group g.
            bool pad[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                pad[i] = r0 + 4 * lane + i >= w.khi;
                if (m[i] >= S.arena_rows || (m[i] >= 0 && !S.arena)) {
                    if (op == 0) atomicOr(P.status, KVP_STATUS_MAP);
                    m[i] = -1;   // out-of-range entry: read the base row
                }
            }
            const bool all_neg = m[0] < 0 && m[1] < 0 && m[2] < 0 && m[3] < 0;
            const bool asc = !pad[3] && m[0] >= 0 && m[1] == m[0] + 1 && m[2] == m[0] + 2 && m[3] == m[0] + 3;
            const bool p_neg = __shfl_xor_sync(0xffffffffu, all_neg, 1);
            const bool p_asc = __shfl_xor_sync(0xffffffffu, asc, 1);
            const long long p_m0 = __shfl_xor_sync(0xffffffffu, m[0], 1);
            const bool even = (lane & 1) == 0;
            // A group whose first row is past the key span (tail padding) is
            // zero-filled by the warp, never fetched by TMA; padding rows inside
            // a group that starts in the span are finite base rows (masked).
            const bool p_pad0 = __shfl_xor_sync(0xffffffffu, pad[0], 1);
            const bool group_pad = even ? pad[0] : p_pad0;
            const bool g_base = all_neg && p_neg && !group_pad;
            const bool g_arena = S.arena_boxes > 0 && asc && p_asc && (even ? p_m0 == m[0] + 4 : m[0] == p_m0 + 4);
            // Every row of the group in the arena, in any slot order (LIFO slot
            // reuse leaves descending runs), none of it padding: two TMA
            // gathers of four rows per panel.
            const bool all_arena = !pad[3] && m[0] >= 0 && m[1] >= 0 && m[2] >= 0 && m[3] >= 0;
            const bool p_all_arena = __shfl_xor_sync(0xffffffffu, all_arena, 1);
            const bool g_gather = S.arena_gather && all_arena && p_all_arena && !g_arena;
            const unsigned base_mask = __ballot_sync(0xffffffffu, g_base);
            const unsigned arena_mask = __ballot_sync(0xffffffffu, g_arena);
            const unsigned gather_mask = __ballot_sync(0xffffffffu, g_gather);
            const unsigned mixed_mask = ~(base_mask | arena_mask | gather_mask);
            // One 128-row box per panel when no row is remapped; the box
            // starts inside the tensor (r0 < khi <= kv_rows).
            const bool whole_base = __all_sync(0xffffffffu, all_neg) && S.base_boxes == kBoxKinds;
            // Runs: a base or arena group continues the previous group's run
            // when it is the same kind and, for arena groups, its slots follow
            // on; each run head issues power-of-two boxes for the whole run.
            const long long prev_m0 = __shfl_up_sync(0xffffffffu, m[0], 2);
            const bool cont = even && lane >= 2 &&
                ((g_base && ((base_mask >> (lane - 2)) & 1u)) ||
                 (g_arena && ((arena_mask >> (lane - 2)) & 1u) && m[0] == prev_m0 + 8));
            const unsigned cont_mask = __ballot_sync(0xffffffffu, cont);
            uint8_t* dst_tile = ring + (size_t)s * kTileBytes;
            uint64_t* full = &bar_full[s];
            if (lane == 0) {
                uint32_t bytes = 0;
                if (whole_base) {
                    bytes = kTileBytes;
                } else {
                    for (int g = 0; g < 16; ++g)
                        if (((base_mask | arena_mask | gather_mask) >> (2 * g)) & 1u) bytes += 2 * kGroupPanel;
                }
                mbar_expect_tx(full, bytes);
                if (whole_base)
                    for (int p = 0; p < 2; ++p)
                        tma_load_2d(dst_tile + p * kPanel, &base_maps[kBoxKinds - 1], hcol + 64 * p,
                                    (int)r0, full);
            }
            __syncwarp();  // expect_tx is registered before any lane issues a group load
            if (!whole_base) {
                if (even && (g_base || g_arena) && !cont) {
                    const int g = lane >> 1;
                    int len = 1;                         // groups in this run
                    while (g + len < 16 && ((cont_mask >> (2 * (g + len))) & 1u)) ++len;
                    const CUtensorMap* mp = g_base ? base_maps : maps.a;
                    const int kinds = g_base ? S.base_boxes : S.arena_boxes;
                    for (int off = 0; off < len;) {
                        int kind = 0;                    // largest box that fits the rest of the run
                        while (kind + 1 < kinds && (2 << kind) <= len - off) ++kind;
                        const int row = g_base ? (int)(r0 + 8 * (g + off)) : (int)(m[0] + 8 * off);
                        const int col = g_base ? hcol : acol;
                        for (int p = 0; p < 2; ++p)
                            tma_load_2d(dst_tile + p * kPanel + (g + off) * kGroupPanel, &mp[kind],
                                        col + 64 * p, row, full);
                        off += 1 << kind;
                    }
                }
                // Scattered arena groups: each lane of the pair gathers its own
                // four rows (rows 0-3 of the group from the even lane, 4-7 from
                // the odd one) into both panels.
                if (g_gather) {
                    const int g = lane >> 1;
                    const uint32_t half = (lane & 1) ? 4u * 128u : 0u;
                    for (int p = 0; p < 2; ++p)
                        tma_gather4(dst_tile + p * kPanel + g * kGroupPanel + half, &maps.a1, acol + 64 * p,
                                    (int)m[0], (int)m[1], (int)m[2], (int)m[3], full);
                }
                // Mixed / padding groups: lane -> (panel = lane/16, row = (lane/2)%8,
                // chunks 4*(lane%2) .. +3); one 16-byte cp.async per chunk into the
                // swizzled layout (zero-filled for padding rows), every group of
                // the tile in flight at once, then one wait.
                unsigned mm = mixed_mask & 0x55555555u;
                const int pnl = lane >> 4, rr = (lane >> 1) & 7, c0 = 4 * (lane & 1);
                while (mm) {
                    const int g = __ffs(mm) >> 1;  // bit 2g set
                    mm &= mm - 1;
                    const int row_in_tile = 8 * g + rr;
                    // Row 8g+rr is entry rr%4 of lane 2g+rr/4: fetch all four, pick one.
                    const int src_lane = 2 * g + (rr >> 2);
                    const long long e0 = __shfl_sync(0xffffffffu, m[0], src_lane);
                    const long long e1 = __shfl_sync(0xffffffffu, m[1], src_lane);
                    const long long e2 = __shfl_sync(0xffffffffu, m[2], src_lane);
                    const long long e3 = __shfl_sync(0xffffffffu, m[3], src_lane);
                    const int sel = rr & 3;
                    const long long m_row = sel == 0 ? e0 : sel == 1 ? e1 : sel == 2 ? e2 : e3;
                    const long long key = r0 + row_in_tile;
                    const bool is_pad = key >= w.khi;
                    // (a padding row reads nothing; its source is any valid address)
                    const __nv_bfloat16* src = is_pad ? base
                        : m_row >= 0 ? S.arena + (size_t)m_row * 2 * D + acol + 64 * pnl
                                     : base + (size_t)key * D + hcol + 64 * pnl;
                    uint8_t* dst = dst_tile + pnl * kPanel;
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        cp_async16(dst + sw128_off(row_in_tile, c0 + c),
                                   reinterpret_cast<const uint4*>(src) + (is_pad ? 0 : c0 + c),
                                   is_pad ? 0u : 16u);
                }
                // the copies have landed; make them visible to the tensor cores
                // (only when some group was copied by hand)
                if (mixed_mask & 0x55555555u) {
                    cp_async_wait_all();
                    fence_proxy_async_smem();
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(full);
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
            if (op == 0)
                for (int q = 0; q < kQTiles; ++q) {
                    if (w.t[q].n_tiles == 0) continue;
                    const unsigned long long t0 = globaltimer();
                    while (!mbar_try_wait(&sm.bar_q[q], 0) && globaltimer() - t0 < kWaitNs) {
                    }
                }
        }
    } else if (warp == 1) {
        // ============================ MMA issuer ==============================
        // Per K/V tile j: S0_j, PV1_{j-1}, S1_j, PV0_j.  tcgen05.mma from one
        // thread executes in issue order, so S_q(j+1) (which overwrites the P
        // columns of S_q) runs after PV_q(j) has read them, and the commit of
        // S_q(j) also covers PV_q(j-1): the softmax may rescale O_q as soon as
        // S_q(j) is visible.
        if (lane == 0) {
            // A lean loop: the tensor core's instruction queue is shallow, so
            // every cycle spent here between two GEMMs is a cycle it idles.
            // Stage descriptors are precomputed (stage s of a ring is 32 KB =
            // +2048 in the descriptor's 16-byte address field), stage indices
            // and parities advance without division.
            constexpr uint32_t idS = idesc_bf16(false);
            constexpr uint32_t idO = idesc_bf16(true);
            constexpr uint64_t kStageDesc = kTileBytes >> 4;
            const int n0 = w.t[0].n_tiles, n1 = w.t[1].n_tiles;
            const uint64_t dq0 = sw128_desc(smem_u32(sm.q[0]), 16, 1024);
            const uint64_t dq1 = sw128_desc(smem_u32(sm.q[1]), 16, 1024);
            const uint64_t dk = sw128_desc(smem_u32(sm.k[0]), 16, 1024);
            const uint64_t dv = sw128_desc(smem_u32(sm.v[0]), kPanel, 1024);
            const uint32_t s0_tm = tmem, s1_tm = tmem + 128u, o0_tm = tmem + 256u, o1_tm = tmem + 384u;
            // K/V stages are released by the softmax warpgroup that sees the
            // tile's last S GEMM land (see soft_release); only the tile
            // counts that never occur in practice fall back to commits here.
            const bool own_release = !soft_release(n0, n1);
            bool ok = n_tiles == 0 || mbar_wait(&sm.bar_q[0], 0, sm, P.status);
            if (ok && n1 > 0) ok = mbar_wait(&sm.bar_q[1], 0, sm, P.status);
            uint32_t ks = 0, kph = 0;          // K ring stage / parity of tile j
            uint32_t vs = 0, vph = 0;          // V ring stage / parity of tile j
            uint32_t pvs = 0, pvph = 0;        // ... of tile j-1
            // While the first six MMAs of a GEMM are queued, the barriers of
            // the next GEMM are tested without blocking; a GEMM whose inputs
            // were seen ready then follows without a wait.  (A completed phase
            // stays completed until this thread's own later MMAs let it move.)
            bool k_known = false;              // K(j) seen landed
            // Steps 1 .. jf-1 have all four GEMMs and no last-step commits:
            // they run in a loop of their own, with nothing between two GEMMs
            // but the barrier tests and waits they need.
            const int jf = own_release ? 0 : (n0 - 1 < n1 ? n0 - 1 : n1);
            for (int j = 0; ok && j < n_tiles; ++j) {
                if (j == 1 && jf > 1) {
                    for (; j < jf; ++j) {
                        if (!k_known && !mbar_wait(&sm.bar_kfull[ks], kph, sm, P.status)) { ok = false; break; }
                        tc_fence_after();
                        const uint64_t kd = dk + ks * kStageDesc;
                        tc_gemm_ss_head(s0_tm, dq0, kd, idS);
                        const bool pv1_ready = mbar_test(&sm.bar_p_full[1], (uint32_t)(j - 1) & 1u);
                        tc_gemm_ss_tail(s0_tm, dq0, kd, idS);
                        tc_commit(&sm.bar_s_full[0]);
                        if (!pv1_ready && !mbar_wait(&sm.bar_p_full[1], (uint32_t)(j - 1) & 1u, sm, P.status)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint64_t vd1 = dv + pvs * kStageDesc;
                        tc_gemm_ts_head(o1_tm, s1_tm, vd1, idO, j > 1 ? 1u : 0u);
                        tc_gemm_ts_tail(o1_tm, s1_tm, vd1, idO);
                        tc_gemm_ss_head(s1_tm, dq1, kd, idS);
                        const bool pv0_ready = mbar_test(&sm.bar_vfull[vs], vph) &&
                                               mbar_test(&sm.bar_p_full[0], (uint32_t)j & 1u);
                        tc_gemm_ss_tail(s1_tm, dq1, kd, idS);
                        tc_commit(&sm.bar_s_full[1]);
                        const uint32_t ks_n = ks + 1 == kKStages ? 0u : ks + 1;
                        const uint32_t kph_n = ks + 1 == kKStages ? kph ^ 1u : kph;
                        if (!pv0_ready && (!mbar_wait(&sm.bar_vfull[vs], vph, sm, P.status) ||
                                           !mbar_wait(&sm.bar_p_full[0], (uint32_t)j & 1u, sm, P.status))) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint64_t vd0 = dv + vs * kStageDesc;
                        tc_gemm_ts_head(o0_tm, s0_tm, vd0, idO, 1u);
                        k_known = mbar_test(&sm.bar_kfull[ks_n], kph_n);
                        tc_gemm_ts_tail(o0_tm, s0_tm, vd0, idO);
                        pvs = vs; pvph = vph;
                        if (++vs == kVStages) { vs = 0; vph ^= 1u; }
                        ks = ks_n; kph = kph_n;
                    }
                    if (!ok || j >= n_tiles) break;
                }
                if (!k_known && !mbar_wait(&sm.bar_kfull[ks], kph, sm, P.status)) { ok = false; break; }
                tc_fence_after();
                const bool pv1 = j >= 1 && j - 1 < n1;
                bool pv1_ready = false;
                if (j < n0) {
                    const uint64_t kd = dk + ks * kStageDesc;
                    tc_gemm_ss_head(s0_tm, dq0, kd, idS);
                    if (pv1)
                        pv1_ready = (j - 1 < n0 || mbar_test(&sm.bar_vfull[pvs], pvph)) &&
                                    mbar_test(&sm.bar_p_full[1], (uint32_t)(j - 1) & 1u);
                    tc_gemm_ss_tail(s0_tm, dq0, kd, idS);
                    tc_commit(&sm.bar_s_full[0]);
                }
                if (pv1) {                     // PV1(j-1)
                    if (!pv1_ready) {
                        if (j - 1 >= n0 && !mbar_wait(&sm.bar_vfull[pvs], pvph, sm, P.status)) { ok = false; break; }
                        if (!mbar_wait(&sm.bar_p_full[1], (uint32_t)(j - 1) & 1u, sm, P.status)) { ok = false; break; }
                    }
                    tc_fence_after();
                    const uint64_t vd = dv + pvs * kStageDesc;
                    tc_gemm_ts_head(o1_tm, s1_tm, vd, idO, j > 1 ? 1u : 0u);
                    tc_gemm_ts_tail(o1_tm, s1_tm, vd, idO);
                    if (j == n1) tc_commit(&sm.bar_o_done[1]);
                    if (own_release) tc_commit(&sm.bar_vempty[pvs]);
                }
                bool pv0_ready = false;
                if (j < n1) {
                    const uint64_t kd = dk + ks * kStageDesc;
                    tc_gemm_ss_head(s1_tm, dq1, kd, idS);
                    if (j < n0)
                        pv0_ready = mbar_test(&sm.bar_vfull[vs], vph) &&
                                    mbar_test(&sm.bar_p_full[0], (uint32_t)j & 1u);
                    tc_gemm_ss_tail(s1_tm, dq1, kd, idS);
                    tc_commit(&sm.bar_s_full[1]);
                }
                if (own_release) tc_commit(&sm.bar_kempty[ks]);
                const uint32_t ks_n = ks + 1 == kKStages ? 0u : ks + 1;
                const uint32_t kph_n = ks + 1 == kKStages ? kph ^ 1u : kph;
                k_known = false;
                if (j < n0) {                  // PV0(j)
                    if (!pv0_ready) {
                        if (!mbar_wait(&sm.bar_vfull[vs], vph, sm, P.status)) { ok = false; break; }
                        if (!mbar_wait(&sm.bar_p_full[0], (uint32_t)j & 1u, sm, P.status)) { ok = false; break; }
                    }
                    tc_fence_after();
                    const uint64_t vd = dv + vs * kStageDesc;
                    tc_gemm_ts_head(o0_tm, s0_tm, vd, idO, j > 0 ? 1u : 0u);
                    if (j + 1 < n_tiles) k_known = mbar_test(&sm.bar_kfull[ks_n], kph_n);
                    tc_gemm_ts_tail(o0_tm, s0_tm, vd, idO);
                    if (j == n0 - 1) tc_commit(&sm.bar_o_done[0]);
                    if (own_release && j >= n1) tc_commit(&sm.bar_vempty[vs]);   // no PV1 reads V(j)
                }
                pvs = vs; pvph = vph;
                if (++vs == kVStages) { vs = 0; vph ^= 1u; }
                ks = ks_n; kph = kph_n;
            }
            if (ok && n_tiles > 0 && n_tiles - 1 < n1) {   // PV1(last)
                const int jl = n_tiles - 1;
                if ((jl < n0 || mbar_wait(&sm.bar_vfull[pvs], pvph, sm, P.status)) &&
                    mbar_wait(&sm.bar_p_full[1], (uint32_t)jl & 1u, sm, P.status)) {
                    tc_fence_after();
                    tc_gemm_ts_head(o1_tm, s1_tm, dv + pvs * kStageDesc, idO, jl > 0 ? 1u : 0u);
                    tc_gemm_ts_tail(o1_tm, s1_tm, dv + pvs * kStageDesc, idO);
                    tc_commit(&sm.bar_o_done[1]);
                    if (own_release) tc_commit(&sm.bar_vempty[pvs]);
                }
            }
            // Drain: every issued MMA lands before TMEM is freed.
            tc_commit(&sm.bar_mma_done);
            const unsigned long long t0 = globaltimer();
            while (!mbar_try_wait(&sm.bar_mma_done, 0) && globaltimer() - t0 < kWaitNs) {
            }
        }
        __syncwarp();
    }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsHigh));
        // ========================== softmax + epilogue ========================
        const int qt = (warp - 4) >> 2;                // query tile of this warpgroup
        const QTile t = qt ? w.t[1] : w.t[0];
        const int row = (warp & 3) * 32 + lane;        // query row in tile == TMEM lane
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t s_tm = tmem + lane_base + 128u * qt;
        const uint32_t o_tm = tmem + lane_base + 256u + 128u * qt;
        const long long my_khi = row < t.split ? t.khi_lo : t.khi;
        const float sl2 = P.scale_log2;
        float m_run = -INFINITY, l_run = 0.f;          // m in log2 units, scaled
        bool ok = true;
        // The warpgroup of the tile whose S GEMM comes last in each K/V step
        // releases the stages: S_q(j) landing means every MMA issued before
        // it has landed too, i.e. K(j) (both S GEMMs) and V(j-1) (both PV
        // GEMMs) are no longer read.
        const bool releaser = soft_release(w.t[0].n_tiles, w.t[1].n_tiles) &&
                              qt == (w.t[1].n_tiles > 0 ? 1 : 0) && (warp & 3) == 0 && lane == 0;
        for (int j = 0; j < t.n_tiles; ++j) {
            if (!warp_wait(&sm.bar_s_full[qt], (uint32_t)j & 1u, sm, P.status)) { ok = false; break; }
            tc_fence_after();
            if (releaser) {
                mbar_arrive(&sm.bar_kempty[j % kKStages]);
                if (j > 0) mbar_arrive(&sm.bar_vempty[(j - 1) % kVStages]);
            }
            const long long left_ll = my_khi - (w.klo + (long long)j * kBN);
            const int left = left_ll >= kBN ? kBN : (left_ll < 0 ? 0 : (int)left_ll);
            const bool masked = !__all_sync(0xffffffffu, left == kBN);
            uint32_t pk[64];
            float rsum = 0.f;
            float m_new = m_run;
            // Exponentials against the running max; a row whose sum overgrows
            // (its max rose by more than 8 in log2 units) triggers one redo of
            // the warp with the new max.  The first tile takes the max first.
            // One copy of each pass in the code.
#pragma unroll 1
            for (int attempt = 0;; ++attempt) {
                if (attempt > 0 || j > 0)
                    rsum = masked ? exp_row<true>(s_tm, m_new, sl2, left, pk)
                                  : exp_row<false>(s_tm, m_new, sl2, left, pk);
                const bool redo = attempt == 0 && (j == 0 || !(rsum <= kRedoSum));
                if (!__any_sync(0xffffffffu, redo)) break;   // warp-uniform: tcgen05.ld is .sync.aligned
                const float tmax = masked ? max_row<true>(s_tm, left) : max_row<false>(s_tm, left);
                if (redo) m_new = fmaxf(m_run, tmax * sl2);
            }
            const float alpha = m_new == m_run ? 1.f : ex2_approx(m_run - m_new);
            l_run = l_run * alpha + rsum;
            m_run = m_new;
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
                // O_q holds PV_q(j-1) (complete: it was issued before S_q(j))
#pragma unroll
                for (int c4 = 0; c4 < 4; ++c4) {
                    uint32_t o[32];
                    KVP_TMEM_LD32(o_tm + 32 * c4, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 32; ++c)
                        o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
                    KVP_TMEM_ST32(o_tm + 32 * c4, o);
                }
            }
            // P -> the first 64 columns of S_q (bf16 pairs, key 2c in the low half)
            KVP_TMEM_ST32(s_tm, pk);
            KVP_TMEM_ST32(s_tm + 32, (pk + 32));
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&sm.bar_p_full[qt]);
        }
        if (P.splits > 1) {
            // partial (O, m, l) of this key chunk, fp32, for combine_splits_kernel
            const long long rr = t.row0 + row - (long long)S.q_frame0 * P.T;
            const size_t slot = ((size_t)w.chunk * (size_t)P.ws_rows + (size_t)rr) * (size_t)S.nheads +
                                (size_t)(w.head - S.head0);
            float* wo = P.ws + slot * kDH;
            float* wml = P.ws + (size_t)P.splits * (size_t)P.ws_rows * (size_t)S.nheads * kDH + slot * 2;
            if (t.nq > 0 && t.n_tiles > 0) {
                if (ok && warp_wait(&sm.bar_o_done[qt], 0, sm, P.status)) {
                    tc_fence_after();
#pragma unroll
                    for (int c4 = 0; c4 < 4; ++c4) {
                        uint32_t o[32];
                        KVP_TMEM_LD32(o_tm + 32 * c4, o);
                        tmem_wait_ld();
                        if (row < t.nq) {
#pragma unroll
                            for (int c = 0; c < 32; c += 4)
                                *reinterpret_cast<uint4*>(wo + 32 * c4 + c) =
                                    make_uint4(o[c], o[c + 1], o[c + 2], o[c + 3]);
                        }
                    }
                    if (row < t.nq) {
                        wml[0] = m_run;
                        wml[1] = l_run;
                    }
                }
            } else if (t.nq > 0 && row < t.nq) {   // empty chunk: identity partial
#pragma unroll
                for (int c = 0; c < kDH; c += 4)
                    *reinterpret_cast<uint4*>(wo + c) = make_uint4(0, 0, 0, 0);
                wml[0] = -INFINITY;
                wml[1] = 0.f;
            }
        } else if (ok && t.n_tiles > 0 && warp_wait(&sm.bar_o_done[qt], 0, sm, P.status)) {
            tc_fence_after();
            const float inv = 1.f / l_run;
            __nv_bfloat16* dst = S.out + (size_t)(t.row0 + row) * D + hcol;
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
                uint32_t o[32];
                KVP_TMEM_LD32(o_tm + 32 * c4, o);
                tmem_wait_ld();
                if (row < t.nq) {
#pragma unroll
                    for (int c = 0; c < 32; c += 8) {
                        uint4 pkt;
                        pkt.x = pack_bf16(__uint_as_float(o[c]) * inv, __uint_as_float(o[c + 1]) * inv);
                        pkt.y = pack_bf16(__uint_as_float(o[c + 2]) * inv, __uint_as_float(o[c + 3]) * inv);
                        pkt.z = pack_bf16(__uint_as_float(o[c + 4]) * inv, __uint_as_float(o[c + 5]) * inv);
                        pkt.w = pack_bf16(__uint_as_float(o[c + 6]) * inv, __uint_as_float(o[c + 7]) * inv);
                        *reinterpret_cast<uint4*>(dst + 32 * c4 + c) = pkt;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}

// ---------------------------------------------------------- split combine
// out[row, head] = sum_c 2^(m_c - M) O_c / sum_c 2^(m_c - M) l_c over the
// key chunks c of a split launch (M = max_c m_c; m in log2 units).  One warp
// per (query row, head), four dims per lane.
__global__ void __launch_bounds__(256)
combine_splits_kernel(const float* __restrict__ ws, __nv_bfloat16* __restrict__ out, int splits,
                      long long rows, int nheads, int D, int head0, long long row0) {
    const long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (gw >= rows * nheads) return;
    const long long rr = gw / nheads;
    const int h = (int)(gw % nheads);
    const float* ml = ws + (size_t)splits * (size_t)rows * (size_t)nheads * kDH;
    float M = -INFINITY;
    for (int c = 0; c < splits; ++c)
        M = fmaxf(M, ml[(((size_t)c * rows + rr) * nheads + h) * 2]);
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c = 0; c < splits; ++c) {
        const size_t slot = ((size_t)c * rows + rr) * nheads + h;
        const float m = ml[slot * 2];
        if (m == -INFINITY) continue;                 // chunk without keys for this row
        const float wgt = exp2f(m - M);
        L += wgt * ml[slot * 2 + 1];
        const float4 o = reinterpret_cast<const float4*>(ws + slot * kDH)[lane];
        acc.x += wgt * o.x; acc.y += wgt * o.y; acc.z += wgt * o.z; acc.w += wgt * o.w;
    }
    const float inv = 1.f / L;
    uint2 pk;
    pk.x = pack_bf16(acc.x * inv, acc.y * inv);
    pk.y = pack_bf16(acc.z * inv, acc.w * inv);
    *reinterpret_cast<uint2*>(out + (size_t)(row0 + rr) * D + (size_t)(head0 + h) * kDH + 4 * lane) = pk;
}

// The split workspace comes from a private, per-device stream-ordered pool
// that keeps freed blocks cached (release threshold = max): the default
// pool would hand its memory back to the driver at every synchronisation
// and each launch would map it again.
cudaError_t workspace_pool(cudaMemPool_t* out) {
    static std::mutex mu;
    static cudaMemPool_t pools[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(mu);
    if (!pools[dev]) {
        cudaMemPoolProps props{};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        cudaMemPool_t p = nullptr;
        e = cudaMemPoolCreate(&p, &props);
        if (e != cudaSuccess) return e;
        uint64_t keep = ~0ull;
        e = cudaMemPoolSetAttribute(p, cudaMemPoolAttrReleaseThreshold, &keep);
        if (e != cudaSuccess) {
            cudaMemPoolDestroy(p);
            return e;
        }
        pools[dev] = p;
    }
    *out = pools[dev];
    return cudaSuccess;
}

// Key chunks per (query tile pair, head) for a per-frame launch: split only
// when the launch has fewer CTAs than SMs; minimise waves x (fixed cost +
// tiles per chunk), the fixed cost (prologue, epilogue) ~ 3 tiles.
int choose_splits(long long items, int tiles_max, int sms) {
    if (items <= 0 || items >= sms || tiles_max < 4) return 1;
    int best = 1;
    long long best_cost = -1;
    for (int c = 1; c <= 8 && c <= tiles_max / 2; ++c) {
        const long long waves = (items * c + sms - 1) / sms;
        const long long cost = waves * (3 + (tiles_max + c - 1) / c);
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best = c;
        }
    }
    return best;
}

// ------------------------------------------------------------ host helpers
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// Encoded maps are cached by (base, rows, cols, pitch, box): a map holds no
// more than these, so an entry stays right even if the memory is freed and
// reused with the same shape.  Per-frame loops launch the same few tensors
// hundreds of times.
struct MapKey {
    const void* base;
    long long rows, cols, pitch;
    uint32_t box;
    bool operator==(const MapKey& o) const {
        return base == o.base && rows == o.rows && cols == o.cols && pitch == o.pitch && box == o.box;
    }
};
struct MapKeyHash {
    size_t operator()(const MapKey& k) const {
        size_t h = std::hash<const void*>()(k.base);
        h ^= std::hash<long long>()(k.rows) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
        h ^= std::hash<long long>()(k.cols * 131 + k.pitch) + (h << 6) + (h >> 2);
        h ^= std::hash<uint32_t>()(k.box) + (h << 6) + (h >> 2);
        return h;
    }
};

int encode_map(CUtensorMap* m, const void* base, long long rows, long long cols, long long pitch,
               uint32_t box_rows);

// 2D bf16 row-major tensor [rows][cols] with row pitch `pitch` elements.
int make_map(CUtensorMap* m, const void* base, long long rows, long long cols, long long pitch,
             uint32_t box_rows) {
    static std::mutex mu;
    static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
    const MapKey key{base, rows, cols, pitch, box_rows};
    {
        std::lock_guard<std::mutex> g(mu);
        auto it = cache.find(key);
        if (it != cache.end()) {
            *m = it->second;
            return KVP_OK;
        }
    }
    const int rc = encode_map(m, base, rows, cols, pitch, box_rows);
    if (rc == KVP_OK) {
        std::lock_guard<std::mutex> g(mu);
        if (cache.size() >= 4096) cache.clear();
        cache.emplace(key, *m);
    }
    return rc;
}

int encode_map(CUtensorMap* m, const void* base, long long rows, long long cols, long long pitch,
               uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        set_error("cuTensorMapEncodeTiled unavailable");
        return KVP_ERR_UNSUPPORTED;
    }
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)pitch * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d) rows=%lld cols=%lld box_rows=%u", (int)r, rows,
                  cols, box_rows);
        return KVP_ERR_ARG;
    }
    return KVP_OK;
}

}  // namespace

int make_bf16_tensor_map(CUtensorMap* m, const void* base, long long rows, long long cols,
                         long long pitch, uint32_t box_rows) {
    return make_map(m, base, rows, cols, pitch, box_rows);
}

int check_attn_bf16(const LayerIO& io, const AttnDesc& d) {
    const long long T = d.tokens;
    if (d.head_dim != kDH || d.heads <= 0 || T <= 0 || d.frames <= 0 || d.q_frame0 < 0 ||
        d.nheads <= 0 || d.head0 < 0 || d.head0 + d.nheads > d.heads || d.window < 0 ||
        (d.mode != 0 && d.mode != 1) || !io.q || !io.k || !io.v || !io.out) {
        set_error("attn_bf16: bad descriptor (head_dim must be %d)", kDH);
        return KVP_ERR_ARG;
    }
    if (d.flat && (d.mode != 1 || d.window != 0 || T < kBM)) {
        set_error("attn_bf16: flat query tiles need causal mode, no window and tokens >= %d", kBM);
        return KVP_ERR_ARG;
    }
    const long long q_end = ((long long)d.q_frame0 + d.frames) * T;
    if (io.q_rows < q_end || io.kv_rows < q_end || (io.kvmap && io.arena && io.arena_rows <= 0)) {
        set_error("attn_bf16: q_rows/kv_rows (%lld/%lld) do not cover frames up to row %lld",
                  io.q_rows, io.kv_rows, q_end);
        return KVP_ERR_ARG;
    }
    if (((uintptr_t)io.q | (uintptr_t)io.k | (uintptr_t)io.v | (uintptr_t)io.out |
         (uintptr_t)io.arena) & 15) {
        set_error("attn_bf16: Q/K/V/Out/Arena must be 16-byte aligned");
        return KVP_ERR_ARG;
    }
    return KVP_OK;
}

namespace {

// Tensor maps and pointers of one layer (check_attn_bf16 has passed).
// Whether two layers' segments would hold the same tensor maps.
bool same_tensors(const LayerIO& a, const AttnDesc& da, const LayerIO& b, const AttnDesc& db) {
    return a.q == b.q && a.k == b.k && a.v == b.v && a.arena == b.arena && a.q_rows == b.q_rows &&
           a.kv_rows == b.kv_rows && (a.arena ? a.arena_rows == b.arena_rows : true) && da.heads == db.heads;
}

// like: a segment filled from a layer with the same tensors (same_tensors),
// whose maps are copied instead of encoded again.
int fill_seg(Seg& g, const LayerIO& io, const AttnDesc& d, const Seg* like = nullptr) {
    const int D = d.heads * kDH;
    if (like) {
        g = *like;
        g.kvmap = io.kvmap;
        g.out = (__nv_bfloat16*)io.out;
        g.head0 = d.head0;
        g.nheads = d.nheads;
        g.cta0 = 0;
        g.q_frame0 = d.q_frame0;
        return KVP_OK;
    }
    std::memset(&g, 0, sizeof g);
    // Box kinds whose height fits the tensor (a box never starts past the
    // end, and a taller box than the tensor is never encoded).
    int base_boxes = 0, arena_boxes = 0;
    while (base_boxes < kBoxKinds && (8LL << base_boxes) <= io.kv_rows) ++base_boxes;
    if (io.arena)
        while (arena_boxes < kBoxKinds && (8LL << arena_boxes) <= io.arena_rows) ++arena_boxes;
    int rc = make_map(&g.maps.q8, io.q, io.q_rows, D, D, 8);
    for (int i = 0; !rc && i < kBoxKinds; ++i) {
        const uint32_t h = 8u << (i < base_boxes ? i : 0);
        rc = make_map(&g.maps.kv[0][i], io.k, io.kv_rows, D, D, h);
        if (!rc) rc = make_map(&g.maps.kv[1][i], io.v, io.kv_rows, D, D, h);
        if (!rc && arena_boxes)
            rc = make_map(&g.maps.a[i], io.arena, io.arena_rows, 2 * D, 2 * D, 8u << (i < arena_boxes ? i : 0));
    }
    if (!rc && arena_boxes) rc = make_map(&g.maps.a1, io.arena, io.arena_rows, 2 * D, 2 * D, 1);
    if (rc) return rc;
    if (base_boxes == 0 || io.q_rows < 8) {
        set_error("attn_bf16: Q and K/V need at least 8 rows");
        return KVP_ERR_ARG;
    }
    g.k = (const __nv_bfloat16*)io.k;
    g.v = (const __nv_bfloat16*)io.v;
    g.arena = (const __nv_bfloat16*)io.arena;
    g.kvmap = io.kvmap;
    g.out = (__nv_bfloat16*)io.out;
    g.q_rows = io.q_rows;
    g.kv_rows = io.kv_rows;
    g.arena_rows = io.arena ? io.arena_rows : 0;
    g.D = D;
    g.head0 = d.head0;
    g.nheads = d.nheads;
    g.cta0 = 0;
    g.q_frame0 = d.q_frame0;
    g.base_boxes = base_boxes;
    g.arena_boxes = arena_boxes;
    g.arena_gather = arena_boxes > 0 ? 1 : 0;
    return KVP_OK;
}

void fill_params(Params& P, const AttnDesc& d, int* d_status) {
    const long long T = d.tokens;
    std::memset(&P, 0, sizeof P);
    P.status = d_status;
    P.T = (int)T;
    P.frames = d.frames;
    P.mode = d.mode;
    P.window = d.window;
    P.flat = d.flat;
    P.n_qt = (int)((T + kBM - 1) / kBM);
    P.n_pairs = (P.n_qt + kQTiles - 1) / kQTiles;
    P.items_per_head = d.flat ? (int)(((long long)d.frames * T + kQTiles * kBM - 1) / (kQTiles * kBM))
                              : d.frames * P.n_pairs;
    P.scale_log2 = 1.4426950408889634f / sqrtf((float)kDH);
    P.splits = 1;
    P.ws = nullptr;
    P.ws_rows = (long long)d.frames * T;
    P.n_segs = 1;
}

// Kernel attributes and the launch checks, once per device and instantiation.
template <int kSegs>
int setup_kernel() {
    const int smem = (int)sizeof(Smem);
    static PerDeviceOnce setup;
    return setup([&](int dev) -> int {
        int optin = 0;
        KVP_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        if (smem > optin) {
            set_error("attn_bf16: needs %d B of shared memory per block, device allows %d", smem, optin);
            return KVP_ERR_UNSUPPORTED;
        }
        // setmaxnreg.inc waits until the warpgroup's registers exist in the
        // CTA's pool: refuse a build whose launch pool is smaller than the split.
        cudaFuncAttributes fa;
        KVP_CUDA(cudaFuncGetAttributes(&fa, attn_bf16_sm100_kernel<kSegs>));
        if ((long long)fa.numRegs * kThreads < (long long)kRegsLow * 128 + 2LL * kRegsHigh * 128) {
            set_error("attn_bf16: kernel built with %d registers per thread, the register split needs %d",
                      fa.numRegs, (kRegsLow * 128 + 2 * kRegsHigh * 128 + kThreads - 1) / kThreads);
            return KVP_ERR_UNSUPPORTED;
        }
        KVP_CUDA(cudaFuncSetAttribute(attn_bf16_sm100_kernel<kSegs>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        return KVP_OK;
    });
}

}  // namespace

int launch_attn_bf16(const LayerIO& io, const AttnDesc& d, int* d_status, cudaStream_t stream,
                     bool allow_split) {
    const long long T = d.tokens;
    const int D = d.heads * kDH;
    const int rc_check = check_attn_bf16(io, d);
    if (rc_check != KVP_OK) return rc_check;
    // KVP_ATTN_PAIR=1: the SM-pair kernel (attn_pair_sm100.cu) instead.
    if (const char* e = std::getenv("KVP_ATTN_PAIR"))
        if (std::atoi(e) == 1 && attn_pair_supported(d)) return launch_attn_bf16_pair(io, d, d_status, stream);
    if (!d_status) {
        set_error("attn_bf16: no status word");
        return KVP_ERR_ARG;
    }
    SegTable<1> tab;
    int rc = fill_seg(tab.seg[0], io, d);
    if (rc) return rc;
    Params P;
    fill_params(P, d, d_status);
    const int rc_setup = setup_kernel<1>();
    if (rc_setup != KVP_OK) return rc_setup;
    const int smem = (int)sizeof(Smem);
    // Key-range split for per-frame launches that would leave SMs idle
    // (KVP_ATTN_SPLITS=n forces n, 1 disables).
    if (!d.flat && allow_split) {
        int sms = 148, dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess)
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const int last = d.q_frame0 + d.frames - 1;
        const long long span = d.mode == 0 ? T
            : (long long)((d.window > 0 && d.window < last + 1) ? d.window : last + 1) * T;
        const int tiles_max = (int)((span + kBN - 1) / kBN);
        int splits = choose_splits((long long)d.nheads * P.items_per_head, tiles_max, sms);
        if (const char* e = std::getenv("KVP_ATTN_SPLITS")) {
            const int f = std::atoi(e);
            if (f >= 1) splits = f < tiles_max ? f : (tiles_max > 0 ? tiles_max : 1);
        }
        P.splits = splits > 1 ? splits : 1;
    }
    if (P.splits > 1) {
        P.items_per_head *= P.splits;
        const size_t ws_bytes = (size_t)P.splits * (size_t)P.ws_rows * (size_t)d.nheads * (kDH + 2) *
                                sizeof(float);
        cudaMemPool_t pool = nullptr;
        KVP_CUDA(workspace_pool(&pool));
        KVP_CUDA(cudaMallocFromPoolAsync(reinterpret_cast<void**>(&P.ws), ws_bytes, pool, stream));
    }
    const long long grid = (long long)d.nheads * P.items_per_head;
    if (grid <= 0 || grid > 0x7fffffffLL) {
        if (P.ws) cudaFreeAsync(P.ws, stream);
        return KVP_ERR_ARG;
    }
    attn_bf16_sm100_kernel<1><<<(unsigned)grid, kThreads, smem, stream>>>(tab, P);
    cudaError_t le = cudaGetLastError();
    if (P.splits > 1) {
        if (le == cudaSuccess) {
            const long long warps = P.ws_rows * d.nheads;
            combine_splits_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, stream>>>(
                P.ws, tab.seg[0].out, P.splits, P.ws_rows, d.nheads, D, d.head0, (long long)d.q_frame0 * T);
            le = cudaGetLastError();
        }
        const cudaError_t fe = cudaFreeAsync(P.ws, stream);
        if (le == cudaSuccess) le = fe;
    }
    if (le != cudaSuccess) return cuda_status(le, "attn_bf16 launch");
    return KVP_OK;
}

int launch_attn_bf16_multi(const LayerIO* ios, const AttnDesc* ds, int n, int* d_status,
                           cudaStream_t stream) {
    if (!ios || !ds || n <= 0) {
        set_error("attn_bf16_multi: no layers");
        return KVP_ERR_ARG;
    }
    const AttnDesc& d0 = ds[0];
    for (int i = 0; i < n; ++i) {
        const AttnDesc& d = ds[i];
        if (d.tokens != d0.tokens || d.frames != d0.frames || d.mode != d0.mode ||
            d.window != d0.window || d.flat != d0.flat) {
            set_error("attn_bf16_multi: layer %d differs from layer 0 in tokens, frames, mode, window or tiling", i);
            return KVP_ERR_ARG;
        }
        const int rc = check_attn_bf16(ios[i], d);
        if (rc != KVP_OK) return rc;
    }
    if (!d_status) {
        set_error("attn_bf16_multi: no status word");
        return KVP_ERR_ARG;
    }
    const int rc_setup = setup_kernel<kMaxSegs>();
    if (rc_setup != KVP_OK) return rc_setup;
    const int smem = (int)sizeof(Smem);
    Params P;
    fill_params(P, d0, d_status);
    SegTable<kMaxSegs> tab;
    // As few launches as the table allows, with the segments spread evenly
    // over them (30 layers: 10 + 10 + 10, not 12 + 12 + 6).
    const int launches = (n + kMaxSegs - 1) / kMaxSegs;
    const int per_launch = (n + launches - 1) / launches;
    for (int first = 0; first < n; first += per_launch) {
        const int cnt = n - first < per_launch ? n - first : per_launch;
        long long cta = 0;
        for (int i = 0; i < cnt; ++i) {
            const int k = first + i;
            const bool like = i > 0 && same_tensors(ios[k], ds[k], ios[k - 1], ds[k - 1]);
            const int rc = fill_seg(tab.seg[i], ios[k], ds[k], like ? &tab.seg[i - 1] : nullptr);
            if (rc) return rc;
            tab.seg[i].cta0 = (int)cta;
            cta += (long long)ds[first + i].nheads * P.items_per_head;
        }
        for (int i = cnt; i < kMaxSegs; ++i) tab.seg[i] = tab.seg[cnt - 1];
        P.n_segs = cnt;
        if (cta <= 0 || cta > 0x7fffffffLL) return KVP_ERR_ARG;
        attn_bf16_sm100_kernel<kMaxSegs><<<(unsigned)cta, kThreads, smem, stream>>>(tab, P);
        const cudaError_t le = cudaGetLastError();
        if (le != cudaSuccess) return cuda_status(le, "attn_bf16_multi launch");
    }
    return KVP_OK;
}

}  // namespace kvp

// ------------------------------------------------------- bounded-wait probe
// Exercises the timeout path of the bounded mbarrier waits without hanging
// anything: the barrier expects two arrivals and only one ever comes, so the
// wait runs out after limit_ns and the kernel records KVP_STATUS_TIMEOUT.
namespace kvp {
namespace {
__global__ void bounded_wait_probe_kernel(int* status, unsigned long long limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 2);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        mbar_arrive(&bar);
        const unsigned long long t0 = globaltimer();
        bool done = false;
        while (!(done = mbar_try_wait(&bar, 0)))
            if (globaltimer() - t0 > limit_ns) break;
        if (!done) atomicOr(status, KVP_STATUS_TIMEOUT);
    }
}
}  // namespace

int launch_bounded_wait_probe(long long limit_ns, int* d_status, cudaStream_t stream) {
    if (limit_ns <= 0 || limit_ns > 5000000000LL || !d_status) {
        set_error("probe: limit must be in (0, 5 s]");
        return KVP_ERR_ARG;
    }
    bounded_wait_probe_kernel<<<1, 32, 0, stream>>>(d_status, (unsigned long long)limit_ns);
    KVP_CUDA(cudaGetLastError());
    return KVP_OK;
}
}  // namespace kvp
