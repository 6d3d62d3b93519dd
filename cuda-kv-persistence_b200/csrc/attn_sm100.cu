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
// CTA = 128 query rows x one head.  Warp roles (256 threads):
//   warp 0      producer: reads the KVMap for each 128-key tile, classifies
//               every 8-row group (all base / one ascending arena run /
//               mixed) and stages K and V with TMA boxes (128 rows when the
//               whole tile is base rows, 8 rows per group otherwise); mixed
//               groups and padding are copied with 16-byte loads into the
//               same 128B-swizzled layout
//   warp 1      TMEM allocation and the single-thread MMA issuer:
//               S_j = Q K_j^T (M128 N128 K16 x8) and O += P_{j-1} V_{j-1}
//   warps 4-7   softmax (thread i owns query row i = TMEM lane i), online
//               max with lazy rescaling (only when the max grows by > 8 in
//               log2 units), P written to shared memory as bf16, then the
//               epilogue O / l -> bf16 -> global
// TMEM columns: S ring of three 128-column accumulators [0,384), O [384,512).  Shared memory: Q
// 32 KB, two K|V stages of 64 KB, P 32 KB.  Every mbarrier wait is bounded
// (about one second of %globaltimer); on expiry the CTA records
// KVP_STATUS_TIMEOUT in the status word and unwinds without hanging.
#include <cuda.h>
#include <cuda_bf16.h>

#include <cstring>
#include <mutex>
#include <unordered_map>

#include "attn_sm100.h"
#include "kvp_common.h"

namespace kvp {

namespace {

constexpr int kBM = 128;           // query rows per CTA
constexpr int kBN = 128;           // keys per tile
constexpr int kDH = 128;           // head dim
constexpr int kStages = 2;         // depth of the K ring and of the V ring
constexpr int kSBuf = 3;           // S accumulators in TMEM: S runs two tiles ahead of PV
constexpr int kThreads = 384;     // producer, MMA, 2 idle, 8 softmax warps
constexpr uint32_t kPanel = 128 * 128;        // one [128 rows][64 bf16] swizzled panel
constexpr uint32_t kTileBytes = 2 * kPanel;   // [128][128] bf16
constexpr uint32_t kGroupPanel = 8 * 128;     // one 8-row group of a panel
constexpr unsigned long long kWaitNs = 1000000000ull;  // bounded waits: ~1 s

struct __align__(1024) Smem {
    uint8_t q[kTileBytes];
    uint8_t k[kStages][kTileBytes];
    uint8_t v[kStages][kTileBytes];
    uint8_t p[2][kTileBytes];       // P double buffer: tile j uses p[j & 1]
    uint64_t bar_q;
    uint64_t bar_full[2][kStages];   // [0] = K ring, [1] = V ring
    uint64_t bar_empty[2][kStages];
    uint64_t bar_s_full[kSBuf];
    uint64_t bar_s_free[kSBuf];
    uint64_t bar_p_full[2];         // P_j written into p[j & 1]
    uint64_t bar_pv_done[2];        // PV_j done -> p[j & 1] free (one barrier per buffer)
    uint64_t bar_red[4][2];      // row-max exchange of the two warps of a row block
    uint64_t bar_sum[4];         // final row-sum exchange
    float red[2][2][128];        // [tile parity][half][row] partial row max
    uint32_t tmem_base;
    int abort_flag;
};

constexpr int kBoxKinds = 5;       // TMA box heights 8, 16, 32, 64, 128 rows

struct TmaMaps {
    CUtensorMap q8;                 // Q [q_rows][D], box 64 x 8
    CUtensorMap kv[2][kBoxKinds];   // K / V [kv_rows][D], box 64 x (8 << i)
    CUtensorMap a[kBoxKinds];       // arena [arena_rows][2D], box 64 x (8 << i)
};

struct Params {
    const __nv_bfloat16* k;      // base rows, for mixed groups
    const __nv_bfloat16* v;
    const __nv_bfloat16* arena;
    const long long* kvmap;
    __nv_bfloat16* out;
    int* status;
    long long q_rows, kv_rows, arena_rows;
    int D, T, frames, q_frame0, mode, window, head0, nheads, flat, items_per_head, n_qt;
    int base_boxes, arena_boxes;   // box kinds usable (heights <= tensor rows); 0 = no arena TMA
    float scale_log2;
};

// ------------------------------------------------------------- primitives
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
// Bounded wait.  Returns false (and raises the CTA abort flag and the global
// status) when the phase did not complete within kWaitNs, or when another
// role already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, Smem& sm, int* status) {
    if (mbar_try_wait(b, parity)) return true;
    const unsigned long long t0 = globaltimer();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(b, parity)) return true;
        if ((it & 63u) == 0) {
            if (*(volatile int*)&sm.abort_flag) return false;
            if (globaltimer() - t0 > kWaitNs) {
                *(volatile int*)&sm.abort_flag = 1;
                atomicOr(status, KVP_STATUS_TIMEOUT);
                return false;
            }
        }
    }
}
// Warp-uniform bounded wait: lane 0 polls, the verdict is broadcast, so the
// warp stays converged for the .sync.aligned tcgen05 and shuffle
// instructions that follow.
__device__ __forceinline__ bool warp_wait(uint64_t* b, uint32_t parity, Smem& sm, int* status) {
    bool ok = true;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait(b, parity, sm, status);
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    __syncwarp();
    return ok;
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"((unsigned long long)map), "r"(x), "r"(y), "r"(smem_u32(bar))
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

// kind::f16 instruction descriptor: bf16 x bf16 -> f32, M=128, N=128.
constexpr uint32_t idesc_bf16(bool b_mn_major) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
           ((uint32_t)(128 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// Byte offset of (row, 16-byte chunk) inside a 128B-swizzled [rows][64 bf16] panel.
__device__ __forceinline__ uint32_t sw128_off(int row, int chunk) {
    return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 2^x on the FMA/ALU pipes: x = n + f with n = round(x) and f in [-1/2, 1/2],
// 2^f by a cubic fitted here by iteratively reweighted least squares on the
// relative error (max relative error 1.4e-4 over x in [-126, 8], against bf16's
// 3.9e-3 rounding of P), 2^n added to the exponent bits.  Inputs below -126
// are clamped to -126 (the result stays a positive number below 2^-125,
// which is 0 in the bf16 P and negligible in the row sum; -inf lands there too).
__device__ __forceinline__ float ex2_poly(float x) {
    x = fmaxf(x, -126.f);
    const float t = x + 12582912.f;           // 1.5 * 2^23: round to nearest integer
    const float f = x - (t - 12582912.f);
    float p = fmaf(5.517162719e-02f, f, 2.426111432e-01f);
    p = fmaf(p, f, 6.932609953e-01f);
    p = fmaf(p, f, 9.999280725e-01f);
    const int n = __float_as_int(t) - 0x4B400000;
    return __int_as_float(__float_as_int(p) + (n << 23));
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// --------------------------------------------------------------- work item
struct Work {
    long long q_row0;    // first query row (absolute in Q/out)
    int nq;              // valid query rows (<= 128)
    long long klo, khi;  // key rows [klo, khi) for rows >= split
    int split;           // rows < split use khi_lo (flat tiles crossing a frame)
    long long khi_lo;
    int head;
};

__device__ __forceinline__ Work decode_work(const Params& P) {
    Work w;
    const int h_local = blockIdx.x / P.items_per_head;
    const int i = blockIdx.x % P.items_per_head;
    w.head = P.head0 + h_local;
    const long long T = P.T;
    if (P.flat) {
        const long long R0 = (long long)P.q_frame0 * T;
        const long long R1 = (long long)(P.q_frame0 + P.frames) * T;
        const long long t = (long long)(P.items_per_head - 1 - i);  // longest first
        w.q_row0 = R0 + t * kBM;
        const long long last = (w.q_row0 + kBM < R1 ? w.q_row0 + kBM : R1) - 1;
        w.nq = (int)(last - w.q_row0 + 1);
        const long long fl = last / T, ff = w.q_row0 / T;
        w.klo = 0;
        w.khi = (fl + 1) * T;
        w.split = ff != fl ? (int)(fl * T - w.q_row0) : 0;
        w.khi_lo = (ff + 1) * T;
    } else {
        const int fr = i / P.n_qt, qt = i % P.n_qt;
        const int f = P.q_frame0 + P.frames - 1 - fr;  // longest key span first
        w.q_row0 = (long long)f * T + (long long)qt * kBM;
        const long long left = T - (long long)qt * kBM;
        w.nq = (int)(left < kBM ? left : kBM);
        if (P.mode == 0) {
            w.klo = (long long)f * T;
        } else {
            const int base = P.window > 0 ? (f - P.window + 1 > 0 ? f - P.window + 1 : 0) : 0;
            w.klo = (long long)base * T;
        }
        w.khi = (long long)(f + 1) * T;
        w.split = 0;
        w.khi_lo = w.khi;
    }
    return w;
}

// ------------------------------------------------------------------ kernel
__global__ void __launch_bounds__(kThreads, 1)
attn_bf16_sm100_kernel(const __grid_constant__ TmaMaps maps, const __grid_constant__ Params P) {
    extern __shared__ uint8_t smem_raw[];
    // The layout needs a 1024-byte aligned base (128B-swizzle atoms) and uses
    // the whole 227 KB, so there is no room to realign: refuse instead.
    if (reinterpret_cast<uintptr_t>(smem_raw) & 1023) {
        if (threadIdx.x == 0) atomicOr(P.status, KVP_STATUS_ALIGN);
        return;
    }
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const Work w = decode_work(P);
    const int n_tiles = (int)((w.khi - w.klo + kBN - 1) / kBN);

    if (threadIdx.x == 0) {
        mbar_init(&sm.bar_q, 1);
        for (int op = 0; op < 2; ++op)
            for (int s = 0; s < kStages; ++s) {
                mbar_init(&sm.bar_full[op][s], 1);
                mbar_init(&sm.bar_empty[op][s], 1);
            }
        for (int b = 0; b < kSBuf; ++b) {
            mbar_init(&sm.bar_s_full[b], 1);
            mbar_init(&sm.bar_s_free[b], 256);
        }
        mbar_init(&sm.bar_p_full[0], 256);
        mbar_init(&sm.bar_p_full[1], 256);
        mbar_init(&sm.bar_pv_done[0], 1);
        mbar_init(&sm.bar_pv_done[1], 1);
        for (int g = 0; g < 4; ++g) {
            mbar_init(&sm.bar_red[g][0], 64);
            mbar_init(&sm.bar_red[g][1], 64);
            mbar_init(&sm.bar_sum[g], 64);
        }
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
    const int D = P.D;
    const int hcol = w.head * kDH;

    if (warp == 0 || warp == 2) {
        // ============================ producers ===============================
        // Warp 0 stages Q and the K ring, warp 2 the V ring; each reads the
        // KVMap rows of its tile itself, so K of tile j+2 can load as soon as
        // S_j = Q K_j^T is done, independently of the slower V ring.
        const int op = warp == 0 ? 0 : 1;
        if (op == 0 && lane == 0) {
            // Q: 8-row groups that start inside the tensor come by TMA (a group
            // running past the end is zero-filled by TMA); groups wholly past
            // q_rows are not loaded -- their rows only feed output rows that are
            // never stored (S, P and O are row-independent).
            uint32_t qbytes = 0;
            for (int g = 0; g < kBM / 8; ++g)
                if (w.q_row0 + 8 * g < P.q_rows) qbytes += 2 * kGroupPanel;
            mbar_arrive_expect_tx(&sm.bar_q, qbytes);
            for (int g = 0; g < kBM / 8; ++g) {
                if (w.q_row0 + 8 * g >= P.q_rows) break;
                for (int p = 0; p < 2; ++p)
                    tma_load_2d(sm.q + p * kPanel + g * kGroupPanel, &maps.q8, hcol + 64 * p,
                                (int)(w.q_row0 + 8 * g), &sm.bar_q);
            }
        }
        const CUtensorMap* base_maps = maps.kv[op];
        const __nv_bfloat16* base = op == 0 ? P.k : P.v;
        const int acol = (op == 0 ? 0 : D) + hcol;     // column of this operand in an arena row
        int last_armed = -1;
        // KVMap rows of a tile are read one tile ahead, so their L2 latency
        // overlaps the wait for a free stage instead of delaying the TMA issue.
        auto map_rows = [&](int jj, long long (&mm)[4]) {
            const long long rr0 = w.klo + (long long)jj * kBN;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const long long row = rr0 + 4 * lane + i;
                mm[i] = (jj < n_tiles && row < w.khi && P.kvmap) ? __ldg(P.kvmap + row) : -1;
            }
        };
        long long m_next[4];
        map_rows(0, m_next);
        for (int j = 0; j < n_tiles; ++j) {
            long long m[4] = {m_next[0], m_next[1], m_next[2], m_next[3]};
            map_rows(j + 1, m_next);
            const int s = j % kStages;
            const uint32_t ph = (uint32_t)(j / kStages) & 1u;
            if (!warp_wait(&sm.bar_empty[op][s], ph ^ 1u, sm, P.status)) break;
            const long long r0 = w.klo + (long long)j * kBN;
            // Lane l classifies rows 4l..4l+3; lanes 2g, 2g+1 form 8-row group g.
            bool pad[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                pad[i] = r0 + 4 * lane + i >= w.khi;
                if (m[i] >= P.arena_rows || (m[i] >= 0 && !P.arena)) {
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
            const bool g_arena = P.arena_boxes > 0 && asc && p_asc && (even ? p_m0 == m[0] + 4 : m[0] == p_m0 + 4);
            const unsigned base_mask = __ballot_sync(0xffffffffu, g_base);
            const unsigned arena_mask = __ballot_sync(0xffffffffu, g_arena);
            const unsigned mixed_mask = ~(base_mask | arena_mask);
            // One 128-row box per panel when no row is remapped; the box
            // starts inside the tensor (r0 < khi <= kv_rows).
            const bool whole_base = __all_sync(0xffffffffu, all_neg) && P.base_boxes == kBoxKinds;
            // Runs: a base or arena group continues the previous group's run
            // when it is the same kind and, for arena groups, its slots follow
            // on; each run head issues power-of-two boxes for the whole run.
            const long long prev_m0 = __shfl_up_sync(0xffffffffu, m[0], 2);
            const bool cont = even && lane >= 2 &&
                ((g_base && ((base_mask >> (lane - 2)) & 1u)) ||
                 (g_arena && ((arena_mask >> (lane - 2)) & 1u) && m[0] == prev_m0 + 8));
            const unsigned cont_mask = __ballot_sync(0xffffffffu, cont);
            uint8_t* dst_tile = op == 0 ? sm.k[s] : sm.v[s];
            uint64_t* full = &sm.bar_full[op][s];
            if (lane == 0) {
                uint32_t bytes = 0;
                if (whole_base) {
                    bytes = kTileBytes;
                } else {
                    for (int g = 0; g < 16; ++g)
                        if (((base_mask | arena_mask) >> (2 * g)) & 1u) bytes += 2 * kGroupPanel;
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
                    const int kinds = g_base ? P.base_boxes : P.arena_boxes;
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
                // Mixed / padding groups: lane -> (panel = lane/16, row = (lane/2)%8,
                // chunks 4*(lane%2) .. +3); 16-byte copies into the swizzled layout.
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
                    const __nv_bfloat16* src = m_row >= 0
                        ? P.arena + (size_t)m_row * 2 * D + acol + 64 * pnl
                        : base + (size_t)key * D + hcol + 64 * pnl;
                    uint4 buf[4];
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        buf[c] = is_pad ? make_uint4(0, 0, 0, 0)
                                        : __ldg(reinterpret_cast<const uint4*>(src) + c0 + c);
                    uint8_t* dst = dst_tile + pnl * kPanel;
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        *reinterpret_cast<uint4*>(dst + sw128_off(row_in_tile, c0 + c)) = buf[c];
                }
                // make the warp's own stores visible to the tensor cores (only
                // when some group was copied by hand)
                if (mixed_mask & 0x55555555u) fence_proxy_async_smem();
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(full);
            last_armed = j;
        }
        // Drain: never leave TMA writes in flight into a CTA that is exiting.
        if (lane == 0 && sm.abort_flag) {
            for (int j = last_armed > 0 ? last_armed - 1 : 0; j <= last_armed; ++j) {
                if (j < 0) continue;
                const unsigned long long t0 = globaltimer();
                while (!mbar_try_wait(&sm.bar_full[op][j % kStages], (uint32_t)(j / kStages) & 1u) &&
                       globaltimer() - t0 < kWaitNs) {
                }
            }
        }
    } else if (warp == 1) {
        // ============================ MMA issuer ==============================
        if (lane == 0) {
            const uint32_t q_s = smem_u32(sm.q);
            const uint32_t p_s0 = smem_u32(sm.p[0]);
            constexpr uint32_t idS = idesc_bf16(false);
            constexpr uint32_t idO = idesc_bf16(true);
            const uint32_t tmem_o = tmem + 128 * kSBuf;
            bool ok = mbar_wait(&sm.bar_q, 0, sm, P.status);
            int issued_pv = 0;
            for (int j = 0; ok && j <= n_tiles + kSBuf - 2; ++j) {
                if (j < n_tiles) {
                    const int s = j % kStages, b = j % kSBuf;
                    if (!mbar_wait(&sm.bar_full[0][s], (uint32_t)(j / kStages) & 1u, sm, P.status)) { ok = false; break; }
                    if (!mbar_wait(&sm.bar_s_free[b], ((uint32_t)(j / kSBuf) & 1u) ^ 1u, sm, P.status)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t k_s = smem_u32(sm.k[s]);
#pragma unroll
                    for (int ks = 0; ks < kDH / 16; ++ks) {
                        const uint32_t off = (uint32_t)(ks >> 2) * kPanel + (uint32_t)(ks & 3) * 32;
                        tc_mma(tmem + 128 * b, sw128_desc(q_s + off, 16, 1024),
                               sw128_desc(k_s + off, 16, 1024), idS, ks > 0 ? 1u : 0u);
                    }
                    tc_commit(&sm.bar_s_full[b]);
                    tc_commit(&sm.bar_empty[0][s]);   // K_j consumed: the K ring moves on
                }
                if (j >= kSBuf - 1 && j - (kSBuf - 1) < n_tiles) {
                    const int jp = j - (kSBuf - 1), s = jp % kStages;
                    if (!mbar_wait(&sm.bar_full[1][s], (uint32_t)(jp / kStages) & 1u, sm, P.status)) { ok = false; break; }
                    if (!mbar_wait(&sm.bar_p_full[jp & 1], (uint32_t)(jp >> 1) & 1u, sm, P.status)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t v_s = smem_u32(sm.v[s]);
#pragma unroll
                    for (int ks = 0; ks < kBN / 16; ++ks) {
                        const uint32_t a_off = (uint32_t)(ks >> 2) * kPanel + (uint32_t)(ks & 3) * 32;
                        tc_mma(tmem_o, sw128_desc(p_s0 + (uint32_t)(jp & 1) * kTileBytes + a_off, 16, 1024),
                               sw128_desc(v_s + (uint32_t)ks * 2048, kPanel, 1024), idO,
                               (jp > 0 || ks > 0) ? 1u : 0u);
                    }
                    tc_commit(&sm.bar_empty[1][s]);
                    tc_commit(&sm.bar_pv_done[jp & 1]);
                    issued_pv = jp + 1;
                }
            }
            // Drain: the last committed PV must land before TMEM is freed.
            if (issued_pv > 0) {
                const unsigned long long t0 = globaltimer();
                const int last = issued_pv - 1;
                while (!mbar_try_wait(&sm.bar_pv_done[last & 1], (uint32_t)(last >> 1) & 1u) &&
                       globaltimer() - t0 < kWaitNs) {
                }
            }
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ========================== softmax + epilogue ========================
        // Warps 4-11: warp w owns query rows 32*(w%4) .. +31 (its TMEM lane
        // quarter) and key columns [64*half, 64*half+64), half = (w-4)/4, of
        // every S tile; the two warps of a row block exchange their partial
        // row max through shared memory once per tile (named barrier of 64).
        const int half = (warp - 4) >> 2;
        const int row = (warp & 3) * 32 + lane;       // query row in tile == TMEM lane
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t col0 = 64u * (uint32_t)half;
        const int rg = warp & 3;                       // row block shared with warp w^4
        const long long my_khi = row < w.split ? w.khi_lo : w.khi;
        const float sl2 = P.scale_log2;
        float m_run = -INFINITY, l_run = 0.f;          // m in log2 units, scaled
        bool ok = true;
        for (int j = 0; j < n_tiles; ++j) {
            const int b = j & 1;           // parity buffer of the row-max exchange
            const int sb = j % kSBuf;      // S accumulator of this tile
            if (!warp_wait(&sm.bar_s_full[sb], (uint32_t)(j / kSBuf) & 1u, sm, P.status)) { ok = false; break; }
            tc_fence_after();
            uint32_t sr[64];
            const uint32_t s_addr = tmem + lane_base + 128 * sb + col0;
            KVP_TMEM_LD32(s_addr + 0, (sr + 0));
            KVP_TMEM_LD32(s_addr + 32, (sr + 32));
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(&sm.bar_s_free[sb]);

            float s[64];
#pragma unroll
            for (int c = 0; c < 64; ++c) s[c] = __uint_as_float(sr[c]);
            const long long key0 = w.klo + (long long)j * kBN + col0;
            const long long left = my_khi - key0;
            if (left < 64) {   // tail tile: keys past the row's span never count
#pragma unroll
                for (int c = 0; c < 64; ++c)
                    if (c >= left) s[c] = -INFINITY;
            }
            // row max over this half: 8 independent chains, then a short tree
            float mx8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) mx8[i] = s[i];
#pragma unroll
            for (int c = 8; c < 64; c += 8)
#pragma unroll
                for (int i = 0; i < 8; ++i) mx8[i] = fmaxf(mx8[i], s[c + i]);
            const float half_max = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                         fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
            sm.red[b][half][row] = half_max;
            mbar_arrive(&sm.bar_red[rg][b]);
            // Lazy rescaling: keep the running max unless the row max grows by
            // more than 8 (log2 units), so p <= 256 and O rarely needs a TMEM
            // round trip.  After the first tile the exponentials are computed
            // with the running max while the partner half's max is still in
            // flight; only a row whose max jumps recomputes them.
            float ps[8];
            uint32_t pk[32];
            auto exp_half = [&](float m) {
                const float neg_m = -m;
#pragma unroll
                for (int i = 0; i < 8; ++i) ps[i] = 0.f;
#pragma unroll
                for (int c = 0; c < 64; c += 2) {
                    const float x0 = fmaf(s[c], sl2, neg_m);
                    const float x1 = fmaf(s[c + 1], sl2, neg_m);
                    // a quarter of the exponentials run on the FMA pipe
                    const bool fma_pipe = (c & 7) == 6;
                    const float p0 = fma_pipe ? ex2_poly(x0) : ex2_approx(x0);
                    const float p1 = fma_pipe ? ex2_poly(x1) : ex2_approx(x1);
                    ps[(c >> 1) & 7] += p0 + p1;
                    pk[c >> 1] = pack_bf16(p0, p1);
                }
            };
            if (j > 0) exp_half(m_run);
            if (!warp_wait(&sm.bar_red[rg][b], (uint32_t)(j >> 1) & 1u, sm, P.status)) { ok = false; break; }
            const float tmax = fmaxf(half_max, sm.red[b][half ^ 1][row]) * sl2;  // both halves agree
            float m_use = m_run, alpha = 1.f;
            if (j == 0) {
                m_use = tmax;
                exp_half(m_use);
            } else if (tmax > m_run + 8.f) {
                m_use = tmax;
                alpha = ex2_approx(m_run - tmax);
                exp_half(m_use);
            }
            const float rsum = ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
            l_run = l_run * alpha + rsum;
            m_run = m_use;
            // warp-uniform: the TMEM round trip is .sync.aligned
            const bool any_rescale = __any_sync(0xffffffffu, alpha != 1.f);
            if (j >= 1 && any_rescale) {
                // O is rescaled only once PV_{j-1} has finished accumulating
                if (!warp_wait(&sm.bar_pv_done[(j - 1) & 1], (uint32_t)((j - 1) >> 1) & 1u, sm, P.status)) { ok = false; break; }
                tc_fence_after();
                const uint32_t o_addr = tmem + lane_base + 128 * kSBuf + col0;
#pragma unroll
                for (int c4 = 0; c4 < 2; ++c4) {
                    uint32_t o[32];
                    KVP_TMEM_LD32(o_addr + 32 * c4, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 32; ++c)
                        o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
                    KVP_TMEM_ST32(o_addr + 32 * c4, o);
                }
                tmem_wait_st();
            } else if (j >= 2) {
                // P buffer j&1 was last read by PV_{j-2}
                if (!warp_wait(&sm.bar_pv_done[j & 1], (uint32_t)((j - 2) >> 1) & 1u, sm, P.status)) { ok = false; break; }
            }
            // P row half -> shared memory panel `half` of buffer j&1 (K-major, 128B swizzle).
            uint8_t* pdst = sm.p[j & 1] + half * kPanel;
#pragma unroll
            for (int c = 0; c < 8; ++c)
                *reinterpret_cast<uint4*>(pdst + sw128_off(row, c)) =
                    make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(&sm.bar_p_full[j & 1]);
        }
        // Row sum = both halves' partial sums (same running max).
        // (the max buffer of parity n_tiles&1 was last read two tiles ago)
        float (&red_sum)[2][128] = sm.red[n_tiles & 1];
        red_sum[half][row] = l_run;
        mbar_arrive(&sm.bar_sum[rg]);
        if (ok) ok = warp_wait(&sm.bar_sum[rg], 0, sm, P.status);
        const float l_row = l_run + red_sum[half ^ 1][row];
        if (ok && n_tiles > 0 &&
            warp_wait(&sm.bar_pv_done[(n_tiles - 1) & 1], (uint32_t)((n_tiles - 1) >> 1) & 1u, sm, P.status)) {
            tc_fence_after();
            const float inv = 1.f / l_row;
            const uint32_t o_addr = tmem + lane_base + 128 * kSBuf + col0;
            __nv_bfloat16* dst = P.out + (size_t)(w.q_row0 + row) * D + hcol + col0;
#pragma unroll
            for (int c4 = 0; c4 < 2; ++c4) {
                uint32_t o[32];
                KVP_TMEM_LD32(o_addr + 32 * c4, o);
                tmem_wait_ld();
                if (row < w.nq) {
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

// 2D bf16 row-major tensor [rows][cols] with row pitch `pitch` elements.
int make_map(CUtensorMap* m, const void* base, long long rows, long long cols, long long pitch,
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

int launch_attn_bf16(const LayerIO& io, const AttnDesc& d, int* d_status, cudaStream_t stream) {
    const long long T = d.tokens;
    const int D = d.heads * kDH;
    if (d.head_dim != kDH || d.heads <= 0 || T <= 0 || d.frames <= 0 || d.q_frame0 < 0 ||
        d.nheads <= 0 || d.head0 < 0 || d.head0 + d.nheads > d.heads || d.window < 0 ||
        (d.mode != 0 && d.mode != 1) || !io.q || !io.k || !io.v || !io.out || !d_status) {
        set_error("attn_bf16: bad descriptor (head_dim must be %d)", kDH);
        return KVP_ERR_ARG;
    }
    if (d.flat && (d.mode != 1 || d.window != 0 || T < kBM)) {
        set_error("attn_bf16: flat query tiles need causal mode, no window and tokens >= %d", kBM);
        return KVP_ERR_ARG;
    }
    const long long q_end = (long long)(d.q_frame0 + d.frames) * T;
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
    TmaMaps maps;
    std::memset(&maps, 0, sizeof maps);
    // Box kinds whose height fits the tensor (a box never starts past the
    // end, and a taller box than the tensor is never encoded).
    int base_boxes = 0, arena_boxes = 0;
    while (base_boxes < kBoxKinds && (8LL << base_boxes) <= io.kv_rows) ++base_boxes;
    if (io.arena)
        while (arena_boxes < kBoxKinds && (8LL << arena_boxes) <= io.arena_rows) ++arena_boxes;
    int rc = make_map(&maps.q8, io.q, io.q_rows, D, D, 8);
    for (int i = 0; !rc && i < kBoxKinds; ++i) {
        const uint32_t h = 8u << (i < base_boxes ? i : 0);
        rc = make_map(&maps.kv[0][i], io.k, io.kv_rows, D, D, h);
        if (!rc) rc = make_map(&maps.kv[1][i], io.v, io.kv_rows, D, D, h);
        if (!rc && arena_boxes)
            rc = make_map(&maps.a[i], io.arena, io.arena_rows, 2 * D, 2 * D, 8u << (i < arena_boxes ? i : 0));
    }
    if (rc) return rc;
    if (base_boxes == 0 || io.q_rows < 8) {
        set_error("attn_bf16: Q and K/V need at least 8 rows");
        return KVP_ERR_ARG;
    }

    Params P;
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
    P.n_qt = (int)((T + kBM - 1) / kBM);
    P.items_per_head = d.flat ? (int)((d.frames * T + kBM - 1) / kBM) : d.frames * P.n_qt;
    P.base_boxes = base_boxes;
    P.arena_boxes = arena_boxes;
    P.scale_log2 = 1.4426950408889634f / sqrtf((float)kDH);

    const int smem = (int)sizeof(Smem);
    {
        int dev = 0, optin = 0;
        KVP_CUDA(cudaGetDevice(&dev));
        KVP_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        if (smem > optin) {
            set_error("attn_bf16: needs %d B of shared memory per block, device allows %d", smem, optin);
            return KVP_ERR_UNSUPPORTED;
        }
    }
    static int configured_smem = 0;
    if (configured_smem != smem) {
        KVP_CUDA(cudaFuncSetAttribute(attn_bf16_sm100_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        configured_smem = smem;
    }
    const long long grid = (long long)d.nheads * P.items_per_head;
    if (grid <= 0 || grid > 0x7fffffffLL) return KVP_ERR_ARG;
    attn_bf16_sm100_kernel<<<(unsigned)grid, kThreads, smem, stream>>>(maps, P);
    KVP_CUDA(cudaGetLastError());
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
