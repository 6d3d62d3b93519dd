// QKV projection for B200 (sm_100a) that writes admitted K/V rows straight
// into the arena, plus the block's LayerNorm.
//
// Semantics: the reference block's attention input (src/backbone.py:13-33):
//   h = LayerNorm(x) (nn.LayerNorm(D), biased variance, eps), then
//   y = h . W^T + b with W = qkv_proj.weight [3D][D], and
//   qkv.view(b, t, 3, heads, head_dim) splits y's columns into Q [0, D),
//   K [D, 2D), V [2D, 3D), head h at columns [h*128, h*128+128) of each,
// computed in bf16 with fp32 accumulation.  Beyond the reference, every K/V
// row whose KVMap entry names an arena slot is also written to that slot (K
// half at column 0, V half at column D of a 2D-wide row), the same bf16
// values as the base row: a session whose rows are produced here needs no
// gather launch, and attention through the arena stays bitwise equal to
// attention over the base rows.
//
// GEMM: persistent CTAs (one per SM) walk the 256 x 256 output tiles in
// row-major tile order (concurrent CTAs share A row blocks; all of W stays
// in L2).  A tile is two 128-row halves that share every B tile: per K block
// an SM takes in 64 KB for 2 x 128 x 256 x 64 MACs, the rate one SM's L2
// port sustains at the tensor pipe's pace (a 128 x 256 tile needs half as
// many MACs per byte and stalls on L2 ingress at ~60% tensor use).  Per CTA
// (384 threads):
//   warp 0      TMA producer: per 64-column K block two A boxes [128][64]
//               and one B box [256][64], 128B swizzle, into a 3-stage ring
//   warp 1      TMEM allocation (all 512 columns: one 256-column accumulator
//               per half) and the single-thread MMA issuer: per K block
//               tcgen05.mma M128 N256 K16 x 4 for each half, then a commit
//               that frees the ring stage; per tile a commit that hands the
//               accumulators to the epilogue
//   warps 4-11  epilogue: warp w reads TMEM lanes 32*(w%4).. of half
//               (w-4)/4 (its 32 rows, all 256 columns), adds the bias, rounds
//               to bf16 and stores 16-byte vectors to the Q/K/V rows and, for
//               admitted rows, to the arena
// TMEM holds one tile, so the next tile's MMAs wait for the epilogue (about a
// tenth of a tile's MMA time).  Every mbarrier wait is bounded (about one
// second): on expiry the CTA records KVP_STATUS_TIMEOUT, waits (bounded) for
// its own TMA loads and MMAs in flight, frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>

#include "attn_sm100.h"
#include "kvp_common.h"
#include "qkv_sm100.h"
#include "sm100_ptx.h"

namespace kvp {

namespace {

using namespace ptx;

constexpr int kGM = 256;          // output rows per tile (two 128-row halves)
constexpr int kGH = 128;          // rows per half (TMEM lanes, MMA M)
constexpr int kGN = 256;          // output columns per tile (MMA N)
constexpr int kGK = 64;           // K block: one 128-byte swizzle row of bf16
constexpr int kGStages = 3;       // depth of the A/B ring
constexpr int kGThreads = 384;    // producer, MMA, 2 idle, 8 epilogue warps
constexpr uint32_t kHalfBytes = kGH * kGK * 2;  // 16 KB: one half's A box
constexpr uint32_t kABytes = kGM * kGK * 2;     // 32 KB
constexpr uint32_t kBBytes = kGN * kGK * 2;     // 32 KB

struct __align__(1024) GSmem {
    uint8_t a[kGStages][kABytes];
    uint8_t b[kGStages][kBBytes];
    uint8_t stage_out[8][32 * 128];  // per epilogue warp: 32 rows x 64 bf16
    uint64_t full[kGStages];      // TMA bytes of the stage landed
    uint64_t empty[kGStages];     // the stage's MMAs completed
    uint64_t acc_full;            // the tile's last MMA completed
    uint64_t acc_empty;           // the epilogue read the accumulators (8 warps)
    uint64_t mma_done;            // every MMA this CTA issued completed
    uint32_t tmem_base;
    int abort_flag;
};
constexpr size_t kGSmemBytes = sizeof(GSmem) + 1024;   // + realignment slack
static_assert(kGSmemBytes <= 227 * 1024, "QKV ring exceeds shared memory");

struct GParams {
    const float* bias;            // [3D] or null
    __nv_bfloat16* q;             // [rows][D] or null
    __nv_bfloat16* k;             // [rows][D]
    __nv_bfloat16* v;             // [rows][D]
    __nv_bfloat16* arena;         // [arena_rows][2D] or null
    const long long* kvmap;       // indexed by map_row0 + row, or null
    int* status;
    long long rows, map_row0, arena_rows;
    int D, kblocks, n_tiles_n, n_tiles;
    uint32_t stage_bytes;         // bytes the two boxes of one stage deliver
};

// kind::f16 instruction descriptor: bf16 x bf16 -> f32, A and B K-major,
// M = 128, N = 256.
constexpr uint32_t kIdescM128N256 = (1u << 4) | (1u << 7) | (1u << 10) |
                                    ((uint32_t)(kGN >> 3) << 17) | ((uint32_t)(kGH >> 4) << 24);

__device__ __forceinline__ void st_global_v4(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}

__global__ void __launch_bounds__(kGThreads, 1)
qkv_proj_sm100_kernel(const __grid_constant__ CUtensorMap map_x,
                      const __grid_constant__ CUtensorMap map_w, const __grid_constant__ GParams P) {
    extern __shared__ uint8_t smem_raw[];
    GSmem& sm = *reinterpret_cast<GSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                          ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kGStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        mbar_init(&sm.acc_full, 1);
        mbar_init(&sm.acc_empty, 8);
        mbar_init(&sm.mma_done, 1);
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

    if (warp == 0) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            long long issued = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < P.n_tiles && ok; t += gridDim.x) {
                const int m0 = (t / P.n_tiles_n) * kGM;
                const int n0 = (t % P.n_tiles_n) * kGN;
                for (int kb = 0; kb < P.kblocks; ++kb) {
                    if (!(ok = mbar_wait(&sm.empty[stage], phase ^ 1u, sm, P.status))) break;
                    mbar_arrive_expect_tx(&sm.full[stage], P.stage_bytes);
                    // (the second half's box may start past the last row: it
                    // reads zeros, and its bytes still count)
                    tma_load_2d(sm.a[stage], &map_x, kb * kGK, m0, &sm.full[stage]);
                    tma_load_2d(sm.a[stage] + kHalfBytes, &map_x, kb * kGK, m0 + kGH, &sm.full[stage]);
                    tma_load_2d(sm.b[stage], &map_w, kb * kGK, n0, &sm.full[stage]);
                    ++issued;
                    if (++stage == kGStages) { stage = 0; phase ^= 1u; }
                }
            }
            if (!ok) {
                // Let the loads already issued land before the CTA exits: the
                // last min(issued, stages) stages, each at the phase it was
                // armed with.
                for (int i = 0; i < kGStages && i < issued; ++i) {
                    if (--stage < 0) { stage = kGStages - 1; phase ^= 1u; }
                    const unsigned long long t0 = globaltimer();
                    while (!mbar_try_wait_sleep(&sm.full[stage], phase) && globaltimer() - t0 < kWaitNs) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------- MMA issuer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int i = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < P.n_tiles && ok; t += gridDim.x, ++i) {
                if (!(ok = mbar_wait(&sm.acc_empty, (i & 1) ^ 1u, sm, P.status))) break;
                tc_fence_after();
                for (int kb = 0; kb < P.kblocks; ++kb) {
                    if (!(ok = mbar_wait(&sm.full[stage], phase, sm, P.status))) break;
                    tc_fence_after();
                    const uint64_t da = sw128_desc(smem_u32(sm.a[stage]), 16, 1024);
                    const uint64_t db = sw128_desc(smem_u32(sm.b[stage]), 16, 1024);
                    // K16 step ks starts 32 bytes further into the 128-byte
                    // swizzle row: +2 in the descriptor's 16-byte address
                    // field; the second half's A box is 16 KB further (+1024).
#pragma unroll
                    for (int ks = 0; ks < kGK / 16; ++ks) {
                        tc_mma(tmem, da + 2 * ks, db + 2 * ks, kIdescM128N256, (kb | ks) != 0);
                        tc_mma(tmem + kGN, da + (kHalfBytes >> 4) + 2 * ks, db + 2 * ks,
                               kIdescM128N256, (kb | ks) != 0);
                    }
                    tc_commit(&sm.empty[stage]);
                    if (++stage == kGStages) { stage = 0; phase ^= 1u; }
                }
                if (ok) tc_commit(&sm.acc_full);
            }
            // Every MMA issued has completed before TMEM is freed.
            tc_commit(&sm.mma_done);
            const unsigned long long t0 = globaltimer();
            while (!mbar_try_wait_sleep(&sm.mma_done, 0) && globaltimer() - t0 < kWaitNs) {
            }
        }
    } else if (warp >= 4) {
        // --------------------------------------------------------- epilogue
        // Per 64-column pair: TMEM -> registers (thread = row), + bias, bf16,
        // into this warp's staging rows; then read back so that one store
        // instruction writes 4 rows x 128 contiguous bytes (full lines)
        // instead of 32 rows x 16 bytes.  Staging row r keeps its eight
        // 16-byte chunks at positions chunk ^ (r & 7): both the row-wise
        // writes and the chunk-wise reads are free of bank conflicts.
        const int quarter = warp & 3;          // TMEM lanes 32*quarter ..
        const int half = (warp - 4) >> 2;      // tile rows [128*half, +128)
        uint8_t* stg = sm.stage_out[warp - 4];
        const int cc = lane & 7;               // store phase: 16-byte chunk of a row
        const int rsub = lane >> 3;            // store phase: row 4*j + rsub
        const long long D = P.D;
        int i = 0;
        for (int t = blockIdx.x; t < P.n_tiles; t += gridDim.x, ++i) {
            if (!warp_wait(&sm.acc_full, i & 1, sm, P.status)) break;
            tc_fence_after();
            const long long wrow0 = (long long)(t / P.n_tiles_n) * kGM + half * kGH + quarter * 32;
            const int n0 = (t % P.n_tiles_n) * kGN;
            const int region = n0 / P.D;                 // 0 Q, 1 K, 2 V (D % 256 == 0)
            const int col0 = n0 - region * P.D;
            long long my_slot = -1;                      // arena slot of row wrow0 + lane
            if (region > 0 && wrow0 + lane < P.rows && P.kvmap && P.arena) {
                const long long sl = P.kvmap[P.map_row0 + wrow0 + lane];
                if (sl >= P.arena_rows) atomicOr(P.status, KVP_STATUS_MAP);
                else if (sl >= 0) my_slot = sl;
            }
            long long slot_j[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) slot_j[j] = __shfl_sync(0xffffffffu, my_slot, 4 * j + rsub);
            __nv_bfloat16* base = region == 0 ? P.q : region == 1 ? P.k : P.v;
            __nv_bfloat16* arena = P.arena ? P.arena + (region - 1) * D + col0 : nullptr;
            const float* bias = P.bias ? P.bias + n0 : nullptr;
            const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(half * kGN);
#pragma unroll 1
            for (int p = 0; p < kGN / 64; ++p) {
#pragma unroll 1
                for (int c2 = 0; c2 < 2; ++c2) {
                    const int c = 2 * p + c2;
                    uint32_t r[32];
                    KVP_TMEM_LD32(taddr + c * 32, r);
                    KVP_TMEM_WAIT_LD_DEP(r);
                    float bv[32];
                    if (bias) {
                        const float4* b4 = reinterpret_cast<const float4*>(bias + c * 32);
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const float4 x = __ldg(b4 + j);
                            bv[4 * j] = x.x; bv[4 * j + 1] = x.y; bv[4 * j + 2] = x.z; bv[4 * j + 3] = x.w;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) bv[j] = 0.f;
                    }
                    uint32_t pk[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        pk[j] = pack_bf16(__uint_as_float(r[2 * j]) + bv[2 * j],
                                          __uint_as_float(r[2 * j + 1]) + bv[2 * j + 1]);
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        *reinterpret_cast<uint4*>(stg + lane * 128 + (((c2 * 4 + j) ^ (lane & 7)) << 4)) =
                            make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
                }
                if (p == kGN / 64 - 1) {
                    // every TMEM column of the tile is in registers or staged:
                    // the next tile's MMAs may start while the stores drain
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sm.acc_empty);
                }
                __syncwarp();
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int rr = 4 * j + rsub;
                    const uint4 val = *reinterpret_cast<const uint4*>(stg + rr * 128 + ((cc ^ (rr & 7)) << 4));
                    const long long grow = wrow0 + rr;
                    if (grow < P.rows) {
                        const int col = p * 64 + cc * 8;
                        if (base) st_global_v4(base + grow * D + col0 + col, val.x, val.y, val.z, val.w);
                        if (slot_j[j] >= 0)
                            st_global_v4(arena + slot_j[j] * 2 * D + col, val.x, val.y, val.z, val.w);
                    }
                }
                __syncwarp();
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

// ----------------------------------------------------------------- LayerNorm
// y = (x - mean) / sqrt(var + eps) * gamma + beta per row, biased variance,
// statistics in fp32 (nn.LayerNorm).  One warp per row, 16-byte loads; the
// row is read three times, the second and third time from L1.
__global__ void __launch_bounds__(256)
layernorm_bf16_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ gamma,
                      const float* __restrict__ beta, __nv_bfloat16* __restrict__ y,
                      long long rows, int D, float eps) {
    const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * D);
    uint4* yr = reinterpret_cast<uint4*>(y + row * D);
    const int chunks = D / 8;
    float s = 0.f;
    for (int c = lane; c < chunks; c += 32) {
        const uint4 u = xr[c];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __bfloat1622float2(h[j]);
            s += f.x + f.y;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / (float)D;
    float ss = 0.f;
    for (int c = lane; c < chunks; c += 32) {
        const uint4 u = xr[c];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __bfloat1622float2(h[j]);
            ss += (f.x - mean) * (f.x - mean) + (f.y - mean) * (f.y - mean);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rstd = 1.f / sqrtf(ss / (float)D + eps);
    for (int c = lane; c < chunks; c += 32) {
        const uint4 u = xr[c];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
        const float4 g0 = __ldg(reinterpret_cast<const float4*>(gamma) + 2 * c);
        const float4 g1 = __ldg(reinterpret_cast<const float4*>(gamma) + 2 * c + 1);
        const float4 b0 = __ldg(reinterpret_cast<const float4*>(beta) + 2 * c);
        const float4 b1 = __ldg(reinterpret_cast<const float4*>(beta) + 2 * c + 1);
        const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        uint4 o;
        uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __bfloat1622float2(h[j]);
            op[j] = pack_bf16((f.x - mean) * rstd * g[2 * j] + b[2 * j],
                              (f.y - mean) * rstd * g[2 * j + 1] + b[2 * j + 1]);
        }
        yr[c] = o;
    }
}

// Same LayerNorm with the row held in registers: each lane keeps its
// kChunks 16-byte chunks, so the row is read from memory once (D = 256 *
// kChunks).  Statistics in the same order as the three-pass kernel.
template <int kChunks>
__global__ void __launch_bounds__(256)
layernorm_bf16_reg_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ gamma,
                          const float* __restrict__ beta, __nv_bfloat16* __restrict__ y,
                          long long rows, float eps) {
    constexpr int D = kChunks * 256;
    const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * D);
    uint4* yr = reinterpret_cast<uint4*>(y + row * D);
    uint4 u[kChunks];
#pragma unroll
    for (int i = 0; i < kChunks; ++i) u[i] = xr[lane + 32 * i];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u[i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __bfloat1622float2(h[j]);
            s += f.x + f.y;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / (float)D;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u[i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __bfloat1622float2(h[j]);
            ss += (f.x - mean) * (f.x - mean) + (f.y - mean) * (f.y - mean);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rstd = 1.f / sqrtf(ss / (float)D + eps);
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
        const int c = lane + 32 * i;
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u[i]);
        const float4 g0 = __ldg(reinterpret_cast<const float4*>(gamma) + 2 * c);
        const float4 g1 = __ldg(reinterpret_cast<const float4*>(gamma) + 2 * c + 1);
        const float4 b0 = __ldg(reinterpret_cast<const float4*>(beta) + 2 * c);
        const float4 b1 = __ldg(reinterpret_cast<const float4*>(beta) + 2 * c + 1);
        const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        uint4 o;
        uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __bfloat1622float2(h[j]);
            op[j] = pack_bf16((f.x - mean) * rstd * g[2 * j] + b[2 * j],
                              (f.y - mean) * rstd * g[2 * j + 1] + b[2 * j + 1]);
        }
        yr[c] = o;
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

int launch_qkv_project_bf16(const QkvIO& io, int* d_status, cudaStream_t stream) {
    const long long D = io.D;
    const long long m_tiles = (io.rows + kGM - 1) / kGM;
    if (!io.x || !io.w || !io.k || !io.v || io.rows < kGH || D < 256 || D % 256 != 0 ||
        D > (1 << 16) || io.map_row0 < 0 || (io.kvmap && (!io.arena || io.arena_rows < 0)) ||
        !aligned16(io.x) || !aligned16(io.w) || !aligned16(io.k) || !aligned16(io.v) ||
        (io.q && !aligned16(io.q)) || (io.arena && !aligned16(io.arena)) ||
        (io.bias && !aligned16(io.bias)) || m_tiles * (3 * D / kGN) > (1LL << 30)) {
        set_error("qkv_project: invalid arguments (rows >= 128, D %% 256 == 0, D >= 256, 16-byte "
                  "aligned buffers, a map needs an arena)");
        return KVP_ERR_ARG;
    }
    if (!d_status) d_status = status_word();   // after the argument checks: they need no device
    if (!d_status) return KVP_ERR_CUDA;
    static PerDeviceOnce setup;
    const int rc_setup = setup([](int) {
        KVP_CUDA(cudaFuncSetAttribute(qkv_proj_sm100_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)kGSmemBytes));
        return (int)KVP_OK;
    });
    if (rc_setup != KVP_OK) return rc_setup;

    // The last row block's boxes reach past `rows`: TMA fills those rows
    // with zeros (and counts their bytes), the epilogue stores no row >= rows.
    CUtensorMap mx, mw;
    int rc = make_bf16_tensor_map(&mx, io.x, io.rows, D, D, kGH);
    if (rc != KVP_OK) return rc;
    rc = make_bf16_tensor_map(&mw, io.w, 3 * D, D, D, kGN);
    if (rc != KVP_OK) return rc;

    GParams P{};
    P.bias = io.bias;
    P.q = static_cast<__nv_bfloat16*>(io.q);
    P.k = static_cast<__nv_bfloat16*>(io.k);
    P.v = static_cast<__nv_bfloat16*>(io.v);
    P.arena = static_cast<__nv_bfloat16*>(io.arena);
    P.kvmap = io.kvmap;
    P.status = d_status;
    P.rows = io.rows;
    P.map_row0 = io.map_row0;
    P.arena_rows = io.arena_rows;
    P.D = (int)D;
    P.kblocks = (int)(D / kGK);
    P.n_tiles_n = (int)(3 * D / kGN);
    P.n_tiles = (int)(m_tiles * P.n_tiles_n);
    P.stage_bytes = kABytes + kBBytes;

    int dev = 0, sms = 148;
    KVP_CUDA(cudaGetDevice(&dev));
    KVP_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int grid = P.n_tiles < sms ? P.n_tiles : sms;
    qkv_proj_sm100_kernel<<<grid, kGThreads, kGSmemBytes, stream>>>(mx, mw, P);
    KVP_CUDA(cudaGetLastError());
    return KVP_OK;
}

int launch_layernorm_bf16(const void* x, const float* gamma, const float* beta, void* y,
                          long long rows, int D, float eps, cudaStream_t stream) {
    if (!x || !gamma || !beta || !y || rows <= 0 || D <= 0 || D % 8 != 0 || !aligned16(x) ||
        !aligned16(y) || !aligned16(gamma) || !aligned16(beta) || !(eps > 0.f)) {
        set_error("layernorm: invalid arguments (D %% 8 == 0, 16-byte aligned buffers, eps > 0)");
        return KVP_ERR_ARG;
    }
    const long long blocks = (rows + 7) / 8;
    const auto* xb = static_cast<const __nv_bfloat16*>(x);
    auto* yb = static_cast<__nv_bfloat16*>(y);
    switch (D % 256 == 0 ? D / 256 : 0) {
        case 1: layernorm_bf16_reg_kernel<1><<<(unsigned)blocks, 256, 0, stream>>>(xb, gamma, beta, yb, rows, eps); break;
        case 2: layernorm_bf16_reg_kernel<2><<<(unsigned)blocks, 256, 0, stream>>>(xb, gamma, beta, yb, rows, eps); break;
        case 3: layernorm_bf16_reg_kernel<3><<<(unsigned)blocks, 256, 0, stream>>>(xb, gamma, beta, yb, rows, eps); break;
        case 4: layernorm_bf16_reg_kernel<4><<<(unsigned)blocks, 256, 0, stream>>>(xb, gamma, beta, yb, rows, eps); break;
        case 5: layernorm_bf16_reg_kernel<5><<<(unsigned)blocks, 256, 0, stream>>>(xb, gamma, beta, yb, rows, eps); break;
        case 6: layernorm_bf16_reg_kernel<6><<<(unsigned)blocks, 256, 0, stream>>>(xb, gamma, beta, yb, rows, eps); break;
        case 8: layernorm_bf16_reg_kernel<8><<<(unsigned)blocks, 256, 0, stream>>>(xb, gamma, beta, yb, rows, eps); break;
        default:
            layernorm_bf16_kernel<<<(unsigned)blocks, 256, 0, stream>>>(xb, gamma, beta, yb, rows, D, eps);
    }
    KVP_CUDA(cudaGetLastError());
    return KVP_OK;
}

}  // namespace kvp
