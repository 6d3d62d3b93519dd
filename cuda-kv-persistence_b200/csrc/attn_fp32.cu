// FP32 remapped multi-head attention on CUDA cores (the FP32 correctness
// path and the engine behind the reference-compatible attn_forward_* entry
// points).
//
// Semantics are those of the reference's attn_forward_kernel
// (src/gated_attention_kernel.cu:34-139): per (query row, head),
// softmax(q.K^T / sqrt(dh)) . V over a span of key rows, where key row j is
// read from arena row KVMap[j] (K half, then V half at +D) when KVMap[j] >= 0
// and from the base K/V otherwise.  The arena holds exact copies of base
// rows, and the arithmetic order below never depends on where a row was read
// from, so results are bitwise identical whatever the policy.
//
// Layout of the work (not the reference's one-warp-per-row design): a CTA
// owns 64 query rows of one head; 256 threads each hold a 4x4 block of the
// 64x64 score tile and a 4x8 block of the 64x128 output, fed by transposed
// Q/K tiles in shared memory (two 128-bit loads per 16 FMAs).  Online softmax
// in exp2 form with the 1/sqrt(dh) scale folded into log2(e).
#include <cfloat>

#include "kernels.h"
#include "kvp_common.h"

namespace kvp {

namespace {

constexpr int kBQ = 64;     // query rows per CTA
constexpr int kBK = 64;     // keys per tile
constexpr int kDH = 128;    // head dim (the reference hard-wires 128)
constexpr int kThreads = 256;

struct __align__(16) Fp32Smem {
    float qt[kDH][kBQ];     // Q^T  (d-major)
    float kt[kDH][kBK];     // K^T
    float vs[kBK][kDH];     // V
    float pt[kBK][kBQ];     // P^T
    long long map[kBK];
};

__global__ void __launch_bounds__(kThreads, 2)
attn_fp32_kernel(const float* __restrict__ Q, const float* __restrict__ K,
                 const float* __restrict__ V, const float* __restrict__ Arena,
                 const int64_t* __restrict__ KVMap, float* __restrict__ Out, int T, int D,
                 int64_t k_lo, int64_t k_hi, int64_t arena_rows, int64_t frame_stride_rows,
                 int* __restrict__ status) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Fp32Smem& sm = *reinterpret_cast<Fp32Smem*>(smem_raw);

    const int tid = threadIdx.x;
    const int ty = tid >> 4;    // 0..15 -> query rows 4*ty .. 4*ty+3
    const int tx = tid & 15;    // 0..15 -> key cols 4*tx.., out cols 4*tx.. and 64+4*tx..
    const int head = blockIdx.y;
    const int q0 = blockIdx.x * kBQ;
    const int64_t z = blockIdx.z;
    const float* Qf = Q + (size_t)z * T * D;
    float* Of = Out + (size_t)z * T * D;
    const int64_t lo = k_lo + z * frame_stride_rows;
    const int64_t hi = k_hi + z * frame_stride_rows;
    const int hc = head * kDH;

    // Q tile, transposed; rows past T are zero (their outputs are dropped).
    for (int idx = tid; idx < kBQ * (kDH / 4); idx += kThreads) {
        const int r = idx % kBQ, d4 = idx / kBQ;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (q0 + r < T) x = *reinterpret_cast<const float4*>(Qf + (size_t)(q0 + r) * D + hc + 4 * d4);
        sm.qt[4 * d4 + 0][r] = x.x;
        sm.qt[4 * d4 + 1][r] = x.y;
        sm.qt[4 * d4 + 2][r] = x.z;
        sm.qt[4 * d4 + 3][r] = x.w;
    }

    const float scale_log2 = 1.4426950408889634f * rsqrtf((float)kDH);
    float m[4], l[4], o[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -FLT_MAX;
        l[i] = 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) o[i][c] = 0.f;
    }

    for (int64_t j0 = lo; j0 < hi; j0 += kBK) {
        const int valid = (int)((hi - j0) < kBK ? (hi - j0) : kBK);
        __syncthreads();  // previous tile fully consumed
        if (tid < kBK) {
            long long mv = -1;
            if (tid < valid && KVMap) {
                mv = (long long)KVMap[j0 + tid];
                if (mv >= arena_rows || (mv >= 0 && !Arena)) {
                    atomicOr(status, 1);   // map entry outside the arena: read the base row
                    mv = -1;
                }
            }
            sm.map[tid] = mv;
        }
        __syncthreads();
        for (int idx = tid; idx < kBK * (kDH / 4); idx += kThreads) {
            const int r = idx % kBK, d4 = idx / kBK;
            float4 kx = make_float4(0.f, 0.f, 0.f, 0.f), vx = kx;
            if (r < valid) {
                const long long mv = sm.map[r];
                const float* krow = mv >= 0 ? Arena + (size_t)mv * 2 * D + hc
                                            : K + (size_t)(j0 + r) * D + hc;
                const float* vrow = mv >= 0 ? Arena + (size_t)mv * 2 * D + D + hc
                                            : V + (size_t)(j0 + r) * D + hc;
                kx = __ldg(reinterpret_cast<const float4*>(krow) + d4);
                vx = __ldg(reinterpret_cast<const float4*>(vrow) + d4);
            }
            sm.kt[4 * d4 + 0][r] = kx.x;
            sm.kt[4 * d4 + 1][r] = kx.y;
            sm.kt[4 * d4 + 2][r] = kx.z;
            sm.kt[4 * d4 + 3][r] = kx.w;
            *reinterpret_cast<float4*>(&sm.vs[r][4 * d4]) = vx;
        }
        __syncthreads();

        // S = Q K^T for this thread's 4x4 block.
        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int c = 0; c < 4; ++c) s[i][c] = 0.f;
#pragma unroll 8
        for (int d = 0; d < kDH; ++d) {
            const float4 qa = *reinterpret_cast<const float4*>(&sm.qt[d][4 * ty]);
            const float4 kb = *reinterpret_cast<const float4*>(&sm.kt[d][4 * tx]);
            const float qv[4] = {qa.x, qa.y, qa.z, qa.w};
            const float kv[4] = {kb.x, kb.y, kb.z, kb.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int c = 0; c < 4; ++c) s[i][c] = fmaf(qv[i], kv[c], s[i][c]);
        }

        // Online softmax: the 16 threads of a half-warp share the same rows.
        float p[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float tmax = -FLT_MAX;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                s[i][c] = (4 * tx + c < valid) ? s[i][c] * scale_log2 : -FLT_MAX;
                tmax = fmaxf(tmax, s[i][c]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1)
                tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
            const float m_new = fmaxf(m[i], tmax);
            const float corr = exp2f(m[i] - m_new);
            float psum = 0.f;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                p[i][c] = (4 * tx + c < valid) ? exp2f(s[i][c] - m_new) : 0.f;
                psum += p[i][c];
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
            l[i] = l[i] * corr + psum;
            m[i] = m_new;
#pragma unroll
            for (int c = 0; c < 8; ++c) o[i][c] *= corr;
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
            *reinterpret_cast<float4*>(&sm.pt[4 * tx + c][4 * ty]) =
                make_float4(p[0][c], p[1][c], p[2][c], p[3][c]);
        __syncthreads();

        // O += P V
#pragma unroll 4
        for (int k = 0; k < kBK; ++k) {
            const float4 pa = *reinterpret_cast<const float4*>(&sm.pt[k][4 * ty]);
            const float4 v0 = *reinterpret_cast<const float4*>(&sm.vs[k][4 * tx]);
            const float4 v1 = *reinterpret_cast<const float4*>(&sm.vs[k][64 + 4 * tx]);
            const float pv[4] = {pa.x, pa.y, pa.z, pa.w};
            const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int c = 0; c < 8; ++c) o[i][c] = fmaf(pv[i], vv[c], o[i][c]);
        }
    }

#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int row = q0 + 4 * ty + i;
        if (row >= T) continue;
        const float inv = 1.f / l[i];
        float* dst = Of + (size_t)row * D + hc;
        *reinterpret_cast<float4*>(dst + 4 * tx) =
            make_float4(o[i][0] * inv, o[i][1] * inv, o[i][2] * inv, o[i][3] * inv);
        *reinterpret_cast<float4*>(dst + 64 + 4 * tx) =
            make_float4(o[i][4] * inv, o[i][5] * inv, o[i][6] * inv, o[i][7] * inv);
    }
}

}  // namespace

int launch_attn_fp32(const float* q, const float* k, const float* v, const float* arena,
                     const int64_t* kvmap, float* out, int T, int D, int heads, int64_t k_lo,
                     int64_t k_hi, int64_t arena_rows, int frames, int64_t frame_stride_rows,
                     int* d_status, cudaStream_t stream) {
    if (!q || !k || !v || !out || !d_status || T <= 0 || heads <= 0 || frames <= 0 ||
        k_hi <= k_lo || D != heads * kDH) {
        set_error("attn_fp32: bad arguments (T=%d D=%d heads=%d span=[%lld,%lld)); head_dim must be %d",
                  T, D, heads, (long long)k_lo, (long long)k_hi, kDH);
        return KVP_ERR_ARG;
    }
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out | (uintptr_t)arena) & 15) {
        set_error("attn_fp32: Q/K/V/Out/Arena must be 16-byte aligned");
        return KVP_ERR_ARG;
    }
    const int smem = (int)sizeof(Fp32Smem);
    static PerDeviceOnce setup;
    const int rc_setup = setup([&](int) -> int {
        KVP_CUDA(cudaFuncSetAttribute(attn_fp32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        return KVP_OK;
    });
    if (rc_setup != KVP_OK) return rc_setup;
    dim3 grid((unsigned)((T + kBQ - 1) / kBQ), (unsigned)heads, (unsigned)frames);
    attn_fp32_kernel<<<grid, kThreads, smem, stream>>>(q, k, v, arena, kvmap, out, T, D, k_lo, k_hi,
                                                       arena_rows, frame_stride_rows, d_status);
    KVP_CUDA(cudaGetLastError());
    return KVP_OK;
}

}  // namespace kvp
