// Softmax arithmetic shared by the sm_100a attention kernels (attn_sm100.cu,
// attn_pair_sm100.cu): packed fp32 pairs, 2^x on MUFU and on the FMA pipe,
// and the two passes over one S row held in tensor memory.
#pragma once

#include <cstdint>

#include "sm100_ptx.h"

namespace kvp {
namespace attn_dev {

using namespace ptx;

// Which of the 16 column pairs of each 32-column chunk take the FMA-pipe
// exponential (ex2_poly2) instead of MUFU: bit p = pair p.  Two pairs in
// sixteen (one exponential in eight) measured fastest on the 21-frame
// layer; four, six and eight pairs were 1 %, 9 % and 12 % slower.
#ifndef KVP_POLY_PAIRS
#define KVP_POLY_PAIRS 0x8080u
#endif
constexpr uint32_t kPolyPairs = KVP_POLY_PAIRS;

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Packed fp32 pairs (sm_100 f32x2 instructions: one issue slot per pair).
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// 2^x for a pair on the FMA/ALU pipes (f32x2 arithmetic): x = n + f with
// n = round(x) and f in [-1/2, 1/2], 2^f by a cubic fitted here by iteratively reweighted least squares on the
// relative error (max relative error 1.4e-4 over x in [-126, 8], against bf16's
// 3.9e-3 rounding of P), 2^n added to the exponent bits.  Inputs below -126
// are clamped to -126 (the result stays a positive number below 2^-125,
// negligible in the row sum and against any unmasked P; -inf lands there
// too), inputs above 127 to 127 (a finite 2^127-ish value, so an overgrown
// speculative exponent still shows up in the row sum instead of wrapping
// the exponent bits).
__device__ __forceinline__ void ex2_poly2(float x0, float x1, float& y0, float& y1) {
    const uint64_t x = f2_pack(fminf(fmaxf(x0, -126.f), 127.f), fminf(fmaxf(x1, -126.f), 127.f));
    const uint64_t magic = f2_pack(12582912.f, 12582912.f);
    const uint64_t t = f2_add(x, magic);
    const uint64_t f = f2_sub(x, f2_sub(t, magic));
    uint64_t q = f2_fma(f2_pack(5.517162719e-02f, 5.517162719e-02f), f, f2_pack(2.426111432e-01f, 2.426111432e-01f));
    q = f2_fma(q, f, f2_pack(6.932609953e-01f, 6.932609953e-01f));
    q = f2_fma(q, f, f2_pack(9.999280725e-01f, 9.999280725e-01f));
    float t0, t1, q0, q1;
    f2_unpack(t, t0, t1);
    f2_unpack(q, q0, q1);
    // t = 1.5*2^23 + n has bits 0x4B400000 + n, and 0x4B400000 << 23 wraps to
    // zero, so (bits(t) << 23) == n << 23.
    y0 = __int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23));
    y1 = __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23));
}

// ----------------------------------------------------------- softmax pieces
// One S row's 32*kChunks columns from s_addr (this thread's TMEM lane) ->
// P = 2^(s*sl2 - m) as packed bf16 pairs in pk, returns their fp32 sum.  Columns at or
// past `left` are masked (-inf) when kMask.  One exponential in eight runs
// on the FMA pipe (ex2_poly2), the rest on MUFU; scaling and the row sum use
// f32x2 arithmetic.
template <bool kMask, int kChunks = 4>
__device__ __forceinline__ float exp_row(uint32_t s_addr, float m, float sl2, int left,
                                         uint32_t (&pk)[16 * kChunks]) {
    const uint64_t sl2x2 = f2_pack(sl2, sl2);
    const uint64_t negm2 = f2_pack(-m, -m);
    uint64_t acc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] = 0ull;   // (+0, +0)
    // 32-column chunks, software-pipelined: chunk h+1 is loading from TMEM
    // while chunk h is computed.
    uint32_t sa[32], sb[32];
    KVP_TMEM_LD32(s_addr, sa);
    KVP_TMEM_WAIT_LD_DEP(sa);
#pragma unroll
    for (int h = 0; h < kChunks; ++h) {
        uint32_t(&cur)[32] = (h & 1) ? sb : sa;
        uint32_t(&nxt)[32] = (h & 1) ? sa : sb;
        if (h < kChunks - 1) KVP_TMEM_LD32(s_addr + 32 * (h + 1), nxt);
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
            float s0 = __uint_as_float(cur[c]);
            float s1 = __uint_as_float(cur[c + 1]);
            if (kMask) {
                if (32 * h + c >= left) s0 = -INFINITY;
                if (32 * h + c + 1 >= left) s1 = -INFINITY;
            }
            float x0, x1, p0, p1;
            f2_unpack(f2_fma(f2_pack(s0, s1), sl2x2, negm2), x0, x1);
            if ((kPolyPairs >> (c >> 1)) & 1u) {   // selected pairs on the FMA pipe
                ex2_poly2(x0, x1, p0, p1);
            } else {
                p0 = ex2_approx(x0);
                p1 = ex2_approx(x1);
            }
            acc[(c >> 1) & 3] = f2_add(acc[(c >> 1) & 3], f2_pack(p0, p1));
            pk[16 * h + (c >> 1)] = pack_bf16(p0, p1);
        }
        if (h < kChunks - 1) KVP_TMEM_WAIT_LD_DEP(nxt);
    }
    const uint64_t a2 = f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3]));
    float lo, hi;
    f2_unpack(a2, lo, hi);
    return lo + hi;
}

// Row max of one S row (raw scores), masked as in exp_row.
template <bool kMask, int kChunks = 4>
__device__ __forceinline__ float max_row(uint32_t s_addr, int left) {
    float mx[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) mx[i] = -INFINITY;
#pragma unroll
    for (int h = 0; h < kChunks; ++h) {
        uint32_t sr[32];
        KVP_TMEM_LD32(s_addr + 32 * h, sr);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) {
            float s = __uint_as_float(sr[c]);
            if (kMask && 32 * h + c >= left) s = -INFINITY;
            mx[c & 7] = fmaxf(mx[c & 7], s);
        }
    }
    return fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                 fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
}

}  // namespace attn_dev
}  // namespace kvp
