// GPU motion-trace producer: dense two-frame optical flow (Farnebaeck's
// polynomial-expansion method) between consecutive frames, then the
// reference's aggregation (traces/gen_motion_from_video.py:101-121): flow
// magnitude, mean per 16 x 16-pixel cell of the 30 x 52 latent grid, mean
// per row-major 16-token tile; change[0] = change[1]; the percentile reuse
// threshold on the host.
//
// Flow, per frame pair, coarse to fine over levels + 1 pyramid layers (the
// full-resolution frame, then copies blurred with sigma = (1/s - 1)/2 and
// resized bilinearly to scale s = 0.5^k):
//   R = polynomial expansion of each layer: per pixel (bx, by, Axx, Ayy,
//       Axy) of the local model x^T A x + b^T x + c, from separable
//       Gaussian-weighted correlations with {1, x, x^2} (poly_n taps)
//   M = (G11, G12, G22, h1, h2), G = A^T A, h = A^T db with
//       A = (A1(x) + A2(x~)) / 2, db = (b1(x) - b2(x~)) / 2 + A d~,
//       x~ = x + d~ (R2 sampled bilinearly)
//   d = (box mean of G)^-1 (box mean of h), winsize x winsize, `iterations`
//       times, M refreshed from the new d between iterations (one
//       shared-memory tile kernel per iteration: both box passes, the solve
//       and the refresh)
// Every image is planar fp32 [channels][h][w] with mirrored borders
// (reflect-101); one plane of the 480 x 832 frame is 1.6 MB, so a layer's
// working set stays in L2.  A frame's expansion is kept and serves as the
// previous frame of the next pair.  A whole trace pass is replayed as one
// CUDA graph (captured on first use for its buffers).  The CPU restatement of the same steps
// is oracle/motion.py; its agreement with OpenCV's implementation of the
// method is tested there.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <vector>

#include "kvp_common.h"
#include "motion_sm100.h"

namespace kvp {

namespace {

constexpr int kMaxTaps = 32;
struct Taps {
    float w[kMaxTaps];
    int n;                       // radius: taps at -n..n
};

__device__ __forceinline__ int mirror(int i, int n) {
    // reflect-101 (d c b | a b c d | c b a), also for offsets past one period
    while (i < 0 || i >= n) i = i < 0 ? -i : 2 * n - 2 - i;
    return i;
}

__global__ void u8_to_f32_kernel(const uint8_t* __restrict__ src, float* __restrict__ dst, long long n) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = (float)src[i];
}

// dst = src correlated with taps along one axis (axis 0 = rows / y, 1 = x).
__global__ void filter1d_kernel(const float* __restrict__ src, float* __restrict__ dst, int H, int W,
                                int axis, Taps t) {
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int y = blockIdx.y;
    if (x >= W) return;
    float acc = 0.f;
    for (int k = -t.n; k <= t.n; ++k) {
        const int xx = axis ? mirror(x + k, W) : x;
        const int yy = axis ? y : mirror(y + k, H);
        acc = fmaf(t.w[k + t.n], src[(size_t)yy * W + xx], acc);
    }
    dst[(size_t)y * W + x] = acc;
}

__device__ __forceinline__ float bilerp(const float* __restrict__ img, int H, int W, float x, float y) {
    x = fminf(fmaxf(x, 0.f), (float)(W - 1));
    y = fminf(fmaxf(y, 0.f), (float)(H - 1));
    const int x0 = min((int)floorf(x), W - 2);
    const int y0 = min((int)floorf(y), H - 2);
    const float fx = x - (float)x0, fy = y - (float)y0;
    const float* r0 = img + (size_t)y0 * W + x0;
    const float* r1 = r0 + W;
    return (1.f - fy) * ((1.f - fx) * r0[0] + fx * r0[1]) + fy * ((1.f - fx) * r1[0] + fx * r1[1]);
}

// Half-pixel-centre bilinear resize of `ch` planes, times `mult`.
__global__ void resize_kernel(const float* __restrict__ src, int Hs, int Ws, float* __restrict__ dst,
                              int Hd, int Wd, int ch, float sy, float sx, float mult) {
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int y = blockIdx.y;
    if (x >= Wd) return;
    const float fy = ((float)y + 0.5f) * sy - 0.5f;
    const float fx = ((float)x + 0.5f) * sx - 0.5f;
    for (int c = 0; c < ch; ++c)
        dst[((size_t)c * Hd + y) * Wd + x] =
            bilerp(src + (size_t)c * Hs * Ws, Hs, Ws, fx, fy) * mult;
}

struct PolyConsts {
    Taps k0, k1, k2;             // g, g*x, g*x^2
    float ix, ixy_half, a, b, c; // rx = cx*ix, Axy = cxy*ixy_half, Axx = a c1 + b cxx + c cyy
};

// Vertical pass: v0 = k0 (*) f, v1 = k1 (*) f, v2 = k2 (*) f along y.
__global__ void poly_v_kernel(const float* __restrict__ f, float* __restrict__ v, int H, int W,
                              PolyConsts P) {
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int y = blockIdx.y;
    if (x >= W) return;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f;
    for (int k = -P.k0.n; k <= P.k0.n; ++k) {
        const float s = f[(size_t)mirror(y + k, H) * W + x];
        a0 = fmaf(P.k0.w[k + P.k0.n], s, a0);
        a1 = fmaf(P.k1.w[k + P.k0.n], s, a1);
        a2 = fmaf(P.k2.w[k + P.k0.n], s, a2);
    }
    const size_t plane = (size_t)H * W, o = (size_t)y * W + x;
    v[o] = a0;
    v[plane + o] = a1;
    v[2 * plane + o] = a2;
}

// Horizontal pass and solve: R = (bx, by, Axx, Ayy, Axy).
__global__ void poly_h_kernel(const float* __restrict__ v, float* __restrict__ R, int H, int W,
                              PolyConsts P) {
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int y = blockIdx.y;
    if (x >= W) return;
    const size_t plane = (size_t)H * W;
    const float* v0 = v + (size_t)y * W;
    const float* v1 = v0 + plane;
    const float* v2 = v1 + plane;
    float c1 = 0.f, cx = 0.f, cxx = 0.f, cy = 0.f, cxy = 0.f, cyy = 0.f;
    for (int k = -P.k0.n; k <= P.k0.n; ++k) {
        const int xx = mirror(x + k, W);
        const float g0 = P.k0.w[k + P.k0.n], g1 = P.k1.w[k + P.k0.n], g2 = P.k2.w[k + P.k0.n];
        const float s0 = v0[xx], s1 = v1[xx], s2 = v2[xx];
        c1 = fmaf(g0, s0, c1);
        cx = fmaf(g1, s0, cx);
        cxx = fmaf(g2, s0, cxx);
        cy = fmaf(g0, s1, cy);
        cxy = fmaf(g1, s1, cxy);
        cyy = fmaf(g0, s2, cyy);
    }
    const size_t o = (size_t)y * W + x;
    R[o] = cx * P.ix;
    R[plane + o] = cy * P.ix;
    R[2 * plane + o] = P.a * c1 + P.b * cxx + P.c * cyy;
    R[3 * plane + o] = P.a * c1 + P.c * cxx + P.b * cyy;
    R[4 * plane + o] = cxy * P.ixy_half;
}

// M at pixel (x, y) for displacement (dx, dy).
__device__ __forceinline__ void matrices_at(const float* __restrict__ R1, const float* __restrict__ R2,
                                            int H, int W, int x, int y, float dx, float dy,
                                            float* __restrict__ M) {
    const size_t plane = (size_t)H * W, o = (size_t)y * W + x;
    const float sx = (float)x + dx, sy = (float)y + dy;
    float s[5];
#pragma unroll
    for (int c = 0; c < 5; ++c) s[c] = bilerp(R2 + c * plane, H, W, sx, sy);
    const float a11 = (R1[2 * plane + o] + s[2]) * 0.5f;
    const float a22 = (R1[3 * plane + o] + s[3]) * 0.5f;
    const float a12 = (R1[4 * plane + o] + s[4]) * 0.5f;
    const float db1 = (R1[o] - s[0]) * 0.5f + a11 * dx + a12 * dy;
    const float db2 = (R1[plane + o] - s[1]) * 0.5f + a12 * dx + a22 * dy;
    M[o] = a11 * a11 + a12 * a12;
    M[plane + o] = a12 * (a11 + a22);
    M[2 * plane + o] = a12 * a12 + a22 * a22;
    M[3 * plane + o] = a11 * db1 + a12 * db2;
    M[4 * plane + o] = a12 * db1 + a22 * db2;
}

__global__ void update_matrices_kernel(const float* __restrict__ R1, const float* __restrict__ R2,
                                       const float* __restrict__ flow, float* __restrict__ M, int H,
                                       int W) {
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int y = blockIdx.y;
    if (x >= W) return;
    const size_t plane = (size_t)H * W, o = (size_t)y * W + x;
    matrices_at(R1, R2, H, W, x, y, flow[o], flow[plane + o], M);
}

// One displacement iteration for a kTH x kTW tile of pixels: the tile's
// window region of the 5 planes of M (mirrored at the image edges) is staged
// in shared memory, summed vertically then horizontally there, and each
// pixel solves its 2x2 system -> flow and, when `update`, writes M for the
// new flow into Mout (a second buffer: neighbouring tiles still read Min).
constexpr int kTW = 32, kTH = 16;
constexpr int kBoxMaxR = 15;
__host__ __device__ constexpr size_t box_tile_smem_floats(int r) {
    return (size_t)5 * (kTH + 2 * r) * (kTW + 2 * r) + (size_t)5 * kTH * (kTW + 2 * r);
}

__global__ void __launch_bounds__(256)
box_solve_tile_kernel(const float* __restrict__ Min, const float* __restrict__ R1,
                      const float* __restrict__ R2, float* __restrict__ flow,
                      float* __restrict__ Mout, int H, int W, int r, float inv2, int update) {
    extern __shared__ float sh[];
    const int IW = kTW + 2 * r, IH = kTH + 2 * r;
    float* in = sh;                                  // [5][IH][IW]
    float* vs = sh + (size_t)5 * IH * IW;            // [5][kTH][IW]
    const int x0 = blockIdx.x * kTW, y0 = blockIdx.y * kTH;
    const size_t plane = (size_t)H * W;
    for (int idx = threadIdx.x; idx < IH * IW; idx += blockDim.x) {
        const int i = idx / IW, j = idx - (idx / IW) * IW;
        const size_t o = (size_t)mirror(y0 - r + i, H) * W + mirror(x0 - r + j, W);
#pragma unroll
        for (int c = 0; c < 5; ++c) in[c * IH * IW + idx] = Min[c * plane + o];
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < kTH * IW; idx += blockDim.x) {
        const int i = idx / IW, j = idx - (idx / IW) * IW;
#pragma unroll
        for (int c = 0; c < 5; ++c) {
            const float* col = in + c * IH * IW + i * IW + j;
            float a = 0.f;
            for (int m = 0; m <= 2 * r; ++m) a += col[m * IW];
            vs[c * kTH * IW + idx] = a;
        }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < kTH * kTW; idx += blockDim.x) {
        const int i = idx / kTW, j = idx - (idx / kTW) * kTW;
        const int x = x0 + j, y = y0 + i;
        if (x >= W || y >= H) continue;
        float g[5];
#pragma unroll
        for (int c = 0; c < 5; ++c) {
            const float* row = vs + c * kTH * IW + i * IW + j;
            float a = 0.f;
            for (int m = 0; m <= 2 * r; ++m) a += row[m];
            g[c] = a * inv2;
        }
        const float det = g[0] * g[2] - g[1] * g[1];
        const float idet = 1.f / (det + 1e-3f);
        const float dx = (g[2] * g[3] - g[1] * g[4]) * idet;
        const float dy = (g[0] * g[4] - g[1] * g[3]) * idet;
        const size_t o = (size_t)y * W + x;
        flow[o] = dx;
        flow[plane + o] = dy;
        if (update) matrices_at(R1, R2, H, W, x, y, dx, dy, Mout);
    }
}

// change[t] = mean |flow| over tile t's cells (cell = ch x cw pixels of the
// rows x cols grid, cells row-major, tiles of tile_cells consecutive cells).
__global__ void tile_scores_kernel(const float* __restrict__ flow, int H, int W, int rows, int cols,
                                   int tile_cells, float* __restrict__ change) {
    const int t = blockIdx.x;
    const int cells = rows * cols;
    const int c0 = t * tile_cells;
    const int nc = min(tile_cells, cells - c0);
    const int ch = H / rows, cw = W / cols;
    const size_t plane = (size_t)H * W;
    // one cell per warp at a time; the tile's cells have equal weight, so its
    // mean is the mean of its cells' means
    __shared__ float part[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    float tile_acc = 0.f;
    for (int c = c0 + warp; c < c0 + nc; c += nw) {
        const int cy = c / cols, cx = c % cols;
        float s = 0.f;
        for (int p = lane; p < ch * cw; p += 32) {
            const size_t o = (size_t)(cy * ch + p / cw) * W + (cx * cw + p % cw);
            const float dx = flow[o], dy = flow[plane + o];
            s += sqrtf(dx * dx + dy * dy);
        }
#pragma unroll
        for (int k = 16; k > 0; k >>= 1) s += __shfl_xor_sync(0xffffffffu, s, k);
        tile_acc += s / (float)(ch * cw);
    }
    if (lane == 0) part[warp] = tile_acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.f;
        for (int w = 0; w < nw; ++w) s += part[w];
        change[t] = s / (float)nc;
    }
}

Taps gaussian_taps(int n, double sigma) {
    Taps t{};
    t.n = n;
    double sum = 0.0;
    for (int i = -n; i <= n; ++i) sum += std::exp(-(double)i * i / (2.0 * sigma * sigma));
    for (int i = -n; i <= n; ++i) t.w[i + n] = (float)(std::exp(-(double)i * i / (2.0 * sigma * sigma)) / sum);
    return t;
}

PolyConsts poly_consts(int n, double sigma) {
    PolyConsts P{};
    double g[kMaxTaps], sum = 0.0;
    for (int i = -n; i <= n; ++i) sum += (g[i + n] = std::exp(-(double)i * i / (2.0 * sigma * sigma)));
    double m0 = 0, m2 = 0, m4 = 0;
    P.k0.n = P.k1.n = P.k2.n = n;
    for (int i = -n; i <= n; ++i) {
        const double w = g[i + n] / sum, x = i;
        P.k0.w[i + n] = (float)w;
        P.k1.w[i + n] = (float)(w * x);
        P.k2.w[i + n] = (float)(w * x * x);
        m0 += w;
        m2 += w * x * x;
        m4 += w * x * x * x * x;
    }
    // inverse of [[m0^2, m0 m2, m0 m2], [m0 m2, m0 m4, m2^2], [m0 m2, m2^2, m0 m4]], row 1
    const double G[3][3] = {{m0 * m0, m0 * m2, m0 * m2}, {m0 * m2, m0 * m4, m2 * m2},
                            {m0 * m2, m2 * m2, m0 * m4}};
    const double det = G[0][0] * (G[1][1] * G[2][2] - G[1][2] * G[2][1]) -
                       G[0][1] * (G[1][0] * G[2][2] - G[1][2] * G[2][0]) +
                       G[0][2] * (G[1][0] * G[2][1] - G[1][1] * G[2][0]);
    // row 1 of the inverse = column 1 of the cofactor matrix / det
    P.a = (float)(-(G[0][1] * G[2][2] - G[0][2] * G[2][1]) / det);
    P.b = (float)((G[0][0] * G[2][2] - G[0][2] * G[2][0]) / det);
    P.c = (float)(-(G[0][0] * G[1][2] - G[0][2] * G[1][0]) / det);
    P.ix = (float)(1.0 / (m0 * m2));
    P.ixy_half = (float)(0.5 / (m2 * m2));
    return P;
}

dim3 grid_of(int H, int W) { return dim3((unsigned)((W + 127) / 128), (unsigned)H); }

}  // namespace

// ------------------------------------------------------------------ producer
struct MotionProducer::Level {
    int h, w;
    float* img[2];     // the two frames' layers (slot by frame parity)
    float* R[2];       // their expansions
};

MotionProducer::MotionProducer(const MotionParams& p) : p_(p) {
    if (p.height < 32 || p.width < 32 || p.levels < 0 || p.levels > 8 || p.winsize < 3 ||
        p.winsize % 2 == 0 || p.winsize / 2 > kBoxMaxR || p.iterations < 1 || p.poly_n < 3 || p.poly_n % 2 == 0 ||
        p.poly_n > 15 || !(p.poly_sigma > 0) || !(p.pyr_scale > 0 && p.pyr_scale < 1) ||
        p.grid_rows <= 0 || p.grid_cols <= 0 || p.height % p.grid_rows || p.width % p.grid_cols ||
        p.tile_cells <= 0) {
        set_error("motion: invalid parameters");
        status_ = KVP_ERR_ARG;
        return;
    }
    tiles_ = (p.grid_rows * p.grid_cols + p.tile_cells - 1) / p.tile_cells;
    cudaError_t e = cudaSuccess;
    size_t maxplane = 0;
    for (int k = 0; k <= p.levels && e == cudaSuccess; ++k) {
        const double s = std::pow((double)p.pyr_scale, k);
        Level L{};
        L.h = (int)std::nearbyint(p.height * s);
        L.w = (int)std::nearbyint(p.width * s);
        if (L.h < 8 || L.w < 8) break;    // no layer below 8 x 8
        const size_t plane = (size_t)L.h * L.w;
        maxplane = std::max(maxplane, plane);
        for (int i = 0; i < 2 && e == cudaSuccess; ++i) {
            e = cudaMalloc(&L.img[i], plane * sizeof(float));
            if (e == cudaSuccess) e = cudaMalloc(&L.R[i], 5 * plane * sizeof(float));
        }
        levels_.push_back(L);
    }
    const size_t full = (size_t)p.height * p.width;
    if (e == cudaSuccess) e = cudaMalloc(&tmp_, 5 * full * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&tmp2_, 5 * full * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&M_, 5 * full * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&M2_, 5 * full * sizeof(float));
    if (e == cudaSuccess && box_tile_smem_floats(p.winsize / 2) * sizeof(float) > 48 * 1024)
        e = cudaFuncSetAttribute(box_solve_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(box_tile_smem_floats(p.winsize / 2) * sizeof(float)));
    if (e == cudaSuccess) e = cudaMalloc(&flow_[0], 2 * full * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&flow_[1], 2 * full * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&fflow_, 2 * full * sizeof(float));
    if (e != cudaSuccess) status_ = cuda_status(e, "motion buffers");
}

MotionProducer::~MotionProducer() {
    if (exec_) cudaGraphExecDestroy(exec_);
    if (cap_stream_) {
        cudaStreamSynchronize(cap_stream_);
        cudaStreamDestroy(cap_stream_);
    }
    if (ev_in_) cudaEventDestroy(ev_in_);
    if (ev_out_) cudaEventDestroy(ev_out_);
    for (auto& L : levels_)
        for (int i = 0; i < 2; ++i) {
            if (L.img[i]) cudaFree(L.img[i]);
            if (L.R[i]) cudaFree(L.R[i]);
        }
    for (float* p : {tmp_, tmp2_, M_, M2_, flow_[0], flow_[1], fflow_})
        if (p) cudaFree(p);
}

int MotionProducer::load_frame(const uint8_t* d_frame, int slot, cudaStream_t s) {
    // layer 0 = the frame; layer k = blur(sigma_k) of the frame, resized
    const Level& L0 = levels_[0];
    const long long n = (long long)L0.h * L0.w;
    u8_to_f32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(d_frame, L0.img[slot], n);
    const PolyConsts P = poly_consts(p_.poly_n / 2, p_.poly_sigma);
    for (size_t k = 0; k < levels_.size(); ++k) {
        const Level& L = levels_[k];
        if (k > 0) {
            const double scale = std::pow((double)p_.pyr_scale, (double)k);
            const double sigma = (1.0 / scale - 1.0) * 0.5;
            const int ks = std::max(3, (int)std::nearbyint(sigma * 5.0) | 1);
            const Taps g = gaussian_taps(ks / 2, sigma);
            filter1d_kernel<<<grid_of(L0.h, L0.w), 128, 0, s>>>(L0.img[slot], tmp_, L0.h, L0.w, 0, g);
            filter1d_kernel<<<grid_of(L0.h, L0.w), 128, 0, s>>>(tmp_, tmp2_, L0.h, L0.w, 1, g);
            resize_kernel<<<grid_of(L.h, L.w), 128, 0, s>>>(tmp2_, L0.h, L0.w, L.img[slot], L.h, L.w, 1,
                                                            (float)((double)L0.h / L.h),
                                                            (float)((double)L0.w / L.w), 1.f);
        }
        poly_v_kernel<<<grid_of(L.h, L.w), 128, 0, s>>>(L.img[slot], tmp_, L.h, L.w, P);
        poly_h_kernel<<<grid_of(L.h, L.w), 128, 0, s>>>(tmp_, L.R[slot], L.h, L.w, P);
    }
    KVP_CUDA(cudaGetLastError());
    return KVP_OK;
}

int MotionProducer::flow(int prev_slot, int next_slot, float* d_out, cudaStream_t s) {
    // Coarsest to finest: level k's flow lands in flow_[k & 1], the finest
    // level's in d_out; each level starts from the coarser one, resized.
    const int r = p_.winsize / 2;
    const float inv = 1.f / (float)p_.winsize;
    const int nl = (int)levels_.size();
    for (int k = nl - 1; k >= 0; --k) {
        const Level& L = levels_[k];
        const size_t plane = (size_t)L.h * L.w;
        float* fl = k == 0 ? d_out : flow_[k & 1];
        if (k == nl - 1) {
            KVP_CUDA(cudaMemsetAsync(fl, 0, 2 * plane * sizeof(float), s));
        } else {
            const Level& C = levels_[k + 1];
            resize_kernel<<<grid_of(L.h, L.w), 128, 0, s>>>(flow_[(k + 1) & 1], C.h, C.w, fl, L.h, L.w,
                                                            2, (float)((double)C.h / L.h),
                                                            (float)((double)C.w / L.w),
                                                            1.f / p_.pyr_scale);
        }
        const float* R1 = L.R[prev_slot];
        const float* R2 = L.R[next_slot];
        update_matrices_kernel<<<grid_of(L.h, L.w), 128, 0, s>>>(R1, R2, fl, M_, L.h, L.w);
        const dim3 gt((unsigned)((L.w + kTW - 1) / kTW), (unsigned)((L.h + kTH - 1) / kTH));
        float* Mb[2] = {M_, M2_};
        for (int it = 0; it < p_.iterations; ++it)
            box_solve_tile_kernel<<<gt, 256, box_tile_smem_floats(r) * sizeof(float), s>>>(
                Mb[it & 1], R1, R2, fl, Mb[(it + 1) & 1], L.h, L.w, r, inv * inv,
                it < p_.iterations - 1);
    }
    KVP_CUDA(cudaGetLastError());
    return KVP_OK;
}

int MotionProducer::pair_flow(const uint8_t* d_prev, const uint8_t* d_next, float* d_flow,
                              cudaStream_t s) {
    if (status_ != KVP_OK) return status_;
    if (!d_prev || !d_next || !d_flow) return KVP_ERR_ARG;
    int rc = load_frame(d_prev, 0, s);
    if (rc == KVP_OK) rc = load_frame(d_next, 1, s);
    if (rc == KVP_OK) rc = flow(0, 1, d_flow, s);
    return rc;
}

int MotionProducer::trace(const uint8_t* d_frames, int frames, float* d_change, cudaStream_t s) {
    if (status_ != KVP_OK) return status_;
    if (!d_frames || !d_change || frames < 2) return KVP_ERR_ARG;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    KVP_CUDA(cudaStreamIsCapturing(s, &cs));
    if (cs != cudaStreamCaptureStatusNone) return enqueue_trace(d_frames, frames, d_change, s);
    // The pass is ~50 small launches per frame pair: replay it as one CUDA
    // graph (captured once per (frames, count, output)) on a private stream
    // joined to the caller's by events.
    if (!cap_stream_) {
        KVP_CUDA(cudaStreamCreateWithFlags(&cap_stream_, cudaStreamNonBlocking));
        KVP_CUDA(cudaEventCreateWithFlags(&ev_in_, cudaEventDisableTiming));
        KVP_CUDA(cudaEventCreateWithFlags(&ev_out_, cudaEventDisableTiming));
    }
    if (!exec_ || g_frames_ != d_frames || g_count_ != frames || g_change_ != d_change) {
        if (exec_) {
            cudaGraphExecDestroy(exec_);
            exec_ = nullptr;
        }
        KVP_CUDA(cudaStreamBeginCapture(cap_stream_, cudaStreamCaptureModeThreadLocal));
        const int rc = enqueue_trace(d_frames, frames, d_change, cap_stream_);
        cudaGraph_t g = nullptr;
        const cudaError_t e = cudaStreamEndCapture(cap_stream_, &g);
        if (rc != KVP_OK || e != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            return rc != KVP_OK ? rc : cuda_status(e, "motion graph capture");
        }
        const cudaError_t ei = cudaGraphInstantiate(&exec_, g, 0);
        cudaGraphDestroy(g);
        if (ei != cudaSuccess) {
            exec_ = nullptr;
            return cuda_status(ei, "motion graph instantiate");
        }
        g_frames_ = d_frames;
        g_count_ = frames;
        g_change_ = d_change;
    }
    KVP_CUDA(cudaEventRecord(ev_in_, s));
    KVP_CUDA(cudaStreamWaitEvent(cap_stream_, ev_in_, 0));
    KVP_CUDA(cudaGraphLaunch(exec_, cap_stream_));
    KVP_CUDA(cudaEventRecord(ev_out_, cap_stream_));
    KVP_CUDA(cudaStreamWaitEvent(s, ev_out_, 0));
    return KVP_OK;
}

int MotionProducer::enqueue_trace(const uint8_t* d_frames, int frames, float* d_change,
                                  cudaStream_t s) {
    const size_t fbytes = (size_t)p_.height * p_.width;
    // frame f's layers and expansion live in slot f & 1: each frame is
    // expanded once and serves both of its pairs
    int rc = load_frame(d_frames, 0, s);
    for (int f = 1; f < frames && rc == KVP_OK; ++f) {
        rc = load_frame(d_frames + (size_t)f * fbytes, f & 1, s);
        if (rc == KVP_OK) rc = flow((f - 1) & 1, f & 1, fflow_, s);
        if (rc != KVP_OK) break;
        tile_scores_kernel<<<(unsigned)tiles_, 256, 0, s>>>(fflow_, p_.height, p_.width, p_.grid_rows,
                                                            p_.grid_cols, p_.tile_cells,
                                                            d_change + (size_t)f * tiles_);
    }
    if (rc != KVP_OK) return rc;
    // change[0] = change[1] (frame 0 borrows the first pair's rates)
    KVP_CUDA(cudaMemcpyAsync(d_change, d_change + tiles_, tiles_ * sizeof(float),
                             cudaMemcpyDeviceToDevice, s));
    KVP_CUDA(cudaGetLastError());
    return KVP_OK;
}

int motion_threshold(const float* change, int frames, int tiles, double percentile,
                     int8_t* reuse, int8_t* is_static, double* tau_out) {
    if (!change || frames < 2 || tiles <= 0 || !(percentile >= 0 && percentile <= 100)) return KVP_ERR_ARG;
    // numpy's default percentile ("linear"), over frames 1..F-1, with its
    // arithmetic: virtual index (n - 1) * q, and the interpolation taken from
    // the upper neighbour when the fraction is >= 0.5
    std::vector<double> v((size_t)(frames - 1) * tiles);
    for (size_t i = 0; i < v.size(); ++i) v[i] = change[(size_t)tiles + i];
    std::sort(v.begin(), v.end());
    const double n = (double)v.size(), q = percentile / 100.0;
    const double vi = (n - 1.0) * q;
    double lo_d = std::floor(vi);
    const double t = vi - lo_d;
    lo_d = std::min(std::max(lo_d, 0.0), n - 1.0);
    const size_t lo = (size_t)lo_d;
    const size_t hi = (size_t)std::min(std::max(lo_d + 1.0, 0.0), n - 1.0);
    const double a = v[lo], b = v[hi], d = b - a;
    const double tau = t >= 0.5 ? b - d * (1.0 - t) : a + d * t;
    for (int f = 0; f < frames; ++f)
        for (int t = 0; t < tiles; ++t) {
            const bool below = (double)change[(size_t)f * tiles + t] < tau;
            if (reuse) reuse[(size_t)f * tiles + t] = (int8_t)(f > 0 && below);
            if (is_static) is_static[(size_t)f * tiles + t] = (int8_t)below;
        }
    if (tau_out) *tau_out = tau;
    return KVP_OK;
}

}  // namespace kvp
