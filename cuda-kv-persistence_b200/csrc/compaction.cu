// Arena compaction / restage: the vectorised gather that replaces the
// reference's two cudaMemcpyAsync per staged row
// (src/kv_tile_manager.cu:111-116,164-171,180-185).
//
// HBM-bound byte movement: every byte is read once and written once with
// 16-byte accesses, consecutive lanes on consecutive 16-byte words.  A row
// here is one token's K row or V row (D elements, 3 KB in bf16 at D=1536).
#include <atomic>

#include "kernels.h"
#include "kvp_common.h"

namespace kvp {

namespace {

// One CTA per copy descriptor (grid-stride over descriptors).
__global__ void __launch_bounds__(256) copy_batch_kernel(const CopyOp* __restrict__ ops, int n) {
    for (int i = blockIdx.x; i < n; i += gridDim.x) {
        const CopyOp op = ops[i];
        const uintptr_t s = (uintptr_t)op.src, d = (uintptr_t)op.dst;
        if (((s | d | op.bytes) & 15u) == 0) {
            const uint4* src = reinterpret_cast<const uint4*>(op.src);
            uint4* dst = reinterpret_cast<uint4*>(op.dst);
            const uint64_t n16 = op.bytes >> 4;
            for (uint64_t j = threadIdx.x; j < n16; j += blockDim.x) dst[j] = __ldg(src + j);
        } else if (((s | d | op.bytes) & 3u) == 0) {
            const uint32_t* src = reinterpret_cast<const uint32_t*>(op.src);
            uint32_t* dst = reinterpret_cast<uint32_t*>(op.dst);
            const uint64_t n4 = op.bytes >> 2;
            for (uint64_t j = threadIdx.x; j < n4; j += blockDim.x) dst[j] = src[j];
        } else {
            const unsigned char* src = reinterpret_cast<const unsigned char*>(op.src);
            unsigned char* dst = reinterpret_cast<unsigned char*>(op.dst);
            for (uint64_t j = threadIdx.x; j < op.bytes; j += blockDim.x) dst[j] = src[j];
        }
    }
}

// One warp per (pair, layer): the K row then the V row of a source token
// land in one arena row [K | V].  row_bytes must be a multiple of 16.  Pairs
// whose source row lies in [skip_lo, skip_hi) are left alone (their arena
// rows were written by the producer of those rows).
__global__ void __launch_bounds__(256) gather_rows_kernel(GatherLayers L, int layers,
                                                          const int2* __restrict__ pairs, int n,
                                                          int64_t row_bytes, int64_t skip_lo,
                                                          int64_t skip_hi) {
    const int warps_per_cta = blockDim.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t total = (int64_t)n * layers;
    const int64_t n16 = row_bytes >> 4;
    for (int64_t w = (int64_t)blockIdx.x * warps_per_cta + (threadIdx.x >> 5); w < total;
         w += (int64_t)gridDim.x * warps_per_cta) {
        const int layer = (int)(w / n);
        const int2 pr = pairs[w - (int64_t)layer * n];
        if (pr.x >= skip_lo && pr.x < skip_hi) continue;
        const uint4* ks = reinterpret_cast<const uint4*>(
            static_cast<const char*>(L.k[layer]) + (int64_t)pr.x * row_bytes);
        const uint4* vs = reinterpret_cast<const uint4*>(
            static_cast<const char*>(L.v[layer]) + (int64_t)pr.x * row_bytes);
        uint4* dst = reinterpret_cast<uint4*>(static_cast<char*>(L.arena[layer]) +
                                              (int64_t)pr.y * 2 * row_bytes);
        for (int64_t j = lane; j < n16; j += 32) {
            const uint4 a = __ldg(ks + j);
            const uint4 b = __ldg(vs + j);
            dst[j] = a;
            dst[n16 + j] = b;
        }
    }
}

int sm_count() {
    static std::atomic<int> counts[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    int n = counts[dev].load(std::memory_order_relaxed);
    if (n <= 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        counts[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

}  // namespace

int launch_copy_batch(const CopyOp* d_ops, int n, cudaStream_t stream) {
    if (n <= 0) return KVP_OK;
    const int grid = n < sm_count() * 16 ? n : sm_count() * 16;
    copy_batch_kernel<<<grid, 256, 0, stream>>>(d_ops, n);
    KVP_CUDA(cudaGetLastError());
    return KVP_OK;
}

int launch_gather_rows(const GatherLayers& L, int layers, const int32_t* d_pairs, int n,
                       int64_t row_bytes, cudaStream_t stream, int64_t skip_lo, int64_t skip_hi) {
    if (n <= 0 || layers <= 0) return KVP_OK;
    if (layers > kMaxLayers || (row_bytes & 15) != 0 || !d_pairs) {
        set_error("gather_rows: layers=%d (max %d), row_bytes=%lld must be a multiple of 16",
                  layers, kMaxLayers, (long long)row_bytes);
        return KVP_ERR_ARG;
    }
    const int64_t warps = (int64_t)n * layers;
    int64_t grid = (warps + 7) / 8;
    const int64_t cap = (int64_t)sm_count() * 8;
    if (grid > cap) grid = cap;
    gather_rows_kernel<<<(unsigned)grid, 256, 0, stream>>>(
        L, layers, reinterpret_cast<const int2*>(d_pairs), n, row_bytes, skip_lo, skip_hi);
    KVP_CUDA(cudaGetLastError());
    return KVP_OK;
}

}  // namespace kvp
