// kvp_attn_bf16_noalloc: the bf16 tcgen05 remapped attention for callers
// that must not allocate device memory.
//
// Who needs it: hosts that hand all device memory to one pre-planned pool
// or custom allocator and forbid stray cudaMalloc calls (an embedding
// runtime that budgets every byte of HBM up front, or a caching allocator
// that has already reserved the device), and latency-critical serving
// loops that cannot afford the first-call allocation stall (cudaMalloc
// synchronises the device).  kvp_attn_bf16 allocates a small device status word on
// its first call per device and expects the KVMap already in device memory,
// so those callers cannot use it.
//
// What this entry point does instead: its scratch -- the status word the
// kernel reports into, and a device copy of a KVMap the caller passes in
// host memory -- lives in one file-scope static __device__ array below,
// which every GPU that loads libkvp.so holds until the process exits.  The
// caller still passes Q/K/V/Out (and the arena) in device memory.
//
// Limits and rules (also stated in include/kvp.h):
//   * at most kMaxMapRows = 65,536 KVMap rows per call (512 KB of int64,
//     a 21-frame x 1560-token stack needs 32,760); larger maps are rejected
//     with KVP_ERR_CAPACITY and a message;
//   * the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current); make that first call
//     before any stream capture begins;
//   * every call shares the one array and it keeps the last call's contents:
//     the status word is cleared at the start of each call, and calls whose
//     work overlaps on the GPU (different streams, no ordering between them)
//     race on it;
//   * it does not issue copies queued by kvtm_* staging calls: call
//     kvtm_flush (or a window call) first;
//   * without host_status the call returns before the map copy has run: a
//     map in pinned host memory must stay unchanged until `stream` has
//     passed the call (a map in pageable memory is staged before return);
//   * the device address of the array is looked up once per device in the
//     primary context: do not use the entry point from another context on
//     that device, or after cudaDeviceReset.
// No cudaMalloc, cudaFree or allocating library routine is called here.
#include <mutex>

#include "../../include/kvp.h"
#include "attn_sm100.h"
#include "kvp_common.h"

namespace {

constexpr long long kMaxMapRows = 65536;
constexpr long long kStatusSlots = 32;   // 256 bytes: status word, padding

// [0, 32): status area (int at slot 0); [32, 32 + kMaxMapRows): KVMap rows.
static __device__ __align__(256) long long g_noalloc_scratch[kStatusSlots + kMaxMapRows];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
long long* g_scratch_addr[kMaxDevices] = {nullptr};

// Device address of g_noalloc_scratch on the current device (looked up once
// per device; the host-side name is only a stand-in for it).
int scratch_for_current_device(long long** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return kvp::cuda_status(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) {
        kvp::set_error("noalloc: device %d out of range", dev);
        return kvp::KVP_ERR_ARG;
    }
    std::lock_guard<std::mutex> g(g_mu);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return kvp::cuda_status(e, "cudaGetSymbolAddress(noalloc scratch)");
        g_scratch_addr[dev] = static_cast<long long*>(p);
    }
    *out = g_scratch_addr[dev];
    return kvp::KVP_OK;
}

}  // namespace

KVP_API int kvp_attn_bf16_noalloc(const kvp_layer_io* io, const kvp_attn_desc* d,
                                  const long long* host_kvmap, int* host_status, void* stream) {
    if (!io || !d) return kvp::KVP_ERR_ARG;
    if (io->kvmap) {
        kvp::set_error("noalloc: pass the KVMap in host memory (host_kvmap), not io->kvmap");
        return kvp::KVP_ERR_ARG;
    }
    kvp::AttnDesc A{d->tokens, d->frames, d->q_frame0, d->mode, d->window,
                    d->heads, d->head_dim, d->head0, d->nheads, d->flat};
    // Bad arguments are reported before the scratch is looked up or written
    // (the map pointer only has to be non-null here; it becomes the scratch).
    // The descriptor is checked first, so a bad descriptor is -1 whatever
    // the map; only a valid one can be refused for its map size (-3).
    kvp::LayerIO L{io->q, io->k, io->v, io->out, io->arena, host_kvmap,
                   io->q_rows, io->kv_rows, io->arena_rows};
    int rc = kvp::check_attn_bf16(L, A);
    if (rc != kvp::KVP_OK) return rc;
    const long long map_rows = ((long long)d->q_frame0 + d->frames) * (long long)d->tokens;
    if (host_kvmap && (map_rows <= 0 || map_rows > kMaxMapRows)) {
        kvp::set_error("noalloc: KVMap of %lld rows exceeds the %lld-row static scratch",
                       map_rows, kMaxMapRows);
        return kvp::KVP_ERR_CAPACITY;
    }
    long long* scratch = nullptr;
    rc = scratch_for_current_device(&scratch);
    if (rc != kvp::KVP_OK) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    int* status = reinterpret_cast<int*>(scratch);
    long long* dmap = scratch + kStatusSlots;
    KVP_CUDA(cudaMemsetAsync(status, 0, sizeof(int), s));
    if (host_kvmap)
        KVP_CUDA(cudaMemcpyAsync(dmap, host_kvmap, (size_t)map_rows * sizeof(long long),
                                 cudaMemcpyHostToDevice, s));
    L.kvmap = host_kvmap ? dmap : nullptr;
    rc = kvp::launch_attn_bf16(L, A, status, s, /*allow_split=*/false);
    if (rc != kvp::KVP_OK) return rc;
    if (host_status) {
        KVP_CUDA(cudaMemcpyAsync(host_status, status, sizeof(int), cudaMemcpyDeviceToHost, s));
        KVP_CUDA(cudaStreamSynchronize(s));
    }
    return kvp::KVP_OK;
}
