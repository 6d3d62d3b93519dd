// Shared definitions for the kvp native library (B200 / sm_100a).
#pragma once

#include <cstddef>
#include <mutex>
#include <cstdint>
#include <cuda_runtime.h>

#define KVP_API extern "C" __attribute__((visibility("default")))

namespace kvp {

// Status codes returned by the kvp_* entry points (0 = success).
enum Status : int {
    KVP_OK = 0,
    KVP_ERR_ARG = -1,        // invalid argument (null pointer, bad shape, ...)
    KVP_ERR_CUDA = -2,       // a CUDA runtime call failed (see kvp_last_error)
    KVP_ERR_CAPACITY = -3,   // a fixed-size buffer would overflow
    KVP_ERR_UNSUPPORTED = -4,// device / shape not supported by this kernel
    KVP_ERR_TIMEOUT = -5,    // a bounded device wait expired (kernel status word)
    KVP_ERR_MAP = -6,        // a KVMap entry pointed outside the arena
};

// Bits of the device status word (kvp_read_status), set by the kernels.
constexpr int KVP_STATUS_MAP = 1;      // a KVMap entry pointed outside the arena (base row used)
constexpr int KVP_STATUS_TIMEOUT = 2;  // a bounded wait expired; the CTA's output is incomplete
constexpr int KVP_STATUS_ALIGN = 4;    // dynamic shared memory not 1024-byte aligned; nothing computed

// The current device's status word (device int, allocated on first use;
// kvp_read_status reads and clears it).  nullptr if it cannot be allocated.
int* status_word();

// False when the primary context of `device` is not active, e.g. after a
// cudaDeviceReset() by this or another CUDA runtime in the process: handles
// made in the context before it was destroyed must not be passed to CUDA.
// True when the state cannot be queried.
bool primary_context_active(int device);

// Records the message of the last failure on this thread.
void set_error(const char* fmt, ...);
const char* last_error();

// Records the message of CUDA error e and returns KVP_ERR_CUDA (call it
// only for e != cudaSuccess; KVP_CUDA below does the check).
int cuda_status(cudaError_t e, const char* what);

// Per-device one-time setup (kernel attributes, launch checks): `run` is
// called under a lock until it succeeds once on the current device; later
// calls on that device return KVP_OK at once.  A failed setup is retried
// (and re-reports its error) on the next call.
struct PerDeviceOnce {
    static constexpr int kMaxDevices = 64;
    std::mutex mu;
    bool done[kMaxDevices] = {};
    template <class F>
    int operator()(F&& run) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return KVP_ERR_CUDA;
        std::lock_guard<std::mutex> g(mu);
        if (done[dev]) return KVP_OK;
        const int rc = run(dev);
        if (rc == KVP_OK) done[dev] = true;
        return rc;
    }
};

}  // namespace kvp

#define KVP_CUDA(call)                                                 \
    do {                                                               \
        cudaError_t e_ = (call);                                       \
        if (e_ != cudaSuccess) return ::kvp::cuda_status(e_, #call);   \
    } while (0)
