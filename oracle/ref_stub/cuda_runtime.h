// Host-only stand-in for <cuda_runtime.h>, used ONLY to compile the
// reference's own host sources (kv_tile_manager.cu, tile_gating_policy.cpp,
// run_policy_experiment.cu) with g++ on a machine without a GPU.
//
// TEST INFRASTRUCTURE: nothing in the product links this.  "Device" memory
// is host memory, copies are memcpy, and every persistence call
// (cudaDeviceSetLimit, cudaStreamSetAttribute, cudaCtxResetPersistingL2Cache)
// is recorded in a text event log so the reference's admission behaviour can
// be replayed and compared row by row.  The log path comes from the
// KVP_REF_LOG environment variable (no log when unset).
#pragma once

#include <cstddef>
#include <cstdint>

typedef int cudaError_t;
static const cudaError_t cudaSuccess = 0;
static const cudaError_t cudaErrorMemoryAllocation = 2;

typedef struct CUstream_st* cudaStream_t;

enum cudaMemcpyKind {
    cudaMemcpyHostToHost = 0,
    cudaMemcpyHostToDevice = 1,
    cudaMemcpyDeviceToHost = 2,
    cudaMemcpyDeviceToDevice = 3,
    cudaMemcpyDefault = 4
};

enum cudaLimit { cudaLimitPersistingL2CacheSize = 0x06 };

enum cudaAccessProperty {
    cudaAccessPropertyNormal = 0,
    cudaAccessPropertyStreaming = 1,
    cudaAccessPropertyPersisting = 2
};

struct cudaAccessPolicyWindow {
    void* base_ptr;
    size_t num_bytes;
    float hitRatio;
    cudaAccessProperty hitProp;
    cudaAccessProperty missProp;
};

union cudaStreamAttrValue {
    cudaAccessPolicyWindow accessPolicyWindow;
    int syncPolicy;
};

enum cudaStreamAttrID { cudaStreamAttributeAccessPolicyWindow = 1 };

extern "C" {
cudaError_t kvpref_malloc(void** p, size_t bytes);
cudaError_t cudaFree(void* p);
cudaError_t cudaMemcpy(void* dst, const void* src, size_t bytes, cudaMemcpyKind k);
cudaError_t cudaMemcpyAsync(void* dst, const void* src, size_t bytes,
                            cudaMemcpyKind k, cudaStream_t s = 0);
cudaError_t cudaDeviceSetLimit(cudaLimit l, size_t v);
cudaError_t cudaDeviceGetLimit(size_t* v, cudaLimit l);
cudaError_t cudaStreamSetAttribute(cudaStream_t s, cudaStreamAttrID id,
                                   const cudaStreamAttrValue* v);
cudaError_t cudaCtxResetPersistingL2Cache(void);
cudaError_t cudaDeviceSynchronize(void);
cudaError_t cudaGetLastError(void);
cudaError_t cudaDeviceReset(void);
const char* cudaGetErrorString(cudaError_t e);
}

template <class T>
static inline cudaError_t cudaMalloc(T** p, size_t bytes) {
    return kvpref_malloc(reinterpret_cast<void**>(p), bytes);
}
