// Host-only implementations behind oracle/ref_stub/cuda_runtime.h, plus the
// attention entry points the reference driver links against.
//
// TEST INFRASTRUCTURE ONLY.  It is linked with the reference's unmodified
// host sources (src/run_policy_experiment.cu, src/kv_tile_manager.cu,
// src/tile_gating_policy.cpp of GauthamMK-0/cuda-kv-persistence) so that the
// reference's own admission / KVMap code runs on a CPU.  Every call that
// touches persistence or copies rows is appended to the event log named by
// KVP_REF_LOG; the attention entry points record the KVMap slice the kernel
// would have received (the reference kernel's only view of policy decisions,
// src/gated_attention_kernel.cu:170-184) instead of computing attention.
#include "cuda_runtime.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>

static FILE* g_log = nullptr;
static bool g_log_init = false;
static size_t g_limit = 0;
static long g_alloc_idx = 0;
static size_t g_last_window = 0;

static FILE* logf_() {
    if (!g_log_init) {
        g_log_init = true;
        const char* p = getenv("KVP_REF_LOG");
        if (p && *p) g_log = fopen(p, "w");
    }
    return g_log;
}

extern "C" {

cudaError_t kvpref_malloc(void** p, size_t bytes) {
    void* q = calloc(bytes ? bytes : 1, 1);
    if (!q) return cudaErrorMemoryAllocation;
    *p = q;
    if (FILE* f = logf_())
        fprintf(f, "A %ld %llu %zu\n", g_alloc_idx, (unsigned long long)(uintptr_t)q, bytes);
    ++g_alloc_idx;
    return cudaSuccess;
}

cudaError_t cudaFree(void* p) {
    if (FILE* f = logf_()) fprintf(f, "F %llu\n", (unsigned long long)(uintptr_t)p);
    free(p);
    return cudaSuccess;
}

static void log_copy(char tag, int kind, void* dst, const void* src, size_t bytes) {
    // Host->device copies of Q/K/V are bulk; only the D2D row copies and the
    // KVMap upload carry admission information, but all are logged.
    if (FILE* f = logf_())
        fprintf(f, "%c %d %llu %llu %zu\n", tag, kind,
                (unsigned long long)(uintptr_t)dst,
                (unsigned long long)(uintptr_t)src, bytes);
}

cudaError_t cudaMemcpy(void* dst, const void* src, size_t bytes, cudaMemcpyKind k) {
    log_copy('C', (int)k, dst, src, bytes);
    memmove(dst, src, bytes);
    return cudaSuccess;
}

cudaError_t cudaMemcpyAsync(void* dst, const void* src, size_t bytes,
                            cudaMemcpyKind k, cudaStream_t) {
    log_copy('c', (int)k, dst, src, bytes);
    memmove(dst, src, bytes);
    return cudaSuccess;
}

cudaError_t cudaDeviceSetLimit(cudaLimit, size_t v) {
    g_limit = v;
    if (FILE* f = logf_()) fprintf(f, "L %zu\n", v);
    return cudaSuccess;
}

cudaError_t cudaDeviceGetLimit(size_t* v, cudaLimit) {
    *v = g_limit;
    return cudaSuccess;
}

cudaError_t cudaStreamSetAttribute(cudaStream_t, cudaStreamAttrID,
                                   const cudaStreamAttrValue* v) {
    g_last_window = v->accessPolicyWindow.num_bytes;
    if (FILE* f = logf_())
        fprintf(f, "W %llu %zu %d\n",
                (unsigned long long)(uintptr_t)v->accessPolicyWindow.base_ptr,
                v->accessPolicyWindow.num_bytes, (int)v->accessPolicyWindow.hitProp);
    return cudaSuccess;
}

cudaError_t cudaCtxResetPersistingL2Cache(void) {
    if (FILE* f = logf_()) fprintf(f, "R\n");
    return cudaSuccess;
}

cudaError_t cudaDeviceSynchronize(void) { return cudaSuccess; }
cudaError_t cudaGetLastError(void) { return cudaSuccess; }
cudaError_t cudaDeviceReset(void) {
    if (g_log) fflush(g_log);
    return cudaSuccess;
}
const char* cudaGetErrorString(cudaError_t) { return "stub"; }

// num_bytes of the last access-policy window set on a stream.
size_t kvpref_last_window_bytes(void) { return g_last_window; }

}  // extern "C"

// ---- attention entry points (declared in the reference's src/attn_kernel.h)

static void log_launch(const float* q, const float* k, const float* v,
                       const float* arena, const long* map, int T, int D,
                       int heads, int cross, int frame_idx) {
    FILE* f = logf_();
    if (!f) return;
    const long n = map ? (cross ? (long)(frame_idx + 1) * T : (long)T) : 0;
    fprintf(f, "K %d %d %d %d %d %llu %llu %llu %llu %llu %ld", frame_idx, cross,
            T, D, heads, (unsigned long long)(uintptr_t)q,
            (unsigned long long)(uintptr_t)k, (unsigned long long)(uintptr_t)v,
            (unsigned long long)(uintptr_t)arena, (unsigned long long)(uintptr_t)map, n);
    for (long i = 0; i < n; ++i)
        if (map[i] >= 0) fprintf(f, " %ld:%ld", i, map[i]);
    fprintf(f, "\n");
}

void attn_forward_single_frame(const float* d_q_f, const float* d_k,
                               const float* d_v, const float* d_arena,
                               const long* d_kvmap_f, float* d_out_f, int T,
                               int D, int heads, int cross, int frame_idx) {
    (void)d_out_f;
    log_launch(d_q_f, d_k, d_v, d_arena, d_kvmap_f, T, D, heads, cross, frame_idx);
}

void attn_forward_launcher(const float* d_q, const float* d_k, const float* d_v,
                           const float* d_arena, const long* d_kvmap, float* d_out,
                           int frames, int T, int D, int heads, bool remap) {
    (void)d_out;
    for (int f = 0; f < (remap ? frames : 1); ++f)
        log_launch(d_q, d_k, d_v, d_arena, remap ? d_kvmap + (size_t)f * T : nullptr,
                   T, D, heads, 0, f);
}
