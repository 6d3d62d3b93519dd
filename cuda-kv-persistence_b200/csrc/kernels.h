// Launchers of the kvp CUDA kernels (sm_100a).  All return a kvp::Status.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "kv_tile_manager.h"

namespace kvp {

// ---- compaction (csrc/compaction.cu) --------------------------------------

// n independent contiguous copies described by a device array of CopyOp.
int launch_copy_batch(const CopyOp* d_ops, int n, cudaStream_t stream);

constexpr int kMaxLayers = 32;

// Per-layer buffers for the session gather: base K/V rows [rows][row_bytes]
// and the arena [cap][2*row_bytes] (K half, then V half).
struct GatherLayers {
    const void* k[kMaxLayers];
    const void* v[kMaxLayers];
    void* arena[kMaxLayers];
};

// For i < n and every layer: arena[slot[i]] = K[row[i]] || V[row[i]],
// except rows in [skip_lo, skip_hi).  pairs is a device int32 array [n][2]
// = (source row, arena slot).
int launch_gather_rows(const GatherLayers& L, int layers, const int32_t* d_pairs, int n,
                       int64_t row_bytes, cudaStream_t stream, int64_t skip_lo = 0,
                       int64_t skip_hi = 0);

// ---- FP32 remapped attention (csrc/attn_fp32.cu) --------------------------

// Query rows [0, T) of q/out (row stride D floats, head h at columns
// h*128..h*128+127) against key rows j in [k_lo, k_hi) of k/v.  Key row j is
// read from arena row kvmap[j] (K half at column 0, V half at column D of a
// 2*D-float row) when kvmap && kvmap[j] >= 0, else from k/v row j.
// arena_rows bounds the map (entries >= arena_rows are reported as
// KVP_ERR_MAP through *status and read from the base instead).
int launch_attn_fp32(const float* q, const float* k, const float* v, const float* arena,
                     const int64_t* kvmap, float* out, int T, int D, int heads, int64_t k_lo,
                     int64_t k_hi, int64_t arena_rows, int frames, int64_t frame_stride_rows,
                     int* d_status, cudaStream_t stream);

// The reference's two fp32 entry points (src/attn_kernel.h:15-29): flush
// every manager's queued staging copies, then launch on the legacy default
// stream.  Exported twice, with C linkage (capi.cpp) and with the C++
// linkage of the reference's header (cxx_abi.cpp).
void fp32_launcher(const float* d_q, const float* d_k, const float* d_v, const float* d_arena,
                   const long* d_kvmap, float* d_out, int frames, int T, int D, int heads,
                   bool remap);
void fp32_single_frame(const float* d_q_f, const float* d_k, const float* d_v,
                       const float* d_arena, const long* d_kvmap_f, float* d_out_f, int T, int D,
                       int heads, int cross, int frame_idx);

}  // namespace kvp
