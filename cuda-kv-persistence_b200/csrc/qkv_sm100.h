// QKV projection with the arena written in the epilogue, and the block's
// LayerNorm (csrc/qkv_sm100.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace kvp {

// One layer's projection: x bf16 [rows][D] (the LayerNorm output, rows >=
// 128, D a multiple of 256, all buffers 16-byte aligned), w bf16
// [3D][D] (nn.Linear(D, 3D).weight: Q rows, then K, then V), bias fp32 [3D]
// (may be null).  Writes Q/K/V bf16 [rows][D] (q may be null) and, for each
// row r with kvmap[map_row0 + r] in [0, arena_rows), that row's K and V into
// arena row kvmap[...] (bf16 [arena_rows][2D], K half then V half).  Map
// entries >= arena_rows set KVP_STATUS_MAP and are skipped.
struct QkvIO {
    const void* x;
    const void* w;
    const float* bias;
    void* q;
    void* k;
    void* v;
    void* arena;
    const long long* kvmap;
    long long rows, map_row0, arena_rows;
    int D;
};

// d_status null = the current device's status word.
int launch_qkv_project_bf16(const QkvIO& io, int* d_status, cudaStream_t stream);

// y = LayerNorm(x) * gamma + beta per row (bf16 in and out, fp32 statistics).
int launch_layernorm_bf16(const void* x, const float* gamma, const float* beta, void* y,
                          long long rows, int D, float eps, cudaStream_t stream);

}  // namespace kvp
