// GPU motion-trace producer (csrc/motion_sm100.cu): dense two-frame optical
// flow between consecutive frames and the per-tile change rates of
// traces/gen_motion_from_video.py.
#pragma once

#include <cstdint>
#include <vector>

#include <cuda_runtime.h>

namespace kvp {

struct MotionParams {
    int height, width;         // frame size (the reference: 480 x 832)
    int levels;                // pyramid layers above the frame (the reference: 3)
    int winsize;               // odd box window of the displacement fit (15)
    int iterations;            // displacement updates per layer (3)
    int poly_n;                // odd taps of the polynomial expansion (5)
    float poly_sigma;          // its Gaussian applicability (1.2)
    float pyr_scale;           // layer scale (0.5)
    int grid_rows, grid_cols;  // latent grid (30 x 52); cells = frame / grid
    int tile_cells;            // cells per tile (16 tokens)
};

class MotionProducer {
public:
    explicit MotionProducer(const MotionParams& p);
    ~MotionProducer();
    int status() const { return status_; }
    int tiles() const { return tiles_; }
    // Flow [2][height][width] (dx plane, dy plane) with next(x + d) ~ prev(x).
    int pair_flow(const uint8_t* d_prev, const uint8_t* d_next, float* d_flow, cudaStream_t s);
    // change [frames][tiles] (fp32, device): mean flow magnitude per tile of
    // pair (f-1, f) for f >= 1, row 0 = row 1.  d_frames is uint8
    // [frames][height][width].  Replays a CUDA graph captured on the first
    // call for these (d_frames, frames, d_change); a call from inside a
    // stream capture enqueues the kernels directly.
    int trace(const uint8_t* d_frames, int frames, float* d_change, cudaStream_t s);

private:
    struct Level;
    int load_frame(const uint8_t* d_frame, int slot, cudaStream_t s);
    int flow(int prev_slot, int next_slot, float* d_out, cudaStream_t s);
    int enqueue_trace(const uint8_t* d_frames, int frames, float* d_change, cudaStream_t s);

    MotionParams p_;
    int status_ = 0;
    int tiles_ = 0;
    std::vector<Level> levels_;
    float* tmp_ = nullptr;
    float* tmp2_ = nullptr;
    float* M_ = nullptr;
    float* M2_ = nullptr;
    float* flow_[2] = {nullptr, nullptr};
    float* fflow_ = nullptr;
    // the captured trace pass and the buffers it was captured for
    cudaStream_t cap_stream_ = nullptr;
    cudaEvent_t ev_in_ = nullptr, ev_out_ = nullptr;
    cudaGraphExec_t exec_ = nullptr;
    const uint8_t* g_frames_ = nullptr;
    int g_count_ = 0;
    float* g_change_ = nullptr;
};

// The reference's threshold (:119-121, :146-151) on host change rates
// [frames][tiles]: tau = the percentile (numpy's linear interpolation) of
// frames 1..F-1; reuse = change < tau except frame 0; is_static = change < tau.
int motion_threshold(const float* change, int frames, int tiles, double percentile,
                     int8_t* reuse, int8_t* is_static, double* tau_out);

}  // namespace kvp
