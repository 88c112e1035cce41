// Arguments of the persistent single-launch decode step (step_kernel.cu).
#pragma once

#include "common.cuh"

namespace fx {

constexpr int kStepThreads = 512;             // 16 warps per CTA, one CTA per SM
constexpr int kStepRingBytes = 192 * 1024;    // TMA staging ring per CTA
constexpr int kStepSlots = 16;                // mbarriers (tiles in flight)
constexpr int kStepReplicas = 4;              // down-projection accumulators per set
constexpr int kStepAttnRows = 64;             // cache rows per attention tile
constexpr int kStepLmRows = 32;               // LM-head rows per tile
constexpr int kStepPartialStride = 68;        // m, l, pad, pad, o[64]

struct StepLayer {
    const float* input_norm;  // [576]
    const float* qkv;         // [960, 576]
    const float* o_proj;      // [576, 576]
    const float* post_norm;   // [576]
    const float* gate_up;     // [3072, 576]
    const float* down_t;      // [1536, 576]: the down projection transposed (runtime-owned)
    float scale;
};

struct StepArgs {
    StepLayer layer[kLayers];
    const float* embedding;   // [vocab, 576]
    const float* final_norm;
    const float* lm_head;     // [vocab, 576]
    const float* cos_table;   // [capacity, 64]
    const float* sin_table;
    int64_t vocab;
    int64_t capacity;
    float eps;
    float* key_cache;         // [30, 3, capacity, 64]
    float* value_cache;
    int64_t* token;
    int64_t* position;
    int64_t* length;
    int64_t* step;
    int64_t* generated;
    float* logits;
    // workspace (cross-CTA traffic goes through L2 with .cg loads)
    float* q;                 // [576] rotated queries of the current layer
    float* attn;              // [576] merged attention output
    float* hidden_mid;        // [576] h' = h + o_proj(attn) of the current layer
    float* accum;             // [2][kStepReplicas][576] down-projection partial sums
    float* partials;          // [3][3][nch][kStepPartialStride]
    float* final_norm_out;    // [576]
    float* cand_value;        // [grid]
    long long* cand_index;    // [grid]
    unsigned* sync;           // [0] grid barrier, [1..3] kv-group merge, [4] LM head
    int* error;               // bit 1: position outside capacity, bit 2: a bounded wait gave up
    int nch;                  // attention chunks per kv head
    unsigned long long* timeline;  // optional [grid][kStepTimelineEvents] %globaltimer stamps
};

// Timeline events per CTA: 0 = start, then per layer 8 stamps (phase A done,
// barrier 1 passed, B done, barrier 2 passed, C done, barrier 3 passed, D
// done, barrier 4 passed), then LM-head start and end.
constexpr int kStepTimelineEvents = 1 + 8 * kLayers + 2;

// Enqueue one decode step as a single cooperative launch of `grid` CTAs.
fx_status launch_step_kernel(const StepArgs& args, int grid, cudaStream_t stream);
// Dynamic shared memory the step kernel needs (bytes).
size_t step_kernel_smem_bytes();
// down [576, 1536] -> down_t [1536, 576] for every layer.
fx_status launch_transpose_down(const float* const* down, float* down_t, cudaStream_t stream);

}  // namespace fx
