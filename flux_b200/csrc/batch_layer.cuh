// One cooperative launch per layer boundary of the batched decode step: the
// projections, split-K-free sums, norms, SwiGLU, RoPE and cache writes that
// sit between two attention launches (batch_layer.cu).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace fx {

constexpr int kLayerThreads = 512;  // 16 warps, every one computing
constexpr int kLayerMinGrid = 128;  // the per-CTA weight slices are sized for grids of >= 128 CTAs
constexpr int kLayerMaxRows = 64;   // activation rows (sequences) per launch

enum BatchLayerMode : int {
    kLayerFirst = 0,   // embedding rows -> layer 0's input norm, QKV, RoPE, cache rows
    kLayerMiddle = 1,  // layer l's attention merge, o_proj .. down, then layer l + 1's input norm, QKV, RoPE, cache rows
    kLayerLast = 2,    // layer l's attention merge, o_proj .. down, then the final norm rows
};

// Tensor maps over the activation matrices the phases stage (box 32 columns x
// 64 rows, 128-byte swizzle; rows past the matrix read as zeros).
struct alignas(64) BatchLayerMaps {
    CUtensorMap attn;  // [rows][576]
    CUtensorMap h2;    // [rows][576]
    CUtensorMap act;   // [rows][1536]
    CUtensorMap h;     // [rows][576]
};

struct alignas(64) BatchLayerArgs {
    BatchLayerMaps maps;
    // layer l (middle / last)
    const float* o_proj;     // [576][576]
    const float* post_norm;  // [576]
    const float* gate_up;    // [3072][576]: gate rows, then up rows
    const float* down;       // [576][1536]
    // layer l + 1 (first / middle); the final norm in next_norm (last)
    const float* next_norm;  // [576]
    const float* next_qkv;   // [960][576]
    const float* embedding;  // first: [vocab][576]
    const int64_t* tokens;   // first: [B]
    int64_t vocab;
    float* attn;             // [B][576] attention output of layer l (merged here from attn_ws)
    const float* attn_ws;    // [B][9][attn_chunks][66] (m, l, o[64]) per attention chunk of layer l
    int64_t attn_chunks;     // chunks per (sequence, head) in attn_ws
    int attn_rows;           // cache rows per attention chunk
    float* h;                // [B][576] residual stream: layer l's input in, layer l + 1's input out
    float* h2;               // [B][576] after the attention block
    float* act;              // [B][1536] SwiGLU
    float* q;                // [B][9][64] roped q of layer l + 1
    float* key_cache;        // layer l + 1: [B][3][cap][64]
    float* value_cache;
    const int64_t* positions;
    int64_t* lengths;        // lengths[b] = positions[b] + 1
    int64_t cap;
    const float* rope_cos;   // [positions][64]
    const float* rope_sin;
    float* norm_out;         // last: final-norm rows [B][576]
    unsigned* barrier;       // [4] arrival counters of this launch, zero before it (C, D, E, F)
    unsigned* error;         // bit 2: a position outside the cache; bit 16: a bounded wait gave up
    float eps;
    int rows;                // B <= 64
    int mode;
};

// Dynamic shared memory of the kernel (bytes).
size_t batch_layer_smem_bytes();
// Configure the kernel on the current device; *grid = CTAs per launch (one
// per SM, all co-resident, >= kLayerMinGrid).
fx_status prepare_batch_layer(int* grid);
// Enqueue one cooperative launch.
fx_status launch_batch_layer(const BatchLayerArgs& a, int grid, cudaStream_t stream);

}  // namespace fx
