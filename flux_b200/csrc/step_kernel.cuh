// Arguments of the persistent single-launch decode step (step_kernel.cu).
#pragma once

#include "common.cuh"

namespace fx {

constexpr int kStepThreads = 512;          // 15 consumer warps + 1 producer warp, one CTA per SM
constexpr int kStepConsumers = 480;
constexpr int kStepSlots = 7;              // TMA staging slots per CTA
constexpr int kStepSlotBytes = 27648;      // 12 rows of 576 floats
constexpr int kStepAttnRows = 54;          // cache rows (K and V) per attention tile
constexpr int kStepLmRows = 12;            // LM-head rows per tile
constexpr int kStepDownRows = 4;           // down-projection rows (1536 floats) per tile
constexpr int kStepPartial = 66;           // m, l, o[64] per (head, chunk)
constexpr int kStepMinGrid = 140;          // the per-CTA slices must fit one slot
constexpr int kStepMaxGrid = 480;

struct StepLayer {
    const float* input_norm;  // [576]
    const float* qkv;         // [960, 576]
    const float* o_proj;      // [576, 576]
    const float* post_norm;   // [576]
    const float* gate_up;     // [3072, 576]
    const float* down;        // [576, 1536]
    float scale;
};

// Cross-CTA exchange buffers, double-buffered by layer parity.  Every word is
// (tag << 32 | float bits): a reader polls the word until it carries the tag
// of the current (step, layer), so one L2 round trip both waits for and
// delivers the value -- no grid barrier, no fence.
struct StepExchange {
    unsigned long long* hidden;    // [2][576]   layer input h (tag of the layer it enters)
    unsigned long long* qkv;       // [2][960]   RoPE'd q | RoPE'd k | v of the current row
    unsigned long long* partial;   // [2][3][3][nch][66] attention split-K partials
    unsigned long long* attn;      // [2][576]   merged attention output
    unsigned long long* mid;       // [2][576]   h' = h + o_proj(attn)
    unsigned long long* swiglu;    // [2][1536]  SwiGLU output
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
    StepExchange x;
    float* final_norm_out;    // [576]
    float* cand_value;        // [grid]
    long long* cand_index;    // [grid]
    unsigned* sync;           // [0] LM-head arrivals, [1] step epoch
    int* error;               // bit 1: position outside capacity, bit 2: a bounded wait gave up
    int nch;                  // attention chunks per kv head
    unsigned long long* timeline;  // optional [grid][kStepTimelineEvents] %globaltimer stamps
};

// Timeline events per CTA: 0 = start, then per layer 15 stamps (A: h polled,
// tile landed, done; B: q polled, cache tiles done, partial published; M:
// partials polled, done; C: attn polled, tile landed, done; D: h' polled,
// done; E: SwiGLU polled, done), then LM-head start and end.
constexpr int kStepTimelinePerLayer = 15;
constexpr int kStepTimelineEvents = 1 + kStepTimelinePerLayer * kLayers + 2;

// Words of the exchange region for `nch` chunks per kv head.
inline size_t step_exchange_words(int nch) {
    return 2ull * (576 + 960 + 9ull * nch * kStepPartial + 576 + 576 + 1536);
}
// Carve the exchange region (base must be 16-byte aligned).
StepExchange step_exchange_views(unsigned long long* base, int nch);

// Enqueue one decode step as a single cooperative launch of `grid` CTAs.
fx_status launch_step_kernel(const StepArgs& args, int grid, cudaStream_t stream);
// Dynamic shared memory the step kernel needs (bytes).
size_t step_kernel_smem_bytes();
// Configure the kernel on `device`; *grid = CTAs to launch (one per SM).
fx_status prepare_step_kernel(int device, int* grid);

}  // namespace fx
