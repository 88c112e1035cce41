// Arguments of the persistent single-launch decode step (step_kernel.cu).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace fx {

constexpr int kStepThreads = 512;          // 15 consumer warps + 1 producer warp, one CTA per SM
constexpr int kStepConsumers = 480;
constexpr int kStepSlots = 7;              // TMA staging slots per CTA
constexpr int kStepSlotBytes = 27648;      // 12 rows of 576 floats
constexpr int kStepAttnRows = 54;          // cache rows (K and V) per attention tile
constexpr int kStepLmRows = 12;            // LM-head rows per tile
constexpr int kStepPartial = 66;           // m, l, o[64] per (head, chunk)
constexpr int kStepBlock = 4;              // columns per split-K strip (one 16-byte TMA box row)
constexpr int kStepStripRows = 192;        // rows per 2-D TMA box of a strip
constexpr int kStepReplicas = 4;           // copies of the published q | k | v words
constexpr int kStepAccReplicas = 4;        // copies of each split-K accumulator (spreads the atomics; 1 / 2 / 4 replicas: 1.02 / 0.445 / 0.428 ms at ctx 8192)
constexpr int kStepFullGridRows = 6144;   // caches of at least this many rows run on every SM
constexpr int kStepMinGrid = 128;          // the per-CTA slices must fit one slot (12 SwiGLU features)
constexpr int kStepMaxGrid = 384;          // every CTA owns at least one block of 4 MLP features

struct StepLayer {
    CUtensorMap o_map;        // o_proj [576, 576]: boxes of 4 columns x 192 rows
    CUtensorMap down_map;     // down   [576, 1536]: boxes of 4 columns x 192 rows
    const float* input_norm;  // [576]
    const float* qkv;         // [960, 576]
    const float* post_norm;   // [576]
    const float* gate_up;     // [3072, 576]
    float scale;
};

// Cross-CTA exchange region.
//  * q | k | v of the current row and the attention partials travel as
//    64-bit words (tag << 32 | float bits), double-buffered by layer parity: a
//    reader polls a word until it carries the tag of the current (step,
//    layer), so one L2 round trip both waits for and delivers it.
//  * o_proj and down are split-K over the CTAs; their partial sums meet in
//    64-bit tally words [contributor count | overflow count | sum of biased
//    2^-29 fixed-point terms] -- integer adds, so the sum is exact and
//    order-independent, and count and sum arrive in one atomic word: a
//    reader polls until every word's count is complete, no fence needed.
//    A partial outside the fixed-point range (|y| >= 2^13) is added to the
//    element's FP64 overflow word instead (then counted with a release add).
//    CTA c adds into replica c % kStepAccReplicas; readers sum the replicas.  Every layer
//    has its own tally and overflow words and the steps alternate between two
//    sets; each step zeroes the set of the next step, which only a later
//    launch reads.
struct StepExchange {
    unsigned long long* qkv;       // [2][kStepReplicas][960]
    unsigned long long* partial;   // [2][3][3][nch][66]
    unsigned long long* tally;     // [2 steps][30][o_proj, down][kStepAccReplicas][576]
    double* overflow;              // [2 steps][30][o_proj, down][576]
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
    // Host-mapped page-locked word of fx_decode_replay_host (null in the
    // device-resident graph): the step also stores the sampled token there,
    // so no device-to-host copy node follows it.  (Its input token still
    // arrives by a copy: 148 CTAs reading one mapped word cost ~0.1 ms.)
    int64_t* host_out;
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
    const int* inject;        // test hook: layer + 1 at which CTA 0 reports a failure (0: none)
    int* stop;                // [0] set once a step produced the EOS token: later steps return at once
                              // [1] EOS token + 1 (0: no EOS)
    int nch;                  // attention chunks per kv head
    unsigned long long* timeline;  // optional [grid][kStepTimelineEvents] (cycle << 32 | globaltimer) stamps
};

// Timeline events per CTA: 0 = start, then per layer 12 stamps (A: h ready,
// done; B: q polled, first cache tiles landed, cache tiles done, partial
// published; M: partials polled, o_proj tile landed, o_proj partial added;
// D: h' ready, gate/up done, down partial added), then LM-head start and end.
constexpr int kStepTimelinePerLayer = 12;
constexpr int kStepTimelineEvents = 1 + kStepTimelinePerLayer * kLayers + 2;

// 64-bit words of the exchange region for `nch` chunks per kv head.
size_t step_exchange_words(int nch);
// Carve the exchange region (base must be 256-byte aligned).
StepExchange step_exchange_views(unsigned long long* base, int nch);
// Fill the layer's tensor maps for the split-K strips of o_proj and down.
fx_status encode_step_maps(const float* o_proj, const float* down, StepLayer* layer);

// Enqueue one decode step as a single cooperative launch of `grid` CTAs.
fx_status launch_step_kernel(const StepArgs& args, int grid, cudaStream_t stream);
// Dynamic shared memory the step kernel needs (bytes).
size_t step_kernel_smem_bytes();
// Configure the kernel on `device`; *grid = CTAs to launch (one per SM).
fx_status prepare_step_kernel(int device, int* grid);

}  // namespace fx
