// Decode attention over the compact cache for SmolLM2's geometry (9 q heads,
// 3 kv heads, head_dim 64): the fast path of fx_gqa_decode_attention_f32 and
// the attention of the batched decode runtime (attention.cu).
#pragma once

#include "common.cuh"

namespace fx {

constexpr int kCompactChunk = 128;  // cache rows per CTA of the op path; workspace [B][9][chunks][66] as the generic op

struct CompactAttention {
    const float* q;              // [B][9][64]
    const float* k;              // [B][3][cap][64] (16-byte aligned)
    const float* v;
    const int64_t* lengths;      // valid length of sequence b: lengths[b * length_stride], clamped to [1, cap]; null: cap
    int64_t length_stride;
    float* out;                  // [B][9][64]
    float* ws;                   // [B][9][chunks][66]
    unsigned* error;             // optional: bit 1 set if a bounded wait gave up
    unsigned* counters;          // optional [B][3] arrival counters, zero before the first launch (every launch
                                 // leaves them zero): the last chunk CTA of a (sequence, kv head) merges, no
                                 // separate merge launch; null: merge kernel
    float scale;
    int64_t batch, cap, chunks;  // chunks = ceil(cap / chunk_rows)
    int chunk_rows;              // 128 (the op's workspace format) or 64
};

// Workspace floats for `batch` sequences of capacity `cap` in chunks of `rows`.
inline int64_t compact_attention_workspace(int64_t batch, int64_t cap, int rows = kCompactChunk) {
    return batch * kQHeads * ((cap + rows - 1) / rows) * (kHeadDim + 2);
}

// Enqueue the chunk kernel (and the merge kernel unless `counters` is set or
// `merge` is false: the caller merges the workspace itself) on `stream`
// (`dependent`: as programmatic dependent launches of the preceding kernel).
fx_status launch_compact_attention(const CompactAttention& a, cudaStream_t stream, bool dependent = false,
                                   bool merge = true);

}  // namespace fx
