// Causal prefill attention on tcgen05 tensor cores (3xTF32), GQA 9 q heads /
// 3 kv heads, head_dim 64: out[s][h] = softmax_k<=s(q[h][s] . k[h/3][k] *
// scale) . v[h/3][k] for s < S.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace fx {

constexpr int kTcAttnQ = 128;   // queries per CTA
constexpr int kTcAttnKeys = 64; // keys per tile

struct alignas(64) TcAttentionArgs {
    CUtensorMap q_hi, q_lo;    // [9 * S][64] (head-major rows), box 32 x 128
    CUtensorMap k_hi, k_lo;    // [3 * padded][64], box 32 x 64
    CUtensorMap vt_hi, vt_lo;  // [3 * 64][padded] (V transposed per kv head), box 32 x 64
    float* out;                // [S][576]
    int* error;                // bit 8: a bounded wait gave up
    int rows;                  // S
    int padded;                // S rounded up to a whole key tile (rows past S are zero)
    float scale;
};

// Rows S of the split operands: padded = ceil(S / 64) * 64.
inline int64_t tc_attention_padded(int64_t rows) { return (rows + kTcAttnKeys - 1) / kTcAttnKeys * kTcAttnKeys; }

fx_status launch_tc_prefill_attention(const TcAttentionArgs& args, cudaStream_t stream);

}  // namespace fx
