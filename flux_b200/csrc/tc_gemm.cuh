// FP32 projections on the 5th-generation tensor cores (tcgen05) with the
// 3xTF32 split: every FP32 operand x is carried as hi = tf32(x) and
// lo = tf32(x - hi), and C = Xhi.Whi + Xlo.Whi + Xhi.Wlo accumulates in FP32
// in tensor memory.  The dropped Xlo.Wlo term is below 2^-22 of each
// product, so results sit at FP32 rounding level (the SIMT paths' ~1e-6
// relative), not TF32's ~1e-3.
//
// Used where the work is a real contraction: the batched decode projections
// (B rows per step, split-K partials) and the prefill projections (S rows).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace fx {

constexpr int kTcTileN = 128;  // weight rows per CTA (the MMA's M)
constexpr int kTcTileK = 32;   // K columns per stage: one 128-byte swizzle row
constexpr int kTcPairN = 192;  // weight rows per CTA pair in the paired form (96 per CTA)
// The paired form runs from this many X rows; below it the pairs' 256-row
// tiles are too few to fill the GPU (a 128-token prompt: 16 pairs, half of
// each tile padding).  Measured prefills (ms, pairs / per-tile): 128 tokens
// 5.70 / 4.90, 1024: 6.96 / 6.81, 2048: 8.92 / 9.48.
constexpr int kTcPairMinRows = 2048;

// C[m][n] (+ R[m][n]) = sum_k X[m][k] W[n][k] over k in split blockIdx.z's
// slice; C points at split 0 and later splits follow at `split_stride`.
struct alignas(64) TcGemmArgs {
    CUtensorMap w_hi;  // [N][K], box 32 x 128, 128-byte swizzle
    CUtensorMap w_lo;
    CUtensorMap x;     // [M][K], box 32 x BM, 128-byte swizzle
    // W with boxes of 96 rows, for the paired form (128-row X tiles, no K
    // split, N a multiple of 192); `has_pair` says they are set.
    CUtensorMap w_hi96, w_lo96;
    bool has_pair;
    // Fused SwiGLU (paired form only): W is the packed gate/up weight split
    // with rows in the order tc_weights_create(..., swiglu_rows) gives, and
    // act[m][f] = silu(gate) * up is written instead of C (row stride act_ld).
    bool swiglu;
    float* act;
    int act_ld;
    float* c;
    const float* residual;  // null, or [M][ldc] added in the epilogue
    int* error;             // bit 8: a wait gave up
    int m, n, k, ldc;
    int k_per_split;        // multiple of kTcTileK
    long long split_stride; // floats between split outputs
};

// Tensor maps over a row-major FP32 matrix [rows][cols] (cols % 4 == 0,
// 16-byte aligned base) with a box of 32 columns x `box_rows` rows.
fx_status tc_encode_map(CUtensorMap* map, const float* base, int64_t rows, int64_t cols, int box_rows,
                        const char* what);

// hi = tf32(w), lo = tf32(w - hi) elementwise (n % 4 == 0, 16-byte aligned).
fx_status tc_split(const float* w, float* hi, float* lo, size_t n, cudaStream_t stream);

// One launch: grid (ceil(N / 128), ceil(M / bm), splits); bm is 64 or 128.
// `stages` (shared-memory pipeline depth, 48 KB each at bm 64): 0 for the
// default (4 at bm 64, 3 at bm 128), or 3 at bm 64 so that a CTA (145 KB)
// shares its SM with a 71 KB attention chunk CTA of a concurrent stream.
fx_status launch_tc_gemm(const TcGemmArgs& args, int bm, int splits, cudaStream_t stream, bool dependent,
                         int stages = 0);

// The hi / lo halves of one projection weight and their tensor maps (boxes
// of 128 rows, and of 96 rows for the paired form).
struct TcWeight {
    CUtensorMap hi, lo, hi96, lo96;
    int rows = 0, cols = 0;
};

// Split copies of the 30 layers' projections (packed QKV, o_proj, packed
// gate/up, down) and optionally the LM head, in one owned allocation.
struct TcModelWeights {
    float* buffer = nullptr;
    TcWeight qkv[kLayers], o[kLayers], gate_up[kLayers], down[kLayers];
    TcWeight lm_head;
    bool has_lm_head = false;
};

// `layers` false: the LM head only (the persistent batched layers multiply
// FP32 weights on the SIMT cores).  `swiglu_rows`: the packed gate/up
// weights are split with their rows reordered for the paired form's fused
// SwiGLU -- in each block of 192 rows, features 96 b + 48 h + [0, 48) as 48
// gate rows then their 48 up rows (h = 0, 1) -- and serve only that form.
fx_status tc_weights_create(const fx_model_desc& model, bool lm_head, TcModelWeights* out, cudaStream_t stream,
                            bool layers = true, bool swiglu_rows = false);
void tc_weights_release(TcModelWeights* w);

// Arguments of C = X . W^T (+ residual) with K split in `k_per_split` slices.
TcGemmArgs tc_args(const TcWeight& w, const CUtensorMap& x, float* c, const float* residual, int* error, int m,
                   int k_per_split);

}  // namespace fx
