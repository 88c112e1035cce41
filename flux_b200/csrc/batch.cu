// Batched greedy decode: B <= 64 independent sequences of SmolLM2-135M advanced
// together, one CUDA-graph replay per step.  The reference has no batched
// runtime (it is batch 1 only); this serves the sequence-sharded batched
// configuration, where each GPU owns its own sequences and replicas of the
// weights and nothing crosses GPUs.
//
// Per layer (10 launches, programmatic dependent launches in the graph):
// QKV split-K GEMM -> split-K sum + RoPE + cache write at each sequence's own
// position -> compact split-K attention over each sequence's valid length
// (attention.cu, chunks + merge) -> o_proj GEMM -> split-K sum + residual +
// RMSNorm -> gate/up GEMM -> split-K sum + SwiGLU -> down GEMM -> split-K sum
// + residual + the next layer's RMSNorm; then the tied LM head GEMM over all
// rows and a per-row greedy argmax that advances each sequence's token and
// position.  The batch runs as two lanes (halves) on two streams forked and
// joined inside the graph, so one half's latency-bound projections and
// reductions overlap the other half's HBM-bound attention.
//
// The projections are skinny GEMMs (M <= 64 rows of activations against the
// weight rows) on tcgen05 tensor cores (tc_gemm.cu) or, optionally, SIMT
// 64 x 64 tiles, over a slice of K so that small N still spreads over the
// SMs; the K slices are summed in a fixed order by the following fused
// kernel -- deterministic, FP32, and a row's result does not depend on the
// other rows of the batch.
#include "attention.cuh"
#include "batch_layer.cuh"
#include "common.cuh"
#include "tc_gemm.cuh"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

namespace fx {
namespace {

constexpr int kMaxBatch = 64;
constexpr int kTileM = 64, kTileN = 64, kTileK = 32, kGemmThreads = 256;
constexpr int64_t kMaxCapacity = 131072;

// ------------------------------------------------------------- kernels

// Row b of the residual stream (one CTA of 576 threads, one element each)
// is written to h and its RMSNorm n = h * rsqrt(mean(h^2) + eps) * w to
// norm_out.
__device__ __forceinline__ void store_row_and_norm(int b, int i, float v, float* __restrict__ h,
                                                   const float* __restrict__ w, float eps, float* __restrict__ norm_out) {
    __shared__ float scratch[32];
    h[static_cast<size_t>(b) * kHidden + i] = v;
    const float ss = block_sum(v * v, scratch);
    const float inv = rsqrtf(ss / static_cast<float>(kHidden) + eps);
    norm_out[static_cast<size_t>(b) * kHidden + i] = v * inv * w[i];
}

// h[b] = embedding[tokens[b]] (zeros for an out-of-range token) and the
// first layer's input norm of it.
__global__ void __launch_bounds__(kHidden) embed_rows_kernel(const int64_t* __restrict__ tokens,
                                                             const float* __restrict__ embedding, int64_t vocab,
                                                             float* __restrict__ h, const float* __restrict__ w,
                                                             float eps, float* __restrict__ norm_out) {
    grid_dependency_wait();

    const int b = blockIdx.x, i = threadIdx.x;
    const int64_t t = tokens[b];
    const bool valid = t >= 0 && t < vocab;
    store_row_and_norm(b, i, valid ? embedding[t * kHidden + i] : 0.0f, h, w, eps, norm_out);
}

// P[split][m][n] = sum over k in the split's slice of X[m][k] * W[n][k]
// (M <= 64).  256 threads, 4 x 4 outputs each; K staged through two
// shared-memory buffers 32 columns at a time (transposed so the inner loop
// reads float4s), the next slice fetched into registers while the current
// one is multiplied: one barrier per slice.
__global__ void __launch_bounds__(kGemmThreads) skinny_gemm_kernel(const float* __restrict__ X,
                                                                   const float* __restrict__ W,
                                                                   float* __restrict__ P, int M, int N, int K,
                                                                   int k_per_split) {
    grid_dependency_wait();
    __shared__ __align__(16) float As[2][kTileK][kTileM + 4];
    __shared__ __align__(16) float Bs[2][kTileK][kTileN + 4];
    const int n0 = blockIdx.x * kTileN;
    const int split = blockIdx.y;
    const int k0 = split * k_per_split;
    const int k1 = min(K, k0 + k_per_split);
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    // loader: float4 j covers row (tid + 256 j) / 8, k quad (tid + 256 j) % 8
    float4 ar[2], br[2];
    auto fetch = [&](int kk) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int idx = tid + kGemmThreads * j, r = idx >> 3, kq = (idx & 7) * 4;
            ar[j] = r < M && kk + kq < k1 ? *reinterpret_cast<const float4*>(X + static_cast<size_t>(r) * K + kk + kq)
                                          : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            br[j] = n0 + r < N && kk + kq < k1
                        ? *reinterpret_cast<const float4*>(W + static_cast<size_t>(n0 + r) * K + kk + kq)
                        : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
    };
    auto stage = [&](int buf) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int idx = tid + kGemmThreads * j, r = idx >> 3, kq = (idx & 7) * 4;
            As[buf][kq + 0][r] = ar[j].x;
            As[buf][kq + 1][r] = ar[j].y;
            As[buf][kq + 2][r] = ar[j].z;
            As[buf][kq + 3][r] = ar[j].w;
            Bs[buf][kq + 0][r] = br[j].x;
            Bs[buf][kq + 1][r] = br[j].y;
            Bs[buf][kq + 2][r] = br[j].z;
            Bs[buf][kq + 3][r] = br[j].w;
        }
    };
    float acc[4][4] = {};
    int buf = 0;
    if (k0 < k1) {
        fetch(k0);
        stage(0);
    }
    __syncthreads();
    for (int kk = k0; kk < k1; kk += kTileK) {
        const bool more = kk + kTileK < k1;
        if (more) fetch(kk + kTileK);
#pragma unroll
        for (int k = 0; k < kTileK; ++k) {
            const float4 a = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4]);
            const float4 b = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4]);
            const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        if (more) stage(buf ^ 1);
        __syncthreads();
        buf ^= 1;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = ty * 4 + i;
        if (m >= M) continue;
        const int n = n0 + tx * 4;
        float* dst = P + (static_cast<size_t>(split) * M + m) * N + n;
        if (n + 3 < N) {
            *reinterpret_cast<float4*>(dst) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (n + j < N) dst[j] = acc[i][j];
        }
    }
}

// Sum of the split-K partials of element i, splits in a fixed order with
// four loads in flight.
__device__ __forceinline__ float split_sum(const float* __restrict__ P, int splits, size_t stride, size_t i) {
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    int s = 0;
    for (; s + 3 < splits; s += 4) {
        a0 += P[(s + 0) * stride + i];
        a1 += P[(s + 1) * stride + i];
        a2 += P[(s + 2) * stride + i];
        a3 += P[(s + 3) * stride + i];
    }
    for (; s < splits; ++s) a0 += P[s * stride + i];
    return (a0 + a1) + (a2 + a3);
}

// out[m][n] = sum_s P[s][m][n] (+ residual[m][n]).
__global__ void reduce_splits_kernel(const float* __restrict__ P, int splits, int M, int N,
                                     const float* __restrict__ residual, float* __restrict__ out) {
    grid_dependency_wait();

    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(M) * N) return;
    const float v = split_sum(P, splits, static_cast<size_t>(M) * N, i);
    out[i] = residual != nullptr ? residual[i] + v : v;
}

// h_out[m] = residual[m] + sum_s P[s][m] (the o_proj / down split-K sum
// onto the residual stream) and the following RMSNorm of it; one CTA of
// 576 threads per row.
__global__ void __launch_bounds__(kHidden) reduce_residual_norm_kernel(const float* __restrict__ P, int splits, int M,
                                                                       const float* __restrict__ residual,
                                                                       float* __restrict__ h_out,
                                                                       const float* __restrict__ w, float eps,
                                                                       float* __restrict__ norm_out) {
    grid_dependency_wait();

    const int b = blockIdx.x, i = threadIdx.x;
    const size_t e = static_cast<size_t>(b) * kHidden + i;
    const float v = residual[e] + split_sum(P, splits, static_cast<size_t>(M) * kHidden, e);
    store_row_and_norm(b, i, v, h_out, w, eps, norm_out);
}

// out[m][i] = swiglu(sum_s P[s][m][i], sum_s P[s][m][I + i]) for the packed gate|up columns.
__global__ void reduce_swiglu_kernel(const float* __restrict__ P, int splits, int M, float* __restrict__ out) {
    grid_dependency_wait();

    const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= static_cast<int64_t>(M) * kInter) return;
    const int64_t m = e / kInter, i = e % kInter;
    const size_t stride = static_cast<size_t>(M) * kGateUp;
    const float g = split_sum(P, splits, stride, m * kGateUp + i);
    const float u = split_sum(P, splits, stride, m * kGateUp + kInter + i);
    out[e] = swiglu(g, u);
}

// The packed QKV projection's split-K sum, then RoPE on q/k of every
// sequence at its own position, K/V rows written into the layer's cache
// [B][3][cap][64], q -> [B][9][64], lengths[b] = pos + 1.  `qkv` holds
// `splits` partials [s][B][960] (one split: the projection itself).  One
// thread per (sequence, pair): q/k pairs (d, d + 32), v single values.
__global__ void rope_cache_rows_kernel(const float* __restrict__ qkv, int splits, const int64_t* __restrict__ positions,
                                       const float* __restrict__ cos_table, const float* __restrict__ sin_table,
                                       float* __restrict__ kc, float* __restrict__ vc, float* __restrict__ q,
                                       int64_t* __restrict__ lengths, int64_t cap, int B, unsigned* __restrict__ error) {
    grid_dependency_wait();

    constexpr int kPairs = (kQHeads + kKVHeads) * (kHeadDim / 2) + kKVHeads * kHeadDim;  // 384 + 192
    const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= static_cast<int64_t>(B) * kPairs) return;
    const int b = static_cast<int>(e / kPairs), t = static_cast<int>(e % kPairs);
    const int64_t pos = positions[b];
    if (pos < 0 || pos >= cap) {
        if (t == 0) atomicOr(error, 2u);
        return;
    }
    if (t == 0) lengths[b] = pos + 1;
    const size_t stride = static_cast<size_t>(B) * kQKV;
    auto value = [&](int n) { return split_sum(qkv, splits, stride, static_cast<size_t>(b) * kQKV + n); };
    if (t < (kQHeads + kKVHeads) * (kHeadDim / 2)) {
        const int head = t / (kHeadDim / 2), d = t % (kHeadDim / 2);  // heads 0..8 q, 9..11 k
        const float x1 = value(head * kHeadDim + d), x2 = value(head * kHeadDim + d + kHeadDim / 2);
        const float* c = cos_table + pos * kHeadDim;
        const float* s = sin_table + pos * kHeadDim;
        const float r1 = rope_value(x1, x2, c[d], s[d], true);
        const float r2 = rope_value(x2, x1, c[d + kHeadDim / 2], s[d + kHeadDim / 2], false);
        if (head < kQHeads) {
            q[(static_cast<size_t>(b) * kQHeads + head) * kHeadDim + d] = r1;
            q[(static_cast<size_t>(b) * kQHeads + head) * kHeadDim + d + kHeadDim / 2] = r2;
        } else {
            float* dst = kc + ((static_cast<size_t>(b) * kKVHeads + (head - kQHeads)) * cap + pos) * kHeadDim;
            dst[d] = r1;
            dst[d + kHeadDim / 2] = r2;
        }
    } else {
        const int u = t - (kQHeads + kKVHeads) * (kHeadDim / 2);
        vc[((static_cast<size_t>(b) * kKVHeads + u / kHeadDim) * cap + pos) * kHeadDim + u % kHeadDim] =
            value(kHidden + kKVHeads * kHeadDim + u);
    }
}

// One CTA per sequence: token = argmax(logits[b]) (NaN as max, lowest index
// on ties), generated[b][step] = token, position += 1; CTA 0 advances step
// (after every CTA read it: the step counter is read again only by the next
// launch).
__global__ void __launch_bounds__(1024) greedy_rows_kernel(const float* __restrict__ logits, int64_t vocab,
                                                           int64_t* __restrict__ tokens, int64_t* __restrict__ positions,
                                                           int64_t* __restrict__ generated, int64_t gen_cap,
                                                           const int64_t* __restrict__ step_in, int64_t* __restrict__ step_out) {
    grid_dependency_wait();

    __shared__ float sv[32];
    __shared__ long long si[32];
    const int b = blockIdx.x;
    const float* row = logits + static_cast<size_t>(b) * vocab;
    float bv = 0.0f;
    long long bi = -1;
    for (int64_t i = threadIdx.x; i < vocab; i += blockDim.x)
        if (argmax_precedes(row[i], i, bv, bi)) {
            bv = row[i];
            bi = i;
        }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float v = __shfl_xor_sync(0xffffffffu, bv, off);
        const long long i = __shfl_xor_sync(0xffffffffu, bi, off);
        if (argmax_precedes(v, i, bv, bi)) {
            bv = v;
            bi = i;
        }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
            if (argmax_precedes(sv[w], si[w], bv, bi)) {
                bv = sv[w];
                bi = si[w];
            }
        const int64_t token = bi < 0 ? 0 : bi;
        const int64_t st = *step_in;
        tokens[b] = token;
        positions[b] += 1;
        if (st >= 0 && st < gen_cap) generated[static_cast<size_t>(b) * gen_cap + st] = token;
    }
}

__global__ void advance_step_kernel(int64_t* step) {
    grid_dependency_wait();

    if (threadIdx.x == 0 && blockIdx.x == 0) *step += 1;
}

__global__ void set_sequence_kernel(int64_t* tokens, int64_t* positions, const int64_t* token, int64_t index,
                                    int64_t position, int64_t* step, int64_t* generated, int64_t gen_cap) {
    if (threadIdx.x == 0) {
        tokens[index] = *token;
        positions[index] = position;
        *step = 0;
    }
    for (int64_t i = threadIdx.x; i < gen_cap; i += blockDim.x) generated[index * gen_cap + i] = 0;
}

struct GemmPlan {
    int splits = 1, k_per_split = 0;
};

GemmPlan plan_gemm(int N, int K, int sms, bool tensor_cores) {
    // About one wave of CTAs; SIMT slices hold at least 64 columns of K,
    // tensor-core slices at least one 32-column stage.
    const int tile_n = tensor_cores ? kTcTileN : kTileN;
    const int min_k = tensor_cores ? kTcTileK : 64;
    const int tiles = (N + tile_n - 1) / tile_n;
    int splits = std::max(1, (sms + tiles - 1) / tiles);
    splits = std::min(splits, std::max(1, K / min_k));
    int kps = (K + splits - 1) / splits;
    const int round = tensor_cores ? kTcTileK : kTileK;
    kps = (kps + round - 1) / round * round;
    GemmPlan p;
    p.k_per_split = kps;
    p.splits = (K + kps - 1) / kps;
    return p;
}

}  // namespace
}  // namespace fx

using namespace fx;

// One lane: a contiguous range of the batch's sequences with its own
// activations, split-K partials and attention workspace.  With two lanes the
// halves of the batch run their layer chains on two streams inside the
// graph, so one half's latency-bound projections and reductions overlap the
// other half's HBM-bound attention; they join before the LM head.
struct BatchLane {
    int row0 = 0, rows = 0;
    float *h = nullptr, *h2 = nullptr, *qkv = nullptr, *q = nullptr;
    float *norm = nullptr, *attn = nullptr, *act = nullptr;  // 64 rows each (rows >= `rows` stay zero)
    float *partials = nullptr, *attn_ws = nullptr;
    CUtensorMap x_norm, x_attn, x_act;
    BatchLayerMaps layer_maps;  // the layer kernel's staging maps (layer-kernel step)
};

struct fx_batch {
    fx_model_desc model{};
    int64_t batch = 0, capacity = 0, gen_cap = 0, vocab = 0;
    int sms = 0;
    int64_t host_max_position = 0;  // host mirror of max(positions): refuses steps past capacity
    bool pending = false;
    cudaStream_t capture_stream = nullptr, lane_stream = nullptr;
    cudaEvent_t done = nullptr, fork = nullptr, join = nullptr;
    cudaGraphExec_t exec = nullptr;
    cudaGraph_t graph = nullptr;
    // owned device memory
    int64_t *tokens = nullptr, *positions = nullptr, *lengths = nullptr, *generated = nullptr, *step = nullptr;
    float *logits = nullptr, *key_cache = nullptr, *value_cache = nullptr;
    float *activations = nullptr, *partials = nullptr, *attn_ws = nullptr;
    float* norm_all = nullptr;  // the final norm of every row (LM head input), max(batch, 64) rows
    unsigned* error = nullptr;
    int lanes = 1;
    int priority_low = 0, priority_high = 0;  // the device's stream priority range
    BatchLane lane[2];
    GemmPlan qkv_plan, o_plan, gu_plan, down_plan, lm_plan;
    // Projections on tcgen05 tensor cores (3xTF32) unless FLUX_B200_BATCH_GEMM=simt.
    bool tensor_cores = true;
    // FLUX_B200_BATCH_STEP=layers: the work between attention launches as one
    // cooperative launch per layer (batch_layer.cu, SIMT FP32), 2 launches per
    // layer; by default the launch chain below (tcgen05 projections, two
    // lanes), which measured slightly faster (2.92-2.94 vs 2.95-2.98 ms per
    // 64-sequence step on one B200).
    bool layer_kernel = false;
    int layer_grid = 0;
    unsigned* barriers = nullptr;  // [kLayers + 1][4] grid-barrier counters, cleared at each step
    fx::TcModelWeights tc;
    CUtensorMap x_norm_all;
    size_t layer_stride() const { return static_cast<size_t>(batch) * kKVHeads * capacity * kHeadDim; }
    size_t sequence_stride() const { return static_cast<size_t>(kKVHeads) * capacity * kHeadDim; }
};

namespace fx {
namespace {

// A projection of M activation rows: split-K partials into `partials`, or
// straight into `direct_out` when there is one split.
fx_status gemm(fx_batch* r, int M, const float* x, const float* w, int N, int K, const GemmPlan& p, float* direct_out,
               float* partials, cudaStream_t s, const TcWeight* tw = nullptr, const CUtensorMap* xmap = nullptr) {
    float* out = p.splits == 1 && direct_out != nullptr ? direct_out : partials;
    if (r->tensor_cores) {
        TcGemmArgs a = tc_args(*tw, *xmap, out, nullptr, reinterpret_cast<int*>(r->error), M, p.k_per_split);
        // With two lanes, 3 pipeline stages (145 KB) let a projection CTA of
        // one lane share an SM with an attention chunk CTA of the other.
        return launch_tc_gemm(a, 64, p.splits, s, true, r->lanes > 1 ? 3 : 0);
    }
    const dim3 grid((N + kTileN - 1) / kTileN, p.splits);
    return launch_dependent(skinny_gemm_kernel, grid, dim3(kGemmThreads), 0, s, "launching a batched projection", x, w,
                            out, M, N, K, p.k_per_split);
}

fx_status reduce(int M, const GemmPlan& p, int N, const float* partials, const float* residual, float* out,
                 cudaStream_t s) {
    const int64_t n = static_cast<int64_t>(M) * N;
    return launch_dependent(reduce_splits_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, s,
                            "launching a split-K reduction", partials, p.splits, M, N, residual, out);
}

// Embedding and the 30 layers for the lane's sequences; the last layer's
// final norm goes to the lane's rows of norm_all.
fx_status run_lane(fx_batch* r, BatchLane& ln, cudaStream_t s) {
    const fx_model_desc& m = r->model;
    const int B = ln.rows;
    int64_t* tokens = r->tokens + ln.row0;
    int64_t* positions = r->positions + ln.row0;
    int64_t* lengths = r->lengths + ln.row0;
    fx_status st;
    if ((st = launch_dependent(embed_rows_kernel, dim3(B), dim3(kHidden), 0, s, "launching the embedding gather",
                               static_cast<const int64_t*>(tokens), m.embedding, r->vocab, ln.h, m.input_norm[0],
                               m.epsilon, ln.norm)) != FX_OK)
        return st;
    auto residual_norm = [&](const GemmPlan& p, const float* residual, float* h_out, const float* w, float* norm_out) {
        return launch_dependent(reduce_residual_norm_kernel, dim3(B), dim3(kHidden), 0, s,
                                "launching the split-K sum / residual / RMSNorm rows",
                                static_cast<const float*>(ln.partials), p.splits, B, residual, h_out, w, m.epsilon,
                                norm_out);
    };
    for (int l = 0; l < kLayers; ++l) {
        float* kc = r->key_cache + l * r->layer_stride() + ln.row0 * r->sequence_stride();
        float* vc = r->value_cache + l * r->layer_stride() + ln.row0 * r->sequence_stride();
        if ((st = gemm(r, B, ln.norm, m.packed_qkv[l], kQKV, kHidden, r->qkv_plan, ln.qkv, ln.partials, s, &r->tc.qkv[l],
                       &ln.x_norm)) != FX_OK)
            return st;
        {
            const int64_t n = static_cast<int64_t>(B) * ((kQHeads + kKVHeads) * (kHeadDim / 2) + kKVHeads * kHeadDim);
            const float* src = r->qkv_plan.splits > 1 ? ln.partials : ln.qkv;
            if ((st = launch_dependent(rope_cache_rows_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, s,
                                       "launching the batched QKV sum / RoPE / cache write", src, r->qkv_plan.splits,
                                       static_cast<const int64_t*>(positions), m.rope_cos, m.rope_sin, kc, vc, ln.q,
                                       lengths, r->capacity, B, r->error)) != FX_OK)
                return st;
        }
        CompactAttention a{};
        a.q = ln.q;
        a.k = kc;
        a.v = vc;
        a.lengths = lengths;
        a.length_stride = 1;
        a.out = ln.attn;
        a.ws = ln.attn_ws;
        a.error = r->error;
        a.scale = m.attention_scale[l];
        a.batch = B;
        a.cap = r->capacity;
        a.chunks = (r->capacity + kCompactChunk - 1) / kCompactChunk;
        a.chunk_rows = kCompactChunk;
        {
            // HBM-bound attention yields the SMs to the other lane's chain
            LaunchPriorityScope low(r->priority_low);
            if ((st = launch_compact_attention(a, s, true)) != FX_OK) return st;
        }
        if ((st = gemm(r, B, ln.attn, m.o_proj[l], kHidden, kHidden, r->o_plan, nullptr, ln.partials, s, &r->tc.o[l],
                       &ln.x_attn)) != FX_OK)
            return st;
        if ((st = residual_norm(r->o_plan, ln.h, ln.h2, m.post_norm[l], ln.norm)) != FX_OK) return st;
        if ((st = gemm(r, B, ln.norm, m.gate_up[l], kGateUp, kHidden, r->gu_plan, nullptr, ln.partials, s,
                       &r->tc.gate_up[l], &ln.x_norm)) != FX_OK)
            return st;
        {
            const int64_t n = static_cast<int64_t>(B) * kInter;
            if ((st = launch_dependent(reduce_swiglu_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, s,
                                       "launching the batched SwiGLU", static_cast<const float*>(ln.partials),
                                       r->gu_plan.splits, B, ln.act)) != FX_OK)
                return st;
        }
        if ((st = gemm(r, B, ln.act, m.down[l], kHidden, kInter, r->down_plan, nullptr, ln.partials, s, &r->tc.down[l],
                       &ln.x_act)) != FX_OK)
            return st;
        // h = h' + down, then the next layer's input norm (the final norm after the last layer)
        const bool last = l + 1 == kLayers;
        if ((st = residual_norm(r->down_plan, ln.h2, ln.h, last ? m.final_norm : m.input_norm[l + 1],
                                last ? r->norm_all + static_cast<size_t>(ln.row0) * kHidden : ln.norm)) != FX_OK)
            return st;
    }
    return FX_OK;
}

// The lane's 30 layers as (layer kernel, attention chunks, merge) x 30 +
// one layer kernel: the first launch embeds and projects layer 0's QKV,
// launch l + 1 takes layer l's attention output through o_proj .. down and
// layer l + 1's QKV (the last one: the final norm rows).
fx_status run_lane_layers(fx_batch* r, BatchLane& ln, cudaStream_t s) {
    const fx_model_desc& m = r->model;
    FX_CUDA_TRY(cudaMemsetAsync(r->barriers, 0, static_cast<size_t>(kLayers + 1) * 4 * sizeof(unsigned), s),
                "clearing the layer kernels' barriers");
    BatchLayerArgs a{};
    a.maps = ln.layer_maps;
    a.embedding = m.embedding;
    a.tokens = r->tokens + ln.row0;
    a.vocab = r->vocab;
    a.attn = ln.attn;
    a.h = ln.h;
    a.h2 = ln.h2;
    a.act = ln.act;
    a.q = ln.q;
    a.positions = r->positions + ln.row0;
    a.lengths = r->lengths + ln.row0;
    a.cap = r->capacity;
    a.rope_cos = m.rope_cos;
    a.rope_sin = m.rope_sin;
    a.norm_out = r->norm_all + static_cast<size_t>(ln.row0) * kHidden;
    a.error = r->error;
    a.eps = m.epsilon;
    a.rows = ln.rows;
    auto cache_of = [&](float* base, int l) { return base + l * r->layer_stride() + ln.row0 * r->sequence_stride(); };
    a.mode = kLayerFirst;
    a.next_norm = m.input_norm[0];
    a.next_qkv = m.packed_qkv[0];
    a.key_cache = cache_of(r->key_cache, 0);
    a.value_cache = cache_of(r->value_cache, 0);
    a.barrier = r->barriers;
    fx_status st = launch_batch_layer(a, r->layer_grid, s);
    if (st != FX_OK) return st;
    for (int l = 0; l < kLayers; ++l) {
        CompactAttention at{};
        at.q = ln.q;
        at.k = cache_of(r->key_cache, l);
        at.v = cache_of(r->value_cache, l);
        at.lengths = a.lengths;
        at.length_stride = 1;
        at.out = ln.attn;
        at.ws = ln.attn_ws;
        at.error = r->error;
        at.scale = m.attention_scale[l];
        at.batch = ln.rows;
        at.cap = r->capacity;
        at.chunks = (r->capacity + kCompactChunk - 1) / kCompactChunk;
        at.chunk_rows = kCompactChunk;
        if ((st = launch_compact_attention(at, s, true, false)) != FX_OK) return st;  // the layer kernel merges
        const bool last = l + 1 == kLayers;
        a.attn_ws = ln.attn_ws;
        a.attn_chunks = at.chunks;
        a.attn_rows = at.chunk_rows;
        a.mode = last ? kLayerLast : kLayerMiddle;
        a.o_proj = m.o_proj[l];
        a.post_norm = m.post_norm[l];
        a.gate_up = m.gate_up[l];
        a.down = m.down[l];
        a.next_norm = last ? m.final_norm : m.input_norm[l + 1];
        a.next_qkv = last ? nullptr : m.packed_qkv[l + 1];
        a.key_cache = last ? nullptr : cache_of(r->key_cache, l + 1);
        a.value_cache = last ? nullptr : cache_of(r->value_cache, l + 1);
        a.barrier = r->barriers + 4 * (l + 1);
        if ((st = launch_batch_layer(a, r->layer_grid, s)) != FX_OK) return st;
    }
    return FX_OK;
}

fx_status run_step(fx_batch* r, cudaStream_t s) {
    const fx_model_desc& m = r->model;
    const int B = static_cast<int>(r->batch);
    fx_status st;
    if (r->layer_kernel) {
        if ((st = run_lane_layers(r, r->lane[0], s)) != FX_OK) return st;
    } else if (r->lanes > 1) {
        // the latency-bound projections and reductions run at high priority,
        // the attention chunks at low (node priorities of the graph)
        LaunchPriorityScope high(r->priority_high);
        FX_CUDA_TRY(cudaEventRecord(r->fork, s), "forking the batched lanes");
        FX_CUDA_TRY(cudaStreamWaitEvent(r->lane_stream, r->fork, 0), "forking the batched lanes");
        if ((st = run_lane(r, r->lane[1], r->lane_stream)) != FX_OK) return st;
        if ((st = run_lane(r, r->lane[0], s)) != FX_OK) return st;
        FX_CUDA_TRY(cudaEventRecord(r->join, r->lane_stream), "joining the batched lanes");
        FX_CUDA_TRY(cudaStreamWaitEvent(s, r->join, 0), "joining the batched lanes");
    } else if ((st = run_lane(r, r->lane[0], s)) != FX_OK) {
        return st;
    }
    if ((st = gemm(r, B, r->norm_all, m.lm_head, static_cast<int>(r->vocab), kHidden, r->lm_plan, r->logits,
                   r->partials, s, &r->tc.lm_head, &r->x_norm_all)) != FX_OK)
        return st;
    if (r->lm_plan.splits > 1 &&
        (st = reduce(B, r->lm_plan, static_cast<int>(r->vocab), r->partials, nullptr, r->logits, s)) != FX_OK)
        return st;
    if ((st = launch_dependent(greedy_rows_kernel, dim3(B), dim3(1024), 0, s, "launching the batched greedy update",
                               static_cast<const float*>(r->logits), r->vocab, r->tokens, r->positions, r->generated,
                               r->gen_cap, static_cast<const int64_t*>(r->step), r->step)) != FX_OK)
        return st;
    return launch_dependent(advance_step_kernel, dim3(1), dim3(32), 0, s, "advancing the batched step", r->step);
}

struct DeviceScope {
    int previous = -1;
    explicit DeviceScope(int device) {
        cudaGetDevice(&previous);
        if (previous != device) cudaSetDevice(device);
    }
    ~DeviceScope() {
        int current = -1;
        cudaGetDevice(&current);
        if (previous >= 0 && current != previous) cudaSetDevice(previous);
    }
};

void destroy_batch(fx_batch* r) {
    if (r == nullptr) return;
    if (r->exec) cudaGraphExecDestroy(r->exec);
    if (r->graph) cudaGraphDestroy(r->graph);
    for (cudaEvent_t e : {r->done, r->fork, r->join})
        if (e) cudaEventDestroy(e);
    if (r->capture_stream) cudaStreamDestroy(r->capture_stream);
    if (r->lane_stream) cudaStreamDestroy(r->lane_stream);
    for (void* p : {static_cast<void*>(r->tokens), static_cast<void*>(r->logits), static_cast<void*>(r->key_cache),
                    static_cast<void*>(r->value_cache), static_cast<void*>(r->activations),
                    static_cast<void*>(r->partials), static_cast<void*>(r->attn_ws), static_cast<void*>(r->barriers)})
        cudaFree(p);
    tc_weights_release(&r->tc);
    delete r;
}

fx_status create_batch(fx_batch* r, cudaStream_t stream) {
    FX_CUDA_TRY(cudaDeviceGetAttribute(&r->sms, cudaDevAttrMultiProcessorCount, r->model.device), "querying SM count");
    FX_CUDA_TRY(cudaDeviceGetStreamPriorityRange(&r->priority_low, &r->priority_high), "querying stream priorities");
    const int64_t B = r->batch;
    // state: tokens, positions, lengths, step, generated (one allocation)
    const size_t state_words = 3 * B + 1 + B * r->gen_cap;
    FX_CUDA_TRY(cudaMalloc(&r->tokens, state_words * sizeof(int64_t) + 256), "allocating batched state");
    r->positions = r->tokens + B;
    r->lengths = r->positions + B;
    r->step = r->lengths + B;
    r->generated = r->step + 1;
    r->error = reinterpret_cast<unsigned*>(r->generated + B * r->gen_cap);
    FX_CUDA_TRY(cudaMalloc(&r->logits, static_cast<size_t>(B) * r->vocab * sizeof(float)), "allocating batched logits");
    const size_t cache = static_cast<size_t>(kLayers) * r->layer_stride() * sizeof(float);
    FX_CUDA_TRY(cudaMalloc(&r->key_cache, cache), "allocating the batched K cache");
    FX_CUDA_TRY(cudaMalloc(&r->value_cache, cache), "allocating the batched V cache");
    const char* mode = std::getenv("FLUX_B200_BATCH_GEMM");
    r->tensor_cores = !(mode != nullptr && std::strcmp(mode, "simt") == 0);
    // Lanes (FLUX_B200_BATCH_LANES=1 runs the whole batch as one chain).  The
    // split-K plans depend only on the configured lane count, never on the
    // batch size, so a sequence's result is the same in any batch.
    const char* step_env = std::getenv("FLUX_B200_BATCH_STEP");
    r->layer_kernel = step_env != nullptr && std::strcmp(step_env, "layers") == 0;
    if (r->layer_kernel) {
        fx_status prep = prepare_batch_layer(&r->layer_grid);
        if (prep != FX_OK) return prep;
        FX_CUDA_TRY(cudaMalloc(&r->barriers, static_cast<size_t>(kLayers + 1) * 4 * sizeof(unsigned)),
                    "allocating the layer kernels' barriers");
    }
    const char* lanes_env = std::getenv("FLUX_B200_BATCH_LANES");
    const int lanes_cfg = r->layer_kernel || (lanes_env != nullptr && std::strcmp(lanes_env, "1") == 0) ? 1 : 2;
    r->lanes = static_cast<int>(std::min<int64_t>(lanes_cfg, B));
    r->lane[0].row0 = 0;
    r->lane[0].rows = static_cast<int>((B + r->lanes - 1) / r->lanes);
    r->lane[1].row0 = r->lane[0].rows;
    r->lane[1].rows = static_cast<int>(B - r->lane[0].rows);
    const bool tc = r->tensor_cores;
    const int plan_sms = std::max(1, r->sms / lanes_cfg);
    r->qkv_plan = plan_gemm(kQKV, kHidden, plan_sms, tc);
    r->o_plan = plan_gemm(kHidden, kHidden, plan_sms, tc);
    r->gu_plan = plan_gemm(kGateUp, kHidden, plan_sms, tc);
    r->down_plan = plan_gemm(kHidden, kInter, plan_sms, tc);
    r->lm_plan = plan_gemm(static_cast<int>(r->vocab), kHidden, r->sms, tc);
    // Activations per lane; the projection inputs (norm, attn, act) hold 64
    // rows so the tensor-core tiles never read past them (rows past the
    // lane's stay zero).  Then norm_all, max(batch, 64) rows.
    const int64_t R = std::max<int64_t>(B, 64);
    auto lane_act = [](int64_t rows) {
        return static_cast<size_t>(rows) * (3 * kHidden + kQKV) + static_cast<size_t>(64) * (2 * kHidden + kInter);
    };
    size_t act_floats = static_cast<size_t>(R) * kHidden;
    for (int i = 0; i < r->lanes; ++i) act_floats += lane_act(r->lane[i].rows);
    FX_CUDA_TRY(cudaMalloc(&r->activations, act_floats * sizeof(float)), "allocating batched activations");
    FX_CUDA_TRY(cudaMemsetAsync(r->activations, 0, act_floats * sizeof(float), stream), "clearing batched activations");
    // split-K partials per lane (gate/up always reduces through them: SwiGLU
    // epilogue); the LM head's, if split, reuse the whole buffer after the join
    auto lane_partials = [&](int64_t rows) {
        size_t n = 0;
        for (const auto& p : {std::pair<const GemmPlan*, int>{&r->qkv_plan, kQKV}, {&r->o_plan, kHidden},
                              {&r->gu_plan, kGateUp}, {&r->down_plan, kHidden}})
            if (p.first->splits > 1 || p.second == kGateUp)
                n = std::max(n, static_cast<size_t>(p.first->splits) * rows * p.second);
        return (n + 63) / 64 * 64;
    };
    size_t partial_floats = 0;
    for (int i = 0; i < r->lanes; ++i) partial_floats += lane_partials(r->lane[i].rows);
    if (r->lm_plan.splits > 1)
        partial_floats = std::max(partial_floats, static_cast<size_t>(r->lm_plan.splits) * B * r->vocab);
    FX_CUDA_TRY(cudaMalloc(&r->partials, partial_floats * sizeof(float)), "allocating split-K partials");
    // attention partials per lane (the merge runs as its own kernel: with
    // thousands of chunk CTAs per layer the in-kernel last-CTA merge measured
    // slower, 3.34 vs 3.12 ms per step)
    auto lane_ws = [&](int64_t rows) {
        return static_cast<size_t>((compact_attention_workspace(rows, r->capacity) + 63) / 64 * 64);
    };
    size_t attn_floats = 0;
    for (int i = 0; i < r->lanes; ++i) attn_floats += lane_ws(r->lane[i].rows);
    FX_CUDA_TRY(cudaMalloc(&r->attn_ws, attn_floats * sizeof(float)), "allocating the attention workspace");
    FX_CUDA_TRY(cudaMemsetAsync(r->attn_ws, 0, attn_floats * sizeof(float), stream), "clearing the attention workspace");
    r->norm_all = r->activations;
    float* act = r->activations + static_cast<size_t>(R) * kHidden;
    float* part = r->partials;
    float* ws = r->attn_ws;
    for (int i = 0; i < r->lanes; ++i) {
        BatchLane& ln = r->lane[i];
        const int64_t n = ln.rows;
        ln.h = act;
        ln.h2 = ln.h + n * kHidden;
        ln.qkv = ln.h2 + n * kHidden;
        ln.q = ln.qkv + n * kQKV;
        ln.norm = ln.q + n * kHidden;
        ln.attn = ln.norm + 64 * kHidden;
        ln.act = ln.attn + 64 * kHidden;
        act += lane_act(n);
        ln.partials = part;
        part += lane_partials(n);
        ln.attn_ws = ws;
        ws += lane_ws(n);
    }
    if (r->layer_kernel) {
        BatchLane& ln = r->lane[0];
        fx_status st0;
        if ((st0 = tc_encode_map(&ln.layer_maps.attn, ln.attn, 64, kHidden, 64, "the batched attention rows")) != FX_OK ||
            (st0 = tc_encode_map(&ln.layer_maps.h2, ln.h2, ln.rows, kHidden, 64, "the batched residual rows")) != FX_OK ||
            (st0 = tc_encode_map(&ln.layer_maps.act, ln.act, 64, kInter, 64, "the batched SwiGLU rows")) != FX_OK ||
            (st0 = tc_encode_map(&ln.layer_maps.h, ln.h, ln.rows, kHidden, 64, "the batched residual rows")) != FX_OK)
            return st0;
    }
    if (tc) {
        fx_status st0 = tc_weights_create(r->model, true, &r->tc, stream, !r->layer_kernel);
        if (st0 != FX_OK) return st0;
        if ((st0 = tc_encode_map(&r->x_norm_all, r->norm_all, R, kHidden, 64, "the batched final-norm rows")) != FX_OK)
            return st0;
        for (int i = 0; i < r->lanes; ++i) {
            BatchLane& ln = r->lane[i];
            if ((st0 = tc_encode_map(&ln.x_norm, ln.norm, 64, kHidden, 64, "the batched norm rows")) != FX_OK) return st0;
            if ((st0 = tc_encode_map(&ln.x_attn, ln.attn, 64, kHidden, 64, "the batched attention rows")) != FX_OK)
                return st0;
            if ((st0 = tc_encode_map(&ln.x_act, ln.act, 64, kInter, 64, "the batched SwiGLU rows")) != FX_OK) return st0;
        }
    }
    FX_CUDA_TRY(cudaMemsetAsync(r->tokens, 0, state_words * sizeof(int64_t) + 256, stream), "clearing batched state");
    FX_CUDA_TRY(cudaMemsetAsync(r->key_cache, 0, cache, stream), "clearing the batched K cache");
    FX_CUDA_TRY(cudaMemsetAsync(r->value_cache, 0, cache, stream), "clearing the batched V cache");
    FX_CUDA_TRY(cudaMemsetAsync(r->logits, 0, static_cast<size_t>(B) * r->vocab * sizeof(float), stream),
                "clearing batched logits");
    FX_CUDA_TRY(cudaStreamCreateWithFlags(&r->capture_stream, cudaStreamNonBlocking), "creating the capture stream");
    FX_CUDA_TRY(cudaStreamCreateWithFlags(&r->lane_stream, cudaStreamNonBlocking), "creating the lane stream");
    FX_CUDA_TRY(cudaEventCreateWithFlags(&r->done, cudaEventDisableTiming), "creating the completion event");
    FX_CUDA_TRY(cudaEventCreateWithFlags(&r->fork, cudaEventDisableTiming), "creating the lane fork event");
    FX_CUDA_TRY(cudaEventCreateWithFlags(&r->join, cudaEventDisableTiming), "creating the lane join event");
    FX_CUDA_TRY(cudaStreamSynchronize(stream), "initialising the batched runtime");
    // Load every kernel once outside capture (function attributes, modules),
    // then restore the cleared state and capture one step.
    fx_status st = run_step(r, r->capture_stream);
    if (st != FX_OK) return st;
    FX_CUDA_TRY(cudaStreamSynchronize(r->capture_stream), "warming the batched step");
    FX_CUDA_TRY(cudaMemsetAsync(r->tokens, 0, state_words * sizeof(int64_t) + 256, r->capture_stream),
                "clearing batched state");
    FX_CUDA_TRY(cudaMemsetAsync(r->key_cache, 0, cache, r->capture_stream), "clearing the batched K cache");
    FX_CUDA_TRY(cudaMemsetAsync(r->value_cache, 0, cache, r->capture_stream), "clearing the batched V cache");
    FX_CUDA_TRY(cudaStreamBeginCapture(r->capture_stream, cudaStreamCaptureModeThreadLocal), "beginning capture");
    st = run_step(r, r->capture_stream);
    cudaGraph_t graph = nullptr;
    const cudaError_t end = cudaStreamEndCapture(r->capture_stream, &graph);
    if (st != FX_OK) {
        if (graph) cudaGraphDestroy(graph);
        return st;
    }
    FX_CUDA_TRY(end, "ending capture");
    r->graph = graph;
    FX_CUDA_TRY(cudaGraphInstantiate(&r->exec, r->graph, cudaGraphInstantiateFlagUseNodePriority),
                "instantiating the batched graph");
    FX_CUDA_TRY(cudaStreamSynchronize(r->capture_stream), "finalising the batched runtime");
    return FX_OK;
}

}  // namespace
}  // namespace fx

extern "C" fx_status fx_batch_create(const fx_model_desc* model, int64_t batch, int64_t generated_capacity,
                                     void* stream, fx_batch** out) {
    FX_REQUIRE(out != nullptr, "fx_batch_create: output pointer is null");
    *out = nullptr;
    FX_REQUIRE(model != nullptr, "flux batched decode: model description is null");
    FX_REQUIRE(batch >= 1 && batch <= kMaxBatch, "flux batched decode: batch must be in [1, 64]");
    FX_REQUIRE(model->vocab > 0 && model->vocab <= 0x7fffffff, "flux batched decode: vocabulary size out of range");
    FX_REQUIRE(model->capacity >= 1 && model->capacity <= kMaxCapacity,
               "flux batched decode: cache capacity must be in [1, 131072]");
    FX_REQUIRE(generated_capacity >= 1 && generated_capacity <= kMaxCapacity,
               "flux batched decode: generated capacity must be in [1, 131072]");
    FX_REQUIRE(std::isfinite(model->epsilon) && model->epsilon > 0.0f, "flux batched decode: epsilon must be positive");
    FX_REQUIRE(model->embedding && model->final_norm && model->lm_head && model->rope_cos && model->rope_sin,
               "flux batched decode: a model tensor pointer is null");
    for (int l = 0; l < kLayers; ++l) {
        FX_REQUIRE(model->input_norm[l] && model->packed_qkv[l] && model->o_proj[l] && model->post_norm[l] &&
                       model->gate_up[l] && model->down[l],
                   "flux batched decode: exactly 30 complete layer descriptors are required");
        for (const void* p : {static_cast<const void*>(model->packed_qkv[l]), static_cast<const void*>(model->o_proj[l]),
                              static_cast<const void*>(model->gate_up[l]), static_cast<const void*>(model->down[l])})
            FX_REQUIRE(reinterpret_cast<uintptr_t>(p) % 16 == 0, "flux batched decode: weights must be 16-byte aligned");
    }
    FX_REQUIRE(reinterpret_cast<uintptr_t>(model->lm_head) % 16 == 0,
               "flux batched decode: LM head must be 16-byte aligned");
    FX_REQUIRE(reinterpret_cast<uintptr_t>(model->embedding) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(model->final_norm) % 16 == 0,
               "flux batched decode: embedding and norm weights must be 16-byte aligned");
    for (int l = 0; l < kLayers; ++l)
        FX_REQUIRE(reinterpret_cast<uintptr_t>(model->input_norm[l]) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(model->post_norm[l]) % 16 == 0,
                   "flux batched decode: embedding and norm weights must be 16-byte aligned");
    DeviceScope scope(model->device);
    fx_batch* r = new fx_batch();
    r->model = *model;
    r->batch = batch;
    r->capacity = model->capacity;
    r->gen_cap = generated_capacity;
    r->vocab = model->vocab;
    const fx_status st = create_batch(r, as_stream(stream));
    if (st != FX_OK) {
        destroy_batch(r);
        return st;
    }
    *out = r;
    return FX_OK;
}

extern "C" fx_status fx_batch_load(fx_batch* r, int64_t sequence, const int64_t* token,
                                   const float* const* key_layers, const float* const* value_layers,
                                   int64_t source_rows, int64_t length, void* stream) {
    FX_REQUIRE(r != nullptr && token != nullptr, "fx_batch_load: null pointer");
    FX_REQUIRE(sequence >= 0 && sequence < r->batch, "flux batched decode: sequence index out of range");
    FX_REQUIRE(length >= 0 && length < r->capacity, "flux batched decode: length must be within cache capacity");
    FX_REQUIRE(length == 0 || (key_layers != nullptr && value_layers != nullptr && source_rows >= length),
               "flux batched decode: K/V sources must hold `length` rows");
    DeviceScope scope(r->model.device);
    cudaStream_t s = as_stream(stream);
    if (r->pending) FX_CUDA_TRY(cudaStreamWaitEvent(s, r->done, 0), "ordering after batched work");
    const size_t dpitch = static_cast<size_t>(r->capacity) * kHeadDim * sizeof(float);
    for (int l = 0; l < kLayers; ++l) {
        float* kd = r->key_cache + l * r->layer_stride() + static_cast<size_t>(sequence) * kKVHeads * r->capacity * kHeadDim;
        float* vd = r->value_cache + l * r->layer_stride() + static_cast<size_t>(sequence) * kKVHeads * r->capacity * kHeadDim;
        FX_CUDA_TRY(cudaMemsetAsync(kd, 0, kKVHeads * dpitch, s), "clearing a sequence's K cache");
        FX_CUDA_TRY(cudaMemsetAsync(vd, 0, kKVHeads * dpitch, s), "clearing a sequence's V cache");
        if (length > 0) {
            FX_REQUIRE(key_layers[l] != nullptr && value_layers[l] != nullptr,
                       "flux batched decode: one K/V tensor per layer is required");
            const size_t spitch = static_cast<size_t>(source_rows) * kHeadDim * sizeof(float);
            const size_t width = static_cast<size_t>(length) * kHeadDim * sizeof(float);
            FX_CUDA_TRY(cudaMemcpy2DAsync(kd, dpitch, key_layers[l], spitch, width, kKVHeads, cudaMemcpyDeviceToDevice, s),
                        "importing a sequence's K cache");
            FX_CUDA_TRY(cudaMemcpy2DAsync(vd, dpitch, value_layers[l], spitch, width, kKVHeads, cudaMemcpyDeviceToDevice, s),
                        "importing a sequence's V cache");
        }
    }
    set_sequence_kernel<<<1, 256, 0, s>>>(r->tokens, r->positions, token, sequence, length, r->step, r->generated,
                                          r->gen_cap);
    FX_CUDA_TRY(cudaGetLastError(), "installing a sequence");
    FX_CUDA_TRY(cudaEventRecord(r->done, s), "recording the load");
    r->pending = true;
    r->host_max_position = std::max(r->host_max_position, length);
    return FX_OK;
}

extern "C" fx_status fx_batch_step(fx_batch* r, int64_t steps, void* stream) {
    FX_REQUIRE(r != nullptr, "fx_batch_step: runtime is null");
    FX_REQUIRE(steps >= 0, "fx_batch_step: steps must be non-negative");
    if (r->host_max_position + steps > r->capacity) {
        set_error("flux batched decode: cache capacity exhausted");
        return FX_ERR_EXHAUSTED;
    }
    DeviceScope scope(r->model.device);
    cudaStream_t s = as_stream(stream);
    if (r->pending) FX_CUDA_TRY(cudaStreamWaitEvent(s, r->done, 0), "ordering after batched work");
    for (int64_t i = 0; i < steps; ++i) FX_CUDA_TRY(cudaGraphLaunch(r->exec, s), "launching the batched step");
    FX_CUDA_TRY(cudaEventRecord(r->done, s), "recording the batched step");
    r->pending = true;
    r->host_max_position += steps;
    return FX_OK;
}

extern "C" fx_status fx_batch_wait(fx_batch* r, void* stream) {
    FX_REQUIRE(r != nullptr, "fx_batch_wait: runtime is null");
    DeviceScope scope(r->model.device);
    if (r->pending) FX_CUDA_TRY(cudaStreamWaitEvent(as_stream(stream), r->done, 0), "ordering after batched work");
    return FX_OK;
}

extern "C" fx_status fx_batch_check(fx_batch* r) {
    FX_REQUIRE(r != nullptr, "fx_batch_check: runtime is null");
    DeviceScope scope(r->model.device);
    if (r->pending) FX_CUDA_TRY(cudaEventSynchronize(r->done), "waiting for batched work");
    unsigned error = 0;
    FX_CUDA_TRY(cudaMemcpy(&error, r->error, sizeof(error), cudaMemcpyDeviceToHost), "reading the batched error word");
    if (error & 2u) {
        set_error("flux batched decode: a sequence position is outside the cache capacity");
        return FX_ERR_DEVICE;
    }
    if (error & 1u) {
        set_error("flux batched decode: a bounded wait in the attention kernel gave up");
        return FX_ERR_DEVICE;
    }
    if (error & 256u) {
        set_error("flux batched decode: a bounded wait in a tensor-core projection gave up");
        return FX_ERR_DEVICE;
    }
    if (error & 16u) {
        set_error("flux batched decode: a bounded wait in the layer kernel gave up");
        return FX_ERR_DEVICE;
    }
    return FX_OK;
}

extern "C" fx_status fx_batch_get_buffers(const fx_batch* r, fx_batch_buffers* out) {
    FX_REQUIRE(r != nullptr && out != nullptr, "fx_batch_get_buffers: null pointer");
    out->tokens = r->tokens;
    out->positions = r->positions;
    out->logits = r->logits;
    out->generated = r->generated;
    out->step = r->step;
    out->key_cache = r->key_cache;
    out->value_cache = r->value_cache;
    out->batch = r->batch;
    out->capacity = r->capacity;
    out->generated_capacity = r->gen_cap;
    out->kernels_per_step = (r->layer_kernel ? 1 + kLayers * 2 : r->lanes * (1 + kLayers * 10)) + 3 +
                            (r->lm_plan.splits > 1 ? 1 : 0);
    return FX_OK;
}

extern "C" void fx_batch_destroy(fx_batch* r) {
    if (r == nullptr) return;
    DeviceScope scope(r->model.device);
    if (r->pending && r->done != nullptr) cudaEventSynchronize(r->done);
    destroy_batch(r);
}
