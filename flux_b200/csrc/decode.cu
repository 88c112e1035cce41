// Batch-1 SmolLM2-135M decode step on sm_100a and the runtime that replays it.
//
// The reference step (csrc/native_decode_runtime/native_decode_runtime_cuda.cu:
// 1042-1098) launches 304 kernels: a prepare kernel, per layer rmsnorm ->
// cuBLASLt QKV -> RoPE/cache -> GQA chunk + reduce -> cuBLASLt o_proj ->
// residual rmsnorm -> gate/up SwiGLU -> SGEMM down -> SGEAM add, then a final
// rmsnorm, an SGEMM LM head and a single-CTA argmax.  Here every projection
// is an HBM-streaming GEMV fused with its neighbours so one layer is five
// kernels and the step 151:
//
//   qkv_rope   input RMSNorm (recomputed per CTA) + packed QKV GEMV + RoPE on
//              q/k (separately rounded products) + K/V cache write at
//              *position; layer 0 also gathers the embedding row and sets
//              cache_length = position + 1.
//   attention  split-K over the valid rows: one CTA per (kv head, chunk)
//              serves the three q heads of that kv head (K/V read once), the
//              last CTA of each kv head merges the partials.
//   o_proj     o_proj GEMV + residual add.
//   gate_up    post-attention RMSNorm (recomputed per CTA) + gate/up GEMV +
//              SwiGLU.
//   down       down GEMV + residual add.
//   lm_head    final RMSNorm + tied LM-head GEMV + per-CTA greedy candidate;
//              the last CTA reduces the candidates and advances the device
//              state (token, generated[step], step, position).
//
// Weights are streamed with 128-bit read-only loads issued before any
// dependent arithmetic; each GEMV row is owned by a half warp (576 columns =
// 16 lanes x 9 float4) so one warp covers a RoPE pair (d, d + 32) and the
// rotation happens in registers.
#include "common.cuh"
#include "step_kernel.cuh"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>
#include <vector>

namespace fx {
namespace {

constexpr int kRow4 = kHidden / 4;          // float4 per 576-wide row (144)
constexpr int kRowPerLane = kRow4 / 16;     // float4 per lane of a half warp (9)
constexpr int kPartialStride = 68;          // m, l, pad, pad, o[64]
constexpr int kLmRowsPerCta = 16;           // 8 warps x 2 half warps
constexpr int kMaxCapacity = 131072;

// ----------------------------------------------------------------- kernels

struct QkvArgs {
    const float* x;          // layer input (unused for layer 0)
    const int64_t* token;    // layer 0: embedding row index, else nullptr
    const float* embedding;
    int64_t vocab;
    float* embedding_out;    // layer 0: hidden buffer that receives E[token]
    const float* norm_w;
    const float* w;          // [960, 576]
    float eps;
    const float* cos_table;
    const float* sin_table;
    const int64_t* position;
    int64_t* length_out;     // layer 0: receives position + 1
    int64_t capacity;
    float* key_cache;        // this layer's [3, capacity, 64]
    float* value_cache;
    float* q_out;            // [9 * 64]
    int* error;
};

// Dot product of one 576-wide weight row (global) with xn (shared), computed
// by a half warp; every lane of the half warp returns the sum.
__device__ __forceinline__ float half_warp_row_dot(const float* __restrict__ row, const float4* xn, int l16) {
    const float4* r4 = reinterpret_cast<const float4*>(row);
    float4 w[kRowPerLane];
#pragma unroll
    for (int j = 0; j < kRowPerLane; ++j) w[j] = __ldg(r4 + l16 + 16 * j);
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < kRowPerLane; ++j) {
        const float4 x = xn[l16 + 16 * j];
        acc = fmaf(w[j].x, x.x, acc);
        acc = fmaf(w[j].y, x.y, acc);
        acc = fmaf(w[j].z, x.z, acc);
        acc = fmaf(w[j].w, x.w, acc);
    }
    return group_sum<16>(acc);
}

// RMSNorm of a 576-vector into shared memory: xn = x * rsqrt(mean(x^2)+eps) * w.
// `src` may be nullptr with `embedding_row` set (layer-0 gather).
__device__ __forceinline__ void norm_to_shared(const float* __restrict__ src, const float* __restrict__ w,
                                               float eps, float* xn, float* scratch, float* copy_out) {
    float ss = 0.0f;
    for (int i = threadIdx.x; i < kHidden; i += blockDim.x) {
        const float v = src != nullptr ? src[i] : 0.0f;
        xn[i] = v;
        if (copy_out != nullptr) copy_out[i] = v;
        ss += v * v;
    }
    ss = block_sum(ss, scratch);
    const float inv = rsqrtf(ss / static_cast<float>(kHidden) + eps);
    for (int i = threadIdx.x; i < kHidden; i += blockDim.x) xn[i] = xn[i] * inv * w[i];
    __syncthreads();
}

// grid 120 x 128 threads: 480 warp tasks = 288 q RoPE pairs + 96 k RoPE pairs
// + 96 v row pairs.
__global__ void __launch_bounds__(128) qkv_rope_kernel(QkvArgs a) {
    __shared__ __align__(16) float xn[kHidden];
    __shared__ float scratch[32];
    const int64_t pos = *a.position;
    const float* src = a.x;
    if (a.token != nullptr) {
        const int64_t tok = *a.token;
        src = (tok >= 0 && tok < a.vocab) ? a.embedding + tok * kHidden : nullptr;
    }
    norm_to_shared(src, a.norm_w, a.eps, xn, scratch, blockIdx.x == 0 ? a.embedding_out : nullptr);
    if (blockIdx.x == 0 && threadIdx.x == 0 && a.length_out != nullptr) *a.length_out = pos + 1;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int half = lane >> 4, l16 = lane & 15;
    const int task = blockIdx.x * 4 + warp;
    int row_a, kind;  // kind 0 = q pair, 1 = k pair, 2 = v pair
    if (task < 288) {
        row_a = (task >> 5) * kHeadDim + (task & 31);
        kind = 0;
    } else if (task < 384) {
        const int t = task - 288;
        row_a = kHidden + (t >> 5) * kHeadDim + (t & 31);
        kind = 1;
    } else {
        row_a = kHidden + kKVHeads * kHeadDim + 2 * (task - 384);
        kind = 2;
    }
    const int row_b = kind == 2 ? row_a + 1 : row_a + kHeadDim / 2;
    const float y = half_warp_row_dot(a.w + static_cast<int64_t>(half ? row_b : row_a) * kHidden,
                                      reinterpret_cast<const float4*>(xn), l16);
    const float ya = __shfl_sync(0xffffffffu, y, 0);
    const float yb = __shfl_sync(0xffffffffu, y, 16);
    if (l16 != 0) return;
    if (pos < 0 || pos >= a.capacity) {
        if (lane == 0) atomicOr(a.error, 1);
        return;
    }
    const int row = half ? row_b : row_a;
    if (kind == 2) {
        const int u = row - kHidden - kKVHeads * kHeadDim;
        a.value_cache[(static_cast<int64_t>(u / kHeadDim) * a.capacity + pos) * kHeadDim + u % kHeadDim] = y;
        return;
    }
    const int d = row % kHeadDim;  // row_a has d < 32, row_b has d + 32
    const float c = a.cos_table[pos * kHeadDim + d];
    const float s = a.sin_table[pos * kHeadDim + d];
    const float r = half ? rope_value(yb, ya, c, s, false) : rope_value(ya, yb, c, s, true);
    if (kind == 0) {
        a.q_out[row] = r;
    } else {
        const int h = (row - kHidden) / kHeadDim;
        a.key_cache[(static_cast<int64_t>(h) * a.capacity + pos) * kHeadDim + d] = r;
    }
}

struct AttnArgs {
    const float* q;          // [9 * 64]
    const float* key_cache;  // this layer's [3, capacity, 64]
    const float* value_cache;
    const int64_t* length;   // valid rows (position + 1)
    int64_t capacity;
    float scale;
    float* partials;         // [3 kv][3 q][nch][kPartialStride]
    unsigned* counters;      // [3]
    float* out;              // [9 * 64]
    int nch;                 // chunks per kv head (grid = 3 * nch)
    int chunk_max;           // rows of score storage per CTA
};

// One CTA per (kv head g, chunk c).  Rows are split in 32-row multiples;
// an 8-lane group owns a row: lane l8 holds dims [4 l8, 4 l8 + 4) and
// [32 + 4 l8, 36 + 4 l8) so a warp's 4 rows are 1 KB of coalesced loads.
__global__ void __launch_bounds__(256) attention_kernel(AttnArgs a) {
    extern __shared__ float scores[];  // [3][chunk_max]
    __shared__ float red[8][kGroup][kHeadDim];
    __shared__ float stats[2][kGroup];
    __shared__ float scratch[32];
    __shared__ int is_last;
    const int g = blockIdx.x / a.nch, c = blockIdx.x % a.nch;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int l8 = lane & 7, grp = warp * 4 + (lane >> 3);  // 32 row groups
    const int64_t len = max(static_cast<int64_t>(1), min(*a.length, a.capacity));
    int64_t chunk = (len + a.nch - 1) / a.nch;
    chunk = ((chunk + 31) / 32) * 32;
    const int active = static_cast<int>((len + chunk - 1) / chunk);
    if (c < active) {
        const int64_t s0 = c * chunk;
        const int n = static_cast<int>(min(chunk, len - s0));
        float4 q0[kGroup], q1[kGroup];
#pragma unroll
        for (int h = 0; h < kGroup; ++h) {
            const float4* qh = reinterpret_cast<const float4*>(a.q + (g * kGroup + h) * kHeadDim);
            q0[h] = qh[l8];
            q1[h] = qh[8 + l8];
        }
        const float* kb = a.key_cache + (static_cast<int64_t>(g) * a.capacity + s0) * kHeadDim;
        for (int p = grp; p < n; p += 32) {
            const float4* kr = reinterpret_cast<const float4*>(kb + static_cast<int64_t>(p) * kHeadDim);
            const float4 k0 = __ldg(kr + l8), k1 = __ldg(kr + 8 + l8);
#pragma unroll
            for (int h = 0; h < kGroup; ++h) {
                float d = q0[h].x * k0.x;
                d = fmaf(q0[h].y, k0.y, d);
                d = fmaf(q0[h].z, k0.z, d);
                d = fmaf(q0[h].w, k0.w, d);
                d = fmaf(q1[h].x, k1.x, d);
                d = fmaf(q1[h].y, k1.y, d);
                d = fmaf(q1[h].z, k1.z, d);
                d = fmaf(q1[h].w, k1.w, d);
                d = group8_sum(d);  // row groups of a warp diverge on the chunk tail
                if (l8 == 0) scores[h * a.chunk_max + p] = d * a.scale;
            }
        }
        __syncthreads();
#pragma unroll
        for (int h = 0; h < kGroup; ++h) {
            float m = -FLT_MAX;
            for (int p = threadIdx.x; p < n; p += blockDim.x) m = fmaxf(m, scores[h * a.chunk_max + p]);
            m = block_max(m, scratch);
            float s = 0.0f;
            for (int p = threadIdx.x; p < n; p += blockDim.x) {
                const float e = expf(scores[h * a.chunk_max + p] - m);
                scores[h * a.chunk_max + p] = e;
                s += e;
            }
            s = block_sum(s, scratch);
            if (threadIdx.x == 0) { stats[0][h] = m; stats[1][h] = s; }
        }
        __syncthreads();
        float acc[kGroup][8];
#pragma unroll
        for (int h = 0; h < kGroup; ++h)
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[h][j] = 0.0f;
        const float* vb = a.value_cache + (static_cast<int64_t>(g) * a.capacity + s0) * kHeadDim;
        for (int p = grp; p < n; p += 32) {
            const float4* vr = reinterpret_cast<const float4*>(vb + static_cast<int64_t>(p) * kHeadDim);
            const float4 v0 = __ldg(vr + l8), v1 = __ldg(vr + 8 + l8);
#pragma unroll
            for (int h = 0; h < kGroup; ++h) {
                const float e = scores[h * a.chunk_max + p];
                acc[h][0] = fmaf(e, v0.x, acc[h][0]);
                acc[h][1] = fmaf(e, v0.y, acc[h][1]);
                acc[h][2] = fmaf(e, v0.z, acc[h][2]);
                acc[h][3] = fmaf(e, v0.w, acc[h][3]);
                acc[h][4] = fmaf(e, v1.x, acc[h][4]);
                acc[h][5] = fmaf(e, v1.y, acc[h][5]);
                acc[h][6] = fmaf(e, v1.z, acc[h][6]);
                acc[h][7] = fmaf(e, v1.w, acc[h][7]);
            }
        }
#pragma unroll
        for (int h = 0; h < kGroup; ++h)
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float v = acc[h][j];
                v += __shfl_xor_sync(0xffffffffu, v, 8);
                v += __shfl_xor_sync(0xffffffffu, v, 16);
                acc[h][j] = v;
            }
        if (lane < 8) {
#pragma unroll
            for (int h = 0; h < kGroup; ++h)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    red[warp][h][4 * lane + j] = acc[h][j];
                    red[warp][h][32 + 4 * lane + j] = acc[h][4 + j];
                }
        }
        __syncthreads();
        if (threadIdx.x < kGroup * kHeadDim) {
            const int h = threadIdx.x / kHeadDim, d = threadIdx.x % kHeadDim;
            float o = 0.0f;
#pragma unroll
            for (int w = 0; w < 8; ++w) o += red[w][h][d];
            float* pw = a.partials + ((static_cast<int64_t>(g) * kGroup + h) * a.nch + c) * kPartialStride;
            pw[4 + d] = o;
            if (d == 0) { pw[0] = stats[0][h]; pw[1] = stats[1][h]; }
        }
    }
    // Last CTA of this kv head merges (threadFenceReduction pattern).
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(&a.counters[g], 1u);
        is_last = prev == static_cast<unsigned>(a.nch - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    if (threadIdx.x < kGroup * kHeadDim) {
        const int h = threadIdx.x / kHeadDim, d = threadIdx.x % kHeadDim;
        const float* base = a.partials + (static_cast<int64_t>(g) * kGroup + h) * a.nch * kPartialStride;
        float m = -FLT_MAX;
        for (int cc = 0; cc < active; ++cc) m = fmaxf(m, __ldcg(base + cc * kPartialStride));
        float total = 0.0f, o = 0.0f;
        for (int cc = 0; cc < active; ++cc) {
            const float f = expf(__ldcg(base + cc * kPartialStride) - m);
            total += __ldcg(base + cc * kPartialStride + 1) * f;
            o += __ldcg(base + cc * kPartialStride + 4 + d) * f;
        }
        a.out[(g * kGroup + h) * kHeadDim + d] = o / total;
    }
    if (threadIdx.x == 0) a.counters[g] = 0u;
}

// grid 72 x 128: each half warp one o_proj row; out = h_in + Wo . attn.
__global__ void __launch_bounds__(128) o_proj_kernel(const float* __restrict__ attn, const float* __restrict__ w,
                                                     const float* __restrict__ h_in, float* __restrict__ h_out) {
    __shared__ __align__(16) float xs[kHidden];
    for (int i = threadIdx.x; i < kHidden; i += blockDim.x) xs[i] = attn[i];
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row = blockIdx.x * 8 + warp * 2 + (lane >> 4);
    const float y = half_warp_row_dot(w + static_cast<int64_t>(row) * kHidden, reinterpret_cast<const float4*>(xs),
                                      lane & 15);
    if ((lane & 15) == 0) h_out[row] = y + h_in[row];
}

// grid 192 x 256: each warp one intermediate feature i (gate row i by the
// first half warp, up row 1536 + i by the second).
__global__ void __launch_bounds__(256) gate_up_kernel(const float* __restrict__ h, const float* __restrict__ norm_w,
                                                      float eps, const float* __restrict__ w,
                                                      float* __restrict__ s_out) {
    __shared__ __align__(16) float xn[kHidden];
    __shared__ float scratch[32];
    norm_to_shared(h, norm_w, eps, xn, scratch, nullptr);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int i = blockIdx.x * 8 + warp;
    const int row = (lane >> 4) ? kInter + i : i;
    const float y = half_warp_row_dot(w + static_cast<int64_t>(row) * kHidden, reinterpret_cast<const float4*>(xn),
                                      lane & 15);
    const float up = __shfl_sync(0xffffffffu, y, 16);
    if (lane == 0) s_out[i] = swiglu(y, up);
}

// grid 144 x 128: one warp per down row (1536 wide = 32 lanes x 12 float4).
__global__ void __launch_bounds__(128) down_kernel(const float* __restrict__ s, const float* __restrict__ w,
                                                   const float* __restrict__ h_mid, float* __restrict__ h_out) {
    __shared__ __align__(16) float ss[kInter];
    for (int i = threadIdx.x; i < kInter; i += blockDim.x) ss[i] = s[i];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row = blockIdx.x * 4 + warp;
    const float4* r4 = reinterpret_cast<const float4*>(w + static_cast<int64_t>(row) * kInter);
    float4 wv[12];
#pragma unroll
    for (int j = 0; j < 12; ++j) wv[j] = __ldg(r4 + lane + 32 * j);
    __syncthreads();
    const float4* s4 = reinterpret_cast<const float4*>(ss);
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < 12; ++j) {
        const float4 x = s4[lane + 32 * j];
        acc = fmaf(wv[j].x, x.x, acc);
        acc = fmaf(wv[j].y, x.y, acc);
        acc = fmaf(wv[j].z, x.z, acc);
        acc = fmaf(wv[j].w, x.w, acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) h_out[row] = h_mid[row] + acc;
}

struct LmArgs {
    int* stop;               // [0] generation ended on EOS (state frozen), [1] EOS token + 1 (0: none)
    const float* h;
    const float* norm_w;
    float eps;
    const float* w;          // [vocab, 576]
    int64_t vocab;
    float* logits;
    float* norm_out;         // [576] final-norm output (written by CTA 0)
    float* cand_value;       // [gridDim]
    long long* cand_index;   // [gridDim]
    unsigned* counter;
    int64_t* token;
    int64_t* generated;
    int64_t generated_capacity;
    int64_t* step;
    int64_t* position;
    const int64_t* length;
};

__device__ __forceinline__ void argmax_combine(float& bv, long long& bi, float v, long long i) {
    if (argmax_precedes(v, i, bv, bi)) { bv = v; bi = i; }
}

__global__ void __launch_bounds__(256) lm_head_kernel(LmArgs a) {
    __shared__ __align__(16) float xn[kHidden];
    __shared__ float scratch[32];
    __shared__ float wv[16];
    __shared__ long long wi[16];
    __shared__ int is_last;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < kHidden; i += blockDim.x) {
        const float v = a.h[i];
        xn[i] = v;
        ss += v * v;
    }
    ss = block_sum(ss, scratch);
    const float inv = rsqrtf(ss / static_cast<float>(kHidden) + a.eps);
    for (int i = threadIdx.x; i < kHidden; i += blockDim.x) {
        xn[i] = xn[i] * inv * a.norm_w[i];
        if (blockIdx.x == 0) a.norm_out[i] = xn[i];
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, l16 = lane & 15;
    float bv = 0.0f;
    long long bi = -1;
    for (int64_t base = static_cast<int64_t>(blockIdx.x) * kLmRowsPerCta; base < a.vocab;
         base += static_cast<int64_t>(gridDim.x) * kLmRowsPerCta) {
        const int64_t row = base + warp * 2 + (lane >> 4);
        // Rows past the vocabulary recompute the last row so every lane
        // takes part in the half-warp shuffles; their result is dropped.
        const int64_t safe_row = row < a.vocab ? row : a.vocab - 1;
        const float y = half_warp_row_dot(a.w + safe_row * kHidden, reinterpret_cast<const float4*>(xn), l16);
        if (l16 == 0 && row < a.vocab) {
            a.logits[row] = y;
            argmax_combine(bv, bi, y, row);
        }
    }
    // Combine the 16 row owners (lanes 0 and 16 of each warp).
    const float ov = __shfl_sync(0xffffffffu, bv, 16);
    const long long oi = __shfl_sync(0xffffffffu, bi, 16);
    if (lane == 0) {
        argmax_combine(bv, bi, ov, oi);
        wv[warp] = bv;
        wi[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; ++w) argmax_combine(bv, bi, wv[w], wi[w]);
        a.cand_value[blockIdx.x] = bv;
        a.cand_index[blockIdx.x] = bi;
        __threadfence();
        is_last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!is_last || warp != 0) return;
    __threadfence();
    bv = 0.0f;
    bi = -1;
    for (unsigned c = lane; c < gridDim.x; c += 32)
        argmax_combine(bv, bi, __ldcg(a.cand_value + c), __ldcg(a.cand_index + c));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v = __shfl_xor_sync(0xffffffffu, bv, o);
        const long long i = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_combine(bv, bi, v, i);
    }
    if (lane == 0) {
        if (a.stop[0] == 0) {  // after an EOS the state stays frozen
            const int64_t selected = bi < 0 ? 0 : bi;
            *a.token = selected;
            const int64_t st = *a.step;
            if (st >= 0 && st < a.generated_capacity) a.generated[st] = selected;
            *a.step = st + 1;
            *a.position = *a.length;
            if (a.stop[1] != 0 && selected == static_cast<int64_t>(a.stop[1]) - 1) a.stop[0] = 1;
        }
        *a.counter = 0u;
    }
}

// Device-side state installation (graph-safe, no host staging).
__global__ void set_state_kernel(int64_t* token, const int64_t* token_src, int64_t* position, int64_t* length,
                                 int64_t* step, int64_t* generated, int64_t value, int64_t step_value,
                                 bool seed_generated, int* stop) {
    if (threadIdx.x != 0) return;
    const int64_t t = *token_src;
    *token = t;
    *position = value;
    *length = value;
    *step = step_value;
    if (seed_generated) generated[0] = t;
    stop[0] = 0;  // a new generation (the EOS token, stop[1], is kept)
}

// ------------------------------------------------------------------ host

struct DeviceGuard {
    int previous = -1;
    explicit DeviceGuard(int device) {
        cudaGetDevice(&previous);
        if (previous != device) cudaSetDevice(device);
    }
    ~DeviceGuard() {
        int current = -1;
        cudaGetDevice(&current);
        if (previous >= 0 && current != previous) cudaSetDevice(previous);
    }
};

}  // namespace
}  // namespace fx

using namespace fx;

struct fx_decode {
    fx_model_desc model{};
    int64_t capacity = 0, vocab = 0;
    int64_t start_position = 0, replay_count = 0;
    bool pending = false, generation_started = false, capture_active = false;
    int sms = 0, nch = 0, chunk_max = 0, lm_blocks = 0;
    bool persistent = true;       // one cooperative launch per step (else 151 kernels)
    int step_grid = 0;
    cudaStream_t capture_stream = nullptr;
    cudaEvent_t done = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int64_t* host_io = nullptr;   // page-locked, mapped [0] token in, [1] token out (fx_decode_replay_host)
    int64_t* host_io_dev = nullptr;  // the same words as the device sees them
    cudaGraph_t graph_host = nullptr;      // persistent step: the step also writing host_io[1]
    cudaGraphExec_t exec_host = nullptr;
    // owned device memory
    int64_t* state = nullptr;     // token, position, length, step, generated[capacity]
    float* logits = nullptr;
    float* key_cache = nullptr;
    float* value_cache = nullptr;
    unsigned long long* timeline = nullptr;  // optional per-CTA phase stamps (persistent step)
    char* workspace = nullptr;
    size_t workspace_bytes = 0;
    // workspace views
    float *h_a, *h_b, *h_mid, *q, *attn, *swiglu_out, *final_norm_out, *partials, *cand_value;
    long long* cand_index;
    unsigned* counters;           // [3] attention + [1] lm head
    unsigned* step_sync;          // persistent step: [0] LM-head arrivals, [1] step epoch
    StepExchange exchange{};      // persistent step: cross-CTA exchange region
    StepLayer step_layers[kLayers]{};  // persistent step: per-layer pointers and strip tensor maps
    int* error;
    int* inject;  // test hook of the persistent step (fx_decode_inject_failure)
    int* stop;    // [0] generation ended on EOS, [1] EOS token + 1 (0: none; fx_decode_set_eos)

    int64_t* token() const { return state; }
    int64_t* position() const { return state + 1; }
    int64_t* length() const { return state + 2; }
    int64_t* step() const { return state + 3; }
    int64_t* generated() const { return state + 4; }
    size_t layer_stride() const { return static_cast<size_t>(kKVHeads) * capacity * kHeadDim; }
};

namespace fx {
namespace {

fx_status validate_model(const fx_model_desc* m) {
    FX_REQUIRE(m != nullptr, "flux native decode: model description is null");
    FX_REQUIRE(m->vocab > 0, "flux native decode: vocabulary must be non-empty");
    FX_REQUIRE(m->capacity >= 1 && m->capacity <= kMaxCapacity,
               "flux native decode: cache capacity must be in [1, 131072]");
    FX_REQUIRE(std::isfinite(m->epsilon) && m->epsilon > 0.0f,
               "flux native decode: every RMSNorm epsilon must be positive");
    FX_REQUIRE(m->embedding && m->final_norm && m->lm_head && m->rope_cos && m->rope_sin,
               "flux native decode: a model tensor pointer is null");
    for (int l = 0; l < kLayers; ++l) {
        FX_REQUIRE(m->input_norm[l] && m->packed_qkv[l] && m->o_proj[l] && m->post_norm[l] && m->gate_up[l] &&
                       m->down[l],
                   "flux native decode: exactly 30 complete layer descriptors are required");
        FX_REQUIRE(std::isfinite(m->attention_scale[l]), "flux native decode: every attention scale must be finite");
        for (const void* p : {static_cast<const void*>(m->packed_qkv[l]), static_cast<const void*>(m->o_proj[l]),
                              static_cast<const void*>(m->gate_up[l]), static_cast<const void*>(m->down[l])})
            FX_REQUIRE(reinterpret_cast<uintptr_t>(p) % 16 == 0, "flux native decode: weights must be 16-byte aligned");
    }
    FX_REQUIRE(reinterpret_cast<uintptr_t>(m->lm_head) % 16 == 0, "flux native decode: LM head must be 16-byte aligned");
    return FX_OK;
}

template <typename T>
T* carve(char*& cursor, size_t count) {
    cursor = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(cursor) + 255) & ~uintptr_t(255));
    T* p = reinterpret_cast<T*>(cursor);
    cursor += count * sizeof(T);
    return p;
}

fx_status allocate(fx_decode* r) {
    const size_t cache = static_cast<size_t>(kLayers) * r->layer_stride();
    FX_CUDA_TRY(cudaMalloc(&r->state, (4 + r->capacity) * sizeof(int64_t)), "allocating decode state");
    FX_CUDA_TRY(cudaMalloc(&r->logits, r->vocab * sizeof(float)), "allocating logits");
    FX_CUDA_TRY(cudaMalloc(&r->key_cache, cache * sizeof(float)), "allocating K cache");
    FX_CUDA_TRY(cudaMalloc(&r->value_cache, cache * sizeof(float)), "allocating V cache");
    if (r->persistent) {
        const char* timeline = std::getenv("FLUX_B200_TIMELINE");
        if (timeline != nullptr && std::strcmp(timeline, "1") == 0) {
            const size_t bytes = static_cast<size_t>(r->step_grid) * kStepTimelineEvents * sizeof(unsigned long long);
            FX_CUDA_TRY(cudaMalloc(&r->timeline, bytes), "allocating the step timeline");
            FX_CUDA_TRY(cudaMemset(r->timeline, 0, bytes), "clearing the step timeline");
        }
    }
    // Lay the workspace out once with a null base to size it, then for real.
    for (int pass = 0; pass < 2; ++pass) {
        char* cursor = pass == 0 ? nullptr : r->workspace;
        r->h_a = carve<float>(cursor, kHidden);
        r->h_b = carve<float>(cursor, kHidden);
        r->h_mid = carve<float>(cursor, kHidden);
        r->q = carve<float>(cursor, kHidden);
        r->attn = carve<float>(cursor, kHidden);
        r->swiglu_out = carve<float>(cursor, kInter);
        r->final_norm_out = carve<float>(cursor, kHidden);
        r->partials = carve<float>(cursor, static_cast<size_t>(kKVHeads) * kGroup * r->nch * kPartialStride);
        unsigned long long* words = carve<unsigned long long>(cursor, step_exchange_words(r->nch));
        r->step_sync = carve<unsigned>(cursor, 4);
        r->cand_value = carve<float>(cursor, r->lm_blocks);
        r->cand_index = carve<long long>(cursor, r->lm_blocks);
        r->counters = carve<unsigned>(cursor, 8);
        r->error = carve<int>(cursor, 4);
        r->inject = carve<int>(cursor, 4);
        r->stop = carve<int>(cursor, 4);
        if (pass == 1) r->exchange = step_exchange_views(words, r->nch);
        if (pass == 0) {
            r->workspace_bytes = static_cast<size_t>(reinterpret_cast<uintptr_t>(cursor)) + 256;
            FX_CUDA_TRY(cudaMalloc(&r->workspace, r->workspace_bytes), "allocating decode workspace");
        }
    }
    return FX_OK;
}

// Reset the caches, copy `position` prefilled rows per layer, install token,
// position = length = position, step = 0 and clear logits and workspace.
fx_status initialize_state(fx_decode* r, const int64_t* token, const float* const* ks, const float* const* vs,
                           int64_t rows, int64_t position, cudaStream_t stream) {
    const size_t cache_bytes = static_cast<size_t>(kLayers) * r->layer_stride() * sizeof(float);
    FX_CUDA_TRY(cudaMemsetAsync(r->key_cache, 0, cache_bytes, stream), "clearing K cache");
    FX_CUDA_TRY(cudaMemsetAsync(r->value_cache, 0, cache_bytes, stream), "clearing V cache");
    if (position > 0) {
        const size_t row_bytes = static_cast<size_t>(position) * kHeadDim * sizeof(float);
        const size_t dpitch = static_cast<size_t>(r->capacity) * kHeadDim * sizeof(float);
        const size_t spitch = static_cast<size_t>(rows) * kHeadDim * sizeof(float);
        for (int l = 0; l < kLayers; ++l) {
            FX_CUDA_TRY(cudaMemcpy2DAsync(r->key_cache + l * r->layer_stride(), dpitch, ks[l], spitch, row_bytes,
                                          kKVHeads, cudaMemcpyDeviceToDevice, stream),
                        "importing K cache");
            FX_CUDA_TRY(cudaMemcpy2DAsync(r->value_cache + l * r->layer_stride(), dpitch, vs[l], spitch, row_bytes,
                                          kKVHeads, cudaMemcpyDeviceToDevice, stream),
                        "importing V cache");
        }
    }
    FX_CUDA_TRY(cudaMemsetAsync(r->logits, 0, r->vocab * sizeof(float), stream), "clearing logits");
    FX_CUDA_TRY(cudaMemsetAsync(r->workspace, 0, r->workspace_bytes, stream), "clearing workspace");
    FX_CUDA_TRY(cudaMemsetAsync(r->generated(), 0, r->capacity * sizeof(int64_t), stream), "clearing generated");
    set_state_kernel<<<1, 32, 0, stream>>>(r->token(), token, r->position(), r->length(), r->step(), r->generated(),
                                           position, 0, false, r->stop);
    FX_CUDA_TRY(cudaGetLastError(), "initializing decode state");
    return FX_OK;
}

// Enqueue one decode step on `stream`: one cooperative launch, or 151 kernels.
fx_status run_body(fx_decode* r, cudaStream_t stream, bool host_io = false) {
    const fx_model_desc& m = r->model;
    if (r->persistent) {
        StepArgs a{};
        if (host_io) a.host_out = r->host_io_dev + 1;
        for (int l = 0; l < kLayers; ++l) a.layer[l] = r->step_layers[l];
        a.embedding = m.embedding;
        a.final_norm = m.final_norm;
        a.lm_head = m.lm_head;
        a.cos_table = m.rope_cos;
        a.sin_table = m.rope_sin;
        a.vocab = r->vocab;
        a.capacity = r->capacity;
        a.eps = m.epsilon;
        a.key_cache = r->key_cache;
        a.value_cache = r->value_cache;
        a.token = r->token();
        a.position = r->position();
        a.length = r->length();
        a.step = r->step();
        a.generated = r->generated();
        a.logits = r->logits;
        a.x = r->exchange;
        a.final_norm_out = r->final_norm_out;
        a.cand_value = r->cand_value;
        a.cand_index = r->cand_index;
        a.sync = r->step_sync;
        a.error = r->error;
        a.inject = r->inject;
        a.stop = r->stop;
        a.nch = r->nch;
        a.timeline = r->timeline;
        return launch_step_kernel(a, r->step_grid, stream);
    }
    const size_t attn_smem = static_cast<size_t>(kGroup) * r->chunk_max * sizeof(float);
    for (int l = 0; l < kLayers; ++l) {
        float* h_in = (l % 2 == 0) ? r->h_a : r->h_b;
        float* h_out = (l % 2 == 0) ? r->h_b : r->h_a;
        float* kc = r->key_cache + l * r->layer_stride();
        float* vc = r->value_cache + l * r->layer_stride();
        QkvArgs qa{};
        qa.x = h_in;
        qa.token = l == 0 ? r->token() : nullptr;
        qa.embedding = m.embedding;
        qa.vocab = r->vocab;
        qa.embedding_out = l == 0 ? r->h_a : nullptr;
        qa.norm_w = m.input_norm[l];
        qa.w = m.packed_qkv[l];
        qa.eps = m.epsilon;
        qa.cos_table = m.rope_cos;
        qa.sin_table = m.rope_sin;
        qa.position = r->position();
        qa.length_out = l == 0 ? r->length() : nullptr;
        qa.capacity = r->capacity;
        qa.key_cache = kc;
        qa.value_cache = vc;
        qa.q_out = r->q;
        qa.error = r->error;
        qkv_rope_kernel<<<120, 128, 0, stream>>>(qa);
        AttnArgs aa{r->q, kc, vc, r->length(), r->capacity, m.attention_scale[l], r->partials, r->counters,
                    r->attn, r->nch, r->chunk_max};
        attention_kernel<<<kKVHeads * r->nch, 256, attn_smem, stream>>>(aa);
        o_proj_kernel<<<kHidden / 8, 128, 0, stream>>>(r->attn, m.o_proj[l], h_in, r->h_mid);
        gate_up_kernel<<<kInter / 8, 256, 0, stream>>>(r->h_mid, m.post_norm[l], m.epsilon, m.gate_up[l],
                                                        r->swiglu_out);
        down_kernel<<<kHidden / 4, 128, 0, stream>>>(r->swiglu_out, m.down[l], r->h_mid, h_out);
    }
    LmArgs la{};
    la.stop = r->stop;
    la.h = r->h_a;  // 30 layers: the last output lands in h_a
    la.norm_w = m.final_norm;
    la.eps = m.epsilon;
    la.w = m.lm_head;
    la.vocab = r->vocab;
    la.logits = r->logits;
    la.norm_out = r->final_norm_out;
    la.cand_value = r->cand_value;
    la.cand_index = r->cand_index;
    la.counter = r->counters + 4;
    la.token = r->token();
    la.generated = r->generated();
    la.generated_capacity = r->capacity;
    la.step = r->step();
    la.position = r->position();
    la.length = r->length();
    lm_head_kernel<<<r->lm_blocks, 256, 0, stream>>>(la);
    FX_CUDA_TRY(cudaGetLastError(), "launching the decode step");
    return FX_OK;
}

void release(fx_decode* r) {
    if (r == nullptr) return;
    DeviceGuard guard(r->model.device);
    if (r->capture_active && r->capture_stream != nullptr) {
        cudaGraph_t abandoned = nullptr;
        cudaStreamEndCapture(r->capture_stream, &abandoned);
        if (abandoned != nullptr) cudaGraphDestroy(abandoned);
        r->capture_active = false;
    }
    if (r->pending && r->done != nullptr) cudaEventSynchronize(r->done);
    if (r->exec) cudaGraphExecDestroy(r->exec);
    if (r->exec_host) cudaGraphExecDestroy(r->exec_host);
    if (r->graph_host) cudaGraphDestroy(r->graph_host);
    if (r->graph) cudaGraphDestroy(r->graph);
    if (r->done) cudaEventDestroy(r->done);
    if (r->capture_stream) {
        cudaStreamSynchronize(r->capture_stream);
        cudaStreamDestroy(r->capture_stream);
    }
    if (r->host_io) cudaFreeHost(r->host_io);
    cudaFree(r->state);
    cudaFree(r->logits);
    cudaFree(r->key_cache);
    cudaFree(r->value_cache);
    cudaFree(r->timeline);
    cudaFree(r->workspace);
    delete r;
}

fx_status create_impl(fx_decode* r, const int64_t* token, const float* const* ks, const float* const* vs,
                      int64_t rows, int64_t position, cudaStream_t stream) {
    FX_CUDA_TRY(cudaDeviceGetAttribute(&r->sms, cudaDevAttrMultiProcessorCount, r->model.device),
                "querying SM count");
    r->nch = std::max(1, std::min(r->sms / kKVHeads, 64));
    int64_t chunk = (r->capacity + r->nch - 1) / r->nch;
    r->chunk_max = static_cast<int>(((chunk + 31) / 32) * 32);
    r->lm_blocks = std::max(1, 2 * r->sms);
    const char* mode = std::getenv("FLUX_B200_DECODE_STEP");
    r->persistent = !(mode != nullptr && std::strcmp(mode, "kernels") == 0);
    if (r->persistent) {
        int sms = 0;
        const fx_status prep = prepare_step_kernel(r->model.device, &sms);
        if (prep != FX_OK) return prep;
        // Short caches: the largest grid that splits the 384 SwiGLU feature
        // blocks evenly (128 on a 148-SM B200: balanced phase D, fewer tally
        // contributors).  Long caches: every SM (the attention chunks get
        // shorter).  Measured on B200: 0.418 vs 0.425 ms/token at context 128
        // and 0.487 vs 0.482 at 8192 (128 vs 148 CTAs).
        r->step_grid = sms;
        if (r->capacity < kStepFullGridRows)
            while (r->step_grid > kStepMinGrid && (kInter / kStepBlock) % r->step_grid != 0) --r->step_grid;
        if (const char* g = std::getenv("FLUX_B200_STEP_GRID")) {  // tuning: another persistent grid
            const int want = std::atoi(g);
            if (want >= kStepMinGrid && want <= sms) r->step_grid = want;
        }
        r->nch = std::max(1, std::min(r->step_grid / kKVHeads, 64));
        chunk = (r->capacity + r->nch - 1) / r->nch;
        r->chunk_max = static_cast<int>(((chunk + 31) / 32) * 32);
        FX_REQUIRE(r->step_grid >= kStepMinGrid && r->step_grid <= kStepMaxGrid && r->step_grid <= r->lm_blocks &&
                       kKVHeads * r->nch <= r->step_grid,
                   "flux native decode: the persistent step needs a GPU with 128 to 384 SMs");
        for (int l = 0; l < kLayers; ++l) {
            StepLayer& L = r->step_layers[l];
            const fx_status enc = encode_step_maps(r->model.o_proj[l], r->model.down[l], &L);
            if (enc != FX_OK) return enc;
            L.input_norm = r->model.input_norm[l];
            L.qkv = r->model.packed_qkv[l];
            L.post_norm = r->model.post_norm[l];
            L.gate_up = r->model.gate_up[l];
            L.scale = r->model.attention_scale[l];
        }
    }
    const size_t attn_smem = static_cast<size_t>(kGroup) * r->chunk_max * sizeof(float);
    if (attn_smem > 48 * 1024) {
        const fx_status raised = raise_smem_limit(reinterpret_cast<const void*>(attention_kernel), attn_smem,
                                                  "raising attention shared memory");
        if (raised != FX_OK) return raised;
    }
    fx_status st = allocate(r);
    if (st != FX_OK) return st;
    FX_CUDA_TRY(cudaStreamCreateWithFlags(&r->capture_stream, cudaStreamNonBlocking), "creating capture stream");
    FX_CUDA_TRY(cudaEventCreateWithFlags(&r->done, cudaEventDisableTiming), "creating completion event");
    FX_CUDA_TRY(cudaHostAlloc(reinterpret_cast<void**>(&r->host_io), 2 * sizeof(int64_t), cudaHostAllocMapped),
                "allocating page-locked token words");
    FX_CUDA_TRY(cudaHostGetDevicePointer(reinterpret_cast<void**>(&r->host_io_dev), r->host_io, 0),
                "mapping the page-locked token words");
    st = initialize_state(r, token, ks, vs, rows, position, stream);
    if (st != FX_OK) return st;
    FX_CUDA_TRY(cudaEventRecord(r->done, stream), "recording setup");
    FX_CUDA_TRY(cudaStreamWaitEvent(r->capture_stream, r->done, 0), "ordering setup");
    // Warm-up step (loads every kernel before capture), then restore the state.
    st = run_body(r, r->capture_stream);
    if (st != FX_OK) return st;
    FX_CUDA_TRY(cudaStreamSynchronize(r->capture_stream), "warming the decode step");
    st = initialize_state(r, token, ks, vs, rows, position, r->capture_stream);
    if (st != FX_OK) return st;
    FX_CUDA_TRY(cudaStreamBeginCapture(r->capture_stream, cudaStreamCaptureModeThreadLocal),
                "beginning CUDA graph capture");
    r->capture_active = true;
    if (std::getenv("FLUX_B200_INJECT_CAPTURE_FAILURE") != nullptr) {  // test hook: a failing launch in capture
        set_error("flux native decode: injected failure during CUDA graph capture");
        st = FX_ERR_CUDA;
    } else {
        st = run_body(r, r->capture_stream);
    }
    cudaGraph_t graph = nullptr;
    const cudaError_t end = cudaStreamEndCapture(r->capture_stream, &graph);
    r->capture_active = false;
    if (st != FX_OK) {
        if (graph) cudaGraphDestroy(graph);
        return st;
    }
    FX_CUDA_TRY(end, "ending CUDA graph capture");
    r->graph = graph;
    FX_CUDA_TRY(cudaGraphInstantiate(&r->exec, r->graph, 0), "instantiating the decode graph");
    if (r->persistent) {
        // the same step also writing its token to the mapped host word
        FX_CUDA_TRY(cudaStreamBeginCapture(r->capture_stream, cudaStreamCaptureModeThreadLocal),
                    "beginning the host-word graph capture");
        r->capture_active = true;
        st = run_body(r, r->capture_stream, true);
        cudaGraph_t host_graph = nullptr;
        const cudaError_t host_end = cudaStreamEndCapture(r->capture_stream, &host_graph);
        r->capture_active = false;
        if (st != FX_OK) {
            if (host_graph) cudaGraphDestroy(host_graph);
            return st;
        }
        FX_CUDA_TRY(host_end, "ending the host-word graph capture");
        r->graph_host = host_graph;
        FX_CUDA_TRY(cudaGraphInstantiate(&r->exec_host, r->graph_host, 0), "instantiating the host-word graph");
    }
    FX_CUDA_TRY(cudaStreamSynchronize(r->capture_stream), "finalizing capture");
    r->start_position = position;
    return FX_OK;
}

}  // namespace
}  // namespace fx

extern "C" fx_status fx_decode_create(const fx_model_desc* model, const int64_t* initial_token,
                                      const float* const* key_sources, const float* const* value_sources,
                                      int64_t source_rows, int64_t initial_position, void* stream,
                                      fx_decode** out) {
    FX_REQUIRE(out != nullptr, "fx_decode_create: output pointer is null");
    *out = nullptr;
    const fx_status valid = validate_model(model);
    if (valid != FX_OK) return valid;
    FX_REQUIRE(initial_token != nullptr, "flux native decode: initial token is null");
    FX_REQUIRE(initial_position >= 0 && initial_position < model->capacity,
               "flux native decode: initial position must be inside capacity");
    if (initial_position > 0) {
        FX_REQUIRE(key_sources && value_sources && source_rows >= initial_position,
                   "flux native decode: every K/V source must be contiguous float32 [1, 3, sequence>=position, 64]");
        for (int l = 0; l < kLayers; ++l)
            FX_REQUIRE(key_sources[l] && value_sources[l], "flux native decode: reset requires one K/V tensor per layer");
    }
    DeviceGuard guard(model->device);
    fx_decode* r = new (std::nothrow) fx_decode();
    FX_REQUIRE(r != nullptr, "flux native decode: out of host memory");
    r->model = *model;
    r->capacity = model->capacity;
    r->vocab = model->vocab;
    const fx_status st = create_impl(r, initial_token, key_sources, value_sources, source_rows, initial_position,
                                     as_stream(stream));
    if (st != FX_OK) {
        const std::string message = fx_last_error();
        release(r);
        set_error(message);
        return st;
    }
    *out = r;
    return FX_OK;
}

extern "C" fx_status fx_decode_replay(fx_decode* r, const int64_t* token, void* stream) {
    FX_REQUIRE(r != nullptr, "fx_decode_replay: runtime is null");
    if (r->replay_count >= r->capacity - r->start_position) {
        set_error("flux native full decode: fixed-capacity state is exhausted");
        return FX_ERR_EXHAUSTED;
    }
    DeviceGuard guard(r->model.device);
    cudaStream_t s = as_stream(stream);
    if (r->pending) FX_CUDA_TRY(cudaStreamWaitEvent(s, r->done, 0), "ordering consecutive replays");
    if (token != nullptr)
        FX_CUDA_TRY(cudaMemcpyAsync(r->token(), token, sizeof(int64_t), cudaMemcpyDeviceToDevice, s),
                    "copying replay token");
    FX_CUDA_TRY(cudaGraphLaunch(r->exec, s), "launching the decode graph");
    FX_CUDA_TRY(cudaEventRecord(r->done, s), "recording replay completion");
    r->pending = true;
    ++r->replay_count;
    return FX_OK;
}

extern "C" fx_status fx_decode_replay_host(fx_decode* r, const int64_t* host_token, int64_t* host_next,
                                          void* stream) {
    FX_REQUIRE(r != nullptr && host_next != nullptr, "fx_decode_replay_host: null pointer");
    if (r->replay_count >= r->capacity - r->start_position) {
        set_error("flux native full decode: fixed-capacity state is exhausted");
        return FX_ERR_EXHAUSTED;
    }
    DeviceGuard guard(r->model.device);
    cudaStream_t s = as_stream(stream);
    if (r->pending) FX_CUDA_TRY(cudaStreamWaitEvent(s, r->done, 0), "ordering consecutive replays");
    // The staging words are free: the previous call returned after its step.
    if (host_token != nullptr) {
        r->host_io[0] = *host_token;
        FX_CUDA_TRY(cudaMemcpyAsync(r->token(), r->host_io, sizeof(int64_t), cudaMemcpyHostToDevice, s),
                    "copying the host replay token");
    }
    if (r->exec_host != nullptr) {
        // the step stores its token to the mapped host word itself
        FX_CUDA_TRY(cudaGraphLaunch(r->exec_host, s), "launching the decode graph");
    } else {
        FX_CUDA_TRY(cudaGraphLaunch(r->exec, s), "launching the decode graph");
        FX_CUDA_TRY(cudaMemcpyAsync(r->host_io + 1, r->token(), sizeof(int64_t), cudaMemcpyDeviceToHost, s),
                    "copying the sampled token to the host");
    }
    FX_CUDA_TRY(cudaEventRecord(r->done, s), "recording replay completion");
    r->pending = true;
    ++r->replay_count;
    FX_CUDA_TRY(cudaEventSynchronize(r->done), "waiting for the replay");
    *host_next = reinterpret_cast<volatile int64_t*>(r->host_io)[1];
    return FX_OK;
}

extern "C" fx_status fx_decode_generate(fx_decode* r, int64_t steps, void* stream) {
    FX_REQUIRE(r != nullptr, "fx_decode_generate: runtime is null");
    FX_REQUIRE(steps >= 0, "flux native full decode: generation step count must be non-negative");
    if (steps > r->capacity - r->start_position - r->replay_count) {
        set_error("flux native full decode: fixed-capacity generation is exhausted");
        return FX_ERR_EXHAUSTED;
    }
    if (r->generation_started) {
        set_error("flux native full decode: prefill or reset is required before reuse");
        return FX_ERR_STATE;
    }
    DeviceGuard guard(r->model.device);
    cudaStream_t s = as_stream(stream);
    if (r->pending) FX_CUDA_TRY(cudaStreamWaitEvent(s, r->done, 0), "ordering greedy generation");
    for (int64_t i = 0; i < steps; ++i) FX_CUDA_TRY(cudaGraphLaunch(r->exec, s), "launching chained decode graph");
    if (steps > 0) {
        FX_CUDA_TRY(cudaEventRecord(r->done, s), "recording generation completion");
        r->pending = true;
        r->replay_count += steps;
    }
    r->generation_started = true;
    return FX_OK;
}

extern "C" fx_status fx_decode_reset(fx_decode* r, const int64_t* token, const float* const* key_sources,
                                     const float* const* value_sources, int64_t source_rows, int64_t position,
                                     void* stream) {
    FX_REQUIRE(r != nullptr, "fx_decode_reset: runtime is null");
    FX_REQUIRE(token != nullptr, "flux native full decode: token is null");
    FX_REQUIRE(position >= 0 && position < r->capacity,
               "flux native full decode: reset position must be inside capacity");
    if (position > 0) {
        FX_REQUIRE(key_sources && value_sources, "flux native full decode: reset requires one K/V tensor per layer");
        for (int l = 0; l < kLayers; ++l)
            FX_REQUIRE(key_sources[l] && value_sources[l],
                       "flux native full decode: reset requires one K/V tensor per layer");
        FX_REQUIRE(source_rows >= position,
                   "flux native full decode: every K/V source must be contiguous float32 [1, 3, sequence>=position, 64]");
    }
    DeviceGuard guard(r->model.device);
    if (r->pending) {
        FX_CUDA_TRY(cudaEventSynchronize(r->done), "waiting to reset");
        r->pending = false;
    }
    cudaStream_t s = as_stream(stream);
    const fx_status st = initialize_state(r, token, key_sources, value_sources, source_rows, position, s);
    if (st != FX_OK) return st;
    FX_CUDA_TRY(cudaStreamSynchronize(s), "resetting decode state");
    r->start_position = position;
    r->replay_count = 0;
    r->generation_started = false;
    return FX_OK;
}

extern "C" fx_status fx_decode_install_prefill(fx_decode* r, const int64_t* token, int64_t position, void* stream) {
    FX_REQUIRE(r != nullptr && token != nullptr, "fx_decode_install_prefill: null pointer");
    FX_REQUIRE(position >= 1 && position <= r->capacity,
               "flux native full decode: prefill position must be in [1, capacity]");
    DeviceGuard guard(r->model.device);
    cudaStream_t s = as_stream(stream);
    set_state_kernel<<<1, 32, 0, s>>>(r->token(), token, r->position(), r->length(), r->step(), r->generated(),
                                      position, 1, true, r->stop);
    FX_CUDA_TRY(cudaGetLastError(), "installing prefill state");
    FX_CUDA_TRY(cudaEventRecord(r->done, s), "recording prefill completion");
    r->start_position = position;
    r->replay_count = 0;
    r->generation_started = false;
    r->pending = true;
    return FX_OK;
}

namespace fx {
int* decode_error_word(fx_decode* runtime) { return runtime == nullptr ? nullptr : runtime->error; }
}  // namespace fx

extern "C" fx_status fx_decode_wait(fx_decode* r, void* stream) {
    FX_REQUIRE(r != nullptr, "fx_decode_wait: runtime is null");
    DeviceGuard guard(r->model.device);
    if (r->pending) FX_CUDA_TRY(cudaStreamWaitEvent(as_stream(stream), r->done, 0), "ordering after decode work");
    return FX_OK;
}

extern "C" fx_status fx_decode_get_buffers(const fx_decode* r, fx_decode_buffers* out) {
    FX_REQUIRE(r != nullptr && out != nullptr, "fx_decode_get_buffers: null pointer");
    out->input_token = r->token();
    out->logits = r->logits;
    out->generated_tokens = r->generated();
    out->generation_step = r->step();
    out->key_cache = r->key_cache;
    out->value_cache = r->value_cache;
    out->position = r->position();
    out->cache_length = r->length();
    out->workspace = reinterpret_cast<float*>(r->workspace);
    out->workspace_bytes = static_cast<int64_t>(r->workspace_bytes);
    out->hidden_a = r->h_a;
    out->hidden_b = r->h_b;
    out->final_norm_output = r->final_norm_out;
    out->attention_workspace = r->partials;
    out->stable_buffer_bytes = static_cast<int64_t>((4 + r->capacity) * sizeof(int64_t) + r->vocab * sizeof(float));
    out->timeline = reinterpret_cast<uint64_t*>(r->timeline);
    out->timeline_ctas = r->timeline != nullptr ? r->step_grid : 0;
    out->timeline_events = r->timeline != nullptr ? kStepTimelineEvents : 0;
    return FX_OK;
}

extern "C" fx_status fx_decode_read_state(fx_decode* r, int32_t which, int64_t* value) {
    FX_REQUIRE(r != nullptr && value != nullptr, "fx_decode_read_state: null pointer");
    FX_REQUIRE(which >= 0 && which <= 2, "fx_decode_read_state: unknown state scalar");
    DeviceGuard guard(r->model.device);
    if (r->pending) FX_CUDA_TRY(cudaEventSynchronize(r->done), "waiting to inspect decode state");
    const int64_t* src = which == FX_STATE_POSITION ? r->position()
                         : which == FX_STATE_CACHE_LENGTH ? r->length()
                                                          : r->step();
    FX_CUDA_TRY(cudaMemcpy(value, src, sizeof(int64_t), cudaMemcpyDeviceToHost), "reading decode state");
    int error = 0;
    FX_CUDA_TRY(cudaMemcpy(&error, r->error, sizeof(int), cudaMemcpyDeviceToHost), "reading decode error flag");
    if (error & 256) {
        set_error("flux native prefill: a bounded wait in a tensor-core projection gave up");
        return FX_ERR_DEVICE;
    }
    if (error & 2) {
        set_error("flux native full decode: a step gave up a bounded wait (or a CTA reported a failure); "
                  "reset the runtime before the next replay");
        return FX_ERR_DEVICE;
    }
    if (error != 0) {
        set_error("flux native full decode: a step ran with its position outside the cache capacity");
        return FX_ERR_DEVICE;
    }
    return FX_OK;
}

extern "C" fx_status fx_decode_set_eos(fx_decode* r, int64_t eos_token) {
    FX_REQUIRE(r != nullptr, "fx_decode_set_eos: null runtime");
    FX_REQUIRE(eos_token >= -1 && eos_token < r->vocab, "fx_decode_set_eos: EOS token must be -1 or a vocabulary id");
    DeviceGuard guard(r->model.device);
    if (r->pending) FX_CUDA_TRY(cudaEventSynchronize(r->done), "waiting before setting the EOS token");
    const int value = static_cast<int>(eos_token + 1);
    FX_CUDA_TRY(cudaMemcpy(r->stop + 1, &value, sizeof(int), cudaMemcpyHostToDevice), "setting the EOS token");
    return FX_OK;
}

extern "C" fx_status fx_decode_inject_failure(fx_decode* r, int32_t layer) {
    FX_REQUIRE(r != nullptr, "fx_decode_inject_failure: null runtime");
    FX_REQUIRE(r->persistent, "fx_decode_inject_failure: only the persistent step has the hook");
    FX_REQUIRE(layer >= -1 && layer < kLayers, "fx_decode_inject_failure: layer must be in [-1, 30)");
    DeviceGuard guard(r->model.device);
    if (r->pending) FX_CUDA_TRY(cudaEventSynchronize(r->done), "waiting before setting the failure hook");
    const int value = layer + 1;
    FX_CUDA_TRY(cudaMemcpy(r->inject, &value, sizeof(int), cudaMemcpyHostToDevice), "setting the failure hook");
    return FX_OK;
}

extern "C" fx_status fx_decode_get_info(const fx_decode* r, fx_decode_info* out) {
    FX_REQUIRE(r != nullptr && out != nullptr, "fx_decode_get_info: null pointer");
    out->capacity = r->capacity;
    out->vocab = r->vocab;
    out->start_position = r->start_position;
    out->replay_count = r->replay_count;
    out->kernels_per_step = r->persistent ? 1 : 5 * kLayers + 1;
    return FX_OK;
}

extern "C" void fx_decode_destroy(fx_decode* r) { release(r); }
