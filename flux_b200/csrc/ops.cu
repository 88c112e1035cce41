// Stand-alone operators behind torch.ops.flux.* (the eager integration path).
//
// These keep the reference operators' semantics (argument meaning, error
// behaviour, rounding of the RoPE products); the fused decode step lives in
// decode.cu.  None of them is on the timed decode path.
#include "attention.cuh"
#include "common.cuh"

#include <cuda.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdint>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

namespace fx {
namespace {

constexpr int64_t kFusedMergeMaxCtas = 512;  // chunk CTAs up to which the op merges in-kernel

// ------------------------------------------------------------------ norms

// One CTA per row.  With `residual` set, v = hidden + residual is written to
// residual_out first (exact FP32 sum) and normalised; otherwise v = input.
// out = v * rsqrt(mean(v^2) + eps) * w   (rmsnorm_cuda.cu:23-64 /
// residual_rmsnorm_cuda.cu:23-104 evaluation order).
__global__ void rmsnorm_rows_kernel(const float* __restrict__ input, const float* __restrict__ residual,
                                    const float* __restrict__ weight, float* __restrict__ out,
                                    float* __restrict__ residual_out, int64_t width, float eps) {
    __shared__ float scratch[32];
    const int64_t base = static_cast<int64_t>(blockIdx.x) * width;
    float ss = 0.0f;
    for (int64_t i = threadIdx.x; i < width; i += blockDim.x) {
        float v = input[base + i];
        if (residual != nullptr) {
            v = v + residual[base + i];
            residual_out[base + i] = v;
        }
        ss += v * v;
    }
    ss = block_sum(ss, scratch);
    const float inv = rsqrtf(ss / static_cast<float>(width) + eps);
    for (int64_t i = threadIdx.x; i < width; i += blockDim.x) {
        const float v = residual != nullptr ? residual_out[base + i] : input[base + i];
        out[base + i] = v * inv * weight[i];
    }
}

__global__ void packed_swiglu_kernel(const float* __restrict__ packed, float* __restrict__ out, int64_t rows,
                                     int64_t inter) {
    const int64_t total = rows * inter;
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = t / inter, i = t - r * inter;
        out[t] = swiglu(packed[r * 2 * inter + i], packed[r * 2 * inter + inter + i]);
    }
}

// Row softmax; with `mask` the row value is (s * scale) + mask (both rounded,
// as torch evaluates scores * scale + mask).
__global__ void softmax_rows_kernel(const float* __restrict__ in, float* __restrict__ out, int64_t width,
                                    const float* __restrict__ mask, int64_t heads, int64_t queries,
                                    int64_t mb, int64_t mh, int64_t mq, int64_t mk, int64_t s0, int64_t s1,
                                    int64_t s2, int64_t s3, float scale) {
    __shared__ float scratch[32];
    const int64_t row = blockIdx.x;
    const float* x = in + row * width;
    float* y = out + row * width;
    int64_t mask_base = 0;
    if (mask != nullptr) {
        const int64_t q = row % queries;
        const int64_t h = (row / queries) % heads;
        const int64_t b = row / (queries * heads);
        mask_base = (mb == 1 ? 0 : b) * s0 + (mh == 1 ? 0 : h) * s1 + (mq == 1 ? 0 : q) * s2;
    }
    auto value = [&](int64_t i) {
        if (mask == nullptr) return x[i];
        return __fadd_rn(__fmul_rn(x[i], scale), mask[mask_base + (mk == 1 ? 0 : i) * s3]);
    };
    float m = -INFINITY;
    for (int64_t i = threadIdx.x; i < width; i += blockDim.x) m = fmaxf(m, value(i));
    m = block_max(m, scratch);
    float s = 0.0f;
    for (int64_t i = threadIdx.x; i < width; i += blockDim.x) {
        const float e = expf(value(i) - m);
        y[i] = e;
        s += e;
    }
    s = block_sum(s, scratch);
    for (int64_t i = threadIdx.x; i < width; i += blockDim.x) y[i] = y[i] / s;
}

// ------------------------------------------------------------------- RoPE

struct Strides4 { int64_t s[4]; };
struct Strides3 { int64_t s[3]; };

__global__ void rope_kernel(const float* __restrict__ q, Strides4 qs, const float* __restrict__ k, Strides4 ks,
                            const float* __restrict__ cos, Strides3 cs, const float* __restrict__ sin,
                            Strides3 ss, float* __restrict__ q_out, float* __restrict__ k_out, int64_t batch,
                            int64_t hq, int64_t hk, int64_t seq, int64_t dim, int64_t rope_batch) {
    const int64_t half = dim / 2;
    const int64_t q_total = batch * hq * seq * dim;
    const int64_t total = q_total + batch * hk * seq * dim;
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const bool is_q = t < q_total;
        const int64_t u = is_q ? t : t - q_total;
        const int64_t heads = is_q ? hq : hk;
        const int64_t d = u % dim;
        const int64_t s = (u / dim) % seq;
        const int64_t h = (u / (dim * seq)) % heads;
        const int64_t b = u / (dim * seq * heads);
        const Strides4& st = is_q ? qs : ks;
        const float* src = is_q ? q : k;
        const int64_t base = b * st.s[0] + h * st.s[1] + s * st.s[2];
        const int64_t partner = d < half ? d + half : d - half;
        const int64_t rb = rope_batch == 1 ? 0 : b;
        const float c = cos[rb * cs.s[0] + s * cs.s[1] + d * cs.s[2]];
        const float sn = sin[rb * ss.s[0] + s * ss.s[1] + d * ss.s[2]];
        const float r = rope_value(src[base + d * st.s[3]], src[base + partner * st.s[3]], c, sn, d < half);
        (is_q ? q_out : k_out)[u] = r;
    }
}

// Reference semantics of packed_qkv_rope_cache_cuda_fp32_kernel
// (packed_qkv_rope_cache_cuda.cu:51-121) with arbitrary positive strides.
__global__ void packed_qkv_rope_cache_kernel(const float* __restrict__ packed, Strides3 ps,
                                             const float* __restrict__ cos, Strides3 cs,
                                             const float* __restrict__ sin, Strides3 ss, float* key_cache,
                                             Strides4 kst, float* value_cache, Strides4 vst, int64_t capacity,
                                             const int64_t* position_ptr, int64_t* advance,
                                             float* __restrict__ q_out) {
    __shared__ int64_t position;
    if (threadIdx.x == 0) position = *position_ptr;
    __syncthreads();
    if (position < 0 || position >= capacity) return;
    for (int t = threadIdx.x; t < kQKV; t += blockDim.x) {
        if (t < kHidden + kKVHeads * kHeadDim) {
            const int head_base = (t / kHeadDim) * kHeadDim;
            const int d = t % kHeadDim;
            const int partner = d < kHeadDim / 2 ? d + kHeadDim / 2 : d - kHeadDim / 2;
            const float v = rope_value(packed[(head_base + d) * ps.s[2]], packed[(head_base + partner) * ps.s[2]],
                                       cos[d * cs.s[2]], sin[d * ss.s[2]], d < kHeadDim / 2);
            if (t < kHidden) {
                q_out[t] = v;
            } else {
                const int h = (t - kHidden) / kHeadDim;
                key_cache[h * kst.s[1] + position * kst.s[2] + d * kst.s[3]] = v;
            }
        } else {
            const int u = t - kHidden - kKVHeads * kHeadDim;
            const int h = u / kHeadDim, d = u % kHeadDim;
            value_cache[h * vst.s[1] + position * vst.s[2] + d * vst.s[3]] = packed[t * ps.s[2]];
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && advance != nullptr) *advance = position + 1;
}

// --------------------------------------------------------------- attention

constexpr int kOpChunk = 128;  // positions per split-K chunk (workspace [B, Hq, chunks, D+2])
constexpr int kOpMaxGroup = 16;
constexpr int kOpMaxDim = 256;

struct GqaArgs {
    const float* q; Strides4 qs;
    const float* k; Strides4 ks;
    const float* v; Strides4 vs;
    const float* mask; int64_t msz[4]; int64_t mst[4];
    const int64_t* length;
    float* out; float* ws;
    float scale;
    int64_t batch, hq, hkv, cap, dim, chunks;
};

__device__ __forceinline__ int64_t valid_length(const int64_t* length, int64_t cap) {
    const int64_t requested = length == nullptr ? cap : *length;
    return std::max<int64_t>(1, std::min<int64_t>(requested, cap));
}

// grid (chunks, hkv, batch); one CTA scores kOpChunk positions for the
// `group` query heads of one kv head and writes (max, sum, unnormalised PV).
__global__ void __launch_bounds__(128) gqa_partial_kernel(GqaArgs a) {
    extern __shared__ float smem[];
    const int64_t group = a.hq / a.hkv;
    float* qsh = smem;                         // [group][dim]
    float* scores = smem + group * a.dim;      // [group][kOpChunk]
    __shared__ float scratch[32];
    const int64_t c = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int64_t len = valid_length(a.length, a.cap);
    const int64_t start = c * kOpChunk;
    if (start >= len) return;
    const int n = static_cast<int>(std::min<int64_t>(kOpChunk, len - start));
    for (int64_t t = threadIdx.x; t < group * a.dim; t += blockDim.x) {
        const int64_t h = g * group + t / a.dim, d = t % a.dim;
        qsh[t] = a.q[b * a.qs.s[0] + h * a.qs.s[1] + d * a.qs.s[3]];
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    const float* kb = a.k + b * a.ks.s[0] + g * a.ks.s[1];
    for (int p = warp; p < n; p += warps) {
        float acc[kOpMaxGroup];
#pragma unroll
        for (int h = 0; h < kOpMaxGroup; ++h) acc[h] = 0.0f;
        for (int64_t d = lane; d < a.dim; d += 32) {
            const float kv = kb[(start + p) * a.ks.s[2] + d * a.ks.s[3]];
#pragma unroll
            for (int h = 0; h < kOpMaxGroup; ++h)
                if (h < group) acc[h] += qsh[h * a.dim + d] * kv;
        }
#pragma unroll
        for (int h = 0; h < kOpMaxGroup; ++h) {
            if (h >= group) break;
            const float dot = warp_sum(acc[h]);
            if (lane == 0) {
                float s = dot * a.scale;
                if (a.mask != nullptr) {
                    const int64_t hh = g * group + h;
                    s += a.mask[(a.msz[0] == 1 ? 0 : b) * a.mst[0] + (a.msz[1] == 1 ? 0 : hh) * a.mst[1] +
                                (a.msz[3] == 1 ? 0 : start + p) * a.mst[3]];
                }
                scores[h * kOpChunk + p] = s;
            }
        }
    }
    __syncthreads();
    for (int64_t h = 0; h < group; ++h) {
        float m = -FLT_MAX;
        for (int p = threadIdx.x; p < n; p += blockDim.x) m = fmaxf(m, scores[h * kOpChunk + p]);
        m = block_max(m, scratch);
        float s = 0.0f;
        for (int p = threadIdx.x; p < n; p += blockDim.x) {
            const float e = expf(scores[h * kOpChunk + p] - m);
            scores[h * kOpChunk + p] = e;
            s += e;
        }
        s = block_sum(s, scratch);
        if (threadIdx.x == 0) {
            float* w = a.ws + ((b * a.hq + g * group + h) * a.chunks + c) * (a.dim + 2);
            w[0] = m;
            w[1] = s;
        }
    }
    __syncthreads();
    const float* vb = a.v + b * a.vs.s[0] + g * a.vs.s[1];
    for (int64_t d = threadIdx.x; d < a.dim; d += blockDim.x) {
        float acc[kOpMaxGroup];
#pragma unroll
        for (int h = 0; h < kOpMaxGroup; ++h) acc[h] = 0.0f;
        for (int p = 0; p < n; ++p) {
            const float vv = vb[(start + p) * a.vs.s[2] + d * a.vs.s[3]];
#pragma unroll
            for (int h = 0; h < kOpMaxGroup; ++h)
                if (h < group) acc[h] += scores[h * kOpChunk + p] * vv;
        }
        for (int64_t h = 0; h < group; ++h)
            a.ws[((b * a.hq + g * group + h) * a.chunks + c) * (a.dim + 2) + 2 + d] = acc[h];
    }
}

// grid (batch * hq): merge the chunk partials of one query head.
__global__ void gqa_merge_kernel(GqaArgs a) {
    const int64_t bh = blockIdx.x;
    const int64_t len = valid_length(a.length, a.cap);
    const int64_t active = (len + kOpChunk - 1) / kOpChunk;
    const float* w = a.ws + bh * a.chunks * (a.dim + 2);
    float m = -FLT_MAX;
    for (int64_t c = 0; c < active; ++c) m = fmaxf(m, w[c * (a.dim + 2)]);
    float total = 0.0f;
    for (int64_t c = 0; c < active; ++c) total += w[c * (a.dim + 2) + 1] * expf(w[c * (a.dim + 2)] - m);
    for (int64_t d = threadIdx.x; d < a.dim; d += blockDim.x) {
        float acc = 0.0f;
        for (int64_t c = 0; c < active; ++c) acc += w[c * (a.dim + 2) + 2 + d] * expf(w[c * (a.dim + 2)] - m);
        a.out[bh * a.dim + d] = acc / total;
    }
}

// ------------------------------------------------------------------ GEMV

// out[i] = swiglu(W[i] . x, W[I + i] . x); one warp per i.
__global__ void gate_up_swiglu_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                      float* __restrict__ out, int64_t inter, int64_t width) {
    const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (i >= inter) return;
    const float* gw = w + i * width;
    const float* uw = w + (inter + i) * width;
    float g = 0.0f, u = 0.0f;
    for (int64_t k = lane; k < width; k += 32) {
        const float xv = x[k];
        g = fmaf(gw[k], xv, g);
        u = fmaf(uw[k], xv, u);
    }
    g = warp_sum(g);
    u = warp_sum(u);
    if (lane == 0) out[i] = swiglu(g, u);
}

// Small-M linear: one warp per output column n computes it for every row m
// (each weight row is streamed once).  Used for m <= 8.
__global__ void linear_small_m_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                      float* __restrict__ out, int64_t m, int64_t k, int64_t n) {
    const int64_t col = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (col >= n) return;
    const float* wr = w + col * k;
    float acc[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) acc[r] = 0.0f;
    for (int64_t kk = lane; kk < k; kk += 32) {
        const float wv = wr[kk];
#pragma unroll
        for (int r = 0; r < 8; ++r)
            if (r < m) acc[r] = fmaf(wv, x[r * k + kk], acc[r]);
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        if (r >= m) break;
        const float s = warp_sum(acc[r]);
        if (lane == 0) out[r * n + col] = s;
    }
}

// ---------------------------------------------------------------- greedy

template <bool Update>
__global__ void __launch_bounds__(1024) greedy_kernel(const float* __restrict__ logits, int64_t vocab,
                                                      int64_t* token, int64_t* generated, int64_t gen_cap,
                                                      int64_t* step, int64_t* position, const int64_t* length) {
    __shared__ float sv[1024];
    __shared__ long long si[1024];
    float bv = 0.0f;
    long long bi = -1;
    for (int64_t i = threadIdx.x; i < vocab; i += blockDim.x) {
        const float v = logits[i];
        if (argmax_precedes(v, i, bv, bi)) { bv = v; bi = i; }
    }
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int width = blockDim.x / 2; width > 0; width >>= 1) {
        if (threadIdx.x < width &&
            argmax_precedes(sv[threadIdx.x + width], si[threadIdx.x + width], sv[threadIdx.x], si[threadIdx.x])) {
            sv[threadIdx.x] = sv[threadIdx.x + width];
            si[threadIdx.x] = si[threadIdx.x + width];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const int64_t selected = si[0] < 0 ? 0 : si[0];
        *token = selected;
        if (Update) {
            const int64_t s = *step;
            if (s >= 0 && s < gen_cap) generated[s] = selected;
            *step = s + 1;
            *position = *length;
        }
    }
}

unsigned grid_for(int64_t work, int threads, int64_t cap = 148 * 16) {
    return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((work + threads - 1) / threads, cap)));
}

}  // namespace

// Launcher shared with the prefill runtime (defined in prefill.cu).
fx_status launch_gemm_nt(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k,
                         cudaStream_t stream);

}  // namespace fx

using namespace fx;

extern "C" fx_status fx_rmsnorm_f32(const float* input, const float* weight, float* output, int64_t rows,
                                    int64_t width, float epsilon, void* stream) {
    FX_REQUIRE(input && weight && output, "fx_rmsnorm_f32: null pointer");
    FX_REQUIRE(rows > 0 && width > 0 && rows <= 0x7fffffff, "fx_rmsnorm_f32: rows and width must be positive");
    FX_REQUIRE(std::isfinite(epsilon) && epsilon >= 0.0f, "fx_rmsnorm_f32: epsilon must be finite and non-negative");
    rmsnorm_rows_kernel<<<static_cast<unsigned>(rows), 256, 0, as_stream(stream)>>>(input, nullptr, weight, output,
                                                                                   nullptr, width, epsilon);
    FX_CUDA_TRY(cudaGetLastError(), "launching rmsnorm");
    return FX_OK;
}

extern "C" fx_status fx_residual_rmsnorm_f32(const float* hidden, const float* residual, const float* weight,
                                             float* norm_out, float* residual_out, int64_t rows, int64_t width,
                                             float epsilon, void* stream) {
    FX_REQUIRE(hidden && residual && weight && norm_out && residual_out, "fx_residual_rmsnorm_f32: null pointer");
    FX_REQUIRE(rows > 0 && width > 0 && rows <= 0x7fffffff,
               "fx_residual_rmsnorm_f32: rows and width must be positive");
    FX_REQUIRE(std::isfinite(epsilon) && epsilon >= 0.0f,
               "fx_residual_rmsnorm_f32: epsilon must be finite and non-negative");
    rmsnorm_rows_kernel<<<static_cast<unsigned>(rows), 256, 0, as_stream(stream)>>>(hidden, residual, weight,
                                                                                   norm_out, residual_out, width,
                                                                                   epsilon);
    FX_CUDA_TRY(cudaGetLastError(), "launching residual rmsnorm");
    return FX_OK;
}

extern "C" fx_status fx_packed_swiglu_f32(const float* packed, float* output, int64_t rows, int64_t intermediate,
                                          void* stream) {
    FX_REQUIRE(packed && output, "fx_packed_swiglu_f32: null pointer");
    FX_REQUIRE(rows > 0 && intermediate > 0, "fx_packed_swiglu_f32: sizes must be positive");
    packed_swiglu_kernel<<<grid_for(rows * intermediate, 256), 256, 0, as_stream(stream)>>>(packed, output, rows,
                                                                                            intermediate);
    FX_CUDA_TRY(cudaGetLastError(), "launching packed swiglu");
    return FX_OK;
}

extern "C" fx_status fx_softmax_f32(const float* input, float* output, int64_t rows, int64_t width, void* stream) {
    FX_REQUIRE(input && output, "fx_softmax_f32: null pointer");
    FX_REQUIRE(rows > 0 && width > 0 && rows <= 0x7fffffff, "fx_softmax_f32: sizes must be positive");
    softmax_rows_kernel<<<static_cast<unsigned>(rows), 256, 0, as_stream(stream)>>>(
        input, output, width, nullptr, 1, 1, 1, 1, 1, 1, 0, 0, 0, 0, 1.0f);
    FX_CUDA_TRY(cudaGetLastError(), "launching softmax");
    return FX_OK;
}

extern "C" fx_status fx_attention_score_softmax_f32(const float* scores, const int64_t* sizes4, const float* mask,
                                                    const int64_t* mask_sizes4, const int64_t* mask_strides4,
                                                    float scale, float* output, void* stream) {
    FX_REQUIRE(scores && sizes4 && mask && mask_sizes4 && mask_strides4 && output,
               "fx_attention_score_softmax_f32: null pointer");
    FX_REQUIRE(std::isfinite(scale), "fx_attention_score_softmax_f32: scale must be finite");
    for (int d = 0; d < 4; ++d) {
        FX_REQUIRE(sizes4[d] > 0, "fx_attention_score_softmax_f32: sizes must be positive");
        FX_REQUIRE(mask_sizes4[d] == 1 || mask_sizes4[d] == sizes4[d],
                   "fx_attention_score_softmax_f32: mask is not broadcastable");
    }
    const int64_t rows = sizes4[0] * sizes4[1] * sizes4[2];
    FX_REQUIRE(rows <= 0x7fffffff, "fx_attention_score_softmax_f32: too many rows");
    softmax_rows_kernel<<<static_cast<unsigned>(rows), 256, 0, as_stream(stream)>>>(
        scores, output, sizes4[3], mask, sizes4[1], sizes4[2], mask_sizes4[0], mask_sizes4[1], mask_sizes4[2],
        mask_sizes4[3], mask_strides4[0], mask_strides4[1], mask_strides4[2], mask_strides4[3], scale);
    FX_CUDA_TRY(cudaGetLastError(), "launching attention score softmax");
    return FX_OK;
}

extern "C" fx_status fx_rope_f32(const float* query, const int64_t* query_strides4, const float* key,
                                 const int64_t* key_strides4, const float* cos, const int64_t* cos_strides3,
                                 const float* sin, const int64_t* sin_strides3, float* query_out, float* key_out,
                                 int64_t batch, int64_t query_heads, int64_t key_heads, int64_t sequence,
                                 int64_t head_dim, int64_t rope_batch, void* stream) {
    FX_REQUIRE(query && key && cos && sin && query_out && key_out && query_strides4 && key_strides4 &&
                   cos_strides3 && sin_strides3,
               "fx_rope_f32: null pointer");
    FX_REQUIRE(batch > 0 && query_heads > 0 && key_heads > 0 && sequence > 0, "fx_rope_f32: sizes must be positive");
    FX_REQUIRE(head_dim > 0 && head_dim % 2 == 0, "fx_rope_f32: head_dim must be positive and even");
    FX_REQUIRE(rope_batch == 1 || rope_batch == batch, "fx_rope_f32: rope batch must be 1 or the batch");
    Strides4 qs{}, ks{};
    Strides3 cs{}, ss{};
    for (int d = 0; d < 4; ++d) { qs.s[d] = query_strides4[d]; ks.s[d] = key_strides4[d]; }
    for (int d = 0; d < 3; ++d) { cs.s[d] = cos_strides3[d]; ss.s[d] = sin_strides3[d]; }
    const int64_t total = batch * (query_heads + key_heads) * sequence * head_dim;
    rope_kernel<<<grid_for(total, 256), 256, 0, as_stream(stream)>>>(query, qs, key, ks, cos, cs, sin, ss, query_out,
                                                                     key_out, batch, query_heads, key_heads,
                                                                     sequence, head_dim, rope_batch);
    FX_CUDA_TRY(cudaGetLastError(), "launching rope");
    return FX_OK;
}

extern "C" fx_status fx_packed_qkv_rope_cache_f32(const float* packed_qkv, const int64_t* packed_strides3,
                                                  const float* cos, const int64_t* cos_strides3, const float* sin,
                                                  const int64_t* sin_strides3, float* key_cache,
                                                  const int64_t* key_strides4, float* value_cache,
                                                  const int64_t* value_strides4, int64_t capacity,
                                                  const int64_t* position, int64_t* advance_length,
                                                  float* query_out, void* stream) {
    FX_REQUIRE(packed_qkv && cos && sin && key_cache && value_cache && position && query_out && packed_strides3 &&
                   cos_strides3 && sin_strides3 && key_strides4 && value_strides4,
               "fx_packed_qkv_rope_cache_f32: null pointer");
    FX_REQUIRE(capacity > 0, "fx_packed_qkv_rope_cache_f32: capacity must be positive");
    Strides3 ps{}, cs{}, ss{};
    Strides4 kst{}, vst{};
    for (int d = 0; d < 3; ++d) { ps.s[d] = packed_strides3[d]; cs.s[d] = cos_strides3[d]; ss.s[d] = sin_strides3[d]; }
    for (int d = 0; d < 4; ++d) { kst.s[d] = key_strides4[d]; vst.s[d] = value_strides4[d]; }
    packed_qkv_rope_cache_kernel<<<1, 256, 0, as_stream(stream)>>>(packed_qkv, ps, cos, cs, sin, ss, key_cache, kst,
                                                                  value_cache, vst, capacity, position,
                                                                  advance_length, query_out);
    FX_CUDA_TRY(cudaGetLastError(), "launching packed QKV/RoPE/cache update");
    return FX_OK;
}

extern "C" int64_t fx_gqa_decode_attention_workspace_floats(int64_t batch, int64_t query_heads, int64_t capacity,
                                                            int64_t head_dim) {
    if (batch <= 0 || query_heads <= 0 || capacity <= 0 || head_dim <= 0) return 0;
    // INT64_MAX when the product does not fit: no workspace is large enough.
    const int64_t chunks = capacity / kOpChunk + (capacity % kOpChunk != 0 ? 1 : 0);
    int64_t floats = 0, width = 0;
    if (__builtin_add_overflow(head_dim, int64_t{2}, &width) || __builtin_mul_overflow(batch, query_heads, &floats) ||
        __builtin_mul_overflow(floats, chunks, &floats) || __builtin_mul_overflow(floats, width, &floats))
        return INT64_MAX;
    return floats;
}

extern "C" fx_status fx_gqa_decode_attention_f32(const float* query, const int64_t* query_strides4,
                                                 const float* key_cache, const int64_t* key_strides4,
                                                 const float* value_cache, const int64_t* value_strides4,
                                                 const float* mask, const int64_t* mask_sizes4,
                                                 const int64_t* mask_strides4, const int64_t* cache_length,
                                                 float* output, float* workspace, int64_t workspace_floats,
                                                 float scale, int64_t batch, int64_t query_heads,
                                                 int64_t kv_heads, int64_t capacity, int64_t head_dim,
                                                 void* stream) {
    FX_REQUIRE(query && key_cache && value_cache && output && workspace && query_strides4 && key_strides4 &&
                   value_strides4,
               "fx_gqa_decode_attention_f32: null pointer");
    FX_REQUIRE(batch > 0 && query_heads > 0 && kv_heads > 0 && capacity > 0 && head_dim > 0,
               "fx_gqa_decode_attention_f32: sizes must be positive");
    FX_REQUIRE(query_heads % kv_heads == 0, "fx_gqa_decode_attention_f32: query heads must be divisible by KV heads");
    FX_REQUIRE(query_heads / kv_heads <= kOpMaxGroup, "fx_gqa_decode_attention_f32: at most 16 query heads per KV head");
    FX_REQUIRE(head_dim <= kOpMaxDim, "fx_gqa_decode_attention_f32: head_dim must be <= 256");
    FX_REQUIRE(std::isfinite(scale), "fx_gqa_decode_attention_f32: scale must be finite");
    FX_REQUIRE(workspace_floats >= fx_gqa_decode_attention_workspace_floats(batch, query_heads, capacity, head_dim),
               "fx_gqa_decode_attention_f32: workspace is too small");
    const int64_t chunks = (capacity + kOpChunk - 1) / kOpChunk;
    FX_REQUIRE(chunks <= 0x7fffffff && kv_heads <= 65535 && batch <= 65535,
               "fx_gqa_decode_attention_f32: grid too large");
    GqaArgs a{};
    a.q = query; a.k = key_cache; a.v = value_cache;
    for (int d = 0; d < 4; ++d) {
        a.qs.s[d] = query_strides4[d]; a.ks.s[d] = key_strides4[d]; a.vs.s[d] = value_strides4[d];
        a.msz[d] = mask ? mask_sizes4[d] : 1; a.mst[d] = mask ? mask_strides4[d] : 0;
    }
    if (mask != nullptr) {
        FX_REQUIRE(mask_sizes4 && mask_strides4, "fx_gqa_decode_attention_f32: mask sizes/strides missing");
        const int64_t target[4] = {batch, query_heads, 1, capacity};
        for (int d = 0; d < 4; ++d)
            FX_REQUIRE(mask_sizes4[d] == 1 || mask_sizes4[d] == target[d],
                       "fx_gqa_decode_attention_f32: mask is not broadcastable");
    }
    // SmolLM2 geometry over contiguous compact caches: the TMA-staged kernel
    // (attention.cu), same workspace format.
    const int64_t q_compact[4] = {query_heads * head_dim, head_dim, head_dim, 1};
    const int64_t kv_compact[4] = {kv_heads * capacity * head_dim, capacity * head_dim, head_dim, 1};
    bool compact = mask == nullptr && head_dim == kHeadDim && query_heads == kQHeads && kv_heads == kKVHeads &&
                   reinterpret_cast<uintptr_t>(key_cache) % 16 == 0 && reinterpret_cast<uintptr_t>(value_cache) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(query) % 16 == 0;
    for (int d = 0; d < 4 && compact; ++d) {
        if (d != 2 && query_strides4[d] != q_compact[d]) compact = false;
        if (key_strides4[d] != kv_compact[d] || value_strides4[d] != kv_compact[d]) compact = false;
    }
    if (compact) {
        CompactAttention c{};
        c.q = query; c.k = key_cache; c.v = value_cache;
        c.lengths = cache_length; c.length_stride = 0;
        c.out = output; c.ws = workspace; c.error = nullptr; c.scale = scale;
        c.batch = batch; c.cap = capacity; c.chunks = chunks; c.chunk_rows = kCompactChunk;
        // Room for merge counters after the partials and a small grid: merge
        // inside the chunk kernel (one launch).  On large grids the per-CTA
        // fence and arrival cost more than the merge launch saves (B200,
        // B = 64, L = 8192: 182 vs 160 us), so they keep the merge kernel.
        const int64_t partials = fx_gqa_decode_attention_workspace_floats(batch, query_heads, capacity, head_dim);
        if (workspace_floats >= partials + batch * kv_heads && batch * kv_heads * chunks <= kFusedMergeMaxCtas)
            c.counters = reinterpret_cast<unsigned*>(workspace + partials);
        return launch_compact_attention(c, as_stream(stream));
    }
    a.mask = mask; a.length = cache_length; a.out = output; a.ws = workspace; a.scale = scale;
    a.batch = batch; a.hq = query_heads; a.hkv = kv_heads; a.cap = capacity; a.dim = head_dim; a.chunks = chunks;
    const size_t smem = static_cast<size_t>((query_heads / kv_heads) * (head_dim + kOpChunk)) * sizeof(float);
    const dim3 grid(static_cast<unsigned>(chunks), static_cast<unsigned>(kv_heads), static_cast<unsigned>(batch));
    gqa_partial_kernel<<<grid, 128, smem, as_stream(stream)>>>(a);
    FX_CUDA_TRY(cudaGetLastError(), "launching GQA decode partials");
    const int merge_threads = static_cast<int>(std::min<int64_t>(256, std::max<int64_t>(32, head_dim)));
    gqa_merge_kernel<<<static_cast<unsigned>(batch * query_heads), merge_threads, 0, as_stream(stream)>>>(a);
    FX_CUDA_TRY(cudaGetLastError(), "launching GQA decode merge");
    return FX_OK;
}

extern "C" fx_status fx_packed_gate_up_swiglu_f32(const float* input, const float* weight, float* output,
                                                  int64_t intermediate, int64_t width, void* stream) {
    FX_REQUIRE(input && weight && output, "fx_packed_gate_up_swiglu_f32: null pointer");
    FX_REQUIRE(intermediate > 0 && width > 0, "fx_packed_gate_up_swiglu_f32: sizes must be positive");
    gate_up_swiglu_kernel<<<grid_for(intermediate * 32, 256, 1LL << 30), 256, 0, as_stream(stream)>>>(
        input, weight, output, intermediate, width);
    FX_CUDA_TRY(cudaGetLastError(), "launching gate/up SwiGLU");
    return FX_OK;
}

extern "C" fx_status fx_linear_f32(const float* input, const float* weight, float* output, int64_t m, int64_t k,
                                   int64_t n, void* stream) {
    FX_REQUIRE(input && weight && output, "fx_linear_f32: null pointer");
    FX_REQUIRE(m > 0 && k > 0 && n > 0, "fx_linear_f32: sizes must be positive");
    if (m <= 8) {
        linear_small_m_kernel<<<grid_for(n * 32, 256, 1LL << 30), 256, 0, as_stream(stream)>>>(input, weight, output,
                                                                                               m, k, n);
        FX_CUDA_TRY(cudaGetLastError(), "launching linear");
        return FX_OK;
    }
    return launch_gemm_nt(input, weight, output, m, n, k, as_stream(stream));
}

extern "C" fx_status fx_greedy_argmax_f32(const float* logits, int64_t vocab, int64_t* token, void* stream) {
    FX_REQUIRE(logits && token, "fx_greedy_argmax_f32: null pointer");
    FX_REQUIRE(vocab > 0, "fx_greedy_argmax_f32: vocabulary must be non-empty");
    greedy_kernel<false><<<1, 1024, 0, as_stream(stream)>>>(logits, vocab, token, nullptr, 0, nullptr, nullptr,
                                                            nullptr);
    FX_CUDA_TRY(cudaGetLastError(), "launching greedy argmax");
    return FX_OK;
}

extern "C" fx_status fx_greedy_argmax_update_f32(const float* logits, int64_t vocab, int64_t* token,
                                                 int64_t* generated, int64_t generated_capacity, int64_t* step,
                                                 int64_t* position, const int64_t* attention_length,
                                                 void* stream) {
    FX_REQUIRE(logits && token && generated && step && position && attention_length,
               "fx_greedy_argmax_update_f32: null pointer");
    FX_REQUIRE(vocab > 0 && generated_capacity > 0, "fx_greedy_argmax_update_f32: sizes must be positive");
    greedy_kernel<true><<<1, 1024, 0, as_stream(stream)>>>(logits, vocab, token, generated, generated_capacity,
                                                           step, position, attention_length);
    FX_CUDA_TRY(cudaGetLastError(), "launching greedy argmax update");
    return FX_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free GQA decode attention.
//
// Some callers cannot allocate device memory: a host that reserves the whole
// device budget for its own pool at start-up and treats any later cudaMalloc
// as an out-of-memory risk and a device-wide synchronisation, or a plugin host
// whose C FFI hands the plugin tensors but no allocator.  For them this entry
// point runs fx_gqa_decode_attention_f32 with its split-K partials in a
// fixed, file-scope device array instead of a caller-provided workspace.
//
// The array holds kStaticScratchFloats floats (1 MiB) and stays resident on
// every device that loads this library until the process exits.  All calls on
// a device share it and it keeps the last call's contents; nothing in it has
// to start at zero (every partial the merge reads is written by the same
// call), but two calls whose kernels overlap on the GPU (different streams
// without ordering between them) race on it.
//
// The array's device address belongs to the CUDA context it was looked up
// in, so it is looked up (cudaGetSymbolAddress) on the first call in each
// context -- the device's primary context, or a context the host made current
// itself -- and cached under that context's unique ID (cuCtxGetId, which a
// context created after a cudaDeviceReset does not share).  Make the first
// call in each context before any stream capture begins.
// ---------------------------------------------------------------------------

namespace fx {
namespace {

constexpr int64_t kStaticScratchFloats = 262144;

static __device__ __align__(256) float g_gqa_static_scratch[kStaticScratchFloats];

std::mutex g_static_scratch_mutex;
std::vector<std::pair<unsigned long long, float*>> g_static_scratch_by_context;

// Device address of g_gqa_static_scratch in the calling thread's current
// context (looked up on the first call in that context).
fx_status static_scratch_address(float** out) {
    unsigned long long id = 0;
    fx_status status = current_context_id(&id);
    if (status != FX_OK) return status;
    std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
    if (id != 0)
        for (const auto& entry : g_static_scratch_by_context)
            if (entry.first == id) {
                *out = entry.second;
                return FX_OK;
            }
    // First call in this context (or none was current yet: the lookup makes
    // the device's primary context current, whose ID is read afterwards).
    void* address = nullptr;
    FX_CUDA_TRY(cudaGetSymbolAddress(&address, g_gqa_static_scratch), "looking up the static GQA scratch address");
    if (id == 0) {
        status = current_context_id(&id);
        if (status != FX_OK) return status;
    }
    if (id != 0) g_static_scratch_by_context.emplace_back(id, static_cast<float*>(address));
    *out = static_cast<float*>(address);
    return FX_OK;
}

}  // namespace
}  // namespace fx

extern "C" int64_t fx_gqa_decode_attention_static_scratch_floats(void) { return fx::kStaticScratchFloats; }

extern "C" fx_status fx_gqa_decode_attention_static_scratch_f32(
    const float* query, const int64_t* query_strides4, const float* key_cache, const int64_t* key_strides4,
    const float* value_cache, const int64_t* value_strides4, const float* mask, const int64_t* mask_sizes4,
    const int64_t* mask_strides4, const int64_t* cache_length, float* output, float scale, int64_t batch,
    int64_t query_heads, int64_t kv_heads, int64_t capacity, int64_t head_dim, void* stream) {
    // The limits fx_gqa_decode_attention_f32 enforces, checked before the
    // scratch size is computed (the size helper also refuses on overflow).
    FX_REQUIRE(batch > 0 && query_heads > 0 && kv_heads > 0 && capacity > 0 && head_dim > 0,
               "fx_gqa_decode_attention_static_scratch_f32: sizes must be positive");
    FX_REQUIRE(batch <= 65535 && kv_heads <= 65535 && query_heads % kv_heads == 0 &&
                   query_heads / kv_heads <= fx::kOpMaxGroup && head_dim <= fx::kOpMaxDim,
               "fx_gqa_decode_attention_static_scratch_f32: batch and KV heads must be <= 65535, at most 16 "
               "query heads per KV head, head_dim <= 256");
    const int64_t needed = fx_gqa_decode_attention_workspace_floats(batch, query_heads, capacity, head_dim);
    if (needed > fx::kStaticScratchFloats) {
        fx::set_error("fx_gqa_decode_attention_static_scratch_f32: batch * query_heads * ceil(capacity / 128) * "
                      "(head_dim + 2) = " + std::to_string(needed) + " floats of split-K scratch exceeds the " +
                      std::to_string(fx::kStaticScratchFloats) + "-float static array");
        return FX_ERR_INVALID;
    }
    float* scratch = nullptr;
    const fx_status status = fx::static_scratch_address(&scratch);
    if (status != FX_OK) return status;
    // exactly the partials (no merge counters: the array is shared by calls of any size)
    return fx_gqa_decode_attention_f32(query, query_strides4, key_cache, key_strides4, value_cache, value_strides4,
                                       mask, mask_sizes4, mask_strides4, cache_length, output, scratch, needed, scale,
                                       batch, query_heads, kv_heads, capacity, head_dim, stream);
}
