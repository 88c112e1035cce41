// Native prompt prefill that fills the decode runtime's compact cache.
//
// Built only as far as the decode loop needs it (reference:
// csrc/native_prefill_runtime/native_prefill_runtime_cuda.cu:553-665):
// embedding gather -> 30 x (RMSNorm, QKV GEMM, RoPE + cache fill, causal
// online-softmax attention, o_proj GEMM + residual, RMSNorm, gate/up GEMM,
// SwiGLU, down GEMM + residual) -> final RMSNorm of the last row -> LM head
// -> greedy token -> decode state handoff (position = prompt length,
// generated[0] = token, step = 1).  The four projections per layer run on
// tcgen05 tensor cores with the 3xTF32 split (FP32-level results; weights
// split once at create); the attention is a flash-style FP32 SIMT kernel.
// The SIMT GEMM below serves the generic fx_linear_f32 op.
#include "common.cuh"
#include "tc_attention.cuh"
#include "tc_gemm.cuh"

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <cmath>
#include <new>
#include <string>

namespace fx {
namespace {

constexpr int kGemmBM = 128, kGemmBN = 128, kGemmBK = 16, kGemmThreads = 256;

// C[M, N] = A[M, K] . B[N, K]^T (+ R[M, N] when R is set).  Row-major, K % 4 == 0,
// 16-byte aligned A and B.  128 x 128 tile, 8 x 8 outputs per thread.
__global__ void __launch_bounds__(kGemmThreads) gemm_nt_kernel(const float* __restrict__ A,
                                                               const float* __restrict__ B, float* __restrict__ C,
                                                               const float* __restrict__ R, int64_t M, int64_t N,
                                                               int64_t K) {
    __shared__ __align__(16) float As[2][kGemmBK][kGemmBM + 4];
    __shared__ __align__(16) float Bs[2][kGemmBK][kGemmBN + 4];
    const int tid = threadIdx.x;
    const int tx = tid % 16, ty = tid / 16;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kGemmBM;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kGemmBN;
    // Loader mapping: 512 float4 per operand tile -> 2 per thread.
    // float4 f: row = f / 4 (0..127), k4 = f % 4.
    float4 ra[2], rb[2];
    auto load_tiles = [&](int64_t k0) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int f = tid + i * kGemmThreads;
            const int row = f >> 2, k4 = f & 3;
            const int64_t kk = k0 + 4 * k4;
            const int64_t am = m0 + row, bn = n0 + row;
            ra[i] = (am < M && kk < K) ? __ldg(reinterpret_cast<const float4*>(A + am * K + kk))
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
            rb[i] = (bn < N && kk < K) ? __ldg(reinterpret_cast<const float4*>(B + bn * K + kk))
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    auto store_tiles = [&](int buf) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int f = tid + i * kGemmThreads;
            const int row = f >> 2, k4 = f & 3;
            As[buf][4 * k4 + 0][row] = ra[i].x;
            As[buf][4 * k4 + 1][row] = ra[i].y;
            As[buf][4 * k4 + 2][row] = ra[i].z;
            As[buf][4 * k4 + 3][row] = ra[i].w;
            Bs[buf][4 * k4 + 0][row] = rb[i].x;
            Bs[buf][4 * k4 + 1][row] = rb[i].y;
            Bs[buf][4 * k4 + 2][row] = rb[i].z;
            Bs[buf][4 * k4 + 3][row] = rb[i].w;
        }
    };
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
    load_tiles(0);
    store_tiles(0);
    __syncthreads();
    int buf = 0;
    for (int64_t k0 = 0; k0 < K; k0 += kGemmBK) {
        const bool more = k0 + kGemmBK < K;
        if (more) load_tiles(k0 + kGemmBK);
#pragma unroll
        for (int kk = 0; kk < kGemmBK; ++kk) {
            float a[8], b[8];
            const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
            a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
            a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
            b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
            b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (more) {
            store_tiles(buf ^ 1);
            __syncthreads();
            buf ^= 1;
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
            if (n >= N) continue;
            float v = acc[i][j];
            if (R != nullptr) v = v + R[m * N + n];
            C[m * N + n] = v;
        }
    }
}

// Fallback for K % 4 != 0 or unaligned operands: one thread per output.
__global__ void gemm_nt_simple_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C,
                                      const float* __restrict__ R, int64_t M, int64_t N, int64_t K) {
    const int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (t >= M * N) return;
    const int64_t m = t / N, n = t % N;
    float acc = 0.0f;
    for (int64_t k = 0; k < K; ++k) acc = fmaf(A[m * K + k], B[n * K + k], acc);
    C[t] = R != nullptr ? acc + R[t] : acc;
}

// The prefill's RMSNorm: one warp per row of kHidden floats (float4 loads,
// shuffle reduction), out = v * rsqrt(mean(v^2) + eps) * w.  The op-level
// kernel (ops.cu) keeps the reference's summation order with a block per
// row; the prefill, whose products are 3xTF32 anyway, only needs FP32
// accuracy, and a block per 576-float row reached ~1.5 TB/s.
constexpr int kNormRowsPerBlock = 8;
__global__ void __launch_bounds__(32 * kNormRowsPerBlock) prefill_rmsnorm_kernel(const float* __restrict__ in,
                                                                                const float* __restrict__ weight,
                                                                                float* __restrict__ out, int64_t rows,
                                                                                float eps) {
    constexpr int kVec = kHidden / 4;                   // 144 float4 per row
    constexpr int kPer = (kVec + 31) / 32;              // 5 per lane (the last partly)
    const int64_t row = static_cast<int64_t>(blockIdx.x) * kNormRowsPerBlock + threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    if (row >= rows) return;
    const float4* x = reinterpret_cast<const float4*>(in + row * kHidden);
    float4 v[kPer];
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int i = lane + 32 * j;
        v[j] = i < kVec ? x[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float inv = rsqrtf(ss / static_cast<float>(kHidden) + eps);
    const float4* w = reinterpret_cast<const float4*>(weight);
    float4* y = reinterpret_cast<float4*>(out + row * kHidden);
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int i = lane + 32 * j;
        if (i < kVec) {
            const float4 g = w[i];
            y[i] = make_float4(v[j].x * inv * g.x, v[j].y * inv * g.y, v[j].z * inv * g.z, v[j].w * inv * g.w);
        }
    }
}

__global__ void embedding_gather_kernel(const int64_t* __restrict__ ids, const float* __restrict__ embedding,
                                        float* __restrict__ out, int64_t rows, int64_t vocab) {
    const int64_t total = rows * kHidden;
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = t / kHidden, c = t % kHidden;
        const int64_t tok = ids[r];
        out[t] = (tok >= 0 && tok < vocab) ? embedding[tok * kHidden + c] : 0.0f;
    }
}

__device__ __forceinline__ float tf32_round(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// The TF32 hi / lo halves of v at index i of the split planes.
__device__ __forceinline__ void store_split(float* __restrict__ hi, float* __restrict__ lo, size_t i, float v) {
    const float h = tf32_round(v);
    hi[i] = h;
    lo[i] = tf32_round(v - h);
}

// Rows [0, S) of packed QKV -> q [9, S, 64] (RoPE), K (RoPE) / V into the
// cache rows [0, S) (native_prefill_runtime_cuda.cu:124-163).  With
// `split` set, also the tensor-core attention's operands: q and K as TF32
// hi / lo planes ([9][S][64], [3][padded][64]) and V transposed per kv head
// ([3][64][padded]).
struct PrefillSplit {
    float *q_hi, *q_lo, *k_hi, *k_lo, *vt_hi, *vt_lo;
    int64_t padded;
};

// One block per kRopeRows rows x one chunk of three heads (blockIdx.y: q
// heads 0-2, 3-5, 6-8, k heads, v heads): every store is coalesced along the
// columns, and the V^T planes (one row per value column) go through a
// shared-memory tile so that each of their rows is written as kRopeRows
// consecutive floats (a store per element at a stride of `padded` floats
// took ~2x the kernel's traffic time).
constexpr int kRopeRows = 16;
constexpr int kRopeChunk = kKVHeads * kHeadDim;  // 192 columns
static_assert(kQKV == 5 * kRopeChunk, "packed QKV is five chunks of three heads");
__global__ void __launch_bounds__(256) prefill_rope_cache_kernel(const float* __restrict__ packed,
                                                                 const float* __restrict__ cos,
                                                                 const float* __restrict__ sin, float* __restrict__ q,
                                                                 float* __restrict__ key_cache,
                                                                 float* __restrict__ value_cache, int64_t rows,
                                                                 int64_t capacity, PrefillSplit split) {
    __shared__ float vt_tile[kKVHeads * kHeadDim][kRopeRows + 1];
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kRopeRows;
    const int nrows = static_cast<int>(min(static_cast<int64_t>(kRopeRows), rows - r0));
    const int chunk = static_cast<int>(blockIdx.y);
    for (int e = threadIdx.x; e < nrows * kRopeChunk; e += blockDim.x) {
        const int rr = e / kRopeChunk, col = chunk * kRopeChunk + e % kRopeChunk;
        const int64_t r = r0 + rr;
        const float* prow = packed + r * kQKV;
        if (col < kHidden + kKVHeads * kHeadDim) {
            const int base = (col / kHeadDim) * kHeadDim, d = col % kHeadDim;
            const int partner = d < kHeadDim / 2 ? d + kHeadDim / 2 : d - kHeadDim / 2;
            const float v = rope_value(prow[base + d], prow[base + partner], cos[r * kHeadDim + d],
                                       sin[r * kHeadDim + d], d < kHeadDim / 2);
            if (col < kHidden) {
                const size_t at = (static_cast<int64_t>(col / kHeadDim) * rows + r) * kHeadDim + d;
                q[at] = v;
                if (split.q_hi != nullptr) store_split(split.q_hi, split.q_lo, at, v);
            } else {
                const int h = (col - kHidden) / kHeadDim;
                key_cache[(static_cast<int64_t>(h) * capacity + r) * kHeadDim + d] = v;
                if (split.k_hi != nullptr)
                    store_split(split.k_hi, split.k_lo, (static_cast<int64_t>(h) * split.padded + r) * kHeadDim + d, v);
            }
        } else {
            const int u = col - kHidden - kKVHeads * kHeadDim;
            value_cache[(static_cast<int64_t>(u / kHeadDim) * capacity + r) * kHeadDim + u % kHeadDim] = prow[col];
            vt_tile[u][rr] = prow[col];
        }
    }
    if (split.vt_hi != nullptr && chunk == 4) {  // uniform over the block
        __syncthreads();
        for (int e = threadIdx.x; e < kKVHeads * kHeadDim * kRopeRows; e += blockDim.x) {
            const int u = e / kRopeRows, rr = e % kRopeRows;
            if (rr < nrows) store_split(split.vt_hi, split.vt_lo, static_cast<size_t>(u) * split.padded + r0 + rr,
                                        vt_tile[u][rr]);
        }
    }
}

// Causal attention over the cache rows [0, S), flash style: grid
// (ceil(S/64), 9), one CTA per 64 queries of one q head, 256 threads.  Key
// tiles of 64 rows stream through shared memory (K transposed, V as is); each
// thread owns a 4 x 4 block of the score tile (rows 4 tr.., keys 4 tc..) and
// a 4 x 4 block of the output (rows 4 tr.., dims 4 tc..), so both products
// are register-blocked (16 FMAs per two 16-byte shared loads).  Online
// softmax per row across the tiles, reduced over the 16 lanes that share the
// rows.  Heaviest query blocks (most key tiles) are scheduled first.
constexpr int kFlash = 64;          // queries and keys per tile
constexpr int kFlashPad = kFlash + 4;
constexpr int kFlashThreads = 256;
constexpr size_t kFlashSmem = 4ull * kFlash * kFlashPad * sizeof(float);

__global__ void __launch_bounds__(kFlashThreads) prefill_flash_kernel(const float* __restrict__ q,
                                                                      const float* __restrict__ key_cache,
                                                                      const float* __restrict__ value_cache,
                                                                      float* __restrict__ out, int64_t rows,
                                                                      int64_t capacity, float scale) {
    extern __shared__ __align__(16) float flash_smem[];
    float (*Qt)[kFlashPad] = reinterpret_cast<float (*)[kFlashPad]>(flash_smem);           // [dim][query]
    float (*Kt)[kFlashPad] = reinterpret_cast<float (*)[kFlashPad]>(flash_smem + kFlash * kFlashPad);  // [dim][key]
    float (*Vs)[kFlashPad] = reinterpret_cast<float (*)[kFlashPad]>(flash_smem + 2 * kFlash * kFlashPad);  // [key][dim]
    float (*Pt)[kFlashPad] = reinterpret_cast<float (*)[kFlashPad]>(flash_smem + 3 * kFlash * kFlashPad);  // [key][query]
    const int qb = static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x);
    const int h = blockIdx.y, g = h / kGroup;
    const int64_t r0 = static_cast<int64_t>(qb) * kFlash;
    const int tid = threadIdx.x, tr = tid >> 4, tc = tid & 15;
    // Q tile (scaled), transposed.
    for (int idx = tid; idx < kFlash * kHeadDim / 4; idx += kFlashThreads) {
        const int r = idx >> 4, d4 = idx & 15;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r0 + r < rows) v = *reinterpret_cast<const float4*>(q + (static_cast<int64_t>(h) * rows + r0 + r) * kHeadDim + 4 * d4);
        Qt[4 * d4 + 0][r] = v.x * scale;
        Qt[4 * d4 + 1][r] = v.y * scale;
        Qt[4 * d4 + 2][r] = v.z * scale;
        Qt[4 * d4 + 3][r] = v.w * scale;
    }
    const float* kb = key_cache + static_cast<int64_t>(g) * capacity * kHeadDim;
    const float* vb = value_cache + static_cast<int64_t>(g) * capacity * kHeadDim;
    float o[4][4] = {}, m[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
    }
    // K / V tile kt is fetched into registers while tile kt - 1 is computed.
    constexpr int kPer = kFlash * kHeadDim / 4 / kFlashThreads;  // float4s per thread per tile (4)
    float4 kreg[kPer], vreg[kPer];
    auto fetch = [&](int64_t k0) {
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int idx = tid + j * kFlashThreads, key = idx >> 4, d4 = idx & 15;
            kreg[j] = vreg[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k0 + key < rows) {
                kreg[j] = __ldg(reinterpret_cast<const float4*>(kb + (k0 + key) * kHeadDim) + d4);
                vreg[j] = __ldg(reinterpret_cast<const float4*>(vb + (k0 + key) * kHeadDim) + d4);
            }
        }
    };
    fetch(0);
    for (int kt = 0; kt <= qb; ++kt) {
        const int64_t k0 = static_cast<int64_t>(kt) * kFlash;
        __syncthreads();  // the previous tile's K / V / P are consumed
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int idx = tid + j * kFlashThreads, key = idx >> 4, d4 = idx & 15;
            Kt[4 * d4 + 0][key] = kreg[j].x;
            Kt[4 * d4 + 1][key] = kreg[j].y;
            Kt[4 * d4 + 2][key] = kreg[j].z;
            Kt[4 * d4 + 3][key] = kreg[j].w;
            *reinterpret_cast<float4*>(&Vs[key][4 * d4]) = vreg[j];
        }
        __syncthreads();
        if (kt < qb) fetch(k0 + kFlash);
        float sc[4][4] = {};
#pragma unroll 8
        for (int d = 0; d < kHeadDim; ++d) {
            const float4 a = *reinterpret_cast<const float4*>(&Qt[d][4 * tr]);
            const float4 b = *reinterpret_cast<const float4*>(&Kt[d][4 * tc]);
            const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) sc[i][j] = fmaf(av[i], bv[j], sc[i][j]);
        }
        // causal / length mask, online softmax per row (16 lanes share a row)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t row = r0 + 4 * tr + i;
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t key = k0 + 4 * tc + j;
                if (key > row || key >= rows) sc[i][j] = -INFINITY;
                mx = fmaxf(mx, sc[i][j]);
            }
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float mn = fmaxf(m[i], mx);
            const float corr = expf(m[i] - mn);  // first tile: m = -inf -> 0
            float sum = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                sc[i][j] = expf(sc[i][j] - mn);  // masked: exp(-inf) = 0
                sum += sc[i][j];
            }
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            l[i] = l[i] * corr + sum;
            m[i] = mn;
#pragma unroll
            for (int c = 0; c < 4; ++c) o[i][c] *= corr;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
            *reinterpret_cast<float4*>(&Pt[4 * tc + j][4 * tr]) = make_float4(sc[0][j], sc[1][j], sc[2][j], sc[3][j]);
        __syncthreads();
#pragma unroll 8
        for (int key = 0; key < kFlash; ++key) {
            const float4 a = *reinterpret_cast<const float4*>(&Pt[key][4 * tr]);
            const float4 b = *reinterpret_cast<const float4*>(&Vs[key][4 * tc]);
            const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int c = 0; c < 4; ++c) o[i][c] = fmaf(av[i], bv[c], o[i][c]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t row = r0 + 4 * tr + i;
        if (row >= rows) continue;
        const float inv = 1.0f / l[i];
        *reinterpret_cast<float4*>(out + row * kHidden + h * kHeadDim + 4 * tc) =
            make_float4(o[i][0] * inv, o[i][1] * inv, o[i][2] * inv, o[i][3] * inv);
    }
}

unsigned blocks_for(int64_t work) {
    return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, 148 * 32)));
}

}  // namespace

fx_status launch_gemm_nt_residual(const float* a, const float* b, float* c, const float* residual, int64_t m,
                                  int64_t n, int64_t k, cudaStream_t stream) {
    const bool aligned = k % 4 == 0 && reinterpret_cast<uintptr_t>(a) % 16 == 0 &&
                         reinterpret_cast<uintptr_t>(b) % 16 == 0;
    if (aligned) {
        const dim3 grid(static_cast<unsigned>((n + kGemmBN - 1) / kGemmBN), static_cast<unsigned>((m + kGemmBM - 1) / kGemmBM));
        gemm_nt_kernel<<<grid, kGemmThreads, 0, stream>>>(a, b, c, residual, m, n, k);
    } else {
        gemm_nt_simple_kernel<<<static_cast<unsigned>((m * n + 255) / 256), 256, 0, stream>>>(a, b, c, residual, m, n, k);
    }
    FX_CUDA_TRY(cudaGetLastError(), "launching GEMM");
    return FX_OK;
}

fx_status launch_gemm_nt(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k,
                         cudaStream_t stream) {
    return launch_gemm_nt_residual(a, b, c, nullptr, m, n, k, stream);
}

}  // namespace fx

using namespace fx;

struct fx_prefill {
    fx_model_desc model{};
    int64_t rows = 0;
    fx_decode* decode = nullptr;
    float* buffer = nullptr;
    size_t buffer_bytes = 0;
    float* logits = nullptr;
    int64_t* initial_token = nullptr;
    float *h_a, *h_b, *norm, *residual, *qkv, *q, *attn, *gate_up, *swiglu_out, *final_hidden;
    fx::TcModelWeights tc;                  // split projection weights
    CUtensorMap x_norm, x_attn, x_swiglu;   // activation maps of the projections
    int bm = 128;                           // activation rows per tensor-core tile
    // From kTcPairMinRows rows the gate/up projection runs on CTA pairs with
    // SwiGLU in its epilogue (gate/up weights split in the fused row order).
    bool fused_swiglu = false;
    // Tensor-core attention (unless FLUX_B200_PREFILL_ATTENTION=simt): split
    // q / K / V^T planes and their maps.
    bool tc_attention = true;
    float* split_buffer = nullptr;
    fx::TcAttentionArgs attn_args{};
};

namespace fx {
namespace {

fx_status prefill_run(fx_prefill* p, const int64_t* ids, cudaStream_t s) {
    // the flash tiles need more than the default 48 KB of shared memory
    const fx_status raised = raise_smem_limit(reinterpret_cast<const void*>(prefill_flash_kernel), kFlashSmem,
                                              "raising prefill attention shared memory");
    if (raised != FX_OK) return raised;
    const fx_model_desc& m = p->model;
    fx_decode_buffers db{};
    fx_status st = fx_decode_get_buffers(p->decode, &db);
    if (st != FX_OK) return st;
    st = fx_decode_wait(p->decode, s);
    if (st != FX_OK) return st;
    const int64_t S = p->rows;
    const int64_t cap = m.capacity;
    int* error = decode_error_word(p->decode);
    p->attn_args.error = error;
    auto project = [&](const TcWeight& w, const CUtensorMap& x, float* c, const float* residual) {
        return launch_tc_gemm(tc_args(w, x, c, residual, error, static_cast<int>(S), w.cols), p->bm, 1, s, false);
    };
    auto prefill_norm = [&](const float* in, const float* weight) -> fx_status {
        if (reinterpret_cast<uintptr_t>(in) % 16 != 0 || reinterpret_cast<uintptr_t>(weight) % 16 != 0)
            return fx_rmsnorm_f32(in, weight, p->norm, S, kHidden, m.epsilon, s);  // float4 loads need 16 bytes
        prefill_rmsnorm_kernel<<<static_cast<unsigned>((S + kNormRowsPerBlock - 1) / kNormRowsPerBlock),
                                 32 * kNormRowsPerBlock, 0, s>>>(in, weight, p->norm, S, m.epsilon);
        FX_CUDA_TRY(cudaGetLastError(), "launching the prefill RMSNorm");
        return FX_OK;
    };
    const size_t layer_stride = static_cast<size_t>(kKVHeads) * cap * kHeadDim;
    embedding_gather_kernel<<<blocks_for(S * kHidden), 256, 0, s>>>(ids, m.embedding, p->h_a, S, m.vocab);
    FX_CUDA_TRY(cudaGetLastError(), "launching embedding gather");
    for (int l = 0; l < kLayers; ++l) {
        float* in = l % 2 == 0 ? p->h_a : p->h_b;
        float* out = l % 2 == 0 ? p->h_b : p->h_a;
        float* kc = db.key_cache + l * layer_stride;
        float* vc = db.value_cache + l * layer_stride;
        if ((st = prefill_norm(in, m.input_norm[l])) != FX_OK) return st;
        if ((st = project(p->tc.qkv[l], p->x_norm, p->qkv, nullptr)) != FX_OK) return st;
        PrefillSplit split{};
        if (p->tc_attention) {
            const int64_t P = tc_attention_padded(S);
            float* b = p->split_buffer;
            split = {b, b + S * kHidden, b + 2 * S * kHidden, b + 2 * S * kHidden + kKVHeads * P * kHeadDim,
                     b + 2 * S * kHidden + 2 * kKVHeads * P * kHeadDim,
                     b + 2 * S * kHidden + 3 * kKVHeads * P * kHeadDim, P};
        }
        prefill_rope_cache_kernel<<<dim3(static_cast<unsigned>((S + kRopeRows - 1) / kRopeRows), 5), 256, 0, s>>>(
            p->qkv, m.rope_cos, m.rope_sin, p->q, kc, vc, S, cap, split);
        FX_CUDA_TRY(cudaGetLastError(), "launching prefill RoPE/cache fill");
        if (p->tc_attention) {
            TcAttentionArgs args = p->attn_args;
            args.scale = m.attention_scale[l];
            if ((st = launch_tc_prefill_attention(args, s)) != FX_OK) return st;
        } else {
            prefill_flash_kernel<<<dim3(static_cast<unsigned>((S + kFlash - 1) / kFlash), kQHeads), kFlashThreads,
                                   kFlashSmem, s>>>(p->q, kc, vc, p->attn, S, cap, m.attention_scale[l]);
            FX_CUDA_TRY(cudaGetLastError(), "launching prefill attention");
        }
        // residual = attn . Wo^T + in; norm = rmsnorm(residual)
        if ((st = project(p->tc.o[l], p->x_attn, p->residual, in)) != FX_OK) return st;
        if ((st = prefill_norm(p->residual, m.post_norm[l])) != FX_OK) return st;
        if (p->fused_swiglu) {
            TcGemmArgs a = tc_args(p->tc.gate_up[l], p->x_norm, nullptr, nullptr, error, static_cast<int>(S),
                                   kHidden);
            a.swiglu = true;
            a.act = p->swiglu_out;
            a.act_ld = kInter;
            if ((st = launch_tc_gemm(a, p->bm, 1, s, false)) != FX_OK) return st;
        } else {
            if ((st = project(p->tc.gate_up[l], p->x_norm, p->gate_up, nullptr)) != FX_OK) return st;
            if ((st = fx_packed_swiglu_f32(p->gate_up, p->swiglu_out, S, kInter, s)) != FX_OK) return st;
        }
        if ((st = project(p->tc.down[l], p->x_swiglu, out, p->residual)) != FX_OK) return st;
    }
    const float* last = p->h_a + (S - 1) * kHidden;  // 30 layers end in h_a
    if ((st = fx_rmsnorm_f32(last, m.final_norm, p->final_hidden, 1, kHidden, m.epsilon, s)) != FX_OK) return st;
    if ((st = fx_linear_f32(p->final_hidden, m.lm_head, p->logits, 1, kHidden, m.vocab, s)) != FX_OK) return st;
    if ((st = fx_greedy_argmax_f32(p->logits, m.vocab, p->initial_token, s)) != FX_OK) return st;
    return fx_decode_install_prefill(p->decode, p->initial_token, S, s);
}

void prefill_release(fx_prefill* p) {
    if (p == nullptr) return;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(p->model.device);
    if (p->decode != nullptr) fx_decode_destroy(p->decode);  // waits for pending work
    tc_weights_release(&p->tc);
    cudaFree(p->split_buffer);
    cudaFree(p->buffer);
    cudaFree(p->logits);
    cudaFree(p->initial_token);
    if (prev >= 0) cudaSetDevice(prev);
    delete p;
}

fx_status prefill_create_impl(fx_prefill* p, const int64_t* ids, cudaStream_t s) {
    const int64_t S = p->rows;
    p->bm = S <= 64 ? 64 : 128;
    // The projection inputs (norm, attn, swiglu_out) hold at least one
    // tensor-core tile of rows; rows past S stay zero.
    const int64_t R = std::max<int64_t>(S, p->bm);
    const size_t counts[] = {static_cast<size_t>(S) * kHidden, static_cast<size_t>(S) * kHidden,
                             static_cast<size_t>(R) * kHidden, static_cast<size_t>(S) * kHidden,
                             static_cast<size_t>(S) * kQKV,    static_cast<size_t>(S) * kHidden,
                             static_cast<size_t>(R) * kHidden, static_cast<size_t>(S) * kGateUp,
                             static_cast<size_t>(R) * kInter,  static_cast<size_t>(kHidden)};
    size_t total = 0;
    for (size_t c : counts) total += (c + 63) / 64 * 64;
    p->buffer_bytes = total * sizeof(float);
    FX_CUDA_TRY(cudaMalloc(&p->buffer, p->buffer_bytes), "allocating prefill workspace");
    FX_CUDA_TRY(cudaMalloc(&p->logits, p->model.vocab * sizeof(float)), "allocating prefill logits");
    FX_CUDA_TRY(cudaMalloc(&p->initial_token, sizeof(int64_t)), "allocating prefill token");
    float** views[] = {&p->h_a, &p->h_b, &p->norm, &p->residual, &p->qkv, &p->q, &p->attn, &p->gate_up,
                       &p->swiglu_out, &p->final_hidden};
    float* cursor = p->buffer;
    for (int i = 0; i < 10; ++i) {
        *views[i] = cursor;
        cursor += (counts[i] + 63) / 64 * 64;
    }
    FX_CUDA_TRY(cudaMemsetAsync(p->buffer, 0, p->buffer_bytes, s), "clearing the prefill workspace");
    p->fused_swiglu = p->bm == 128 && S >= kTcPairMinRows;
    fx_status st0 = tc_weights_create(p->model, false, &p->tc, s, true, p->fused_swiglu);
    if (st0 != FX_OK) return st0;
    const char* attention_mode = std::getenv("FLUX_B200_PREFILL_ATTENTION");
    p->tc_attention = !(attention_mode != nullptr && std::strcmp(attention_mode, "simt") == 0);
    if (p->tc_attention) {
        const int64_t P = tc_attention_padded(S);
        const size_t floats = 2 * static_cast<size_t>(S) * kHidden + 4 * static_cast<size_t>(kKVHeads) * P * kHeadDim;
        FX_CUDA_TRY(cudaMalloc(&p->split_buffer, floats * sizeof(float)), "allocating the split attention operands");
        FX_CUDA_TRY(cudaMemsetAsync(p->split_buffer, 0, floats * sizeof(float), s), "clearing the split operands");
        float* b = p->split_buffer;
        TcAttentionArgs& a = p->attn_args;
        float* k_hi = b + 2 * S * kHidden;
        float* k_lo = k_hi + kKVHeads * P * kHeadDim;
        float* vt_hi = k_lo + kKVHeads * P * kHeadDim;
        float* vt_lo = vt_hi + kKVHeads * P * kHeadDim;
        if ((st0 = tc_encode_map(&a.q_hi, b, kQHeads * S, kHeadDim, kTcAttnQ, "the split queries")) != FX_OK ||
            (st0 = tc_encode_map(&a.q_lo, b + S * kHidden, kQHeads * S, kHeadDim, kTcAttnQ, "the split queries")) !=
                FX_OK ||
            (st0 = tc_encode_map(&a.k_hi, k_hi, kKVHeads * P, kHeadDim, kTcAttnKeys, "the split keys")) != FX_OK ||
            (st0 = tc_encode_map(&a.k_lo, k_lo, kKVHeads * P, kHeadDim, kTcAttnKeys, "the split keys")) != FX_OK ||
            (st0 = tc_encode_map(&a.vt_hi, vt_hi, kKVHeads * kHeadDim, P, kTcAttnKeys, "the split values")) != FX_OK ||
            (st0 = tc_encode_map(&a.vt_lo, vt_lo, kKVHeads * kHeadDim, P, kTcAttnKeys, "the split values")) != FX_OK)
            return st0;
        a.out = p->attn;
        a.error = nullptr;  // set at run time (the decode runtime's error word)
        a.rows = static_cast<int>(S);
        a.padded = static_cast<int>(P);
    }
    if ((st0 = tc_encode_map(&p->x_norm, p->norm, R, kHidden, p->bm, "the prefill norm rows")) != FX_OK) return st0;
    if ((st0 = tc_encode_map(&p->x_attn, p->attn, R, kHidden, p->bm, "the prefill attention rows")) != FX_OK) return st0;
    if ((st0 = tc_encode_map(&p->x_swiglu, p->swiglu_out, R, kInter, p->bm, "the prefill SwiGLU rows")) != FX_OK)
        return st0;
    FX_CUDA_TRY(cudaMemsetAsync(p->initial_token, 0, sizeof(int64_t), s), "initializing decode token");
    fx_status st = fx_decode_create(&p->model, p->initial_token, nullptr, nullptr, 0, 0, s, &p->decode);
    if (st != FX_OK) return st;
    return prefill_run(p, ids, s);
}

}  // namespace
}  // namespace fx

extern "C" fx_status fx_prefill_create(const fx_model_desc* model, const int64_t* input_ids, int64_t prompt_length,
                                       void* stream, fx_prefill** out) {
    FX_REQUIRE(out != nullptr && model != nullptr && input_ids != nullptr, "fx_prefill_create: null pointer");
    *out = nullptr;
    FX_REQUIRE(prompt_length >= 1 && prompt_length <= model->capacity,
               "flux native prefill: prompt length must be in [1, capacity]");
    fx_prefill* p = new (std::nothrow) fx_prefill();
    FX_REQUIRE(p != nullptr, "flux native prefill: out of host memory");
    p->model = *model;
    p->rows = prompt_length;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(model->device);
    const fx_status st = prefill_create_impl(p, input_ids, as_stream(stream));
    if (prev >= 0) cudaSetDevice(prev);
    if (st != FX_OK) {
        const std::string message = fx_last_error();
        prefill_release(p);
        set_error(message);
        return st;
    }
    *out = p;
    return FX_OK;
}

extern "C" fx_status fx_prefill_run(fx_prefill* p, const int64_t* input_ids, void* stream) {
    FX_REQUIRE(p != nullptr && input_ids != nullptr, "fx_prefill_run: null pointer");
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(p->model.device);
    const fx_status st = prefill_run(p, input_ids, as_stream(stream));
    if (prev >= 0) cudaSetDevice(prev);
    return st;
}

extern "C" fx_decode* fx_prefill_decode(fx_prefill* p) { return p == nullptr ? nullptr : p->decode; }

extern "C" fx_status fx_prefill_get_buffers(const fx_prefill* p, fx_prefill_buffers* out) {
    FX_REQUIRE(p != nullptr && out != nullptr, "fx_prefill_get_buffers: null pointer");
    out->prefill_logits = p->logits;
    out->workspace = p->buffer;
    out->workspace_bytes = static_cast<int64_t>(p->buffer_bytes);
    out->attention_output = p->attn;
    out->final_hidden = p->final_hidden;
    out->initial_token = p->initial_token;
    return FX_OK;
}

extern "C" int64_t fx_prefill_prompt_length(const fx_prefill* p) { return p == nullptr ? 0 : p->rows; }

extern "C" void fx_prefill_destroy(fx_prefill* p) { prefill_release(p); }
