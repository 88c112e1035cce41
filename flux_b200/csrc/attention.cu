// Split-K decode attention over the compact cache [B][3][cap][64] (GQA, 3 q
// heads per kv head), ragged valid lengths per sequence.
//
// Chunk kernel, grid (chunks, 3 kv heads, B), 256 threads: one CTA owns 128
// cache rows of one (sequence, kv head).  Thread 0 starts two 1-D TMA bulk
// copies (K rows, V rows; no multicast) into shared memory on separate
// mbarriers, so scoring starts as soon as K has landed.  Scores: 4-lane
// groups, one row each, 3 heads from one K load; softmax in base 2 over the
// chunk; P.V with one thread per (4-dim quad, head, row split).  Each CTA
// writes (max, sum, unnormalised o[64]) per q head -- the workspace format of
// gqa_decode_attention_cuda.cu:551-633 -- and the merge kernel combines the
// active chunks of each (sequence, q head).
//
// HBM: every K/V row of the valid lengths is read once; with 64 KB in
// flight per CTA and three CTAs per SM the kernel streams at HBM rate when
// the grid is large.
#include "attention.cuh"

namespace fx {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kPart = kHeadDim + 2;
constexpr int kSplits = 5;                     // P.V row splits (5 x 3 heads x 16 quads = 240 threads)
constexpr float kLog2e = 1.4426950408889634f;  // log2(e)
constexpr float kLn2 = 0.6931471805599453f;    // ln(2)
constexpr unsigned long long kWaitNs = 2000000000ull;
constexpr int kMergeMaxChunks = 2048;          // 131072 rows / 64

template <int kRows>
struct ChunkShared {
    uint64_t bar[2];
    alignas(16) float p[kGroup][kRows];
    float wmax[kWarps][kGroup];
    float wsum[kWarps][kGroup];
    alignas(16) float o[kSplits][kGroup][kHeadDim];
    float l[kSplits][kGroup];
    float mscr[kGroup][2];  // in-kernel merge: per-head max / total of the two warps of a head
    float tscr[kGroup][2];
    int failed;
    int last;
};
template <int kRows>
constexpr size_t tile_bytes() { return static_cast<size_t>(kRows) * kHeadDim * sizeof(float); }
template <int kRows>
constexpr size_t shared_head() { return (sizeof(ChunkShared<kRows>) + 127) / 128 * 128; }
template <int kRows>
constexpr size_t chunk_smem() { return shared_head<kRows>() + 2 * tile_bytes<kRows>(); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait for phase 0 of `bar`; false if it gave up.
__device__ bool wait_landed(uint64_t* bar) {
    if (try_wait(bar, 0)) return true;
    const unsigned long long t0 = global_timer();
    while (!try_wait(bar, 0))
        if (global_timer() - t0 > kWaitNs) return false;
    return true;
}

__device__ __forceinline__ int64_t sequence_length(const CompactAttention& a, int64_t b) {
    const int64_t requested = a.lengths == nullptr ? a.cap : a.lengths[b * a.length_stride];
    return requested < 1 ? 1 : (requested > a.cap ? a.cap : requested);
}

template <int kRows>
// Three CTAs per SM (shared memory allows three 128-row CTAs); the bound
// also steers register allocation: 2.885 vs 2.919 ms per batched step
// against the unbounded build on one B200.
__global__ void __launch_bounds__(kThreads, 3) compact_chunk_kernel(const __grid_constant__ CompactAttention a) {
    grid_dependency_wait();

    extern __shared__ __align__(128) unsigned char smem[];
    ChunkShared<kRows>& sh = *reinterpret_cast<ChunkShared<kRows>*>(smem);
    float* ktile = reinterpret_cast<float*>(smem + shared_head<kRows>());
    float* vtile = ktile + kRows * kHeadDim;
    const int64_t c = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int64_t len = sequence_length(a, b);
    const int64_t start = c * kRows;
    if (start >= len) return;
    const int n = static_cast<int>(len - start < kRows ? len - start : kRows);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const size_t row0 = ((static_cast<size_t>(b) * kKVHeads + g) * a.cap + start) * kHeadDim;
    if (tid == 0) {
        sh.failed = 0;
        for (int i = 0; i < 2; ++i)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&sh.bar[i])) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        const uint32_t bytes = static_cast<uint32_t>(n) * kHeadDim * sizeof(float);
        const float* src[2] = {a.k + row0, a.v + row0};
        float* dst[2] = {ktile, vtile};
        for (int i = 0; i < 2; ++i) {
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&sh.bar[i])),
                         "r"(bytes)
                         : "memory");
            asm volatile(
                "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                    smem_u32(dst[i])),
                "l"(src[i]), "r"(bytes), "r"(smem_u32(&sh.bar[i]))
                : "memory");
        }
    }
    // Scores: 4-lane groups (8 per warp), one row each; lane (gl, l4) covers
    // the 16-byte chunks l4 + 4 m of a row, visiting m = (j + gl) % 4 at step
    // j so the 32 lanes of one load hit 8 distinct bank groups.  q (pre-scaled
    // to base-2 units) is loaded in the same rotated order.
    const int l4 = lane & 3, gl = lane >> 2;
    const float scale2 = a.scale * kLog2e;
    float4 q[kGroup][4];
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
        const float4* qh = reinterpret_cast<const float4*>(a.q + (static_cast<size_t>(b) * kQHeads + g * kGroup + h) * kHeadDim);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float4 v = qh[l4 + 4 * ((j + gl) & 3)];
            v.x *= scale2;
            v.y *= scale2;
            v.z *= scale2;
            v.w *= scale2;
            q[h][j] = v;
        }
    }
    __syncthreads();  // barriers initialised
    if (!wait_landed(&sh.bar[0])) sh.failed = 1;
    float mloc[kGroup] = {-INFINITY, -INFINITY, -INFINITY};
    for (int r0 = warp * 8; r0 < n; r0 += 8 * kWarps) {  // warp-uniform: full-mask shuffles
        const int r = r0 + gl;
        const float4* k4 = reinterpret_cast<const float4*>(ktile + (r < n ? r : r0) * kHeadDim);
        float d[kGroup] = {0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float4 kv = k4[l4 + 4 * ((j + gl) & 3)];
#pragma unroll
            for (int h = 0; h < kGroup; ++h) {
                d[h] = fmaf(q[h][j].x, kv.x, d[h]);
                d[h] = fmaf(q[h][j].y, kv.y, d[h]);
                d[h] = fmaf(q[h][j].z, kv.z, d[h]);
                d[h] = fmaf(q[h][j].w, kv.w, d[h]);
            }
        }
#pragma unroll
        for (int off = 1; off < 4; off <<= 1)
#pragma unroll
            for (int h = 0; h < kGroup; ++h) d[h] += __shfl_xor_sync(0xffffffffu, d[h], off);
        if (r < n) {
#pragma unroll
            for (int h = 0; h < kGroup; ++h) mloc[h] = fmaxf(mloc[h], d[h]);
            if (l4 < kGroup) sh.p[l4][r] = l4 == 0 ? d[0] : (l4 == 1 ? d[1] : d[2]);
        }
    }
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
        mloc[h] = warp_max(mloc[h]);
        if (lane == 0) sh.wmax[warp][h] = mloc[h];
    }
    __syncthreads();
    float m[kGroup], lsum[kGroup];
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
        float v = lane < kWarps ? sh.wmax[lane][h] : -INFINITY;
        m[h] = warp_max(v);
        lsum[h] = 0.0f;
    }
    for (int r = tid; r < n; r += kThreads)
#pragma unroll
        for (int h = 0; h < kGroup; ++h) {
            const float e = exp2f(sh.p[h][r] - m[h]);
            sh.p[h][r] = e;
            lsum[h] += e;
        }
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
        lsum[h] = warp_sum(lsum[h]);
        if (lane == 0) sh.wsum[warp][h] = lsum[h];
    }
    if (!wait_landed(&sh.bar[1])) sh.failed = 1;
    __syncthreads();
    // P.V: thread (quad, head, split) sums rows split, split + 5, ...
    const int pq = tid & 15, ph = (tid >> 4) % kGroup, psplit = tid / (16 * kGroup);
    if (psplit < kSplits) {
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        float4 acc2 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        const float* prow = sh.p[ph];
        int r = psplit;
        for (; r + kSplits < n; r += 2 * kSplits) {
            const float p0 = prow[r], p1 = prow[r + kSplits];
            const float4 v0 = reinterpret_cast<const float4*>(vtile + r * kHeadDim)[pq];
            const float4 v1 = reinterpret_cast<const float4*>(vtile + (r + kSplits) * kHeadDim)[pq];
            acc.x = fmaf(p0, v0.x, acc.x);
            acc.y = fmaf(p0, v0.y, acc.y);
            acc.z = fmaf(p0, v0.z, acc.z);
            acc.w = fmaf(p0, v0.w, acc.w);
            acc2.x = fmaf(p1, v1.x, acc2.x);
            acc2.y = fmaf(p1, v1.y, acc2.y);
            acc2.z = fmaf(p1, v1.z, acc2.z);
            acc2.w = fmaf(p1, v1.w, acc2.w);
        }
        if (r < n) {
            const float p0 = prow[r];
            const float4 v0 = reinterpret_cast<const float4*>(vtile + r * kHeadDim)[pq];
            acc.x = fmaf(p0, v0.x, acc.x);
            acc.y = fmaf(p0, v0.y, acc.y);
            acc.z = fmaf(p0, v0.z, acc.z);
            acc.w = fmaf(p0, v0.w, acc.w);
        }
        acc.x += acc2.x;
        acc.y += acc2.y;
        acc.z += acc2.z;
        acc.w += acc2.w;
        reinterpret_cast<float4*>(sh.o[psplit][ph])[pq] = acc;
    }
    __syncthreads();
    if (tid < kGroup * kHeadDim) {
        const int h = tid / kHeadDim, d = tid % kHeadDim;
        float o = 0.0f;
#pragma unroll
        for (int s = 0; s < kSplits; ++s) o += sh.o[s][h][d];
        float* w = a.ws + ((static_cast<size_t>(b) * kQHeads + g * kGroup + h) * a.chunks + c) * kPart;
        if (sh.failed) o = __int_as_float(0x7fc00000);
        w[2 + d] = o;
        if (d == 0) {
            float total = 0.0f;
#pragma unroll
            for (int w8 = 0; w8 < kWarps; ++w8) total += sh.wsum[w8][h];
            w[0] = (h == 0 ? m[0] : (h == 1 ? m[1] : m[2])) * kLn2;  // natural-log units
            w[1] = total;
        }
    }
    if (tid == 0 && sh.failed && a.error != nullptr) atomicOr(a.error, 1u);
    if (a.counters == nullptr) return;
    // The last chunk CTA of (b, g) to arrive merges the 3 heads over every
    // chunk, in chunk order (the merge kernel's arithmetic: bitwise the same
    // result whichever CTA is last), then rearms the counter.
    const int active = static_cast<int>((len + kRows - 1) / kRows);
    __syncthreads();  // this CTA's partials are written
    if (tid == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(&a.counters[b * kKVHeads + g], 1u);
        sh.last = prev + 1 == static_cast<unsigned>(active) ? 1 : 0;
    }
    __syncthreads();
    if (!sh.last) return;
    __threadfence();
    float* weight = ktile;  // [3][active], the K / V tiles are no longer needed
    const int mh = tid / kHeadDim, d = tid % kHeadDim, mw = (tid % kHeadDim) >> 5;
    const bool merger = tid < kGroup * kHeadDim;
    const float* w = a.ws + (static_cast<size_t>(b) * kQHeads + g * kGroup + (merger ? mh : 0)) * a.chunks * kPart;
    float mx = -INFINITY;
    if (merger)
        for (int cc = d; cc < active; cc += kHeadDim) mx = fmaxf(mx, __ldcg(w + static_cast<size_t>(cc) * kPart));
    mx = warp_max(mx);
    if (merger && lane == 0) sh.mscr[mh][mw] = mx;
    __syncthreads();
    mx = merger ? fmaxf(sh.mscr[mh][0], sh.mscr[mh][1]) : 0.0f;
    float total = 0.0f;
    if (merger)
        for (int cc = d; cc < active; cc += kHeadDim) {
            const float f = expf(__ldcg(w + static_cast<size_t>(cc) * kPart) - mx);
            weight[mh * active + cc] = f;
            total = fmaf(__ldcg(w + static_cast<size_t>(cc) * kPart + 1), f, total);
        }
    total = warp_sum(total);
    if (merger && lane == 0) sh.tscr[mh][mw] = total;
    __syncthreads();
    if (!merger) return;
    total = sh.tscr[mh][0] + sh.tscr[mh][1];
    const float* wf = weight + mh * active;
    float acc = 0.0f, acc2 = 0.0f;
    int cc = 0;
    for (; cc + 1 < active; cc += 2) {
        acc = fmaf(__ldcg(w + static_cast<size_t>(cc) * kPart + 2 + d), wf[cc], acc);
        acc2 = fmaf(__ldcg(w + static_cast<size_t>(cc + 1) * kPart + 2 + d), wf[cc + 1], acc2);
    }
    if (cc < active) acc = fmaf(__ldcg(w + static_cast<size_t>(cc) * kPart + 2 + d), wf[cc], acc);
    a.out[(static_cast<size_t>(b) * kQHeads + g * kGroup + mh) * kHeadDim + d] = (acc + acc2) / total;
    if (tid == 0) a.counters[b * kKVHeads + g] = 0u;
}

// grid (B * 9), 64 threads: combine the active chunks of one (sequence, q
// head).  The chunk weights exp(m_c - max) / sum are computed once per chunk
// (cooperatively) into shared memory, then thread d sums o_c[d] over chunks.
__global__ void __launch_bounds__(kHeadDim) compact_merge_kernel(const __grid_constant__ CompactAttention a) {
    grid_dependency_wait();

    __shared__ float weight[kMergeMaxChunks];
    __shared__ float scratch[2];
    const int64_t bh = blockIdx.x, b = bh / kQHeads;
    const int rows = a.chunk_rows;
    const int active = static_cast<int>((sequence_length(a, b) + rows - 1) / rows);
    const float* w = a.ws + bh * a.chunks * kPart;
    const int d = threadIdx.x, lane = d & 31, warp = d >> 5;
    float m = -INFINITY;
    for (int c = d; c < active; c += kHeadDim) m = fmaxf(m, w[static_cast<size_t>(c) * kPart]);
    m = warp_max(m);
    if (lane == 0) scratch[warp] = m;
    __syncthreads();
    m = fmaxf(scratch[0], scratch[1]);
    __syncthreads();
    float total = 0.0f;
    for (int c = d; c < active; c += kHeadDim) {
        const float f = expf(w[static_cast<size_t>(c) * kPart] - m);
        weight[c] = f;
        total = fmaf(w[static_cast<size_t>(c) * kPart + 1], f, total);
    }
    total = warp_sum(total);
    if (lane == 0) scratch[warp] = total;
    __syncthreads();
    total = scratch[0] + scratch[1];
    float acc = 0.0f, acc2 = 0.0f;
    int c = 0;
    for (; c + 1 < active; c += 2) {
        acc = fmaf(w[static_cast<size_t>(c) * kPart + 2 + d], weight[c], acc);
        acc2 = fmaf(w[static_cast<size_t>(c + 1) * kPart + 2 + d], weight[c + 1], acc2);
    }
    if (c < active) acc = fmaf(w[static_cast<size_t>(c) * kPart + 2 + d], weight[c], acc);
    a.out[bh * kHeadDim + d] = (acc + acc2) / total;
}

}  // namespace

namespace {

template <int kRows>
fx_status launch_chunks(const CompactAttention& a, dim3 grid, cudaStream_t stream, bool dependent) {
    const fx_status st = raise_smem_limit(reinterpret_cast<const void*>(compact_chunk_kernel<kRows>), chunk_smem<kRows>(),
                                          "raising attention shared memory");
    if (st != FX_OK) return st;
    if (dependent)
        return launch_dependent(compact_chunk_kernel<kRows>, grid, dim3(kThreads), chunk_smem<kRows>(), stream,
                                "launching compact attention chunks", a);
    compact_chunk_kernel<kRows><<<grid, kThreads, chunk_smem<kRows>(), stream>>>(a);
    FX_CUDA_TRY(cudaGetLastError(), "launching compact attention chunks");
    return FX_OK;
}

}  // namespace

fx_status launch_compact_attention(const CompactAttention& a, cudaStream_t stream, bool dependent, bool merge) {
    FX_REQUIRE(a.chunk_rows == 64 || a.chunk_rows == 128, "flux attention: chunks are 64 or 128 rows");
    FX_REQUIRE(a.batch >= 1 && a.batch <= 65535 && a.chunks >= 1 && a.chunks <= kMergeMaxChunks &&
                   a.chunks * a.chunk_rows >= a.cap,
               "flux attention: batch or capacity out of range");
    const dim3 grid(static_cast<unsigned>(a.chunks), kKVHeads, static_cast<unsigned>(a.batch));
    const dim3 merge_grid(static_cast<unsigned>(a.batch * kQHeads));
    const fx_status st = a.chunk_rows == 128 ? launch_chunks<128>(a, grid, stream, dependent)
                                             : launch_chunks<64>(a, grid, stream, dependent);
    if (st != FX_OK || a.counters != nullptr || !merge) return st;
    if (dependent)
        return launch_dependent(compact_merge_kernel, merge_grid, dim3(kHeadDim), 0, stream,
                                "launching compact attention merge", a);
    compact_merge_kernel<<<merge_grid, kHeadDim, 0, stream>>>(a);
    FX_CUDA_TRY(cudaGetLastError(), "launching compact attention merge");
    return FX_OK;
}

}  // namespace fx
