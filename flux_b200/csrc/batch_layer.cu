// The work between two attention launches of the batched decode step, as one
// cooperative launch of G CTAs (one per SM, 512 threads): the same layer
// boundary that packed_qkv_rope_cache, residual_rmsnorm,
// packed_gate_up_gemv + packed_swiglu and the o_proj / down GEMVs cover in
// the reference's batch-1 runtime (native_decode_runtime_cuda.cu:1042-1098),
// here for B <= 64 independent sequences at once.
//
// Phases (middle launch, layer l), separated by bounded grid barriers:
//   C  attn = the merge of layer l's attention chunks (one warp per
//      (sequence, q head): max, weights exp(m_c - max), sum of l_c and o_c)
//   D  h2 = h + attn . o_proj^T          CTA c owns output columns [n0, n1)
//   E  act = swiglu(norm(h2) . gate^T, norm(h2) . up^T)   features [f0, f1)
//   F  h = h2 + act . down^T             output columns [n0, n1)
//   A  layer l + 1: norm(h) . qkv^T for its row pairs, RoPE at each
//      sequence's own position, q out, K / V rows into the cache
// The first launch runs A on the embedding rows; the last runs C, D, E, F
// and writes the final-norm rows for the LM head.
//
// Each phase multiplies its activation rows by the CTA's weight slice.  The
// slice (<= 24 rows, padded pitch) lands in shared memory by 1-D bulk copies
// issued one phase ahead, as soon as the previous phase's products are done,
// so HBM streams it during that phase's epilogue and grid barrier.  The
// activation rows are staged by TMA 2-D boxes (32 columns x 64 rows, 128-byte
// swizzle: the 16-byte units of row b are permuted by b % 8, so the row groups
// of a warp's loads are bank-conflict-free) in 288-column chunks through two
// buffers, the next chunk in flight while one is multiplied.  Warp w takes a
// block of 2 R weight rows and a slice of the columns; lane (g, wg)
// accumulates batch rows g + 16 i (i < 4) x weight rows R wg .. R wg + R - 1
// in registers (R = 4 for gate/up and QKV, 2 for the 3-5 rows of o_proj and
// down); the K slices are summed in a fixed order after one barrier.  A row's result depends only on its own
// activations, never on the batch, and the sums run in a fixed order:
// deterministic and batch-invariant.
//
// The RMSNorms fold as in the persistent batch-1 step: the norm weight
// multiplies the weight slice in shared memory, and each dot product is
// scaled by the row's 1 / rms (from the staged rows) afterwards.
#include "batch_layer.cuh"
#include "tcgen05.cuh"

namespace fx {
namespace {

constexpr int kWarps = kLayerThreads / 32;                                    // 16
constexpr int kBoxCols = 32;                                                  // columns per TMA box (128 bytes)
constexpr int kChunk = 288;                                                   // columns per staged chunk
constexpr int kChunkBoxes = kChunk / kBoxCols;                                // 9
constexpr uint32_t kBoxBytes = kLayerMaxRows * kBoxCols * 4;                  // 8 KB
constexpr int kWs = kHidden + 4;                                              // weight row pitch, K = 576
constexpr int kWsDown = kInter + 4;                                           // weight row pitch, K = 1536
constexpr int kMaxOut = (kHidden + kLayerMinGrid - 1) / kLayerMinGrid;        // 5 columns of o_proj / down
constexpr int kMaxFeat = (kInter + kLayerMinGrid - 1) / kLayerMinGrid;        // 12 SwiGLU features
constexpr int kQkvTasks = kQKV / 2;                                           // 480 row pairs
constexpr int kMaxTasks = (kQkvTasks + kLayerMinGrid - 1) / kLayerMinGrid;    // 4
constexpr int kWFloats = 2 * kMaxFeat * kWs;                                  // the largest slice (gate/up)
static_assert(kMaxOut * kWsDown <= kWFloats && 2 * kMaxTasks * kWs <= kWFloats, "weight slice buffer");
constexpr unsigned long long kWaitNs = 2000000000ull;                         // 2 s per wait
constexpr unsigned long long kPeerCheckNs = 1000000ull;                       // look at the error word after 1 ms
constexpr unsigned kErrPosition = 2u;
constexpr unsigned kErrWait = 16u;

struct LayerShared {
    // two chunk buffers, box j = columns 32 j.. of the chunk, rows swizzled;
    // after a phase's last chunk they hold the warps' K-slice sums
    float x[2][kChunkBoxes][kLayerMaxRows][kBoxCols];
    alignas(16) float w[kWFloats];                        // the phase's weight slice (padded rows)
    float ss[kLayerMaxRows];                              // sums of squares of the staged rows
    uint64_t xbar[2], wbar;                               // chunk buffers / weight slice landed
    volatile int abort;
};
constexpr size_t kLayerSmem = sizeof(LayerShared) + 1024;  // + alignment of the swizzled boxes
static_assert(kWarps * kLayerMaxRows * 8 <= 2 * kChunkBoxes * kLayerMaxRows * kBoxCols, "partials fit the chunks");

// ------------------------------------------------------------- PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
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

// 1-D bulk copy global -> shared completing on `bar` (16-byte aligned, size a multiple of 16; no multicast).
__device__ __forceinline__ void bulk_row(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned ld_relaxed(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// ------------------------------------------------------- bounded waits

// Every calling thread waits (bounded) for phase `parity` of an mbarrier;
// the caller's next barrier makes a give-up (sh.abort) uniform.
__device__ void wait_bar(LayerShared& sh, const BatchLayerArgs& a, uint64_t* bar, uint32_t parity) {
    if (mbar_test(bar, parity)) return;
    const unsigned long long t0 = now_ns();
    while (!mbar_test(bar, parity)) {
        if (sh.abort) return;
        const unsigned long long dt = now_ns() - t0;
        if (dt > kPeerCheckNs && (ld_relaxed(a.error) & kErrWait) != 0) {
            sh.abort = 1;
            return;
        }
        if (dt > kWaitNs) {
            atomicOr(a.error, kErrWait);
            sh.abort = 1;
            return;
        }
    }
}

// Grid barrier k of this launch: every CTA's writes before it are visible to
// every CTA after it, to its TMA loads as well.  Bounded; false (uniformly
// over the CTA) when this CTA or another gave up.
__device__ bool grid_sync(LayerShared& sh, const BatchLayerArgs& a, int k) {
    __syncthreads();
    if (threadIdx.x == 0 && !sh.abort) {
        __threadfence();
        atomicAdd(a.barrier + k, 1u);
        const unsigned long long t0 = now_ns();
        while (ld_acquire(a.barrier + k) < gridDim.x) {
            const unsigned long long dt = now_ns() - t0;
            if (dt > kPeerCheckNs && (ld_relaxed(a.error) & kErrWait) != 0) {
                sh.abort = 1;
                break;
            }
            if (dt > kWaitNs) {
                atomicOr(a.error, kErrWait);
                sh.abort = 1;
                break;
            }
        }
        __threadfence();
        asm volatile("fence.proxy.async.global;" ::: "memory");  // the TMA loads that follow see those writes
    }
    __syncthreads();
    return !sh.abort;
}

// ------------------------------------------------------------ staging

// The chunk buffers' uses: issued (thread 0) and waited for, per buffer
// (scalars, selected by the buffer index: no local-memory array).
struct Chunks {
    uint32_t issued0 = 0, issued1 = 0, used0 = 0, used1 = 0;
    __device__ __forceinline__ uint32_t& issued(int buf) { return buf ? issued1 : issued0; }
    __device__ __forceinline__ uint32_t& used(int buf) { return buf ? used1 : used0; }
};

// Address of the float4 of batch row b at float4 column c4 of chunk buffer
// `buf` (box c4 / 8, 16-byte unit c4 % 8 permuted by b % 8).
__device__ __forceinline__ float4* x_at(LayerShared& sh, int buf, int b, int c4) {
    return reinterpret_cast<float4*>(&sh.x[buf][c4 >> 3][b][((c4 & 7) ^ (b & 7)) << 2]);
}

// Thread 0: TMA boxes for chunk c (columns 288 c .. of a K-column `map`, rows
// 0..63) into buffer c % 2, completing on sh.xbar[c % 2].
__device__ void issue_chunk(LayerShared& sh, Chunks& ch, const CUtensorMap* map, int K, int c) {
    const int buf = c & 1, col0 = c * kChunk, boxes = min(kChunk, K - col0) / kBoxCols;
    ++ch.issued(buf);
    mbar_expect(&sh.xbar[buf], static_cast<uint32_t>(boxes) * kBoxBytes);
    for (int j = 0; j < boxes; ++j) tc::tma_box(&sh.x[buf][j][0][0], map, col0 + j * kBoxCols, 0, &sh.xbar[buf]);
}

// Thread 0: `nr` weight rows (row i from rows(i), k floats each) into the
// slice buffer at pitch ws, completing on sh.wbar (`issued` counts phases).
template <typename RowSrc>
__device__ void issue_w(LayerShared& sh, int nr, int k, int ws, RowSrc rows, uint32_t& issued) {
    ++issued;
    mbar_expect(&sh.wbar, static_cast<uint32_t>(nr * k * 4));
    for (int i = 0; i < nr; ++i)
        bulk_row(sh.w + static_cast<size_t>(i) * ws, rows(i), static_cast<uint32_t>(k * 4), &sh.wbar);
}

// sh.ss[b] (+)= sum of squares of row b of chunk buffer `buf` (ncols columns),
// 8 threads per row in a fixed order.
__device__ void row_squares(LayerShared& sh, int buf, int ncols, bool first) {
    const int t = threadIdx.x, b = t >> 3, c8 = t & 7;
    float ss = 0.0f;
    for (int c4 = c8; c4 < ncols / 4; c4 += 8) {
        const float4 v = *x_at(sh, buf, b, c4);
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
    }
    ss += __shfl_xor_sync(0xffffffffu, ss, 4);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    if (c8 == 0) sh.ss[b] = first ? ss : sh.ss[b] + ss;
}

// w[i][k] *= norm[k] for the slice's nr rows (pitch kWs, 576 columns).
__device__ void fold_norm(LayerShared& sh, int nr, const float* norm) {
    for (int e = threadIdx.x; e < nr * (kHidden / 4); e += kLayerThreads) {
        const int i = e / (kHidden / 4), c4 = e % (kHidden / 4);
        float4* p = reinterpret_cast<float4*>(sh.w + static_cast<size_t>(i) * kWs) + c4;
        const float4 n = __ldg(reinterpret_cast<const float4*>(norm) + c4);
        float4 v = *p;
        v.x *= n.x;
        v.y *= n.y;
        v.z *= n.z;
        v.w *= n.w;
        *p = v;
    }
}

// ------------------------------------------------------------ projection

struct Units {
    int nblk, nks, n;  // blocks of 2 R weight rows, K slices per block, working warps
};

template <int R>
__device__ __forceinline__ Units units_for(int nr) {
    Units u;
    u.nblk = (nr + 2 * R - 1) / (2 * R);
    u.nks = kWarps / u.nblk;
    u.n = u.nblk * u.nks;
    return u;
}

// This warp's products over chunk buffer `buf` (ncols columns; weight columns
// from kw0): weight rows blk * 2R + R wg + j (clamped to nr - 1; those
// results are dropped), batch rows g + 16 i, float4 columns of K slice ks.
template <int R>
__device__ __forceinline__ void gemm_chunk(const LayerShared& sh, int buf, int ws, int nr, int kw0, int ncols,
                                           float (&acc)[4][R]) {
    const Units u = units_for<R>(nr);
    const int warp = threadIdx.x >> 5;
    if (warp >= u.n) return;
    const int blk = warp / u.nks, ks = warp % u.nks;
    const int n4 = ncols >> 2, k4a = ks * n4 / u.nks, k4b = (ks + 1) * n4 / u.nks;
    const int lane = threadIdx.x & 31, g = lane & 15, wg = lane >> 4;
    const float4* wp[R];
#pragma unroll
    for (int j = 0; j < R; ++j)
        wp[j] = reinterpret_cast<const float4*>(sh.w + static_cast<size_t>(min(blk * 2 * R + R * wg + j, nr - 1)) * ws +
                                                kw0);
    const int sw = g & 7;  // (g + 16 i) % 8
    const float* xrow = &sh.x[buf][0][g][0];
#pragma unroll 2
    for (int k4 = k4a; k4 < k4b; ++k4) {
        float4 wv[R], xv[4];
#pragma unroll
        for (int j = 0; j < R; ++j) wv[j] = wp[j][k4];
        const float* xb = xrow + (k4 >> 3) * (kLayerMaxRows * kBoxCols) + (((k4 & 7) ^ sw) << 2);
#pragma unroll
        for (int i = 0; i < 4; ++i) xv[i] = *reinterpret_cast<const float4*>(xb + 16 * i * kBoxCols);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < R; ++j) {
                acc[i][j] = fmaf(xv[i].x, wv[j].x, acc[i][j]);
                acc[i][j] = fmaf(xv[i].y, wv[j].y, acc[i][j]);
                acc[i][j] = fmaf(xv[i].z, wv[j].z, acc[i][j]);
                acc[i][j] = fmaf(xv[i].w, wv[j].w, acc[i][j]);
            }
    }
}

// The warps' K-slice sums of the phase's products (they replace the staged
// chunks, which are consumed by then; a barrier follows before unit_sum).
template <int R>
__device__ __forceinline__ void store_partials(LayerShared& sh, int nr, const float (&acc)[4][R]) {
    const int warp = threadIdx.x >> 5;
    if (warp >= units_for<R>(nr).n) return;
    float* part = &sh.x[0][0][0][0] + warp * (kLayerMaxRows * 2 * R);
    const int lane = threadIdx.x & 31, g = lane & 15, wg = lane >> 4;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < R; ++j) part[(g + 16 * i) * 2 * R + R * wg + j] = acc[i][j];
}

// Output (batch row b, weight row r): its K slices in order.
template <int R>
__device__ __forceinline__ float unit_sum(const LayerShared& sh, int nr, int b, int r) {
    const Units u = units_for<R>(nr);
    constexpr int kPart = kLayerMaxRows * 2 * R;
    const float* p = &sh.x[0][0][0][0] + (r / (2 * R)) * u.nks * kPart + b * 2 * R + r % (2 * R);
    float v = 0.0f;
    for (int ks = 0; ks < u.nks; ++ks) v += p[ks * kPart];
    return v;
}

// The products of a K-column activation matrix (TMA `map`, chunks 0 and 1
// already issued) with the slice's nr weight rows (pitch ws), chunk by chunk
// through the two buffers; with want_ss, sh.ss gets the rows' sums of squares.
// Ends with the K-slice sums stored and published by a barrier.
template <int R>
__device__ void project(LayerShared& sh, const BatchLayerArgs& a, Chunks& ch, const CUtensorMap* map, int K, int ws,
                        int nr, bool want_ss) {
    float acc[4][R];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < R; ++j) acc[i][j] = 0.0f;
    const int nch = (K + kChunk - 1) / kChunk;
    for (int c = 0; c < nch; ++c) {
        const int buf = c & 1, nc = min(kChunk, K - c * kChunk);
        wait_bar(sh, a, &sh.xbar[buf], ch.used(buf)++ & 1u);
        if (want_ss) row_squares(sh, buf, nc, c == 0);
        gemm_chunk<R>(sh, buf, ws, nr, c * kChunk, nc, acc);
        __syncthreads();  // buffer `buf` is free again
        if (threadIdx.x == 0 && c + 2 < nch && !sh.abort) issue_chunk(sh, ch, map, K, c + 2);
    }
    store_partials<R>(sh, nr, acc);
    __syncthreads();
}

// Packed-QKV task -> its two rows: q / k pairs (d, d + 32) for RoPE, v pairs (2t, 2t + 1).
__device__ __forceinline__ void task_rows(int task, int& ra, int& rb) {
    if (task < 288) {
        ra = (task >> 5) * kHeadDim + (task & 31);
        rb = ra + kHeadDim / 2;
    } else if (task < 384) {
        const int t = task - 288;
        ra = kHidden + (t >> 5) * kHeadDim + (t & 31);
        rb = ra + kHeadDim / 2;
    } else {
        ra = kHidden + kKVHeads * kHeadDim + 2 * (task - 384);
        rb = ra + 1;
    }
}

// ------------------------------------------------------------------ kernel

__global__ void __launch_bounds__(kLayerThreads, 1) batch_layer_kernel(const __grid_constant__ BatchLayerArgs a) {
    extern __shared__ unsigned char layer_raw[];
    LayerShared& sh = *reinterpret_cast<LayerShared*>(layer_raw + ((1024u - (smem_u32(layer_raw) & 1023u)) & 1023u));
    const int tid = threadIdx.x, G = gridDim.x, cta = blockIdx.x;
    const int B = a.rows;
    const int n0 = cta * kHidden / G, n1 = (cta + 1) * kHidden / G, nr = n1 - n0;
    const int f0 = cta * kInter / G, f1 = (cta + 1) * kInter / G, nf = f1 - f0;
    const int t0 = cta * kQkvTasks / G, t1 = (cta + 1) * kQkvTasks / G, nt = t1 - t0;
    const bool proj = a.mode != kLayerFirst;  // D, E, F
    const bool qkv = a.mode != kLayerLast;    // A
    Chunks ch;
    uint32_t wused = 0, wissued = 0;  // weight-slice phases waited for / issued (thread 0)
    auto qkv_rows = [&](int i) {
        int ra, rb;
        task_rows(t0 + i / 2, ra, rb);
        return a.next_qkv + static_cast<size_t>(i % 2 == 0 ? ra : rb) * kHidden;
    };

    if (tid == 0) {
        mbar_init(&sh.xbar[0], 1);
        mbar_init(&sh.xbar[1], 1);
        mbar_init(&sh.wbar, 1);
        sh.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        // weights do not depend on the previous kernel: they stream in while it drains
        if (proj)
            issue_w(sh, nr, kHidden, kWs, [&](int i) { return a.o_proj + static_cast<size_t>(n0 + i) * kHidden; },
                    wissued);
        else
            issue_w(sh, 2 * nt, kHidden, kWs, qkv_rows, wissued);
    }
    grid_dependency_wait();  // the previous kernels' attention chunks, residual rows, positions
    __syncthreads();

    if (proj) {
        // Thread e < B * nr owns output (b, n0 + r) = (e / nr, e % nr) of D
        // and F: it holds h (prefetched now) and then h2 in registers.
        const bool owner = tid < B * nr;
        const size_t at = owner ? static_cast<size_t>(tid / nr) * kHidden + n0 + tid % nr : 0;
        const float h_in = owner ? __ldcg(a.h + at) : 0.0f;
        float h2v = 0.0f;

        // ------------------------------------------------ C: attn = merge of layer l's attention chunks
        {
            const int warp = tid >> 5, lane = tid & 31;
            for (int p = warp * G + cta; p < B * kQHeads; p += G * kWarps) {
                const int64_t len = min(max(a.lengths[p / kQHeads], static_cast<int64_t>(1)), a.cap);
                const int active = static_cast<int>((len + a.attn_rows - 1) / a.attn_rows);
                const float* w = a.attn_ws + static_cast<size_t>(p) * a.attn_chunks * (kHeadDim + 2);
                float m = -INFINITY;
                for (int c = lane; c < active; c += 32) m = fmaxf(m, __ldcg(w + static_cast<size_t>(c) * (kHeadDim + 2)));
                m = warp_max(m);
                float total = 0.0f, acc0 = 0.0f, acc1 = 0.0f;
                for (int c0 = 0; c0 < active; c0 += 32) {
                    const int c = c0 + lane;
                    const float* wc = w + static_cast<size_t>(c) * (kHeadDim + 2);
                    const float f = c < active ? expf(__ldcg(wc) - m) : 0.0f;
                    if (c < active) total = fmaf(__ldcg(wc + 1), f, total);
                    const int n = min(32, active - c0);
                    const float* o = w + static_cast<size_t>(c0) * (kHeadDim + 2) + 2 + lane;
                    int j = 0;
                    for (; j + 8 <= n; j += 8) {  // 16 loads in flight per lane
                        float v0[8], v1[8];
#pragma unroll
                        for (int u = 0; u < 8; ++u) {
                            v0[u] = __ldcg(o + static_cast<size_t>(j + u) * (kHeadDim + 2));
                            v1[u] = __ldcg(o + static_cast<size_t>(j + u) * (kHeadDim + 2) + 32);
                        }
#pragma unroll
                        for (int u = 0; u < 8; ++u) {
                            const float fj = __shfl_sync(0xffffffffu, f, j + u);
                            acc0 = fmaf(v0[u], fj, acc0);
                            acc1 = fmaf(v1[u], fj, acc1);
                        }
                    }
                    for (; j < n; ++j) {
                        const float fj = __shfl_sync(0xffffffffu, f, j);
                        acc0 = fmaf(__ldcg(o + static_cast<size_t>(j) * (kHeadDim + 2)), fj, acc0);
                        acc1 = fmaf(__ldcg(o + static_cast<size_t>(j) * (kHeadDim + 2) + 32), fj, acc1);
                    }
                }
                total = warp_sum(total);
                a.attn[static_cast<size_t>(p) * kHeadDim + lane] = acc0 / total;
                a.attn[static_cast<size_t>(p) * kHeadDim + lane + 32] = acc1 / total;
            }
        }
        if (!grid_sync(sh, a, 0)) goto done;

        // ------------------------------------------------ D: h2 = h + attn . o_proj^T
        if (tid == 0) {
            issue_chunk(sh, ch, &a.maps.attn, kHidden, 0);
            issue_chunk(sh, ch, &a.maps.attn, kHidden, 1);
        }
        wait_bar(sh, a, &sh.wbar, wused++ & 1u);
        project<2>(sh, a, ch, &a.maps.attn, kHidden, kWs, nr, false);
        if (sh.abort) goto done;
        if (tid == 0)  // the gate/up slice streams in during the epilogue and the grid barrier
            issue_w(
                sh, 2 * nf, kHidden, kWs,
                [&](int i) {
                    const int row = i < nf ? f0 + i : kInter + f0 + (i - nf);
                    return a.gate_up + static_cast<size_t>(row) * kHidden;
                },
                wissued);
        if (owner) {
            h2v = h_in + unit_sum<2>(sh, nr, tid / nr, tid % nr);
            a.h2[at] = h2v;
        }
        if (!grid_sync(sh, a, 1)) goto done;

        // ------------------------------------------------ E: act = swiglu(norm(h2) . gate, norm(h2) . up)
        if (tid == 0) {
            issue_chunk(sh, ch, &a.maps.h2, kHidden, 0);
            issue_chunk(sh, ch, &a.maps.h2, kHidden, 1);
        }
        wait_bar(sh, a, &sh.wbar, wused++ & 1u);
        fold_norm(sh, 2 * nf, a.post_norm);
        __syncthreads();
        project<4>(sh, a, ch, &a.maps.h2, kHidden, kWs, 2 * nf, true);
        if (sh.abort) goto done;
        if (tid == 0)
            issue_w(sh, nr, kInter, kWsDown, [&](int i) { return a.down + static_cast<size_t>(n0 + i) * kInter; },
                    wissued);
        for (int e = tid; e < B * nf; e += kLayerThreads) {
            const int b = e / nf, f = e % nf;
            const float inv = rsqrtf(sh.ss[b] / static_cast<float>(kHidden) + a.eps);
            const float gv = unit_sum<4>(sh, 2 * nf, b, f) * inv;
            const float uv = unit_sum<4>(sh, 2 * nf, b, nf + f) * inv;
            a.act[static_cast<size_t>(b) * kInter + f0 + f] = swiglu(gv, uv);
        }
        if (!grid_sync(sh, a, 2)) goto done;

        // ------------------------------------------------ F: h = h2 + act . down^T
        if (tid == 0) {
            issue_chunk(sh, ch, &a.maps.act, kInter, 0);
            issue_chunk(sh, ch, &a.maps.act, kInter, 1);
        }
        wait_bar(sh, a, &sh.wbar, wused++ & 1u);
        project<2>(sh, a, ch, &a.maps.act, kInter, kWsDown, nr, false);
        if (sh.abort) goto done;
        if (tid == 0 && qkv) issue_w(sh, 2 * nt, kHidden, kWs, qkv_rows, wissued);
        if (owner) a.h[at] = h2v + unit_sum<2>(sh, nr, tid / nr, tid % nr);
        if (!grid_sync(sh, a, 3)) goto done;
    }

    if (qkv) {
        // ------------------------------------------------ A: norm(h) . qkv^T, RoPE, q and cache rows
        if (a.mode == kLayerFirst) {
            // the embedding rows (zeros for an out-of-range token) staged by
            // the threads (a gather: TMA boxes take contiguous rows) into
            // both chunk buffers, as if two chunks had landed; CTA 0 also
            // starts the residual stream with them
            const int b = tid >> 3, c8 = tid & 7;
            const int64_t tok = b < B ? a.tokens[b] : -1;
            const float* src = tok >= 0 && tok < a.vocab ? a.embedding + tok * kHidden : nullptr;
            for (int c4 = c8; c4 < kHidden / 4; c4 += 8) {
                const float4 v = src != nullptr ? __ldg(reinterpret_cast<const float4*>(src) + c4)
                                                : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                *x_at(sh, c4 / (kChunk / 4), b, c4 % (kChunk / 4)) = v;
                if (cta == 0 && b < B) reinterpret_cast<float4*>(a.h + static_cast<size_t>(b) * kHidden)[c4] = v;
            }
            if (tid == 0) {  // complete one phase of each chunk barrier (no bytes)
                ++ch.issued0;
                ++ch.issued1;
                mbar_expect(&sh.xbar[0], 0);
                mbar_expect(&sh.xbar[1], 0);
            }
        } else if (tid == 0) {
            issue_chunk(sh, ch, &a.maps.h, kHidden, 0);
            issue_chunk(sh, ch, &a.maps.h, kHidden, 1);
        }
        wait_bar(sh, a, &sh.wbar, wused++ & 1u);
        fold_norm(sh, 2 * nt, a.next_norm);
        __syncthreads();
        project<4>(sh, a, ch, &a.maps.h, kHidden, kWs, 2 * nt, true);
        if (sh.abort) goto done;
        for (int e = tid; e < B * nt; e += kLayerThreads) {
            const int b = e / nt, j = e % nt;
            const int64_t pos = a.positions[b];
            if (pos < 0 || pos >= a.cap) {
                if (j == 0) atomicOr(a.error, kErrPosition);
                continue;
            }
            if (cta == 0 && j == 0) a.lengths[b] = pos + 1;
            const float inv = rsqrtf(sh.ss[b] / static_cast<float>(kHidden) + a.eps);
            const float ya = unit_sum<4>(sh, 2 * nt, b, 2 * j) * inv;
            const float yb = unit_sum<4>(sh, 2 * nt, b, 2 * j + 1) * inv;
            const int task = t0 + j;
            int ra, rb;
            task_rows(task, ra, rb);
            if (task < 384) {
                const int d = ra % kHeadDim;  // < 32: partner d + 32
                const float* c = a.rope_cos + pos * kHeadDim;
                const float* s = a.rope_sin + pos * kHeadDim;
                const float r1 = rope_value(ya, yb, c[d], s[d], true);
                const float r2 = rope_value(yb, ya, c[d + kHeadDim / 2], s[d + kHeadDim / 2], false);
                if (task < 288) {
                    float* q = a.q + static_cast<size_t>(b) * kHidden + ra;
                    q[0] = r1;
                    q[kHeadDim / 2] = r2;
                } else {
                    const int kv = (ra - kHidden) / kHeadDim;
                    float* k = a.key_cache + ((static_cast<size_t>(b) * kKVHeads + kv) * a.cap + pos) * kHeadDim + d;
                    k[0] = r1;
                    k[kHeadDim / 2] = r2;
                }
            } else {
                const int u = ra - kHidden - kKVHeads * kHeadDim;  // even: u, u + 1 in one head
                float* v = a.value_cache +
                           ((static_cast<size_t>(b) * kKVHeads + u / kHeadDim) * a.cap + pos) * kHeadDim + u % kHeadDim;
                v[0] = ya;
                v[1] = yb;
            }
        }
    } else {
        // ------------------------------------------------ the final norm rows (LM-head input)
        for (int b = cta; b < B; b += G) {
            const float* hr = a.h + static_cast<size_t>(b) * kHidden;
            const float x0 = tid < kHidden ? __ldcg(hr + tid) : 0.0f;
            const float x1 = tid + kLayerThreads < kHidden ? __ldcg(hr + tid + kLayerThreads) : 0.0f;
            const float ss = block_sum(fmaf(x0, x0, x1 * x1), sh.ss);
            const float inv = rsqrtf(ss / static_cast<float>(kHidden) + a.eps);
            float* out = a.norm_out + static_cast<size_t>(b) * kHidden;
            if (tid < kHidden) out[tid] = x0 * inv * a.next_norm[tid];
            if (tid + kLayerThreads < kHidden) out[tid + kLayerThreads] = x1 * inv * a.next_norm[tid + kLayerThreads];
            __syncthreads();
        }
    }
done:
    __syncthreads();
    if (tid == 0) {
        // copies issued but never waited for (after a give-up) land before the CTA leaves
        for (uint32_t i = wused; i < wissued; ++i) {
            const unsigned long long tw = now_ns();
            while (!mbar_test(&sh.wbar, i & 1u))
                if (now_ns() - tw > kWaitNs) break;
        }
        for (int buf = 0; buf < 2; ++buf)
            for (uint32_t i = ch.used(buf); i < ch.issued(buf); ++i) {
                const unsigned long long tw = now_ns();
                while (!mbar_test(&sh.xbar[buf], i & 1u))
                    if (now_ns() - tw > kWaitNs) break;
            }
    }
}

}  // namespace

size_t batch_layer_smem_bytes() { return kLayerSmem; }

fx_status prepare_batch_layer(int* grid) {
    const size_t smem = batch_layer_smem_bytes();
    const fx_status raised = raise_smem_limit(reinterpret_cast<const void*>(batch_layer_kernel), smem,
                                              "raising the batched layer kernel's shared memory");
    if (raised != FX_OK) return raised;
    int device = 0, sms = 0, per_sm = 0;
    FX_CUDA_TRY(cudaGetDevice(&device), "querying the device");
    FX_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device), "querying the SM count");
    FX_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, batch_layer_kernel, kLayerThreads, smem),
                "querying the batched layer kernel's occupancy");
    if (per_sm < 1 || sms < kLayerMinGrid) {
        set_error("flux batched decode: the layer kernel needs 128 co-resident CTAs of 512 threads");
        return FX_ERR_CUDA;
    }
    *grid = sms;
    return FX_OK;
}

fx_status launch_batch_layer(const BatchLayerArgs& a, int grid, cudaStream_t stream) {
    cudaLaunchConfig_t config{};
    config.gridDim = dim3(static_cast<unsigned>(grid));
    config.blockDim = dim3(kLayerThreads);
    config.dynamicSmemBytes = batch_layer_smem_bytes();
    config.stream = stream;
    cudaLaunchAttribute attributes[2]{};
    attributes[0].id = cudaLaunchAttributeCooperative;
    attributes[0].val.cooperative = 1;
    // a programmatic dependent launch: the weight prefetch of the prologue
    // overlaps the end of the previous kernel (grid_dependency_wait guards the rest)
    attributes[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attributes[1].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attributes;
    config.numAttrs = 2;
    FX_CUDA_TRY(cudaLaunchKernelEx(&config, batch_layer_kernel, a), "launching the batched layer kernel");
    return FX_OK;
}

}  // namespace fx
