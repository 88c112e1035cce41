// 3xTF32 projection GEMM on tcgen05 tensor cores (sm_100a).
//
// One CTA computes a 128 (weight rows) x BM (activation rows) tile of
// C = X . W^T over its K slice.  320 threads in three roles:
//   warp 0, lane 0  TMA producer: per 32-column stage, W_hi and W_lo boxes
//                   (128 x 32) and the raw X box (BM x 32), 128-byte
//                   swizzled, completing on full[stage];
//   warp 1          allocates 4 BM TMEM columns; lane 0 issues the MMAs
//                   (M = 128, N = BM, K = 8 per instruction, 3 products per
//                   K step), commits each stage back to empty[stage] and its
//                   hi.hi accumulator (fresh every second stage, two
//                   buffers) to acc_full;
//   warps 2-9       split the staged X tile in shared memory into hi (in
//                   place) and lo (a second buffer), publish it to the
//                   tensor core with fence.proxy.async, arrive on
//                   conv[stage]; they add the hi.hi accumulator of every
//                   second stage into FP32 registers (warp w reads TMEM
//                   lanes 32 (w % 4) .., half the columns), then the
//                   cross-term accumulator, and write C,
//                   transposed so each store is 32 consecutive floats of one
//                   output row.
// The operands are K-major with the canonical 128-byte swizzle: 8-row groups
// 1024 bytes apart (SBO), the 8-column K steps 32 bytes apart inside a row.
// Every mbarrier wait is bounded by %globaltimer; a wait that gives up sets
// bit 8 of the error word, stops the CTA's loops, lets copies and MMAs in
// flight finish (bounded), frees TMEM and returns.
#include "tc_gemm.cuh"
#include "tcgen05.cuh"

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>

namespace fx {
namespace {

using namespace tc;

constexpr int kTcThreads = 320;  // producer warp, MMA warp, 8 split/epilogue warps
constexpr int kTcEpi = kTcThreads - 64;
constexpr int kTcPromote = 2;    // stages per hi.hi accumulator before it is added into registers
constexpr uint32_t kWBox = kTcTileN * kTcTileK * 4;  // 16 KB

// Default stage counts: 4 for 64-row tiles, 3 for 128-row tiles.
constexpr int tc_default_stages(int bm) { return bm == 64 ? 4 : 3; }

template <int BM, int STAGES>
struct TcLayout {
    static constexpr uint32_t kX = BM * kTcTileK * 4;
    static constexpr uint32_t kStage = 2 * kWBox + 2 * kX;  // W_hi, W_lo, X (-> X_hi), X_lo
    static constexpr int kStages = STAGES;
    static constexpr size_t kSmem = static_cast<size_t>(kStages) * kStage + 1024 + 256;
    // TMEM columns: [0, BM) the cross terms, [BM, 2 BM) and [2 BM, 3 BM)
    // the per-stage hi.hi products (double-buffered); allocation 4 BM.
    static constexpr uint32_t kTmemCols = 4 * BM;
};

template <int BM, int STAGES>
__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm_kernel(const __grid_constant__ TcGemmArgs a) {
    using L = TcLayout<BM, STAGES>;
    constexpr int S = L::kStages;
    extern __shared__ unsigned char tc_raw[];
    unsigned char* smem = tc_raw + ((1024u - (smem_addr(tc_raw) & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * L::kStage);
    uint64_t* conv = full + S;
    uint64_t* empty = conv + S;
    uint64_t* acc_full = empty + S;   // [2] a stage's hi.hi products are in TMEM
    uint64_t* acc_empty = acc_full + 2;  // [2] the epilogue has taken them
    uint64_t* done = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int n0 = blockIdx.x * kTcTileN, m0 = blockIdx.y * BM;
    const int k0 = blockIdx.z * a.k_per_split;
    const int k1 = min(a.k, k0 + a.k_per_split);
    const int nk = k1 > k0 ? (k1 - k0 + kTcTileK - 1) / kTcTileK : 0;
    auto w_hi = [&](int s) { return smem + s * L::kStage; };
    auto w_lo = [&](int s) { return smem + s * L::kStage + kWBox; };
    auto x_hi = [&](int s) { return smem + s * L::kStage + 2 * kWBox; };
    auto x_lo = [&](int s) { return smem + s * L::kStage + 2 * kWBox + L::kX; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            bar_init(&full[s], 1);
            bar_init(&conv[s], kTcEpi);
            bar_init(&empty[s], 1);
        }
        for (int j = 0; j < 2; ++j) {
            bar_init(&acc_full[j], 1);
            bar_init(&acc_empty[j], kTcEpi);
        }
        bar_init(done, 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(L::kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int issued = 0;
            for (int i = 0; i < nk; ++i) {
                const int s = i % S;
                if (i >= S && !bar_wait(&empty[s], static_cast<uint32_t>(i / S - 1) & 1u, abort, a.error)) break;
                if (*abort) break;
                const int kx = k0 + i * kTcTileK;
                bar_expect(&full[s], 2 * kWBox + L::kX);
                tma_box(w_hi(s), &a.w_hi, kx, n0, &full[s]);
                tma_box(w_lo(s), &a.w_lo, kx, n0, &full[s]);
                if (i == 0) grid_dependency_wait();  // X comes from the previous kernel
                tma_box(x_hi(s), &a.x, kx, m0, &full[s]);
                issued = i + 1;
            }
            if (nk == 0) grid_dependency_wait();
            // Copies still in flight land before the CTA leaves (a no-op
            // unless a consumer gave up early).
            for (int i = max(0, issued - S); i < issued; ++i) {
                const unsigned long long t0 = now_ns();
                while (!bar_test(&full[i % S], static_cast<uint32_t>(i / S) & 1u))
                    if (now_ns() - t0 > kTcWaitNs) break;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = tf32_idesc(BM);
            for (int i = 0; i < nk; ++i) {
                const int s = i % S, g = i / kTcPromote, j = g & 1;
                const bool first = i % kTcPromote == 0, last = i % kTcPromote == kTcPromote - 1 || i == nk - 1;
                if (!bar_wait(&conv[s], static_cast<uint32_t>(i / S) & 1u, abort, a.error)) break;
                if (first && g >= 2 &&
                    !bar_wait(&acc_empty[j], static_cast<uint32_t>(g / 2 - 1) & 1u, abort, a.error))
                    break;
                fence_after_sync();
                const uint64_t ah = sw128_desc(smem_addr(w_hi(s))), al = sw128_desc(smem_addr(w_lo(s)));
                const uint64_t bh = sw128_desc(smem_addr(x_hi(s))), bl = sw128_desc(smem_addr(x_lo(s)));
                const uint32_t main_acc = tmem + static_cast<uint32_t>((1 + j) * BM);
#pragma unroll
                for (int kk = 0; kk < kTcTileK / 8; ++kk) {
                    const uint64_t step = static_cast<uint64_t>(kk * 32 >> 4);  // 8 TF32 = 32 bytes
                    mma_tf32(tmem, ah + step, bl + step, idesc, (i | kk) != 0 ? 1u : 0u);
                    mma_tf32(tmem, al + step, bh + step, idesc, 1u);
                    mma_tf32(main_acc, ah + step, bh + step, idesc, (!first || kk != 0) ? 1u : 0u);
                }
                mma_commit(&empty[s]);
                if (last) mma_commit(&acc_full[j]);
            }
            mma_commit(done);  // arrives once every MMA issued above has completed
        }
        __syncwarp();
    } else {
        // The tensor core's accumulation truncates, so a long chain of MMAs
        // into one accumulator drifts by about one unit in the last place
        // per step.  Every kTcPromote stages the hi.hi products start a
        // fresh accumulator and are added here in FP32 with
        // round-to-nearest; the cross terms (2^-11 of the result) stay in one
        // accumulator.  Warps w and w + 4 share TMEM lane quarter w % 4 and
        // take one half of the columns each.
        constexpr int kHalf = BM / 2;
        const int t = threadIdx.x - 64;  // 0..255
        const int quarter = warp & 3;
        const int c0 = (warp - 2) / 4 * kHalf;
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        const int groups = (nk + kTcPromote - 1) / kTcPromote;
        float acc[kHalf];
#pragma unroll
        for (int c = 0; c < kHalf; ++c) acc[c] = 0.0f;
        bool ok = true;
        int promoted = 0;
        auto promote = [&](int g) {
            const int j = g & 1;
            ok = ok && bar_wait(&acc_full[j], static_cast<uint32_t>(g / 2) & 1u, abort, a.error);
            __syncwarp();
            fence_after_sync();
#pragma unroll
            for (int col = 0; col < kHalf; col += 32) {
                float v[32];
                tmem_load32(tmem + lane_base + static_cast<uint32_t>((1 + j) * BM + c0 + col), v);
#pragma unroll
                for (int c = 0; c < 32; ++c) acc[col + c] += v[c];
            }
            fence_before_sync();
            bar_arrive(&acc_empty[j]);
        };
        for (int i = 0; i < nk && ok; ++i) {
            const int s = i % S;
            if (!bar_wait(&full[s], static_cast<uint32_t>(i / S) & 1u, abort, a.error)) {
                ok = false;
                break;
            }
            float4* xh = reinterpret_cast<float4*>(x_hi(s));
            float4* xl = reinterpret_cast<float4*>(x_lo(s));
#pragma unroll
            for (int q = t; q < BM * kTcTileK / 4; q += kTcEpi) {
                // integer-ALU rounding (the conversion pipe is quarter rate)
                const float4 v = xh[q];
                float4 h, r;
                h.x = tf32_round_int(v.x);
                h.y = tf32_round_int(v.y);
                h.z = tf32_round_int(v.z);
                h.w = tf32_round_int(v.w);
                r.x = tf32_round_int(v.x - h.x);
                r.y = tf32_round_int(v.y - h.y);
                r.z = tf32_round_int(v.z - h.z);
                r.w = tf32_round_int(v.w - h.w);
                xh[q] = h;
                xl[q] = r;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            bar_arrive(&conv[s]);
            if (promoted < i / kTcPromote) promote(promoted++);
        }
        while (ok && promoted < groups) promote(promoted++);
        grid_dependency_wait();  // the residual and C belong to earlier kernels too
        ok = ok && bar_wait(done, 0, abort, a.error) && !*abort;
        __syncwarp();
        fence_after_sync();
        const int n = n0 + quarter * 32 + lane;
        float* c = a.c + static_cast<long long>(blockIdx.z) * a.split_stride;
#pragma unroll
        for (int col = 0; col < kHalf; col += 32) {
            float v[32];
            if (nk > 0) {
                tmem_load32(tmem + lane_base + static_cast<uint32_t>(c0 + col), v);
            } else {
#pragma unroll
                for (int q = 0; q < 32; ++q) v[q] = 0.0f;
            }
            if (ok && n < a.n) {
#pragma unroll
                for (int q = 0; q < 32; ++q) {
                    const int m = m0 + c0 + col + q;
                    if (m < a.m) {
                        const long long at = static_cast<long long>(m) * a.ldc + n;
                        const float r = acc[col + q] + v[q];
                        c[at] = a.residual != nullptr ? r + a.residual[at] : r;
                    }
                }
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::kTmemCols)
                     : "memory");
    }
}

// Persistent form for large M (the prefill's projections, 128-row tiles, no
// K split): one CTA per SM walks the tiles t = blockIdx.x + u * gridDim.x
// (weight block fastest), so the TMA ring, TMEM and the barriers persist
// across tiles and a tile's first loads are issued while the previous tile
// still multiplies.  448 threads:
//   warp 0, lane 0  TMA producer over every (tile, stage) in order: W_hi,
//                   W_lo and raw X boxes into a 4-stage ring (48 KB each);
//   warp 1          512 TMEM columns: [0, 128) the tile's cross terms,
//                   [128, 512) three hi.hi group buffers; lane 0 issues the
//                   MMAs, commits each stage to empty[stage], each group to
//                   acc_full and each tile's last stage to tile_full;
//   warps 2-5       split each staged X tile into hi (in place) and lo (one
//                   of two 16 KB buffers, reused once empty[] shows the MMAs
//                   of the stage two back done);
//   warps 6-13      promote the hi.hi groups into FP32 registers, then take
//                   the tile's cross terms, free them for the next tile and
//                   store C while the next tile multiplies (three group
//                   buffers let the MMAs run six stages ahead of the store).
// Each tile's sums are formed as in tc_gemm_kernel<128, *>: the same
// products, the same groups of kTcPromote stages and the same order of the
// FP32 adds.  Every mbarrier operation and tcgen05.commit of the MMA thread
// costs ~110-170 cycles that do not overlap the queued MMAs (measured on
// B200), so the MMA thread commits once per stage plus once per group.
constexpr int kPtThreads = 448;
constexpr int kPtSplit = 128;
constexpr int kPtEpi = 256;
constexpr int kPtStages = 4;
constexpr uint32_t kPtX = 128 * kTcTileK * 4;    // 16 KB
constexpr uint32_t kPtStage = 2 * kWBox + kPtX;  // W_hi, W_lo, X (-> X_hi)
constexpr size_t kPtSmem = static_cast<size_t>(kPtStages) * kPtStage + 2 * kPtX + 1024 + 256;
static_assert(kPtSmem <= 232448, "the persistent GEMM's shared memory exceeds one CTA's limit");

__global__ void __launch_bounds__(kPtThreads, 1) tc_gemm_persistent_kernel(const __grid_constant__ TcGemmArgs a) {
    constexpr int S = kPtStages;
    extern __shared__ unsigned char tc_raw[];
    unsigned char* smem = tc_raw + ((1024u - (smem_addr(tc_raw) & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * kPtStage + 2 * kPtX);
    uint64_t* conv = full + S;
    uint64_t* empty = conv + S;
    uint64_t* acc_full = empty + S;     // [3] a group's hi.hi products are in TMEM
    uint64_t* acc_empty = acc_full + 3; // [3] the epilogue has taken them
    uint64_t* tile_full = acc_empty + 3;   // a tile's cross terms are complete
    uint64_t* tile_empty = tile_full + 1;  // the epilogue has taken them
    uint64_t* done = tile_empty + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int nblocks = (a.n + kTcTileN - 1) / kTcTileN;
    const int tiles = nblocks * ((a.m + 127) / 128);
    const int mine = static_cast<int>(blockIdx.x) < tiles ? (tiles - 1 - static_cast<int>(blockIdx.x)) / gridDim.x + 1 : 0;
    const int nk = a.k / kTcTileK;
    auto tile_n0 = [&](int u) { return (static_cast<int>(blockIdx.x) + u * static_cast<int>(gridDim.x)) % nblocks * kTcTileN; };
    auto tile_m0 = [&](int u) { return (static_cast<int>(blockIdx.x) + u * static_cast<int>(gridDim.x)) / nblocks * 128; };
    auto w_hi = [&](int s) { return smem + s * kPtStage; };
    auto w_lo = [&](int s) { return smem + s * kPtStage + kWBox; };
    auto x_hi = [&](int s) { return smem + s * kPtStage + 2 * kWBox; };
    auto x_lo = [&](int b) { return smem + S * kPtStage + b * kPtX; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            bar_init(&full[s], 1);
            bar_init(&conv[s], kPtSplit);
            bar_init(&empty[s], 1);
        }
        for (int j = 0; j < 3; ++j) {
            bar_init(&acc_full[j], 1);
            bar_init(&acc_empty[j], kPtEpi);
        }
        bar_init(tile_full, 1);
        bar_init(tile_empty, kPtEpi);
        bar_init(done, 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int issued = 0;
            bool ok = true;
            for (int u = 0; ok && u < mine; ++u) {
                const int n0 = tile_n0(u), m0 = tile_m0(u);
                for (int j = 0; j < nk; ++j) {
                    const int i = u * nk + j, s = i % S;
                    if (i >= S && !bar_wait(&empty[s], static_cast<uint32_t>(i / S - 1) & 1u, abort, a.error)) {
                        ok = false;
                        break;
                    }
                    if (*abort) {
                        ok = false;
                        break;
                    }
                    bar_expect(&full[s], kPtStage);
                    tma_box(w_hi(s), &a.w_hi, j * kTcTileK, n0, &full[s]);
                    tma_box(w_lo(s), &a.w_lo, j * kTcTileK, n0, &full[s]);
                    if (i == 0) grid_dependency_wait();  // X comes from the previous kernel
                    tma_box(x_hi(s), &a.x, j * kTcTileK, m0, &full[s]);
                    issued = i + 1;
                }
            }
            if (issued == 0) grid_dependency_wait();
            // Copies still in flight land before the CTA leaves (a no-op
            // unless a consumer gave up early).
            for (int i = max(0, issued - S); i < issued; ++i) {
                const unsigned long long t0 = now_ns();
                while (!bar_test(&full[i % S], static_cast<uint32_t>(i / S) & 1u))
                    if (now_ns() - t0 > kTcWaitNs) break;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = tf32_idesc(128);
            bool ok = true;
            int group = 0;
            for (int u = 0; ok && u < mine; ++u) {
                for (int j = 0; j < nk; ++j) {
                    const int i = u * nk + j, s = i % S, b = i & 1;
                    const bool first = j % kTcPromote == 0, last = j % kTcPromote == kTcPromote - 1 || j == nk - 1;
                    if (!bar_wait(&conv[s], static_cast<uint32_t>(i / S) & 1u, abort, a.error) ||
                        (j == 0 && u >= 1 &&
                         !bar_wait(tile_empty, static_cast<uint32_t>(u - 1) & 1u, abort, a.error)) ||
                        (first && group >= 3 &&
                         !bar_wait(&acc_empty[group % 3], static_cast<uint32_t>(group / 3 - 1) & 1u, abort,
                                   a.error))) {
                        ok = false;
                        break;
                    }
                    fence_after_sync();
                    const uint64_t ah = sw128_desc(smem_addr(w_hi(s))), al = sw128_desc(smem_addr(w_lo(s)));
                    const uint64_t bh = sw128_desc(smem_addr(x_hi(s))), bl = sw128_desc(smem_addr(x_lo(b)));
                    const uint32_t cross = tmem, main_acc = tmem + static_cast<uint32_t>(128 + group % 3 * 128);
#pragma unroll
                    for (int kk = 0; kk < kTcTileK / 8; ++kk) {
                        const uint64_t step = static_cast<uint64_t>(kk * 32 >> 4);  // 8 TF32 = 32 bytes
                        mma_tf32(cross, ah + step, bl + step, idesc, (j | kk) != 0 ? 1u : 0u);
                        mma_tf32(cross, al + step, bh + step, idesc, 1u);
                        mma_tf32(main_acc, ah + step, bh + step, idesc, (!first || kk != 0) ? 1u : 0u);
                    }
                    mma_commit(&empty[s]);
                    if (last) mma_commit(&acc_full[group++ % 3]);
                    if (j == nk - 1) mma_commit(tile_full);
                }
            }
            // every MMA issued above completes before TMEM is freed
            mma_commit(done);
            const unsigned long long t0 = now_ns();
            while (!bar_test(done, 0))
                if (now_ns() - t0 > kTcWaitNs) break;
        }
        __syncwarp();
    } else if (warp < 6) {
        const int t = threadIdx.x - 64;  // 0..127
        bool ok = true;
        for (int u = 0; ok && u < mine; ++u) {
            for (int j = 0; j < nk; ++j) {
                const int i = u * nk + j, s = i % S, b = i & 1;
                // X_lo buffer b was last read by the MMAs of stage i - 2; empty[(i - 2) % S]
                // cannot run a phase past them, since stage i + 2 needs this split first.
                if (!bar_wait(&full[s], static_cast<uint32_t>(i / S) & 1u, abort, a.error) ||
                    (i >= 2 && !bar_wait(&empty[(i - 2) % S], static_cast<uint32_t>((i - 2) / S) & 1u, abort,
                                         a.error))) {
                    ok = false;
                    break;
                }
                float4* xh = reinterpret_cast<float4*>(x_hi(s)) + t;
                float4* xl = reinterpret_cast<float4*>(x_lo(b)) + t;
                // a fixed trip count, so that all eight loads are in flight at once
                constexpr int kPer = 128 * kTcTileK / 4 / kPtSplit;
                float4 v[kPer];
#pragma unroll
                for (int r = 0; r < kPer; ++r) v[r] = xh[r * kPtSplit];
#pragma unroll
                for (int r = 0; r < kPer; ++r) {
                    // integer-ALU rounding (the conversion pipe is quarter rate)
                    float4 h, l;
                    h.x = tf32_round_int(v[r].x);
                    h.y = tf32_round_int(v[r].y);
                    h.z = tf32_round_int(v[r].z);
                    h.w = tf32_round_int(v[r].w);
                    l.x = tf32_round_int(v[r].x - h.x);
                    l.y = tf32_round_int(v[r].y - h.y);
                    l.z = tf32_round_int(v[r].z - h.z);
                    l.w = tf32_round_int(v[r].w - h.w);
                    xh[r * kPtSplit] = h;
                    xl[r * kPtSplit] = l;
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                bar_arrive(&conv[s]);
            }
        }
    } else {
        // Warps w and w + 4 share TMEM lane quarter w % 4 and take one half
        // of the 128 columns each (see tc_gemm_kernel for the promotion).
        const int quarter = warp & 3;
        const int c0 = (warp - 6) / 4 * 64;
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        const int groups = (nk + kTcPromote - 1) / kTcPromote;
        bool ok = true;
        int group = 0;
        bool waited = false;
        for (int u = 0; ok && u < mine; ++u) {
            float acc[64];
#pragma unroll
            for (int c = 0; c < 64; ++c) acc[c] = 0.0f;
            for (int g = 0; g < groups; ++g, ++group) {
                const int j = group % 3;
                if (!bar_wait(&acc_full[j], static_cast<uint32_t>(group / 3) & 1u, abort, a.error)) {
                    ok = false;
                    break;
                }
                __syncwarp();
                fence_after_sync();
#pragma unroll
                for (int col = 0; col < 64; col += 32) {
                    float v[32];
                    tmem_load32(tmem + lane_base + static_cast<uint32_t>(128 + j * 128 + c0 + col), v);
#pragma unroll
                    for (int c = 0; c < 32; ++c) acc[col + c] += v[c];
                }
                fence_before_sync();
                bar_arrive(&acc_empty[j]);
            }
            if (!ok || !bar_wait(tile_full, static_cast<uint32_t>(u) & 1u, abort, a.error)) {
                ok = false;
                break;
            }
            __syncwarp();
            fence_after_sync();
            float out[64];
#pragma unroll
            for (int col = 0; col < 64; col += 32) {
                float v[32];
                tmem_load32(tmem + lane_base + static_cast<uint32_t>(c0 + col), v);
#pragma unroll
                for (int c = 0; c < 32; ++c) out[col + c] = acc[col + c] + v[c];
            }
            fence_before_sync();
            bar_arrive(tile_empty);
            if (!waited) {
                grid_dependency_wait();  // the residual and C belong to earlier kernels too
                waited = true;
            }
            if (*abort) {
                ok = false;
                break;
            }
            const int n = tile_n0(u) + quarter * 32 + lane, m0 = tile_m0(u) + c0;
            if (n < a.n) {
#pragma unroll
                for (int q = 0; q < 64; ++q) {
                    const int m = m0 + q;
                    if (m < a.m) {
                        const long long at = static_cast<long long>(m) * a.ldc + n;
                        a.c[at] = a.residual != nullptr ? out[q] + a.residual[at] : out[q];
                    }
                }
            }
        }
        if (!waited) grid_dependency_wait();
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
    }
}

// Paired form for large M (the prefill's projections; N a multiple of 192,
// no K split): a cluster of two CTAs on two SMs walks tiles of 256 X rows x
// 192 W rows, t = pair + u * pairs (W block fastest).  The pair's MMAs
// (tcgen05 cta_group::2, M = 256, N = 192) take A = X (128 rows from each
// CTA) and B = W (96 rows from each), so one instruction does 1.5 times the
// per-SM work of a 128 x 128 MMA (128 x 192 on each SM) while each CTA
// stages only 96 W rows, for the same issue, wait and commit cost on the MMA
// thread -- those cost ~110-170 cycles each and do not overlap the queued
// MMAs.  D in each CTA's TMEM: its 128 X rows x the 192 outputs.
// 448 threads per CTA:
//   warp 0, lane 0  TMA producer (each CTA): per 32-column stage the CTA's
//                   raw X box (32 x 128) and W_hi / W_lo boxes (32 x 96)
//                   into a 4-stage ring, refilled when the leader's commit
//                   reaches empty[stage] in both CTAs;
//   warp 1          allocates 512 TMEM columns for the pair; on the leader
//                   (rank 0) lane 0 waits for both CTAs' split stage
//                   (conv[stage], 2 arrivals) and issues 12 MMAs per
//                   stage into one of two 192-column group accumulators
//                   (every product of 2 stages: Xhi.Wlo + Xlo.Whi + Xhi.Whi
//                   per K step), committing to both CTAs' empty[stage] and,
//                   per group, acc_full[group % 2];
//                   on the peer lane 0 forwards each split stage: it waits
//                   for the peer's sdone[stage] and arrives on the leader's
//                   conv[stage] (a cluster-scope release takes ~0.5 us, so
//                   the split warps do not make it themselves);
//   warps 2-5       split each staged X tile into hi (in place) and lo (one
//                   of three 16 KB buffers), then one thread arrives on
//                   conv[stage] (leader) or sdone[stage] (peer);
//   warps 6-13      add each group into FP32 registers (warp w: TMEM lane
//                   quarter w % 4, 96 of the 192 columns), release the group
//                   on the leader's acc_empty, and after a tile's last group
//                   store its rows (float4 stores, + residual), or with the
//                   fused SwiGLU silu(gate) * up of its 48 gate / up column
//                   pairs.
// The tensor core's accumulation truncates, so each group of 2 stages (8
// hi.hi products) starts a fresh accumulator and is added in FP32 with
// round-to-nearest, as in the other forms.
constexpr int kPrThreads = 448;
constexpr int kPrSplit = 128;
constexpr int kPrEpiWarps = 8;
constexpr int kPrStages = 4;
constexpr int kPrXlo = 3;
constexpr uint32_t kPrX = 128 * kTcTileK * 4;            // 16 KB
constexpr uint32_t kPrW = (kTcPairN / 2) * kTcTileK * 4;  // 12 KB
constexpr uint32_t kPrStage = kPrX + 2 * kPrW;            // X (-> X_hi), W_hi, W_lo
constexpr size_t kPrSmem = static_cast<size_t>(kPrStages) * kPrStage + kPrXlo * kPrX + 1024 + 256;
static_assert(kPrSmem <= 232448, "the paired GEMM's shared memory exceeds one CTA's limit");
static_assert(kPrW % 1024 == 0 && kPrStage % 1024 == 0, "operand tiles keep the 1024-byte swizzle alignment");

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPrThreads, 1)
    tc_gemm_pair_kernel(const __grid_constant__ TcGemmArgs a) {
    constexpr int S = kPrStages;
    extern __shared__ unsigned char tc_raw[];
    unsigned char* smem = tc_raw + ((1024u - (smem_addr(tc_raw) & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * kPrStage + kPrXlo * kPrX);
    uint64_t* empty = full + S;         // the leader's MMAs of a stage are done (both CTAs)
    uint64_t* conv = empty + S;         // leader: both CTAs split the stage
    uint64_t* acc_full = conv + S;      // [2] a group is in TMEM (both CTAs)
    uint64_t* acc_empty = acc_full + 2; // [2] leader: both CTAs' epilogues took it
    uint64_t* sdone = acc_empty + 2;    // peer: its split of a stage is done (for the forwarder)
    uint64_t* done = sdone + S;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t rank = cluster_rank();
    const int pair = static_cast<int>(blockIdx.x) / 2, pairs = static_cast<int>(gridDim.x) / 2;
    const int nblocks = a.n / kTcPairN;
    const int tiles = nblocks * ((a.m + 255) / 256);
    const int mine = pair < tiles ? (tiles - 1 - pair) / pairs + 1 : 0;
    const int nk = a.k / kTcTileK;
    auto tile_n0 = [&](int u) { return (pair + u * pairs) % nblocks * kTcPairN; };
    auto tile_m0 = [&](int u) { return (pair + u * pairs) / nblocks * 256 + static_cast<int>(rank) * 128; };
    auto x_hi = [&](int s) { return smem + s * kPrStage; };
    auto w_hi = [&](int s) { return smem + s * kPrStage + kPrX; };
    auto w_lo = [&](int s) { return smem + s * kPrStage + kPrX + kPrW; };
    auto x_lo = [&](int b) { return smem + S * kPrStage + b * kPrX; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            bar_init(&full[s], 1);
            bar_init(&empty[s], 1);
            bar_init(&conv[s], 2);
            bar_init(&sdone[s], 1);
        }
        for (int j = 0; j < 2; ++j) {
            bar_init(&acc_full[j], 1);
            bar_init(&acc_empty[j], 2 * kPrEpiWarps);
        }
        bar_init(done, 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    cluster_sync();  // both CTAs' barriers exist before either arrives on the other's
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int issued = 0;
            bool ok = true;
            const int w0 = static_cast<int>(rank) * (kTcPairN / 2);
            for (int u = 0; ok && u < mine; ++u) {
                const int n0 = tile_n0(u) + w0, m0 = tile_m0(u);
                for (int j = 0; j < nk; ++j) {
                    const int i = u * nk + j, s = i % S;
                    if (i >= S && !bar_wait(&empty[s], static_cast<uint32_t>(i / S - 1) & 1u, abort, a.error)) {
                        ok = false;
                        break;
                    }
                    if (*abort) {
                        ok = false;
                        break;
                    }
                    bar_expect(&full[s], kPrStage);
                    tma_box(w_hi(s), &a.w_hi96, j * kTcTileK, n0, &full[s]);
                    tma_box(w_lo(s), &a.w_lo96, j * kTcTileK, n0, &full[s]);
                    if (i == 0) grid_dependency_wait();  // X comes from the previous kernel
                    tma_box(x_hi(s), &a.x, j * kTcTileK, m0, &full[s]);
                    issued = i + 1;
                }
            }
            if (issued == 0) grid_dependency_wait();
            // Copies still in flight land before the CTA leaves (a no-op
            // unless a consumer gave up early).
            for (int i = max(0, issued - S); i < issued; ++i) {
                const unsigned long long t0 = now_ns();
                while (!bar_test(&full[i % S], static_cast<uint32_t>(i / S) & 1u))
                    if (now_ns() - t0 > kTcWaitNs) break;
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = tf32_idesc_pair(kTcPairN);
            bool ok = true;
            int group = 0;
            for (int u = 0; ok && u < mine; ++u) {
                for (int j = 0; j < nk; ++j) {
                    const int i = u * nk + j, s = i % S;
                    const bool first = j % kTcPromote == 0, last = j % kTcPromote == kTcPromote - 1 || j == nk - 1;
                    if (!bar_wait_cluster(&conv[s], static_cast<uint32_t>(i / S) & 1u, abort, a.error) ||
                        (first && group >= 2 &&
                         !bar_wait_cluster(&acc_empty[group & 1], static_cast<uint32_t>(group / 2 - 1) & 1u, abort,
                                           a.error))) {
                        ok = false;
                        break;
                    }
                    fence_after_sync();
                    const uint64_t ah = sw128_desc(smem_addr(x_hi(s))), al = sw128_desc(smem_addr(x_lo(i % kPrXlo)));
                    const uint64_t bh = sw128_desc(smem_addr(w_hi(s))), bl = sw128_desc(smem_addr(w_lo(s)));
                    const uint32_t acc = tmem + static_cast<uint32_t>((group & 1) * 256);
#pragma unroll
                    for (int kk = 0; kk < kTcTileK / 8; ++kk) {
                        const uint64_t step = static_cast<uint64_t>(kk * 32 >> 4);  // 8 TF32 = 32 bytes
                        mma_tf32_pair(acc, ah + step, bl + step, idesc, (!first || kk != 0) ? 1u : 0u);
                        mma_tf32_pair(acc, al + step, bh + step, idesc, 1u);
                        mma_tf32_pair(acc, ah + step, bh + step, idesc, 1u);
                    }
                    mma_commit_pair(&empty[s]);
                    if (last) mma_commit_pair(&acc_full[group++ & 1]);
                }
            }
            // every MMA issued above completes before TMEM is freed
            mma_commit_pair(done);
        }
        if (lane == 0 && rank != 0) {
            // the peer's forwarder: its split stages to the leader's conv[]
            for (int i = 0; i < mine * nk; ++i) {
                if (!bar_wait(&sdone[i % S], static_cast<uint32_t>(i / S) & 1u, abort, a.error)) break;
                bar_arrive_rank(&conv[i % S], 0);
            }
        }
        if (lane == 0) {
            const unsigned long long t0 = now_ns();
            while (!bar_test(done, 0))
                if (now_ns() - t0 > kTcWaitNs) break;
        }
        __syncwarp();
    } else if (warp < 2 + kPrSplit / 32) {
        const int t = threadIdx.x - 64;  // 0..127
        bool stop = false;
        for (int u = 0; !stop && u < mine; ++u) {
            for (int j = 0; j < nk; ++j) {
                const int i = u * nk + j, s = i % S;
                // X_lo buffer i % 3 was last read by the MMAs of stage i - 3;
                // empty[(i - 3) % S] cannot run a phase past them, since stage
                // i + 1 needs this split first.
                const bool ready =
                    bar_wait(&full[s], static_cast<uint32_t>(i / S) & 1u, abort, a.error) &&
                    (i < kPrXlo ||
                     bar_wait(&empty[(i - kPrXlo) % S], static_cast<uint32_t>((i - kPrXlo) / S) & 1u, abort, a.error));
                if (ready) {
                    float4* xh = reinterpret_cast<float4*>(x_hi(s)) + t;
                    float4* xl = reinterpret_cast<float4*>(x_lo(i % kPrXlo)) + t;
                    constexpr int kHalf = 128 * kTcTileK / 4 / kPrSplit / 2;  // 4 float4 per pass
#pragma unroll
                    for (int pass = 0; pass < 2; ++pass) {
                        float4 v[kHalf];
#pragma unroll
                        for (int r = 0; r < kHalf; ++r) v[r] = xh[(pass * kHalf + r) * kPrSplit];
#pragma unroll
                        for (int r = 0; r < kHalf; ++r) {
                            // integer-ALU rounding (the conversion pipe is quarter rate)
                            float4 h, l;
                            h.x = tf32_round_int(v[r].x);
                            h.y = tf32_round_int(v[r].y);
                            h.z = tf32_round_int(v[r].z);
                            h.w = tf32_round_int(v[r].w);
                            l.x = tf32_round_int(v[r].x - h.x);
                            l.y = tf32_round_int(v[r].y - h.y);
                            l.z = tf32_round_int(v[r].z - h.z);
                            l.w = tf32_round_int(v[r].w - h.w);
                            xh[(pass * kHalf + r) * kPrSplit] = h;
                            xl[(pass * kHalf + r) * kPrSplit] = l;
                        }
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                }
                // One arrival per CTA and stage: the split threads meet on a
                // named barrier that also ORs their stop flags, so every one
                // of them leaves the loop at the same stage and none waits
                // there alone.
                uint32_t any_stop;
                asm volatile(
                    "{\n\t.reg .pred q, r;\n\t"
                    "setp.ne.u32 q, %1, 0;\n\t"
                    "bar.red.or.pred r, 1, %2, q;\n\t"
                    "selp.u32 %0, 1, 0, r;\n\t}"
                    : "=r"(any_stop)
                    : "r"(ready && !*abort ? 0u : 1u), "n"(kPrSplit)
                    : "memory");
                if (any_stop != 0) {
                    stop = true;
                    break;
                }
                if (t == 0) bar_arrive(rank == 0 ? &conv[s] : &sdone[s]);
            }
        }
    } else {
        const int quarter = warp & 3;
        const int c0 = (warp - 6) / 4 * (kTcPairN / 2);  // 0 or 96
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        const int groups = (nk + kTcPromote - 1) / kTcPromote;
        bool ok = true;
        int group = 0;
        bool waited = false;
        for (int u = 0; ok && u < mine; ++u) {
            float acc[kTcPairN / 2];
#pragma unroll
            for (int c = 0; c < kTcPairN / 2; ++c) acc[c] = 0.0f;
            for (int g = 0; g < groups; ++g, ++group) {
                const int j = group & 1;
                if (!bar_wait(&acc_full[j], static_cast<uint32_t>(group / 2) & 1u, abort, a.error)) {
                    ok = false;
                    break;
                }
                __syncwarp();
                fence_after_sync();
#pragma unroll
                for (int col = 0; col < kTcPairN / 2; col += 16) {
                    float v[16];
                    tmem_load16(tmem + lane_base + static_cast<uint32_t>(j * 256 + c0 + col), v);
#pragma unroll
                    for (int c = 0; c < 16; ++c) acc[col + c] += v[c];
                }
                fence_before_sync();
                __syncwarp();
                if (lane == 0) bar_arrive_rank(&acc_empty[j], 0);
            }
            if (!ok) break;
            if (!waited) {
                grid_dependency_wait();  // the residual and C belong to earlier kernels too
                waited = true;
            }
            if (*abort) {
                ok = false;
                break;
            }
            const int m = tile_m0(u) + quarter * 32 + lane, n0 = tile_n0(u) + c0;
            if (a.swiglu) {
                // columns [0, 48) are gates and [48, 96) their ups: features
                // (tile_n0 + c0) / 2 + [0, 48)
                if (m < a.m) {
                    float* arow = a.act + static_cast<long long>(m) * a.act_ld + n0 / 2;
#pragma unroll
                    for (int q = 0; q < kTcPairN / 4; q += 4)
                        *reinterpret_cast<float4*>(arow + q) =
                            make_float4(swiglu(acc[q], acc[kTcPairN / 4 + q]), swiglu(acc[q + 1], acc[kTcPairN / 4 + q + 1]),
                                        swiglu(acc[q + 2], acc[kTcPairN / 4 + q + 2]),
                                        swiglu(acc[q + 3], acc[kTcPairN / 4 + q + 3]));
                }
            } else if (m < a.m) {
                float* crow = a.c + static_cast<long long>(m) * a.ldc + n0;
                const float* rrow = a.residual != nullptr ? a.residual + static_cast<long long>(m) * a.ldc + n0 : nullptr;
#pragma unroll
                for (int q = 0; q < kTcPairN / 2; q += 4) {
                    float4 o = make_float4(acc[q], acc[q + 1], acc[q + 2], acc[q + 3]);
                    if (rrow != nullptr) {
                        const float4 r = *reinterpret_cast<const float4*>(rrow + q);
                        o.x += r.x;
                        o.y += r.y;
                        o.z += r.z;
                        o.w += r.w;
                    }
                    *reinterpret_cast<float4*>(crow + q) = o;
                }
            }
        }
        if (!waited) grid_dependency_wait();
    }
    fence_before_sync();
    __syncthreads();
    cluster_sync();  // neither CTA frees TMEM or leaves while the pair may still use it
    if (warp == 1) {
        fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
    }
}

__global__ void tf32_split_kernel(const float4* __restrict__ w, float4* __restrict__ hi, float4* __restrict__ lo,
                                  size_t n4) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const float4 v = w[i];
        float4 h, r;
        h.x = tf32_rna(v.x);
        h.y = tf32_rna(v.y);
        h.z = tf32_rna(v.z);
        h.w = tf32_rna(v.w);
        r.x = tf32_rna(v.x - h.x);
        r.y = tf32_rna(v.y - h.y);
        r.z = tf32_rna(v.z - h.z);
        r.w = tf32_rna(v.w - h.w);
        hi[i] = h;
        lo[i] = r;
    }
}

// The packed gate/up weight split with its rows in the fused-SwiGLU order:
// destination row r of block b = r / 192, c = r % 192 takes feature
// f = 96 b + 48 (c / 96) + c % 48, its gate row f when c % 96 < 48, else its
// up row inter + f.
__global__ void tf32_split_swiglu_rows_kernel(const float4* __restrict__ w, float4* __restrict__ hi,
                                              float4* __restrict__ lo, int rows, int cols4, int inter) {
    const size_t n4 = static_cast<size_t>(rows) * cols4;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int r = static_cast<int>(i / cols4), col = static_cast<int>(i % cols4);
        const int b = r / kTcPairN, c = r % kTcPairN;
        const int f = (kTcPairN / 2) * b + (kTcPairN / 4) * (c / (kTcPairN / 2)) + c % (kTcPairN / 4);
        const int src = c % (kTcPairN / 2) < kTcPairN / 4 ? f : inter + f;
        const float4 v = w[static_cast<size_t>(src) * cols4 + col];
        float4 h, l;
        h.x = tf32_rna(v.x);
        h.y = tf32_rna(v.y);
        h.z = tf32_rna(v.z);
        h.w = tf32_rna(v.w);
        l.x = tf32_rna(v.x - h.x);
        l.y = tf32_rna(v.y - h.y);
        l.z = tf32_rna(v.z - h.z);
        l.w = tf32_rna(v.w - h.w);
        hi[i] = h;
        lo[i] = l;
    }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

template <int BM, int STAGES>
fx_status launch_variant(const TcGemmArgs& args, dim3 grid, cudaStream_t stream, bool dependent) {
    constexpr size_t smem = TcLayout<BM, STAGES>::kSmem;
    const fx_status raised = raise_smem_limit(reinterpret_cast<const void*>(tc_gemm_kernel<BM, STAGES>), smem,
                                              "raising the tensor-core GEMM's shared memory");
    if (raised != FX_OK) return raised;
    if (dependent)
        return launch_dependent(tc_gemm_kernel<BM, STAGES>, grid, dim3(kTcThreads), smem, stream,
                                "launching the tensor-core GEMM", args);
    tc_gemm_kernel<BM, STAGES><<<grid, kTcThreads, smem, stream>>>(args);
    FX_CUDA_TRY(cudaGetLastError(), "launching the tensor-core GEMM");
    return FX_OK;
}

fx_status launch_persistent(const TcGemmArgs& args, cudaStream_t stream) {
    const fx_status raised = raise_smem_limit(reinterpret_cast<const void*>(tc_gemm_persistent_kernel), kPtSmem,
                                              "raising the persistent tensor-core GEMM's shared memory");
    if (raised != FX_OK) return raised;
    int device = 0, sms = 0;
    FX_CUDA_TRY(cudaGetDevice(&device), "querying the current device");
    FX_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device), "querying the SM count");
    const long long tiles = static_cast<long long>((args.n + kTcTileN - 1) / kTcTileN) * ((args.m + 127) / 128);
    const unsigned grid = static_cast<unsigned>(std::min<long long>(tiles, sms));
    tc_gemm_persistent_kernel<<<grid, kPtThreads, kPtSmem, stream>>>(args);
    FX_CUDA_TRY(cudaGetLastError(), "launching the persistent tensor-core GEMM");
    return FX_OK;
}

fx_status launch_pair(const TcGemmArgs& args, cudaStream_t stream) {
    const fx_status raised = raise_smem_limit(reinterpret_cast<const void*>(tc_gemm_pair_kernel), kPrSmem,
                                              "raising the paired tensor-core GEMM's shared memory");
    if (raised != FX_OK) return raised;
    // every pair of a persistent grid must be resident at once
    cudaLaunchConfig_t config{};
    config.gridDim = dim3(2, 1, 1);
    config.blockDim = dim3(kPrThreads, 1, 1);
    config.dynamicSmemBytes = kPrSmem;
    config.stream = stream;
    cudaLaunchAttribute cluster{};
    cluster.id = cudaLaunchAttributeClusterDimension;
    cluster.val.clusterDim.x = 2;
    cluster.val.clusterDim.y = 1;
    cluster.val.clusterDim.z = 1;
    config.attrs = &cluster;
    config.numAttrs = 1;
    // resident pairs per device, queried once (the query costs host time on every launch otherwise)
    static std::atomic<int> resident[64];
    int device = 0;
    FX_CUDA_TRY(cudaGetDevice(&device), "querying the current device");
    int clusters = device >= 0 && device < 64 ? resident[device].load(std::memory_order_relaxed) : 0;
    if (clusters <= 0) {
        FX_CUDA_TRY(cudaOccupancyMaxActiveClusters(&clusters, tc_gemm_pair_kernel, &config),
                    "querying the resident CTA pairs of the paired GEMM");
        if (device >= 0 && device < 64) resident[device].store(clusters, std::memory_order_relaxed);
    }
    if (clusters <= 0) {
        set_error("paired tensor-core GEMM: no CTA pair fits on this device");
        return FX_ERR_CUDA;
    }
    const long long tiles = static_cast<long long>(args.n / kTcPairN) * ((args.m + 255) / 256);
    const unsigned grid = static_cast<unsigned>(2 * std::min<long long>(tiles, clusters));
    tc_gemm_pair_kernel<<<grid, kPrThreads, kPrSmem, stream>>>(args);
    FX_CUDA_TRY(cudaGetLastError(), "launching the paired tensor-core GEMM");
    return FX_OK;
}

}  // namespace

fx_status tc_encode_map(CUtensorMap* map, const float* base, int64_t rows, int64_t cols, int box_rows,
                        const char* what) {
    static std::once_flag once;
    static EncodeTiledFn encode = nullptr;
    std::call_once(once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult found{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &found) == cudaSuccess &&
            found == cudaDriverEntryPointSuccess)
            encode = reinterpret_cast<EncodeTiledFn>(fn);
    });
    if (encode == nullptr) {
        set_error("flux tensor-core GEMM: cuTensorMapEncodeTiled is unavailable from the driver");
        return FX_ERR_CUDA;
    }
    if (rows <= 0 || cols <= 0 || cols % 4 != 0 || reinterpret_cast<uintptr_t>(base) % 16 != 0 || box_rows <= 0 ||
        box_rows > 256) {
        set_error(std::string("flux tensor-core GEMM: ") + what + " is not a 16-byte aligned row-major matrix");
        return FX_ERR_INVALID;
    }
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * sizeof(float)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kTcTileK), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t element_strides[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box,
                              element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error(std::string("flux tensor-core GEMM: encoding the tensor map of ") + what + " failed (CUresult " +
                  std::to_string(static_cast<int>(r)) + ")");
        return FX_ERR_CUDA;
    }
    return FX_OK;
}

fx_status tc_split(const float* w, float* hi, float* lo, size_t n, cudaStream_t stream) {
    FX_REQUIRE(n % 4 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0 && reinterpret_cast<uintptr_t>(hi) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(lo) % 16 == 0,
               "tf32 split: sizes and pointers must be multiples of 4 floats / 16 bytes");
    if (n == 0) return FX_OK;
    const size_t n4 = n / 4;
    const unsigned blocks = static_cast<unsigned>(std::min<size_t>((n4 + 255) / 256, 148 * 16));
    tf32_split_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<const float4*>(w), reinterpret_cast<float4*>(hi),
                                                  reinterpret_cast<float4*>(lo), n4);
    FX_CUDA_TRY(cudaGetLastError(), "launching the tf32 split");
    return FX_OK;
}

fx_status launch_tc_gemm(const TcGemmArgs& args, int bm, int splits, cudaStream_t stream, bool dependent,
                         int stages) {
    FX_REQUIRE(args.k % kTcTileK == 0 && args.k_per_split % kTcTileK == 0 && args.k_per_split > 0 && splits >= 1 &&
                   args.m > 0 && args.n > 0 && args.ldc >= args.n,
               "tensor-core GEMM: K and its slices must be multiples of 32, M, N > 0");
    const dim3 grid(static_cast<unsigned>((args.n + kTcTileN - 1) / kTcTileN),
                    static_cast<unsigned>((args.m + bm - 1) / bm), static_cast<unsigned>(splits));
    // 128-row tiles without a K split (the prefill's projections): CTA pairs
    // when M fills them (at least kTcPairMinRows rows) and N is a multiple of
    // 192, else one persistent CTA per SM.
    if (bm == 128 && splits == 1 && stages == 0 && !dependent && args.k_per_split == args.k && args.has_pair &&
        args.m >= kTcPairMinRows &&
        args.n % kTcPairN == 0 && args.ldc % 4 == 0 && reinterpret_cast<uintptr_t>(args.c) % 16 == 0 &&
        (args.residual == nullptr || reinterpret_cast<uintptr_t>(args.residual) % 16 == 0) &&
        (!args.swiglu || (args.act != nullptr && args.act_ld % 4 == 0 && reinterpret_cast<uintptr_t>(args.act) % 16 == 0)))
        return launch_pair(args, stream);
    if (args.swiglu) {
        set_error("tensor-core GEMM: the fused SwiGLU runs only in the paired form (M >= 2048, N % 192 == 0, bm 128)");
        return FX_ERR_INVALID;
    }
    if (bm == 128 && splits == 1 && stages == 0 && !dependent && args.k_per_split == args.k)
        return launch_persistent(args, stream);
    if (stages == 0) stages = tc_default_stages(bm);
    if (bm == 64 && stages == 4) return launch_variant<64, 4>(args, grid, stream, dependent);
    if (bm == 64 && stages == 3) return launch_variant<64, 3>(args, grid, stream, dependent);
    if (bm == 128 && stages == 3) return launch_variant<128, 3>(args, grid, stream, dependent);
    set_error("tensor-core GEMM: the tile must be 64 rows (3 or 4 stages) or 128 rows (3 stages)");
    return FX_ERR_INVALID;
}

fx_status tc_weights_create(const fx_model_desc& model, bool lm_head, TcModelWeights* out, cudaStream_t stream,
                            bool layers, bool swiglu_rows) {
    static_assert(kInter % (kTcPairN / 2) == 0, "the gate/up features fill whole 192-row blocks");
    const size_t per_layer =
        layers ? static_cast<size_t>(kQKV + kHidden + kGateUp) * kHidden + static_cast<size_t>(kHidden) * kInter : 0;
    const size_t lm = lm_head ? static_cast<size_t>(model.vocab) * kHidden : 0;
    const size_t total = 2 * (per_layer * kLayers + lm);
    FX_CUDA_TRY(cudaMalloc(&out->buffer, total * sizeof(float)), "allocating the split projection weights");
    float* cursor = out->buffer;
    auto make = [&](TcWeight& w, const float* src, int rows, int cols, const char* what,
                    bool reorder = false) -> fx_status {
        const size_t n = static_cast<size_t>(rows) * cols;
        float* hi = cursor;
        float* lo = cursor + n;
        cursor += 2 * n;
        w.rows = rows;
        w.cols = cols;
        fx_status st = FX_OK;
        if (reorder) {
            FX_REQUIRE(reinterpret_cast<uintptr_t>(src) % 16 == 0 && cols % 4 == 0,
                       "tf32 split: the gate/up weight must be 16-byte aligned rows of a multiple of 4 floats");
            const size_t n4 = n / 4;
            const unsigned blocks = static_cast<unsigned>(std::min<size_t>((n4 + 255) / 256, 148 * 16));
            tf32_split_swiglu_rows_kernel<<<blocks, 256, 0, stream>>>(
                reinterpret_cast<const float4*>(src), reinterpret_cast<float4*>(hi), reinterpret_cast<float4*>(lo),
                rows, cols / 4, kInter);
            FX_CUDA_TRY(cudaGetLastError(), "launching the reordered tf32 split");
        } else {
            st = tc_split(src, hi, lo, n, stream);
        }
        if (st != FX_OK) return st;
        if ((st = tc_encode_map(&w.hi, hi, rows, cols, kTcTileN, what)) != FX_OK ||
            (st = tc_encode_map(&w.lo, lo, rows, cols, kTcTileN, what)) != FX_OK ||
            (st = tc_encode_map(&w.hi96, hi, rows, cols, kTcPairN / 2, what)) != FX_OK)
            return st;
        return tc_encode_map(&w.lo96, lo, rows, cols, kTcPairN / 2, what);
    };
    fx_status st;
    for (int l = 0; l < (layers ? kLayers : 0); ++l) {
        if ((st = make(out->qkv[l], model.packed_qkv[l], kQKV, kHidden, "packed_qkv")) != FX_OK) return st;
        if ((st = make(out->o[l], model.o_proj[l], kHidden, kHidden, "o_proj")) != FX_OK) return st;
        if ((st = make(out->gate_up[l], model.gate_up[l], kGateUp, kHidden, "gate_up", swiglu_rows)) != FX_OK)
            return st;
        if ((st = make(out->down[l], model.down[l], kHidden, kInter, "down")) != FX_OK) return st;
    }
    out->has_lm_head = lm_head;
    if (lm_head && (st = make(out->lm_head, model.lm_head, static_cast<int>(model.vocab), kHidden, "lm_head")) != FX_OK)
        return st;
    return FX_OK;
}

void tc_weights_release(TcModelWeights* w) {
    if (w == nullptr) return;
    cudaFree(w->buffer);
    w->buffer = nullptr;
}

TcGemmArgs tc_args(const TcWeight& w, const CUtensorMap& x, float* c, const float* residual, int* error, int m,
                   int k_per_split) {
    TcGemmArgs a{};
    a.w_hi = w.hi;
    a.w_lo = w.lo;
    a.x = x;
    a.c = c;
    a.residual = residual;
    a.error = error;
    a.m = m;
    a.n = w.rows;
    a.k = w.cols;
    a.ldc = w.rows;
    a.k_per_split = k_per_split;
    a.split_stride = static_cast<long long>(m) * w.rows;
    a.w_hi96 = w.hi96;
    a.w_lo96 = w.lo96;
    a.has_pair = true;
    return a;
}

}  // namespace fx

using namespace fx;

extern "C" fx_status fx_tf32_split_f32(const float* input, float* hi, float* lo, int64_t n, void* stream) {
    FX_REQUIRE(input && hi && lo, "fx_tf32_split_f32: null pointer");
    FX_REQUIRE(n >= 0, "fx_tf32_split_f32: negative size");
    return tc_split(input, hi, lo, static_cast<size_t>(n), as_stream(stream));
}

extern "C" fx_status fx_linear_3xtf32_f32(const float* input, const float* weight_hi, const float* weight_lo,
                                          const float* residual, float* output, int64_t m, int64_t k, int64_t n,
                                          int* error, void* stream) {
    FX_REQUIRE(input && weight_hi && weight_lo && output && error, "fx_linear_3xtf32_f32: null pointer");
    FX_REQUIRE(m > 0 && n > 0 && k > 0 && k % kTcTileK == 0 && m < (1LL << 31) && n < (1LL << 31) && k < (1LL << 31),
               "fx_linear_3xtf32_f32: M, N > 0 and K a positive multiple of 32");
    const int bm = m <= 64 ? 64 : 128;
    TcGemmArgs args{};
    fx_status st;
    if ((st = tc_encode_map(&args.w_hi, weight_hi, n, k, kTcTileN, "weight_hi")) != FX_OK) return st;
    if ((st = tc_encode_map(&args.w_lo, weight_lo, n, k, kTcTileN, "weight_lo")) != FX_OK) return st;
    if ((st = tc_encode_map(&args.x, input, m, k, bm, "input")) != FX_OK) return st;
    if (bm == 128 && n % kTcPairN == 0) {
        if ((st = tc_encode_map(&args.w_hi96, weight_hi, n, k, kTcPairN / 2, "weight_hi")) != FX_OK ||
            (st = tc_encode_map(&args.w_lo96, weight_lo, n, k, kTcPairN / 2, "weight_lo")) != FX_OK)
            return st;
        args.has_pair = true;
    }
    args.c = output;
    args.residual = residual;
    args.error = error;
    args.m = static_cast<int>(m);
    args.n = static_cast<int>(n);
    args.k = static_cast<int>(k);
    args.ldc = static_cast<int>(n);
    args.k_per_split = static_cast<int>(k);
    args.split_stride = 0;
    return launch_tc_gemm(args, bm, 1, as_stream(stream), false);
}

