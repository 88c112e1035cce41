// Causal prefill attention on tcgen05 tensor cores with the 3xTF32 split.
//
// One CTA per (128 queries, q head); key tiles of 64 rows up to the causal
// limit.  Q, K and V^T arrive already split into TF32 hi / lo planes (the
// RoPE / cache-fill kernel writes them), so no operand is converted here.
// 352 threads:
//   warp 0, lane 0   TMA: Q (hi, lo; two 32-column boxes each) once, then per
//                    key tile K (hi, lo) into a 2-stage ring, a stage freed
//                    by the commit of that tile's scores (s_full);
//   warp 10, lane 0  TMA: V^T (hi, lo) per key tile into a 2-stage ring, a
//                    stage freed by the commit of that tile's P V (o_full);
//   warp 1           owns TMEM (512 columns); lane 0 issues the MMAs:
//                    S = Q K^T as two accumulators (head dims 0-31 and 32-63,
//                    12 MMAs each: Qhi.Klo + Qlo.Khi + Qhi.Khi per K step),
//                    then O_tile = P V (A = P from TMEM, 8 key steps x 3);
//   warps 2-5 / 6-9  two softmax sets taking alternate key tiles (so one
//                    set's softmax overlaps the other's MMAs).  Warp w reads
//                    TMEM lanes 32 (w % 4) .., i.e. one query row per thread:
//                    t = S_a + S_b, causal mask on diagonal tiles, running
//                    max m of t c (c = scale log2(e) > 0), p = 2^(t c - m),
//                    row sum; p split into hi / lo written
//                    back over S_a / S_b with tcgen05.st; after the P V MMAs
//                    O_acc = O_acc * alpha + O_tile in FP32 through registers
//                    (each tile's P V product starts a fresh accumulator: the
//                    tensor core's accumulation truncates).
// At the end the two sets' (m, l, O) are merged through shared memory and
// row s of head h is written to out[s][h * 64 ..].
// TMEM columns: set X at 256 X: S_a / P_hi [0, 64), S_b / P_lo [64, 128),
// O_tile [128, 192), O_acc [192, 256).  Every mbarrier wait is bounded (bit 8 of the error
// word, then the CTA drains and frees TMEM).
#include "tc_attention.cuh"
#include "tcgen05.cuh"

#include <mutex>

namespace fx {
namespace {

using namespace tc;

constexpr int kAttnThreads = 352;  // K producer, MMA, 8 softmax warps, V producer
constexpr int kKStages = 2;         // K is free once the scores are done ...
constexpr int kVStages = 2;         // ... V^T only after P V
constexpr uint32_t kQBox = kTcAttnQ * 128;              // 128 rows x 32 floats (16 KB)
constexpr uint32_t kKBox = kTcAttnKeys * 128;           // 64 rows x 32 floats (8 KB)
constexpr uint32_t kQBytes = 4 * kQBox;                 // hi b0, hi b1, lo b0, lo b1
constexpr uint32_t kHalfStage = 4 * kKBox;              // K: hi b0 b1, lo b0 b1 / V^T: hi b0 b1, lo b0 b1
constexpr uint32_t kRingBytes = (kKStages + kVStages) * kHalfStage;
constexpr size_t kAttnSmem = kQBytes + kRingBytes + 1024 + 256;
constexpr uint32_t kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;

// 2^x on the SFU (ex2.approx.ftz: relative error ~2^-22; 2^-inf = 0).
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__global__ void __launch_bounds__(kAttnThreads, 1) tc_prefill_attention_kernel(const __grid_constant__ TcAttentionArgs a) {
    extern __shared__ unsigned char attn_raw[];
    unsigned char* smem = attn_raw + ((1024u - (smem_addr(attn_raw) & 1023u)) & 1023u);
    unsigned char* qs = smem;
    auto kstage = [&](int s) { return smem + kQBytes + s * kHalfStage; };
    auto vstage = [&](int s) { return smem + kQBytes + (kKStages + s) * kHalfStage; };
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kQBytes + kRingBytes);
    uint64_t* q_full = bars;
    uint64_t* k_full = bars + 1;
    uint64_t* v_full = k_full + kKStages;
    uint64_t* s_full = v_full + kVStages;
    uint64_t* p_full = s_full + 2;
    uint64_t* o_full = p_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 2);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int nqb = (a.rows + kTcAttnQ - 1) / kTcAttnQ;
    const int qb = nqb - 1 - static_cast<int>(blockIdx.x);  // heaviest query blocks first
    const int head = blockIdx.y, g = head / kGroup;
    const int q0 = qb * kTcAttnQ;
    const int key_end = min(a.rows, q0 + kTcAttnQ);
    const int nt = (key_end + kTcAttnKeys - 1) / kTcAttnKeys;

    if (threadIdx.x == 0) {
        bar_init(q_full, 1);
        for (int s = 0; s < kKStages; ++s) {
            bar_init(&k_full[s], 1);
        }
        for (int s = 0; s < kVStages; ++s) bar_init(&v_full[s], 1);
        for (int x = 0; x < 2; ++x) {
            bar_init(&s_full[x], 1);
            bar_init(&p_full[x], 128);
            bar_init(&o_full[x], 1);
        }
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    // One producer lane per ring: warp 0 loads Q and the K tiles, warp 9 the
    // V^T tiles.
    // `freed(t)` waits until the stage of tile t - stages may be refilled.
    auto produce = [&](int stages, uint64_t* full, auto&& freed, auto&& load) {
        int issued = 0;
        for (int t = 0; t < nt; ++t) {
            const int s = t % stages;
            if (t >= stages && !freed(t)) break;
            bar_expect(&full[s], kHalfStage);
            load(t, s, &full[s]);
            issued = t + 1;
        }
        // Copies in flight land before the CTA leaves (a no-op unless a
        // consumer gave up early).
        for (int t = max(0, issued - stages); t < issued; ++t) {
            const unsigned long long t0 = now_ns();
            while (!bar_test(&full[t % stages], static_cast<uint32_t>(t / stages) & 1u))
                if (now_ns() - t0 > kTcWaitNs) break;
        }
    };
    if (warp == 0) {
        if (lane == 0) {
            bar_expect(q_full, kQBytes);
            const int qy = head * a.rows + q0;
            tma_box(qs + 0 * kQBox, &a.q_hi, 0, qy, q_full);
            tma_box(qs + 1 * kQBox, &a.q_hi, 32, qy, q_full);
            tma_box(qs + 2 * kQBox, &a.q_lo, 0, qy, q_full);
            tma_box(qs + 3 * kQBox, &a.q_lo, 32, qy, q_full);
            auto k_freed = [&](int t) {
                // K stage t % 2 is free once the scores of tile t - 2 are
                // done: s_full[t % 2] of that tile (its next phase needs this
                // very tile, so the parity cannot alias).
                return bar_wait(&s_full[t & 1], static_cast<uint32_t>((t - kKStages) >> 1) & 1u, abort, a.error);
            };
            produce(kKStages, k_full, k_freed, [&](int t, int s, uint64_t* bar) {
                unsigned char* st = kstage(s);
                const int ky = g * a.padded + t * kTcAttnKeys;
                tma_box(st + 0 * kKBox, &a.k_hi, 0, ky, bar);
                tma_box(st + 1 * kKBox, &a.k_hi, 32, ky, bar);
                tma_box(st + 2 * kKBox, &a.k_lo, 0, ky, bar);
                tma_box(st + 3 * kKBox, &a.k_lo, 32, ky, bar);
            });
            const unsigned long long t0 = now_ns();
            while (!bar_test(q_full, 0))
                if (now_ns() - t0 > kTcWaitNs) break;
        }
    } else if (warp == kAttnThreads / 32 - 1) {
        if (lane == 0) {
            // V^T stage t % 2 is free once the P V products of tile t - 2 are
            // done: o_full[t % 2] of that tile (its next phase needs this very
            // tile, so the parity cannot alias), one commit fewer per tile.
            auto v_freed = [&](int t) {
                return bar_wait(&o_full[t & 1], static_cast<uint32_t>((t - kVStages) >> 1) & 1u, abort, a.error);
            };
            produce(kVStages, v_full, v_freed, [&](int t, int s, uint64_t* bar) {
                unsigned char* st = vstage(s);
                const int vx = t * kTcAttnKeys;
                tma_box(st + 0 * kKBox, &a.vt_hi, vx, g * kHeadDim, bar);
                tma_box(st + 1 * kKBox, &a.vt_hi, vx + 32, g * kHeadDim, bar);
                tma_box(st + 2 * kKBox, &a.vt_lo, vx, g * kHeadDim, bar);
                tma_box(st + 3 * kKBox, &a.vt_lo, vx + 32, g * kHeadDim, bar);
            });
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = tf32_idesc(64);
            bool ok = bar_wait(q_full, 0, abort, a.error);
            const uint64_t qh0 = sw128_desc(smem_addr(qs)), qh1 = sw128_desc(smem_addr(qs + kQBox));
            const uint64_t ql0 = sw128_desc(smem_addr(qs + 2 * kQBox)), ql1 = sw128_desc(smem_addr(qs + 3 * kQBox));
            auto issue_scores = [&](int t) -> bool {
                const int s = t % kKStages, x = t & 1, u = t >> 1;
                if (!bar_wait(&k_full[s], static_cast<uint32_t>(t / kKStages) & 1u, abort, a.error)) return false;
                // S_x / P_x of tile t - 2 are free once its P V products are done.
                if (u >= 1 && !bar_wait(&o_full[x], static_cast<uint32_t>(u - 1) & 1u, abort, a.error)) return false;
                fence_after_sync();
                unsigned char* st = kstage(s);
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    const uint32_t d = tmem + static_cast<uint32_t>(x * 256 + b * 64);
                    const uint64_t qh = b == 0 ? qh0 : qh1, ql = b == 0 ? ql0 : ql1;
                    const uint64_t kh = sw128_desc(smem_addr(st + b * kKBox));
                    const uint64_t kl = sw128_desc(smem_addr(st + (2 + b) * kKBox));
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t step = static_cast<uint64_t>(kk * 2);  // 8 TF32 = 32 bytes
                        mma_tf32(d, qh + step, kl + step, idesc, kk != 0 ? 1u : 0u);
                        mma_tf32(d, ql + step, kh + step, idesc, 1u);
                        mma_tf32(d, qh + step, kh + step, idesc, 1u);
                    }
                }
                mma_commit(&s_full[x]);
                return true;
            };
            ok = ok && nt > 0 && issue_scores(0);
            for (int t = 0; ok && t < nt; ++t) {
                if (t + 1 < nt && !issue_scores(t + 1)) break;
                const int s = t % kVStages, x = t & 1, u = t >> 1;
                if (!bar_wait(&v_full[s], static_cast<uint32_t>(t / kVStages) & 1u, abort, a.error)) break;
                if (!bar_wait(&p_full[x], static_cast<uint32_t>(u) & 1u, abort, a.error)) break;
                fence_after_sync();
                unsigned char* st = vstage(s);
                const uint32_t o = tmem + static_cast<uint32_t>(x * 256 + 128);
                const uint32_t ph = tmem + static_cast<uint32_t>(x * 256), pl = ph + 64;
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const int vb = kk / 4;
                    const uint64_t step = static_cast<uint64_t>((kk % 4) * 2);
                    const uint64_t vh = sw128_desc(smem_addr(st + vb * kKBox)) + step;
                    const uint64_t vl = sw128_desc(smem_addr(st + (2 + vb) * kKBox)) + step;
                    const uint32_t col = static_cast<uint32_t>(kk * 8);
                    mma_tf32_ts(o, ph + col, vl, idesc, kk != 0 ? 1u : 0u);
                    mma_tf32_ts(o, pl + col, vh, idesc, 1u);
                    mma_tf32_ts(o, ph + col, vh, idesc, 1u);
                }
                mma_commit(&o_full[x]);
            }
        }
        __syncwarp();
    } else {
        const int set = (warp - 2) / 4;  // 0: even key tiles, 1: odd
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const int qpos = q0 + row;
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t sa = tmem + lane_base + static_cast<uint32_t>(set * 256);
        const float c = a.scale * kLog2e;
        float m_run = -INFINITY, l_run = 0.0f;
        bool ok = true, first = true;
        for (int t = set; ok && t < nt; t += 2) {
            const int u = t >> 1;
            ok = bar_wait(&s_full[set], static_cast<uint32_t>(u) & 1u, abort, a.error);
            __syncwarp();
            fence_after_sync();
            // Raw scores t = S_a + S_b (the scale c > 0 is applied inside the
            // exponent: max(t) c is the max of the scaled scores).
            const int k0 = t * kTcAttnKeys;
            float tv[kTcAttnKeys];
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float va[32], vb[32];
                tmem_load32(sa + static_cast<uint32_t>(half * 32), va);
                tmem_load32(sa + static_cast<uint32_t>(64 + half * 32), vb);
#pragma unroll
                for (int j = 0; j < 32; ++j) tv[half * 32 + j] = va[j] + vb[j];
            }
            if (k0 + kTcAttnKeys - 1 > q0) {  // a tile on the causal diagonal (block-uniform)
#pragma unroll
                for (int j = 0; j < kTcAttnKeys; ++j)
                    if (k0 + j > qpos) tv[j] = -INFINITY;
            }
            float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int j = 0; j < kTcAttnKeys; ++j) mx[j & 3] = fmaxf(mx[j & 3], tv[j]);
            const float m_new = fmaxf(m_run, fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * c);
            const float mref = m_new == -INFINITY ? 0.0f : m_new;  // a row with no key yet
            const float alpha = fast_exp2(m_run - mref);
            float sum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float ph[32], pl[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const float p = fast_exp2(fmaf(tv[half * 32 + j], c, -mref));
                    sum[j & 3] += p;
                    ph[j] = tf32_round_int(p);
                    pl[j] = tf32_round_int(p - ph[j]);
                }
                tmem_store32(sa + static_cast<uint32_t>(half * 32), ph);
                tmem_store32(sa + static_cast<uint32_t>(64 + half * 32), pl);
            }
            const float rs = (sum[0] + sum[1]) + (sum[2] + sum[3]);
            tmem_store_wait();
            fence_before_sync();
            bar_arrive(&p_full[set]);
            l_run = l_run * alpha + rs;
            m_run = m_new;
            ok = ok && bar_wait(&o_full[set], static_cast<uint32_t>(u) & 1u, abort, a.error);
            __syncwarp();
            fence_after_sync();
            // O_acc = O_acc * alpha + O_tile in FP32 (O_acc at columns 192..255).
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float ov[32], acc[32];
                tmem_load32(sa + static_cast<uint32_t>(128 + half * 32), ov);
                if (!first) {
                    tmem_load32(sa + static_cast<uint32_t>(192 + half * 32), acc);
#pragma unroll
                    for (int j = 0; j < 32; ++j) ov[j] = fmaf(acc[j], alpha, ov[j]);
                }
                tmem_store32(sa + static_cast<uint32_t>(192 + half * 32), ov);
            }
            tmem_store_wait();
            first = false;
        }
        // Merge the two sets' rows: set 1 hands (m, l, O) to set 0 through the
        // (now idle) K / V stages.
        asm volatile("bar.sync 1, 256;" ::: "memory");  // every MMA has completed
        float* scratch = reinterpret_cast<float*>(kstage(0)) + row * (kHeadDim + 4);
        if (set == 1) {
            scratch[0] = m_run;
            scratch[1] = l_run;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float ov[32];
                if (!first) {
                    tmem_load32(sa + static_cast<uint32_t>(192 + half * 32), ov);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) ov[j] = 0.0f;  // no key tile in this set
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) scratch[4 + half * 32 + j] = ov[j];
            }
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (set == 0) {
            const float mb = scratch[0], lb = scratch[1];
            const float m = fmaxf(m_run, mb);
            const float fa = fast_exp2(m_run - m), fb = mb == -INFINITY ? 0.0f : fast_exp2(mb - m);
            const float inv = 1.0f / (l_run * fa + lb * fb);
            float4* dst = reinterpret_cast<float4*>(a.out + static_cast<size_t>(qpos) * kHidden + head * kHeadDim);
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float ov[32];
                tmem_load32(sa + static_cast<uint32_t>(192 + half * 32), ov);
                if (qpos < a.rows && !*abort) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        const float* sb = scratch + 4 + half * 32 + j;
                        dst[(half * 32 + j) / 4] = make_float4((ov[j] * fa + sb[0] * fb) * inv,
                                                               (ov[j + 1] * fa + sb[1] * fb) * inv,
                                                               (ov[j + 2] * fa + sb[2] * fb) * inv,
                                                               (ov[j + 3] * fa + sb[3] * fb) * inv);
                    }
                }
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        fence_after_sync();
        tmem_free(tmem, kTmemCols);
    }
}

}  // namespace

fx_status launch_tc_prefill_attention(const TcAttentionArgs& args, cudaStream_t stream) {
    const fx_status raised = raise_smem_limit(reinterpret_cast<const void*>(tc_prefill_attention_kernel), kAttnSmem,
                                              "raising the tensor-core attention's shared memory");
    if (raised != FX_OK) return raised;
    FX_REQUIRE(args.rows > 0 && args.padded >= args.rows && args.padded % kTcAttnKeys == 0,
               "tensor-core attention: bad row counts");
    FX_REQUIRE(args.scale > 0.0f, "tensor-core attention: the attention scale must be positive");
    const dim3 grid(static_cast<unsigned>((args.rows + kTcAttnQ - 1) / kTcAttnQ), kQHeads);
    tc_prefill_attention_kernel<<<grid, kAttnThreads, kAttnSmem, stream>>>(args);
    FX_CUDA_TRY(cudaGetLastError(), "launching the tensor-core prefill attention");
    return FX_OK;
}

}  // namespace fx
