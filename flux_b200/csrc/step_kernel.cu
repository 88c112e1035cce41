// The whole batch-1 decode step as ONE persistent cooperative launch.
//
// One CTA per SM (512 threads, ~213 KB shared memory).  Each CTA owns a fixed
// slice of every projection and one (kv head, chunk) of the attention, and
// walks 30 layers x 4 phases separated by grid barriers:
//
//   A  h = h' + sum(replicas) (or the embedding row); RMSNorm; its QKV row
//      pairs; RoPE; K/V row written at `position`; q published.
//   B  split-K attention over its chunk of the valid rows for the 3 q heads
//      of its kv head (online softmax per 8-lane row group), partial
//      published; the last CTA of each kv head merges -> attn.
//   C  its o_proj rows: h'[r] = h[r] + Wo[r] . attn.
//   D  RMSNorm(h'); its gate/up features; SwiGLU; its slice of the down
//      projection (rows of the transposed weight) added into one of four
//      replica accumulators with 16-byte vector reductions.
//
// then the LM head (its vocab rows, greedy candidate; the last CTA picks the
// token and advances the device state).  Weights and K/V rows never depend
// on the barriers, so a producer thread streams them into a 192 KB shared
// ring with 1-D TMA bulk copies (cp.async.bulk, mbarrier completion, no
// multicast) as far ahead as the ring allows -- HBM keeps streaming while
// the CTAs wait at a barrier.  Only the K/V row of the current position
// (written in phase A of the same step) is read directly from L2.
//
// Every wait (grid barrier, mbarrier) is bounded by %globaltimer; on expiry
// the CTA sets error bit 2, waits (bounded) for its own copies in flight and
// returns, and the other CTAs see the flag at their next barrier.
#include "step_kernel.cuh"

#include <algorithm>

namespace fx {
namespace {

constexpr int kMaxSeg = 16;
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s per wait
constexpr int kWarps = kStepThreads / 32;
constexpr int kRowBytes = kHidden * 4;                  // 2304

// ------------------------------------------------------------- PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Optional timeline stamp by thread 0 of each CTA.
#define STEP_MARK(event)                                                                        \
    do {                                                                                      \
        if (a.timeline != nullptr && threadIdx.x == 0)                                         \
            a.timeline[static_cast<size_t>(blockIdx.x) * kStepTimelineEvents + (event)] = global_timer(); \
    } while (0)

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
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

// 1-D bulk copy global -> shared completing on `bar` (no multicast).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ int ld_relaxed_s32(const int* p) {
    int v;
    asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void red_add_v4(float* p, float4 v) {
    asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z),
                 "f"(v.w)
                 : "memory");
}

// ------------------------------------------------------------ shared state

struct Shared {
    float xs[kHidden];                 // normalised input vector of the phase
    float sv[64];                      // SwiGLU outputs of this CTA's features
    float wm[kWarps][kGroup];          // attention per-warp states
    float wl[kWarps][kGroup];
    float wo[kWarps][kGroup][kHeadDim];
    float scratch[32];
    float cv[kWarps];
    long long ci[kWarps];
    uint64_t bars[kStepSlots];
    uint32_t slot_off[kStepSlots];
    uint32_t slot_end[kStepSlots];
    uint32_t head, tail;               // ring bytes issued / released (monotonic)
    int issued, released;              // tiles issued / released
    int abort;
    int is_last;
};

constexpr size_t kRingOffset = (sizeof(Shared) + 1023) / 1024 * 1024;

// Per-CTA work split; every thread of the CTA computes the same values.
struct Sched {
    int t0, t1;           // QKV row-pair tasks
    int o0, o1;           // o_proj rows
    int i0, i1;           // intermediate features
    int64_t v0, v1;       // vocab rows
    int g, c;             // attention kv head / chunk (g < 0: none)
    int64_t a0, a1;       // attention rows [a0, a1) of the valid length
    int64_t cached_end;   // rows [a0, cached_end) stream through the ring
    bool owns_new;        // this chunk holds row `pos`
    bool has_rows;        // chunk is active
    int active;           // active chunks per kv head
    int n_att, per_layer, n_lm, total;
    int64_t pos;
    int64_t tok;
};

struct Tile {
    int nseg;
    const float* src[kMaxSeg];
    uint32_t bytes[kMaxSeg];
    uint32_t total;
};

__device__ __forceinline__ void task_rows(int task, int& row_a, int& row_b, int& kind) {
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
    row_b = kind == 2 ? row_a + 1 : row_a + kHeadDim / 2;
}

__device__ void make_sched(const StepArgs& a, int G, int cta, Sched& s) {
    s.t0 = cta * 480 / G;
    s.t1 = (cta + 1) * 480 / G;
    s.o0 = cta * kHidden / G;
    s.o1 = (cta + 1) * kHidden / G;
    s.i0 = cta * kInter / G;
    s.i1 = (cta + 1) * kInter / G;
    s.v0 = static_cast<int64_t>(cta) * a.vocab / G;
    s.v1 = static_cast<int64_t>(cta + 1) * a.vocab / G;
    s.pos = *a.position;
    s.tok = *a.token;
    const int64_t len = s.pos + 1;
    s.g = -1;
    s.c = 0;
    s.a0 = s.a1 = s.cached_end = 0;
    s.owns_new = false;
    s.has_rows = false;
    s.active = 0;
    if (cta < kKVHeads * a.nch) {
        s.g = cta / a.nch;
        s.c = cta % a.nch;
        const int64_t chunk = (len + a.nch - 1) / a.nch;
        s.active = static_cast<int>((len + chunk - 1) / chunk);
        if (s.c < s.active) {
            s.has_rows = true;
            s.a0 = s.c * chunk;
            s.a1 = min(len, s.a0 + chunk);
            s.cached_end = min(s.a1, s.pos);
            s.owns_new = s.pos >= s.a0 && s.pos < s.a1;
        }
    }
    const int64_t cached = s.cached_end > s.a0 ? s.cached_end - s.a0 : 0;
    s.n_att = static_cast<int>((cached + kStepAttnRows - 1) / kStepAttnRows);
    s.per_layer = (s.t1 > s.t0) + s.n_att + (s.o1 > s.o0) + 2 * (s.i1 > s.i0);
    s.n_lm = static_cast<int>((s.v1 - s.v0 + kStepLmRows - 1) / kStepLmRows);
    s.total = kLayers * s.per_layer + s.n_lm;
}

__device__ void make_tile(const StepArgs& a, const Sched& s, int k, Tile& t) {
    t.nseg = 0;
    t.total = 0;
    auto add = [&](const float* src, uint32_t bytes) {
        t.src[t.nseg] = src;
        t.bytes[t.nseg] = bytes;
        t.total += bytes;
        ++t.nseg;
    };
    if (k < kLayers * s.per_layer) {
        const int l = k / s.per_layer;
        int sub = k % s.per_layer;
        const StepLayer& L = a.layer[l];
        if (s.t1 > s.t0) {
            if (sub == 0) {
                for (int task = s.t0; task < s.t1; ++task) {
                    int ra, rb, kind;
                    task_rows(task, ra, rb, kind);
                    add(L.qkv + static_cast<int64_t>(ra) * kHidden, kRowBytes);
                    add(L.qkv + static_cast<int64_t>(rb) * kHidden, kRowBytes);
                }
                return;
            }
            --sub;
        }
        if (sub < s.n_att) {
            const int64_t r0 = s.a0 + static_cast<int64_t>(sub) * kStepAttnRows;
            const int64_t n = min(static_cast<int64_t>(kStepAttnRows), s.cached_end - r0);
            const int64_t base = ((static_cast<int64_t>(l) * kKVHeads + s.g) * a.capacity + r0) * kHeadDim;
            add(a.key_cache + base, static_cast<uint32_t>(n * kHeadDim * 4));
            add(a.value_cache + base, static_cast<uint32_t>(n * kHeadDim * 4));
            return;
        }
        sub -= s.n_att;
        if (s.o1 > s.o0) {
            if (sub == 0) {
                add(L.o_proj + static_cast<int64_t>(s.o0) * kHidden, (s.o1 - s.o0) * kRowBytes);
                return;
            }
            --sub;
        }
        const int ni = s.i1 - s.i0;
        if (sub == 0) {
            add(L.gate_up + static_cast<int64_t>(s.i0) * kHidden, ni * kRowBytes);
            add(L.gate_up + static_cast<int64_t>(kInter + s.i0) * kHidden, ni * kRowBytes);
        } else {
            add(L.down_t + static_cast<int64_t>(s.i0) * kHidden, ni * kRowBytes);
        }
        return;
    }
    const int64_t r0 = s.v0 + static_cast<int64_t>(k - kLayers * s.per_layer) * kStepLmRows;
    const int64_t n = min(static_cast<int64_t>(kStepLmRows), s.v1 - r0);
    add(a.lm_head + r0 * kHidden, static_cast<uint32_t>(n * kRowBytes));
}

// Producer (thread 0 only): issue tiles in consumption order while the ring
// has room and an mbarrier slot is free.
__device__ void pump(const StepArgs& a, const Sched& s, Shared& sh, unsigned char* ring) {
    while (sh.issued < s.total) {
        if (sh.issued - sh.released >= kStepSlots) return;
        Tile t;
        make_tile(a, s, sh.issued, t);
        const uint32_t size = (t.total + 127u) & ~127u;
        uint32_t off = sh.head % kStepRingBytes;
        const uint32_t pad = off + size > static_cast<uint32_t>(kStepRingBytes) ? kStepRingBytes - off : 0u;
        if (sh.head + pad + size - sh.tail > static_cast<uint32_t>(kStepRingBytes)) return;
        sh.head += pad;
        off = sh.head % kStepRingBytes;
        const int slot = sh.issued % kStepSlots;
        sh.slot_off[slot] = off;
        sh.head += size;
        sh.slot_end[slot] = sh.head;
        // Order earlier generic-proxy reads of the reused bytes before the async writes.
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive_expect_tx(&sh.bars[slot], t.total);
        uint32_t o = off;
        for (int i = 0; i < t.nseg; ++i) {
            bulk_load(ring + o, t.src[i], t.bytes[i], &sh.bars[slot]);
            o += t.bytes[i];
        }
        ++sh.issued;
    }
}

// Wait for tile k; returns its shared-memory address (nullptr on timeout, uniform).
__device__ const float* acquire(const StepArgs& a, const Sched& s, Shared& sh, unsigned char* ring, int k) {
    if (threadIdx.x == 0) pump(a, s, sh, ring);
    const int slot = k % kStepSlots;
    const uint32_t parity = static_cast<uint32_t>(k / kStepSlots) & 1u;
    if (!mbar_try_wait(&sh.bars[slot], parity)) {
        const unsigned long long t0 = global_timer();
        while (!mbar_try_wait(&sh.bars[slot], parity)) {
            if (global_timer() - t0 > kWaitNs) {
                sh.abort = 1;
                break;
            }
        }
    }
    __syncthreads();
    if (sh.abort) return nullptr;
    return reinterpret_cast<const float*>(ring + sh.slot_off[slot]);
}

__device__ void release(const StepArgs& a, const Sched& s, Shared& sh, unsigned char* ring, int k) {
    __syncthreads();
    if (threadIdx.x == 0) {
        sh.tail = sh.slot_end[k % kStepSlots];
        sh.released = k + 1;
        pump(a, s, sh, ring);
    }
}

// Grid-wide barrier number `index` (monotonic counter, reset by the last CTA
// of the step).  Returns false (uniformly) when any CTA has given up.
__device__ bool grid_sync(const StepArgs& a, const Sched& s, Shared& sh, unsigned char* ring, unsigned index) {
    __syncthreads();
    if (threadIdx.x == 0) {
        pump(a, s, sh, ring);  // keep HBM busy while waiting
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        red_release_add(&a.sync[0], 1u);
        const unsigned target = (index + 1) * gridDim.x;
        if (ld_acquire_u32(&a.sync[0]) < target) {
            const unsigned long long t0 = global_timer();
            while (ld_acquire_u32(&a.sync[0]) < target) {
                if (ld_relaxed_s32(a.error) != 0) {
                    sh.abort = 1;
                    break;
                }
                if (global_timer() - t0 > kWaitNs) {
                    atomicOr(a.error, 2);
                    sh.abort = 1;
                    break;
                }
            }
        }
    }
    __syncthreads();
    return sh.abort == 0;
}

// Hidden state entering layer l (l == 30: the final hidden state), element i.
__device__ __forceinline__ float hidden_in(const StepArgs& a, const Sched& s, int l, int i) {
    if (l == 0) {
        return (s.tok >= 0 && s.tok < a.vocab) ? __ldg(a.embedding + s.tok * kHidden + i) : 0.0f;
    }
    const float* acc = a.accum + ((l - 1) & 1) * kStepReplicas * kHidden;
    float v = __ldcg(a.hidden_mid + i);
#pragma unroll
    for (int r = 0; r < kStepReplicas; ++r) v += __ldcg(acc + r * kHidden + i);
    return v;
}

// xs = RMSNorm(x) * w for the 576-vector produced by `load(i)`.
template <typename Load>
__device__ __forceinline__ void norm_into(Shared& sh, Load load, const float* __restrict__ w, float eps) {
    float ss = 0.0f;
    for (int i = threadIdx.x; i < kHidden; i += kStepThreads) {
        const float v = load(i);
        sh.xs[i] = v;
        ss += v * v;
    }
    ss = block_sum(ss, sh.scratch);
    const float inv = rsqrtf(ss / static_cast<float>(kHidden) + eps);
    for (int i = threadIdx.x; i < kHidden; i += kStepThreads) sh.xs[i] = sh.xs[i] * inv * __ldg(w + i);
    __syncthreads();
}

// Half-warp dot of a 576-float row in shared memory with sh.xs.
__device__ __forceinline__ float row_dot(const float* row, const float* xs, int l16) {
    const float4* r4 = reinterpret_cast<const float4*>(row);
    const float4* x4 = reinterpret_cast<const float4*>(xs);
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < kHidden / 64; ++j) {
        const float4 w = r4[l16 + 16 * j];
        const float4 x = x4[l16 + 16 * j];
        acc = fmaf(w.x, x.x, acc);
        acc = fmaf(w.y, x.y, acc);
        acc = fmaf(w.z, x.z, acc);
        acc = fmaf(w.w, x.w, acc);
    }
    return group_sum<16>(acc);
}

__device__ __forceinline__ void argmax_take(float& bv, long long& bi, float v, long long i) {
    if (argmax_precedes(v, i, bv, bi)) {
        bv = v;
        bi = i;
    }
}

// Online-softmax update of one 8-lane row group with one cache row.
__device__ __forceinline__ void attend_row(const float4 (&qa)[kGroup], const float4 (&qb)[kGroup], float4 k0,
                                           float4 k1, float4 v0, float4 v1, float scale, float (&m)[kGroup],
                                           float (&l)[kGroup], float (&o)[kGroup][8]) {
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
        float d = qa[h].x * k0.x;
        d = fmaf(qa[h].y, k0.y, d);
        d = fmaf(qa[h].z, k0.z, d);
        d = fmaf(qa[h].w, k0.w, d);
        d = fmaf(qb[h].x, k1.x, d);
        d = fmaf(qb[h].y, k1.y, d);
        d = fmaf(qb[h].z, k1.z, d);
        d = fmaf(qb[h].w, k1.w, d);
        const float sc = group8_sum(d) * scale;  // only this row group need be active
        const float mn = fmaxf(m[h], sc);
        const float f = expf(m[h] - mn);  // m = -inf on the first row: f = 0
        const float e = expf(sc - mn);
        l[h] = l[h] * f + e;
        o[h][0] = fmaf(o[h][0], f, e * v0.x);
        o[h][1] = fmaf(o[h][1], f, e * v0.y);
        o[h][2] = fmaf(o[h][2], f, e * v0.z);
        o[h][3] = fmaf(o[h][3], f, e * v0.w);
        o[h][4] = fmaf(o[h][4], f, e * v1.x);
        o[h][5] = fmaf(o[h][5], f, e * v1.y);
        o[h][6] = fmaf(o[h][6], f, e * v1.z);
        o[h][7] = fmaf(o[h][7], f, e * v1.w);
        m[h] = mn;
    }
}

// ------------------------------------------------------------------ kernel

__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const __grid_constant__ StepArgs a) {
    extern __shared__ __align__(1024) unsigned char smem[];
    Shared& sh = *reinterpret_cast<Shared*>(smem);
    unsigned char* ring = smem + kRingOffset;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int half = lane >> 4, l16 = lane & 15;
    const int G = gridDim.x, cta = blockIdx.x;

    Sched s;
    make_sched(a, G, cta, s);
    if (s.pos < 0 || s.pos >= a.capacity) {
        if (cta == 0 && tid == 0) atomicOr(a.error, 1);
        return;
    }
    if (tid == 0) {
        for (int i = 0; i < kStepSlots; ++i) mbar_init(&sh.bars[i], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        sh.head = sh.tail = 0;
        sh.issued = sh.released = 0;
        sh.abort = 0;
        if (cta == 0) *a.length = s.pos + 1;
    }
    __syncthreads();
    STEP_MARK(0);
    if (tid == 0) pump(a, s, sh, ring);

    int tile = 0;
    unsigned barrier = 0;
    const int64_t cap = a.capacity;
    for (int l = 0; l < kLayers; ++l) {
        const StepLayer& L = a.layer[l];
        // -------------------------------------------------------- phase A
        norm_into(sh, [&](int i) { return hidden_in(a, s, l, i); }, L.input_norm, a.eps);
        {
            // Zero this CTA's share of the replica set that phase D of this layer fills.
            float* acc = a.accum + (l & 1) * kStepReplicas * kHidden;
            const int n = kStepReplicas * kHidden;
            for (int i = cta * n / G + tid; i < (cta + 1) * n / G; i += kStepThreads) acc[i] = 0.0f;
        }
        if (s.t1 > s.t0) {
            const float* t = acquire(a, s, sh, ring, tile);
            if (t == nullptr) goto abort;
            if (warp < s.t1 - s.t0) {
                int ra, rb, kind;
                task_rows(s.t0 + warp, ra, rb, kind);
                const float y = row_dot(t + (2 * warp + half) * kHidden, sh.xs, l16);
                const float ya = __shfl_sync(0xffffffffu, y, 0);
                const float yb = __shfl_sync(0xffffffffu, y, 16);
                if (l16 == 0) {
                    const int row = half ? rb : ra;
                    if (kind == 2) {
                        const int u = row - kHidden - kKVHeads * kHeadDim;
                        a.value_cache[((static_cast<int64_t>(l) * kKVHeads + u / kHeadDim) * cap + s.pos) * kHeadDim +
                                      u % kHeadDim] = y;
                    } else {
                        const int d = row % kHeadDim;
                        const float c = __ldg(a.cos_table + s.pos * kHeadDim + d);
                        const float sn = __ldg(a.sin_table + s.pos * kHeadDim + d);
                        const float r = half ? rope_value(yb, ya, c, sn, false) : rope_value(ya, yb, c, sn, true);
                        if (kind == 0) {
                            a.q[row] = r;
                        } else {
                            const int h = (row - kHidden) / kHeadDim;
                            a.key_cache[((static_cast<int64_t>(l) * kKVHeads + h) * cap + s.pos) * kHeadDim + d] = r;
                        }
                    }
                }
            }
            release(a, s, sh, ring, tile++);
        }
        STEP_MARK(1 + 8 * l);
        if (!grid_sync(a, s, sh, ring, barrier++)) goto abort;
        STEP_MARK(2 + 8 * l);

        // -------------------------------------------------------- phase B
        if (s.g >= 0) {
            if (s.has_rows) {
                const int l8 = lane & 7, grp = warp * 4 + (lane >> 3);
                float4 qa[kGroup], qb[kGroup];
#pragma unroll
                for (int h = 0; h < kGroup; ++h) {
                    const float4* q4 = reinterpret_cast<const float4*>(a.q + (s.g * kGroup + h) * kHeadDim);
                    qa[h] = __ldcg(q4 + l8);
                    qb[h] = __ldcg(q4 + 8 + l8);
                }
                float m[kGroup], lsum[kGroup], o[kGroup][8];
#pragma unroll
                for (int h = 0; h < kGroup; ++h) {
                    m[h] = -INFINITY;
                    lsum[h] = 0.0f;
#pragma unroll
                    for (int j = 0; j < 8; ++j) o[h][j] = 0.0f;
                }
                for (int j = 0; j < s.n_att; ++j) {
                    const float* t = acquire(a, s, sh, ring, tile);
                    if (t == nullptr) goto abort;
                    const int64_t r0 = s.a0 + static_cast<int64_t>(j) * kStepAttnRows;
                    const int n = static_cast<int>(min(static_cast<int64_t>(kStepAttnRows), s.cached_end - r0));
                    if (grp < n) {
                        const float4* k4 = reinterpret_cast<const float4*>(t + grp * kHeadDim);
                        const float4* v4 = reinterpret_cast<const float4*>(t + (n + grp) * kHeadDim);
                        attend_row(qa, qb, k4[l8], k4[8 + l8], v4[l8], v4[8 + l8], L.scale, m, lsum, o);
                    }
                    release(a, s, sh, ring, tile++);
                }
                if (s.owns_new && grp == 0) {
                    const int64_t base = ((static_cast<int64_t>(l) * kKVHeads + s.g) * cap + s.pos) * kHeadDim;
                    const float4* k4 = reinterpret_cast<const float4*>(a.key_cache + base);
                    const float4* v4 = reinterpret_cast<const float4*>(a.value_cache + base);
                    attend_row(qa, qb, __ldcg(k4 + l8), __ldcg(k4 + 8 + l8), __ldcg(v4 + l8), __ldcg(v4 + 8 + l8),
                               L.scale, m, lsum, o);
                }
                // Combine the four row groups of each warp, then the 16 warps.
#pragma unroll
                for (int h = 0; h < kGroup; ++h) {
#pragma unroll
                    for (int off = 8; off <= 16; off <<= 1) {
                        const float mo = __shfl_xor_sync(0xffffffffu, m[h], off);
                        const float lo = __shfl_xor_sync(0xffffffffu, lsum[h], off);
                        const float mn = fmaxf(m[h], mo);
                        const float fa = m[h] == -INFINITY ? 0.0f : expf(m[h] - mn);
                        const float fb = mo == -INFINITY ? 0.0f : expf(mo - mn);
                        lsum[h] = lsum[h] * fa + lo * fb;
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const float oo = __shfl_xor_sync(0xffffffffu, o[h][j], off);
                            o[h][j] = o[h][j] * fa + oo * fb;
                        }
                        m[h] = mn;
                    }
                    if (lane < 8) {
                        if (lane == 0) {
                            sh.wm[warp][h] = m[h];
                            sh.wl[warp][h] = lsum[h];
                        }
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            sh.wo[warp][h][4 * l8 + j] = o[h][j];
                            sh.wo[warp][h][32 + 4 * l8 + j] = o[h][4 + j];
                        }
                    }
                }
                __syncthreads();
                if (tid < kGroup * kHeadDim) {
                    const int h = tid / kHeadDim, d = tid % kHeadDim;
                    float mx = -INFINITY;
#pragma unroll
                    for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, sh.wm[w][h]);
                    float total = 0.0f, acc = 0.0f;
#pragma unroll
                    for (int w = 0; w < kWarps; ++w) {
                        const float f = sh.wm[w][h] == -INFINITY ? 0.0f : expf(sh.wm[w][h] - mx);
                        total += sh.wl[w][h] * f;
                        acc += sh.wo[w][h][d] * f;
                    }
                    float* pw = a.partials +
                                ((static_cast<int64_t>(s.g) * kGroup + h) * a.nch + s.c) * kStepPartialStride;
                    pw[4 + d] = acc;
                    if (d == 0) {
                        pw[0] = mx;
                        pw[1] = total;
                    }
                }
            }
            // The last CTA of this kv head merges the active chunks.
            __syncthreads();
            if (tid == 0) {
                __threadfence();
                sh.is_last = atomicAdd(&a.sync[1 + s.g], 1u) == static_cast<unsigned>(a.nch - 1);
            }
            __syncthreads();
            if (sh.is_last) {
                __threadfence();
                if (tid < kGroup * kHeadDim) {
                    const int h = tid / kHeadDim, d = tid % kHeadDim;
                    const float* base = a.partials + (static_cast<int64_t>(s.g) * kGroup + h) * a.nch * kStepPartialStride;
                    float mx = -INFINITY;
                    for (int cc = 0; cc < s.active; ++cc) mx = fmaxf(mx, __ldcg(base + cc * kStepPartialStride));
                    float total = 0.0f, acc = 0.0f;
                    for (int cc = 0; cc < s.active; ++cc) {
                        const float* pc = base + cc * kStepPartialStride;
                        const float f = expf(__ldcg(pc) - mx);
                        total += __ldcg(pc + 1) * f;
                        acc += __ldcg(pc + 4 + d) * f;
                    }
                    a.attn[(s.g * kGroup + h) * kHeadDim + d] = acc / total;
                }
                if (tid == 0) a.sync[1 + s.g] = 0u;
            }
        }
        STEP_MARK(3 + 8 * l);
        if (!grid_sync(a, s, sh, ring, barrier++)) goto abort;
        STEP_MARK(4 + 8 * l);

        // -------------------------------------------------------- phase C
        for (int i = tid; i < kHidden; i += kStepThreads) sh.xs[i] = __ldcg(a.attn + i);
        __syncthreads();
        if (s.o1 > s.o0) {
            const float* t = acquire(a, s, sh, ring, tile);
            if (t == nullptr) goto abort;
            const int nrows = s.o1 - s.o0;
            const int w2 = warp * 2 + half;
            if (warp * 2 < nrows) {  // whole warps take part in the half-warp shuffles
                const int rr = w2 < nrows ? w2 : 0;
                const float y = row_dot(t + rr * kHidden, sh.xs, l16);
                if (l16 == 0 && w2 < nrows) {
                    const int r = s.o0 + w2;
                    a.hidden_mid[r] = y + hidden_in(a, s, l, r);
                }
            }
            release(a, s, sh, ring, tile++);
        }
        STEP_MARK(5 + 8 * l);
        if (!grid_sync(a, s, sh, ring, barrier++)) goto abort;
        STEP_MARK(6 + 8 * l);

        // -------------------------------------------------------- phase D
        norm_into(sh, [&](int i) { return __ldcg(a.hidden_mid + i); }, L.post_norm, a.eps);
        if (s.i1 > s.i0) {
            const int ni = s.i1 - s.i0;
            const float* t = acquire(a, s, sh, ring, tile);
            if (t == nullptr) goto abort;
            if (warp < ni) {
                const float y = row_dot(t + (half * ni + warp) * kHidden, sh.xs, l16);
                const float up = __shfl_sync(0xffffffffu, y, 16);
                if (lane == 0) sh.sv[warp] = swiglu(y, up);
            }
            release(a, s, sh, ring, tile++);
            const float* wd = acquire(a, s, sh, ring, tile);
            if (wd == nullptr) goto abort;
            if (tid < kHidden / 4) {
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int w = 0; w < ni; ++w) {
                    const float sw = sh.sv[w];
                    const float4 v = reinterpret_cast<const float4*>(wd + w * kHidden)[tid];
                    acc.x = fmaf(sw, v.x, acc.x);
                    acc.y = fmaf(sw, v.y, acc.y);
                    acc.z = fmaf(sw, v.z, acc.z);
                    acc.w = fmaf(sw, v.w, acc.w);
                }
                red_add_v4(a.accum + ((l & 1) * kStepReplicas + cta % kStepReplicas) * kHidden + 4 * tid, acc);
            }
            release(a, s, sh, ring, tile++);
        }
        STEP_MARK(7 + 8 * l);
        if (!grid_sync(a, s, sh, ring, barrier++)) goto abort;
        STEP_MARK(8 + 8 * l);
    }

    // ------------------------------------------------------------ LM head
    {
        STEP_MARK(1 + 8 * kLayers);
        norm_into(sh, [&](int i) { return hidden_in(a, s, kLayers, i); }, a.final_norm, a.eps);
        if (cta == 0)
            for (int i = tid; i < kHidden; i += kStepThreads) a.final_norm_out[i] = sh.xs[i];
        float bv = 0.0f;
        long long bi = -1;
        for (int j = 0; j < s.n_lm; ++j) {
            const float* t = acquire(a, s, sh, ring, tile);
            if (t == nullptr) goto abort;
            const int64_t r0 = s.v0 + static_cast<int64_t>(j) * kStepLmRows;
            const int n = static_cast<int>(min(static_cast<int64_t>(kStepLmRows), s.v1 - r0));
            const int w2 = warp * 2 + half;
            if (warp * 2 < n) {
                const int rr = w2 < n ? w2 : 0;
                const float y = row_dot(t + rr * kHidden, sh.xs, l16);
                if (l16 == 0 && w2 < n) {
                    a.logits[r0 + w2] = y;
                    argmax_take(bv, bi, y, r0 + w2);
                }
            }
            release(a, s, sh, ring, tile++);
        }
        const float ov = __shfl_sync(0xffffffffu, bv, 16);
        const long long oi = __shfl_sync(0xffffffffu, bi, 16);
        if (lane == 0) {
            argmax_take(bv, bi, ov, oi);
            sh.cv[warp] = bv;
            sh.ci[warp] = bi;
        }
        __syncthreads();
        STEP_MARK(2 + 8 * kLayers);
        if (tid == 0) {
            for (int w = 1; w < kWarps; ++w) argmax_take(bv, bi, sh.cv[w], sh.ci[w]);
            a.cand_value[cta] = bv;
            a.cand_index[cta] = bi;
            __threadfence();
            sh.is_last = atomicAdd(&a.sync[4], 1u) == static_cast<unsigned>(G - 1);
        }
        __syncthreads();
        if (sh.is_last && warp == 0) {
            __threadfence();
            bv = 0.0f;
            bi = -1;
            for (int c = lane; c < G; c += 32) argmax_take(bv, bi, __ldcg(a.cand_value + c), __ldcg(a.cand_index + c));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const float v = __shfl_xor_sync(0xffffffffu, bv, off);
                const long long i = __shfl_xor_sync(0xffffffffu, bi, off);
                argmax_take(bv, bi, v, i);
            }
            if (lane == 0) {
                const int64_t selected = bi < 0 ? 0 : bi;
                *a.token = selected;
                const int64_t st = *a.step;
                if (st >= 0 && st < cap) a.generated[st] = selected;
                *a.step = st + 1;
                *a.position = s.pos + 1;
                a.sync[0] = 0u;
                a.sync[4] = 0u;
            }
        }
    }
    return;

abort:
    // Give up: wait (bounded) for this CTA's copies in flight, then leave.
    if (tid == 0) {
        for (int k = sh.released; k < sh.issued; ++k) {
            const unsigned long long t0 = global_timer();
            while (!mbar_try_wait(&sh.bars[k % kStepSlots], static_cast<uint32_t>(k / kStepSlots) & 1u))
                if (global_timer() - t0 > kWaitNs) break;
        }
        atomicOr(a.error, 2);
    }
}

__global__ void transpose_down_kernel(const float* __restrict__ src, float* __restrict__ dst) {
    // src [576, 1536] -> dst [1536, 576]
    __shared__ float tile[32][33];
    const int x = blockIdx.x * 32 + threadIdx.x;  // column of src (0..1535)
    const int y0 = blockIdx.y * 32;               // row of src (0..575)
    for (int j = threadIdx.y; j < 32; j += blockDim.y) tile[j][threadIdx.x] = src[(y0 + j) * kInter + x];
    __syncthreads();
    const int ox = y0 + threadIdx.x;
    for (int j = threadIdx.y; j < 32; j += blockDim.y)
        dst[static_cast<int64_t>(blockIdx.x * 32 + j) * kHidden + ox] = tile[threadIdx.x][j];
}

}  // namespace

size_t step_kernel_smem_bytes() { return kRingOffset + kStepRingBytes; }

fx_status launch_step_kernel(const StepArgs& args, int grid, cudaStream_t stream) {
    cudaLaunchConfig_t config{};
    config.gridDim = dim3(static_cast<unsigned>(grid));
    config.blockDim = dim3(kStepThreads);
    config.dynamicSmemBytes = step_kernel_smem_bytes();
    config.stream = stream;
    cudaLaunchAttribute attribute{};
    attribute.id = cudaLaunchAttributeCooperative;
    attribute.val.cooperative = 1;
    config.attrs = &attribute;
    config.numAttrs = 1;
    FX_CUDA_TRY(cudaLaunchKernelEx(&config, decode_step_kernel, args), "launching the persistent decode step");
    return FX_OK;
}

fx_status prepare_step_kernel(int device, int* grid) {
    const size_t smem = step_kernel_smem_bytes();
    FX_CUDA_TRY(cudaFuncSetAttribute(decode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem)),
                "raising the step kernel's shared memory");
    int per_sm = 0;
    FX_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_step_kernel, kStepThreads, smem),
                "querying step kernel occupancy");
    int sms = 0;
    FX_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device), "querying SM count");
    if (per_sm < 1) {
        set_error("flux native decode: the persistent step kernel does not fit on one SM");
        return FX_ERR_CUDA;
    }
    *grid = sms;
    return FX_OK;
}

fx_status launch_transpose_down(const float* const* down, float* down_t, cudaStream_t stream) {
    for (int l = 0; l < kLayers; ++l) {
        transpose_down_kernel<<<dim3(kInter / 32, kHidden / 32), dim3(32, 8), 0, stream>>>(
            down[l], down_t + static_cast<int64_t>(l) * kInter * kHidden);
    }
    FX_CUDA_TRY(cudaGetLastError(), "transposing the down projections");
    return FX_OK;
}

}  // namespace fx
