// The whole batch-1 decode step as ONE persistent cooperative launch.
//
// One CTA per SM, 512 threads: 15 consumer warps do the math, one producer
// warp streams weights and cache rows into a ring of 7 x 27 KB shared-memory
// slots with 1-D TMA bulk copies (cp.async.bulk, no multicast) completing on
// full/empty mbarrier pairs.  The producer walks the CTA's tiles in the order
// the consumers use them and runs up to 7 tiles ahead, so HBM keeps streaming
// while the consumers wait for values from other CTAs.
//
// Each CTA owns a fixed slice of every projection and one (kv head, chunk)
// of the attention.  Per layer, six dependent phases and no grid barrier:
//
//   A  poll h (576); RMSNorm; its QKV row pairs; RoPE; publish q / k / v of
//      the current row; write the K / V row into the cache.
//   B  poll q of its kv head (and the new K/V row if its chunk holds it);
//      online softmax over its chunk of cache rows for the 3 q heads;
//      publish (m, l, o) per head.
//   M  every attention CTA merges 3-4 of the 192 output dims of its kv head
//      over the partials of all chunks and publishes them.
//   C  poll attn; its o_proj rows; publish h' = h + o_proj(attn).
//   D  poll h'; RMSNorm; its gate and up rows; publish SwiGLU.
//   E  poll SwiGLU (1536); its down rows; publish h_next = h' + down(SwiGLU).
//
// then the LM head (its vocab rows and greedy candidate; the last CTA to
// arrive picks the token, advances the device state and the step epoch).
//
// Cross-CTA values travel as 64-bit words (tag << 32 | float bits): a reader
// polls a word with relaxed gpu-scope loads until it carries the tag of the
// current (step, layer), so one L2 round trip both waits for and delivers the
// value.  Every wait (mbarrier or poll) is bounded by %globaltimer; on expiry
// the CTA sets error bit 2, drains its copies in flight and returns, and the
// other CTAs give up at their next wait once they see the error word.
#include "step_kernel.cuh"

#include <algorithm>

namespace fx {
namespace {

constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s per wait
constexpr unsigned long long kPeerCheckNs = 1000000ull;  // look at the error word after 1 ms
constexpr int kConsumerWarps = kStepConsumers / 32;     // 15
constexpr int kProducerWarp = kConsumerWarps;           // warp 15
constexpr int kRowBytes = kHidden * 4;                  // one 576-float row
constexpr int kMaxSeg = 10;
constexpr int kMaxChunks = 64;
constexpr int kMergeDims = 8;  // output dims merged per attention CTA (192 / chunks, chunks >= 24)

// ------------------------------------------------------------- PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ unsigned long long ld_word(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ int ld_error(const int* p) {
    int v;
    asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_word(unsigned long long* p, uint32_t tag, float x) {
    const unsigned long long v = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(x);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint32_t word_tag(unsigned long long v) { return static_cast<uint32_t>(v >> 32); }
__device__ __forceinline__ float word_value(unsigned long long v) {
    return __uint_as_float(static_cast<uint32_t>(v));
}

// Named barrier of the 15 consumer warps (the producer warp never joins it).
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 480;" ::: "memory"); }

__device__ __forceinline__ int64_t min64(int64_t x, int64_t y) { return x < y ? x : y; }

#define LAYER_MARK(event) STEP_MARK(1 + kStepTimelinePerLayer * l + (event))
#define STEP_MARK(event)                                                                                  \
    do {                                                                                                  \
        if (a.timeline != nullptr && threadIdx.x == 0)                                                     \
            a.timeline[static_cast<size_t>(blockIdx.x) * kStepTimelineEvents + (event)] = global_timer(); \
    } while (0)

// ------------------------------------------------------------ shared state

struct AttnCombine {
    float wm[kConsumerWarps][kGroup];
    float wl[kConsumerWarps][kGroup];
    float wo[kConsumerWarps][kGroup][kHeadDim];
};

struct Shared {
    uint64_t full[kStepSlots];
    uint64_t empty[kStepSlots];
    alignas(16) float hraw[kHidden];          // layer input h (residual of phase C)
    alignas(16) float mid[kHidden];           // h' (phase D input)
    alignas(16) float xs[kHidden];            // normalised vector / attention output
    alignas(16) float qs[kGroup * kHeadDim];  // q of this CTA's kv head
    alignas(16) float knew[kHeadDim];
    alignas(16) float vnew[kHeadDim];
    float gate[32];
    float mid_rows[8];                        // h' of this CTA's o_proj / down rows
    float scratch[32];
    float cv[kConsumerWarps];
    long long ci[kConsumerWarps];
    float mm[kMergeDims][kMaxChunks];  // phase M: m, l, o[d] per (output dim, chunk)
    float ml[kMergeDims][kMaxChunks];
    float mo[kMergeDims][kMaxChunks];
    union {
        AttnCombine att;
        alignas(16) float s[kInter];
    } u;
    volatile int abort;
    int is_last;
    int consumed;  // tiles released by the consumers
    int issued;    // tiles issued by the producer
};

constexpr size_t kRingOffset = (sizeof(Shared) + 127) / 128 * 128;

// The CTA's fixed share of every phase, derived from (grid, CTA, position).
struct Sched {
    int t0, t1;          // QKV row-pair tasks
    int o0, o1;          // o_proj / down rows
    int i0, i1;          // intermediate features
    int64_t v0, v1;      // vocab rows
    int g, c;            // attention kv head / chunk (g < 0: none)
    int64_t a0, a1;      // rows [a0, a1) of the valid length
    int64_t cached_end;  // rows [a0, cached_end) stream through the ring
    bool owns_new;       // the chunk holds row `pos` (read from the exchange)
    bool has_rows;
    int active;          // active chunks per kv head
    int n_att, n_down, n_lm, per_layer, total;
    int64_t pos, tok;
    uint32_t epoch;
};

struct Tile {
    int nseg;
    const float* src[kMaxSeg];
    uint32_t bytes[kMaxSeg];
    uint32_t total;
};

// QKV task -> its two rows.  Tasks 0..287: q (head, d < 32) with partner
// d + 32; 288..383: k likewise; 384..479: v rows 2t, 2t + 1.
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
    s.epoch = a.sync[1];
    const int64_t len = s.pos + 1;
    s.g = -1;
    s.c = 0;
    s.a0 = s.a1 = s.cached_end = 0;
    s.owns_new = s.has_rows = false;
    s.active = 0;
    if (cta < kKVHeads * a.nch) {
        s.g = cta / a.nch;
        s.c = cta % a.nch;
        const int64_t chunk = (len + a.nch - 1) / a.nch;
        s.active = static_cast<int>((len + chunk - 1) / chunk);
        if (s.c < s.active) {
            s.has_rows = true;
            s.a0 = s.c * chunk;
            s.a1 = min64(len, s.a0 + chunk);
            s.cached_end = min64(s.a1, s.pos);
            s.owns_new = s.pos >= s.a0 && s.pos < s.a1;
        }
    }
    const int64_t cached = s.cached_end > s.a0 ? s.cached_end - s.a0 : 0;
    s.n_att = static_cast<int>((cached + kStepAttnRows - 1) / kStepAttnRows);
    s.n_down = (s.o1 - s.o0 + kStepDownRows - 1) / kStepDownRows;
    s.per_layer = 1 + s.n_att + 3 + s.n_down;
    s.n_lm = s.v1 > s.v0 ? 1 + static_cast<int>((s.v1 - s.v0 + kStepLmRows - 1) / kStepLmRows) : 0;
    s.total = kLayers * s.per_layer + s.n_lm;
}

// The k-th tile of this CTA, in consumption order.
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
        if (sub == 0) {  // [input norm][row_a, row_b per task]
            add(L.input_norm, kRowBytes);
            for (int task = s.t0; task < s.t1; ++task) {
                int ra, rb, kind;
                task_rows(task, ra, rb, kind);
                add(L.qkv + static_cast<int64_t>(ra) * kHidden, kRowBytes);
                add(L.qkv + static_cast<int64_t>(rb) * kHidden, kRowBytes);
            }
            return;
        }
        sub -= 1;
        if (sub < s.n_att) {  // [K rows][V rows]
            const int64_t r0 = s.a0 + static_cast<int64_t>(sub) * kStepAttnRows;
            const int64_t n = min64(kStepAttnRows, s.cached_end - r0);
            const int64_t base = ((static_cast<int64_t>(l) * kKVHeads + s.g) * a.capacity + r0) * kHeadDim;
            add(a.key_cache + base, static_cast<uint32_t>(n * kHeadDim * 4));
            add(a.value_cache + base, static_cast<uint32_t>(n * kHeadDim * 4));
            return;
        }
        sub -= s.n_att;
        const int ni = s.i1 - s.i0;
        if (sub == 0) {
            add(L.o_proj + static_cast<int64_t>(s.o0) * kHidden, (s.o1 - s.o0) * kRowBytes);
        } else if (sub == 1) {  // [post norm][gate rows]
            add(L.post_norm, kRowBytes);
            add(L.gate_up + static_cast<int64_t>(s.i0) * kHidden, ni * kRowBytes);
        } else if (sub == 2) {  // [up rows]
            add(L.gate_up + static_cast<int64_t>(kInter + s.i0) * kHidden, ni * kRowBytes);
        } else {  // [down rows] (1536 floats each)
            const int r0 = s.o0 + (sub - 3) * kStepDownRows;
            const int n = min(kStepDownRows, s.o1 - r0);
            add(L.down + static_cast<int64_t>(r0) * kInter, n * kInter * 4);
        }
        return;
    }
    const int j = k - kLayers * s.per_layer;
    if (j == 0) {
        add(a.final_norm, kRowBytes);
        return;
    }
    const int64_t r0 = s.v0 + static_cast<int64_t>(j - 1) * kStepLmRows;
    const int64_t n = min64(kStepLmRows, s.v1 - r0);
    add(a.lm_head + r0 * kHidden, static_cast<uint32_t>(n * kRowBytes));
}

__device__ __forceinline__ void fail(const StepArgs& a, Shared& sh) {
    sh.abort = 1;
    atomicOr(a.error, 2);
}

// Bounded mbarrier wait; false when the wait gave up or the CTA aborted.
__device__ bool wait_bar(const StepArgs& a, Shared& sh, uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_timer();
    while (!mbar_try_wait(bar, parity)) {
        if (sh.abort) return false;
        if (global_timer() - t0 > kWaitNs) {
            fail(a, sh);
            return false;
        }
    }
    return true;
}

// Consumer side of tile k: wait until it landed; nullptr (uniformly) on abort.
__device__ const float* acquire(const StepArgs& a, Shared& sh, unsigned char* ring, int k) {
    const int slot = k % kStepSlots;
    wait_bar(a, sh, &sh.full[slot], static_cast<uint32_t>(k / kStepSlots) & 1u);
    consumer_sync();
    if (sh.abort) return nullptr;
    return reinterpret_cast<const float*>(ring + static_cast<size_t>(slot) * kStepSlotBytes);
}

__device__ void release(Shared& sh, int k) {
    consumer_sync();
    if (threadIdx.x == 0) {
        mbar_arrive(&sh.empty[k % kStepSlots]);
        sh.consumed = k + 1;
    }
}

// Spin (bounded) until the word at p carries `tag`; returns the word.
__device__ unsigned long long poll_word(const StepArgs& a, Shared& sh, const unsigned long long* p,
                                        unsigned long long v, uint32_t tag) {
    const unsigned long long t0 = global_timer();
    while (word_tag(v) != tag) {
        __nanosleep(32);
        v = ld_word(p);
        if (sh.abort) break;
        const unsigned long long dt = global_timer() - t0;
        if (dt > kPeerCheckNs && ld_error(a.error) != 0) {
            sh.abort = 1;
            break;
        }
        if (dt > kWaitNs) {
            fail(a, sh);
            break;
        }
    }
    return v;
}

// The consumers poll n tagged words into dst; false (uniformly) on abort.
__device__ bool poll_into(const StepArgs& a, Shared& sh, const unsigned long long* src, int n, uint32_t tag,
                          float* dst) {
    const int ct = threadIdx.x;
    const unsigned long long ready = static_cast<unsigned long long>(tag) << 32;
    for (int base = ct; base < n; base += 4 * kStepConsumers) {
        unsigned long long v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = base + j * kStepConsumers;
            v[j] = i < n ? ld_word(src + i) : ready;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = base + j * kStepConsumers;
            if (word_tag(v[j]) != tag) v[j] = poll_word(a, sh, src + i, v[j], tag);
            if (i < n) dst[i] = word_value(v[j]);
        }
    }
    consumer_sync();
    return !sh.abort;
}

// Sum over the 480 consumer threads (fixed order); every consumer gets it.
__device__ float consumer_sum(Shared& sh, float v) {
    v = warp_sum(v);
    consumer_sync();
    if ((threadIdx.x & 31) == 0) sh.scratch[threadIdx.x >> 5] = v;
    consumer_sync();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) t += sh.scratch[w];
    return t;
}

// xs = src * rsqrt(mean(src^2) + eps) * w (rmsnorm_cuda.cu:23-89).
__device__ void normalise(Shared& sh, const float* src, const float* w, float eps) {
    float ss = 0.0f;
    for (int i = threadIdx.x; i < kHidden; i += kStepConsumers) ss = fmaf(src[i], src[i], ss);
    ss = consumer_sum(sh, ss);
    const float inv = rsqrtf(ss / static_cast<float>(kHidden) + eps);
    for (int i = threadIdx.x; i < kHidden; i += kStepConsumers) sh.xs[i] = src[i] * inv * w[i];
    consumer_sync();
}

// Half-warp dot product of a 576-float row with xs (both in shared memory).
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
        const float f = expf(m[h] - mn);  // m = -inf before the first row: f = 0
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

__device__ __forceinline__ size_t buf(int l) { return static_cast<size_t>(l & 1); }

// ------------------------------------------------------------------ kernel

__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const __grid_constant__ StepArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    Shared& sh = *reinterpret_cast<Shared*>(smem);
    unsigned char* ring = smem + kRingOffset;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, cta = blockIdx.x;

    Sched s;
    make_sched(a, G, cta, s);
    if (s.pos < 0 || s.pos >= a.capacity) {
        if (cta == 0 && tid == 0) atomicOr(a.error, 1);
        return;
    }
    if (tid == 0) {
        for (int i = 0; i < kStepSlots; ++i) {
            mbar_init(&sh.full[i], 1);
            mbar_init(&sh.empty[i], 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        sh.abort = 0;
        sh.consumed = 0;
        sh.issued = 0;
        if (cta == 0) *a.length = s.pos + 1;
    }
    __syncthreads();
    STEP_MARK(0);

    if (warp == kProducerWarp) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            for (int k = 0; k < s.total; ++k) {
                const int slot = k % kStepSlots;
                if (!wait_bar(a, sh, &sh.empty[slot], (static_cast<uint32_t>(k / kStepSlots) & 1u) ^ 1u)) break;
                Tile t;
                make_tile(a, s, k, t);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive_expect_tx(&sh.full[slot], t.total);
                uint32_t off = 0;
                unsigned char* dst = ring + static_cast<size_t>(slot) * kStepSlotBytes;
                for (int i = 0; i < t.nseg; ++i) {
                    bulk_load(dst + off, t.src[i], t.bytes[i], &sh.full[slot]);
                    off += t.bytes[i];
                }
                sh.issued = k + 1;
            }
        }
    } else {
        // --------------------------------------------------------- consumers
        const int half = lane >> 4, l16 = lane & 15;
        const int64_t cap = a.capacity;
        int k = 0;
        for (int l = 0; l < kLayers; ++l) {
            const uint32_t tag = s.epoch * 64u + static_cast<uint32_t>(l) + 1u;
            // ------------------------------------------------------ phase A
            if (l == 0) {
                const bool valid = s.tok >= 0 && s.tok < a.vocab;
                for (int i = tid; i < kHidden; i += kStepConsumers)
                    sh.hraw[i] = valid ? __ldg(a.embedding + s.tok * kHidden + i) : 0.0f;
                consumer_sync();
            } else if (!poll_into(a, sh, a.x.hidden + buf(l) * kHidden, kHidden, tag, sh.hraw)) {
                goto done;
            }
            LAYER_MARK(0);
            {
                const float* t = acquire(a, sh, ring, k);
                if (t == nullptr) goto done;
                LAYER_MARK(1);
                normalise(sh, sh.hraw, t, a.eps);
                if (warp < s.t1 - s.t0) {
                    int ra, rb, kind;
                    task_rows(s.t0 + warp, ra, rb, kind);
                    const float y = row_dot(t + kHidden * (1 + 2 * warp + half), sh.xs, l16);
                    const float ya = __shfl_sync(0xffffffffu, y, 0);
                    const float yb = __shfl_sync(0xffffffffu, y, 16);
                    if (l16 == 0) {
                        const int row = half ? rb : ra;
                        unsigned long long* out = a.x.qkv + buf(l) * kQKV;
                        if (kind == 2) {
                            const int u = row - kHidden - kKVHeads * kHeadDim;
                            a.value_cache[((static_cast<int64_t>(l) * kKVHeads + u / kHeadDim) * cap + s.pos) *
                                              kHeadDim +
                                          u % kHeadDim] = y;
                            st_word(out + row, tag, y);
                        } else {
                            const int d = row % kHeadDim;
                            const float c = __ldg(a.cos_table + s.pos * kHeadDim + d);
                            const float sn = __ldg(a.sin_table + s.pos * kHeadDim + d);
                            const float r = half ? rope_value(yb, ya, c, sn, false) : rope_value(ya, yb, c, sn, true);
                            if (kind == 1) {
                                const int h = (row - kHidden) / kHeadDim;
                                a.key_cache[((static_cast<int64_t>(l) * kKVHeads + h) * cap + s.pos) * kHeadDim + d] = r;
                            }
                            st_word(out + row, tag, r);
                        }
                    }
                }
                release(sh, k++);
            }
            LAYER_MARK(2);

            // ------------------------------------------------------ phase B
            if (s.has_rows) {
                const unsigned long long* qkv = a.x.qkv + buf(l) * kQKV;
                if (!poll_into(a, sh, qkv + s.g * kGroup * kHeadDim, kGroup * kHeadDim, tag, sh.qs)) goto done;
                if (s.owns_new) {
                    if (!poll_into(a, sh, qkv + kHidden + s.g * kHeadDim, kHeadDim, tag, sh.knew)) goto done;
                    if (!poll_into(a, sh, qkv + kHidden + kKVHeads * kHeadDim + s.g * kHeadDim, kHeadDim, tag,
                                   sh.vnew))
                        goto done;
                }
                LAYER_MARK(3);
                const float scale = a.layer[l].scale;
                const int l8 = lane & 7, grp = warp * 4 + (lane >> 3);
                float4 qa[kGroup], qb[kGroup];
#pragma unroll
                for (int h = 0; h < kGroup; ++h) {
                    qa[h] = reinterpret_cast<const float4*>(sh.qs + h * kHeadDim)[l8];
                    qb[h] = reinterpret_cast<const float4*>(sh.qs + h * kHeadDim)[8 + l8];
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
                    const float* t = acquire(a, sh, ring, k);
                    if (t == nullptr) goto done;
                    const int64_t r0 = s.a0 + static_cast<int64_t>(j) * kStepAttnRows;
                    const int n = static_cast<int>(min64(kStepAttnRows, s.cached_end - r0));
                    if (grp < n) {
                        const float4* k4 = reinterpret_cast<const float4*>(t + grp * kHeadDim);
                        const float4* v4 = reinterpret_cast<const float4*>(t + (n + grp) * kHeadDim);
                        attend_row(qa, qb, k4[l8], k4[8 + l8], v4[l8], v4[8 + l8], scale, m, lsum, o);
                    }
                    release(sh, k++);
                }
                LAYER_MARK(4);
                if (s.owns_new && grp == 0) {
                    const float4* k4 = reinterpret_cast<const float4*>(sh.knew);
                    const float4* v4 = reinterpret_cast<const float4*>(sh.vnew);
                    attend_row(qa, qb, k4[l8], k4[8 + l8], v4[l8], v4[8 + l8], scale, m, lsum, o);
                }
                // Combine the four row groups of each warp, then the 15 warps.
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
                            sh.u.att.wm[warp][h] = m[h];
                            sh.u.att.wl[warp][h] = lsum[h];
                        }
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            sh.u.att.wo[warp][h][4 * l8 + j] = o[h][j];
                            sh.u.att.wo[warp][h][32 + 4 * l8 + j] = o[h][4 + j];
                        }
                    }
                }
                consumer_sync();
                if (tid < kGroup * kHeadDim) {
                    const int h = tid / kHeadDim, d = tid % kHeadDim;
                    float mx = -INFINITY;
#pragma unroll
                    for (int w = 0; w < kConsumerWarps; ++w) mx = fmaxf(mx, sh.u.att.wm[w][h]);
                    float total = 0.0f, acc = 0.0f;
#pragma unroll
                    for (int w = 0; w < kConsumerWarps; ++w) {
                        const float f = sh.u.att.wm[w][h] == -INFINITY ? 0.0f : expf(sh.u.att.wm[w][h] - mx);
                        total = fmaf(sh.u.att.wl[w][h], f, total);
                        acc = fmaf(sh.u.att.wo[w][h][d], f, acc);
                    }
                    unsigned long long* pw = a.x.partial + buf(l) * (static_cast<size_t>(kQHeads) * a.nch * kStepPartial) +
                                             ((static_cast<size_t>(s.g) * kGroup + h) * a.nch + s.c) * kStepPartial;
                    st_word(pw + 2 + d, tag, acc);
                    if (d == 0) {
                        st_word(pw, tag, mx);
                        st_word(pw + 1, tag, total);
                    }
                }
                consumer_sync();
            }
            LAYER_MARK(5);

            // ------------------------------------------------------ phase M
            // Every attention CTA (g, c) merges output dims j = c, c + nch, ...
            // (< 192) of kv head g over the active chunks: one round of loads.
            if (s.g >= 0) {
                const unsigned long long* part = a.x.partial +
                                                 buf(l) * (static_cast<size_t>(kQHeads) * a.nch * kStepPartial) +
                                                 static_cast<size_t>(s.g) * kGroup * a.nch * kStepPartial;
                const int act = s.active;
                const int nd = (kGroup * kHeadDim - s.c + a.nch - 1) / a.nch;
                if (tid < nd * act) {
                    const int q = tid / act, cc = tid % act;
                    const int j = s.c + q * a.nch, h = j / kHeadDim, d = j % kHeadDim;
                    const unsigned long long* p = part + (static_cast<size_t>(h) * a.nch + cc) * kStepPartial;
                    unsigned long long vm = ld_word(p), vl = ld_word(p + 1), vo = ld_word(p + 2 + d);
                    if (word_tag(vm) != tag) vm = poll_word(a, sh, p, vm, tag);
                    if (word_tag(vl) != tag) vl = poll_word(a, sh, p + 1, vl, tag);
                    if (word_tag(vo) != tag) vo = poll_word(a, sh, p + 2 + d, vo, tag);
                    sh.mm[q][cc] = word_value(vm);
                    sh.ml[q][cc] = word_value(vl);
                    sh.mo[q][cc] = word_value(vo);
                }
                consumer_sync();
                if (sh.abort) goto done;
                LAYER_MARK(6);
                if (warp < nd) {
                    float mx = -INFINITY;
                    for (int cc = lane; cc < act; cc += 32) mx = fmaxf(mx, sh.mm[warp][cc]);
                    mx = warp_max(mx);
                    float total = 0.0f, acc = 0.0f;
                    for (int cc = lane; cc < act; cc += 32) {
                        const float w = expf(sh.mm[warp][cc] - mx);
                        total = fmaf(w, sh.ml[warp][cc], total);
                        acc = fmaf(w, sh.mo[warp][cc], acc);
                    }
                    total = warp_sum(total);
                    acc = warp_sum(acc);
                    if (lane == 0) {
                        const int j = s.c + warp * a.nch;
                        st_word(a.x.attn + buf(l) * kHidden + s.g * kGroup * kHeadDim + j, tag, acc / total);
                    }
                }
            }
            LAYER_MARK(7);

            // ------------------------------------------------------ phase C
            if (!poll_into(a, sh, a.x.attn + buf(l) * kHidden, kHidden, tag, sh.xs)) goto done;
            LAYER_MARK(8);
            {
                const float* t = acquire(a, sh, ring, k);
                if (t == nullptr) goto done;
                LAYER_MARK(9);
                const int nrows = s.o1 - s.o0;
                const int w2 = warp * 2 + half;
                if (warp * 2 < nrows) {  // whole warps enter the half-warp shuffles
                    const int rr = w2 < nrows ? w2 : 0;
                    const float y = row_dot(t + rr * kHidden, sh.xs, l16);
                    if (l16 == 0 && w2 < nrows) {
                        const int r = s.o0 + w2;
                        const float mid = sh.hraw[r] + y;
                        sh.mid_rows[w2] = mid;
                        st_word(a.x.mid + buf(l) * kHidden + r, tag, mid);
                    }
                }
                release(sh, k++);
            }
            LAYER_MARK(10);

            // ------------------------------------------------------ phase D
            if (!poll_into(a, sh, a.x.mid + buf(l) * kHidden, kHidden, tag, sh.mid)) goto done;
            LAYER_MARK(11);
            {
                const int ni = s.i1 - s.i0;
                const int w2 = warp * 2 + half;
                const float* t = acquire(a, sh, ring, k);
                if (t == nullptr) goto done;
                normalise(sh, sh.mid, t, a.eps);
                if (warp * 2 < ni) {
                    const int rr = w2 < ni ? w2 : 0;
                    const float y = row_dot(t + kHidden * (1 + rr), sh.xs, l16);
                    if (l16 == 0 && w2 < ni) sh.gate[w2] = y;
                }
                release(sh, k++);
                const float* tu = acquire(a, sh, ring, k);
                if (tu == nullptr) goto done;
                if (warp * 2 < ni) {
                    const int rr = w2 < ni ? w2 : 0;
                    const float y = row_dot(tu + rr * kHidden, sh.xs, l16);
                    if (l16 == 0 && w2 < ni)
                        st_word(a.x.swiglu + buf(l) * kInter + s.i0 + w2, tag, swiglu(sh.gate[w2], y));
                }
                release(sh, k++);
            }
            LAYER_MARK(12);

            // ------------------------------------------------------ phase E
            if (!poll_into(a, sh, a.x.swiglu + buf(l) * kInter, kInter, tag, sh.u.s)) goto done;
            LAYER_MARK(13);
            for (int j = 0; j < s.n_down; ++j) {
                const float* t = acquire(a, sh, ring, k);
                if (t == nullptr) goto done;
                const int r0 = s.o0 + j * kStepDownRows;
                const int n = min(kStepDownRows, s.o1 - r0);
                if (warp < n) {
                    const float4* w4 = reinterpret_cast<const float4*>(t + warp * kInter);
                    const float4* s4 = reinterpret_cast<const float4*>(sh.u.s);
                    float acc = 0.0f;
#pragma unroll
                    for (int q = 0; q < kInter / 128; ++q) {
                        const float4 w = w4[lane + 32 * q];
                        const float4 x = s4[lane + 32 * q];
                        acc = fmaf(w.x, x.x, acc);
                        acc = fmaf(w.y, x.y, acc);
                        acc = fmaf(w.z, x.z, acc);
                        acc = fmaf(w.w, x.w, acc);
                    }
                    acc = warp_sum(acc);
                    if (lane == 0) {
                        const int r = r0 + warp;
                        st_word(a.x.hidden + buf(l + 1) * kHidden + r, tag + 1u, sh.mid_rows[r - s.o0] + acc);
                    }
                }
                release(sh, k++);
            }
            LAYER_MARK(14);
        }

        // ---------------------------------------------------------- LM head
        {
            STEP_MARK(1 + kStepTimelinePerLayer * kLayers);
            float bv = 0.0f;
            long long bi = -1;
            if (s.n_lm > 0) {
                const uint32_t tag = s.epoch * 64u + static_cast<uint32_t>(kLayers) + 1u;
                if (!poll_into(a, sh, a.x.hidden + buf(kLayers) * kHidden, kHidden, tag, sh.hraw)) goto done;
                const float* t = acquire(a, sh, ring, k);
                if (t == nullptr) goto done;
                normalise(sh, sh.hraw, t, a.eps);
                if (s.v0 == 0)
                    for (int i = tid; i < kHidden; i += kStepConsumers) a.final_norm_out[i] = sh.xs[i];
                release(sh, k++);
                for (int j = 1; j < s.n_lm; ++j) {
                    const float* tl = acquire(a, sh, ring, k);
                    if (tl == nullptr) goto done;
                    const int64_t r0 = s.v0 + static_cast<int64_t>(j - 1) * kStepLmRows;
                    const int n = static_cast<int>(min64(kStepLmRows, s.v1 - r0));
                    const int w2 = warp * 2 + half;
                    if (warp * 2 < n) {
                        const int rr = w2 < n ? w2 : 0;
                        const float y = row_dot(tl + rr * kHidden, sh.xs, l16);
                        if (l16 == 0 && w2 < n) {
                            a.logits[r0 + w2] = y;
                            argmax_take(bv, bi, y, r0 + w2);
                        }
                    }
                    release(sh, k++);
                }
            }
            const float ov = __shfl_sync(0xffffffffu, bv, 16);
            const long long oi = __shfl_sync(0xffffffffu, bi, 16);
            if (lane == 0) {
                argmax_take(bv, bi, ov, oi);
                sh.cv[warp] = bv;
                sh.ci[warp] = bi;
            }
            consumer_sync();
            STEP_MARK(2 + kStepTimelinePerLayer * kLayers);
            if (tid == 0) {
                for (int w = 1; w < kConsumerWarps; ++w) argmax_take(bv, bi, sh.cv[w], sh.ci[w]);
                a.cand_value[cta] = bv;
                a.cand_index[cta] = bi;
                __threadfence();
                sh.is_last = atomicAdd(&a.sync[0], 1u) == static_cast<unsigned>(G - 1);
            }
            consumer_sync();
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
                    a.sync[1] = s.epoch + 1u;  // the next step's tags
                }
            }
        }
    }
done:
    __syncthreads();
    if (tid == kProducerWarp * 32) {
        // After an abort: wait (bounded) for copies the consumers never released.
        for (int kk = sh.consumed; kk < sh.issued; ++kk) {
            const unsigned long long t0 = global_timer();
            while (!mbar_try_wait(&sh.full[kk % kStepSlots], static_cast<uint32_t>(kk / kStepSlots) & 1u))
                if (global_timer() - t0 > kWaitNs) break;
        }
    }
}

}  // namespace

StepExchange step_exchange_views(unsigned long long* base, int nch) {
    StepExchange x{};
    unsigned long long* p = base;
    x.hidden = p;
    p += 2 * kHidden;
    x.qkv = p;
    p += 2 * kQKV;
    x.partial = p;
    p += 2ull * kQHeads * nch * kStepPartial;
    x.attn = p;
    p += 2 * kHidden;
    x.mid = p;
    p += 2 * kHidden;
    x.swiglu = p;
    return x;
}

size_t step_kernel_smem_bytes() { return kRingOffset + static_cast<size_t>(kStepSlots) * kStepSlotBytes; }

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
    FX_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device), "querying the SM count");
    if (per_sm < 1) {
        set_error("flux native decode: the persistent step kernel does not fit on one SM");
        return FX_ERR_CUDA;
    }
    if (sms < kStepMinGrid || sms > kStepMaxGrid) {
        set_error("flux native decode: the persistent step needs a GPU with 140 to 480 SMs");
        return FX_ERR_INVALID;
    }
    *grid = sms;
    return FX_OK;
}

}  // namespace fx
