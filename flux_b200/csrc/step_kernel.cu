// The whole batch-1 decode step as ONE persistent cooperative launch.
//
// One CTA per SM, 512 threads: 15 consumer warps do the math, one producer
// warp streams weights and cache rows into a 189 KB shared-memory ring with
// TMA (1-D cp.async.bulk for rows, 2-D cp.async.bulk.tensor for column
// strips; never multicast) completing on full/empty mbarrier pairs.  Each
// tile takes its own size (128-byte aligned, <= 27 KB) of the ring, not a
// fixed slot, so short tiles (a chunk's last few cache rows) do not hold a
// whole slot: the producer walks the CTA's tiles in consumption order and
// runs as far ahead as the bytes allow, so HBM keeps streaming while the
// consumers wait for values from other CTAs.
//
// Each CTA owns a fixed slice of every projection and one (kv head, chunk)
// of the attention.  Per layer four dependent steps (no grid barrier):
//
//   A  h = h' + sum(down partials) once every CTA has added its down
//      partial (arrival counter); RMSNorm; its QKV row pairs; RoPE;
//      publish q / k / v of the current row; write K / V into the cache.
//   B  poll q of its kv head (and the new K/V row if its chunk holds it);
//      online softmax over its chunk of cache rows for the 3 q heads;
//      publish (m, l, o) per head.
//   M  poll the partials of the 4-8 attention dims it owns; merge them;
//      multiply by those 4-8 columns of o_proj (a split-K slice of the GEMV)
//      and add the 576 products into the fixed-point h' accumulator.
//   D  h' = h + sum(o_proj partials) once every CTA has added; RMSNorm; its
//      8-12 gate/up features; SwiGLU; multiply by those columns of down and
//      add the 576 products into the fixed-point down accumulator.
//
// then the LM head (its vocab rows and greedy candidate; the last CTA to
// arrive picks the token, advances the device state and the step epoch).
//
// The split-K sums are exact integer adds of values rounded to 2^-29, so the
// result does not depend on the order the CTAs arrive in (partials of 2^13 or
// more in magnitude go through an FP64 overflow word instead).  Every wait
// (mbarrier, tagged word, counter) is bounded by %globaltimer; on expiry the
// CTA sets error bit 2, drains its copies in flight and returns, and the
// other CTAs give up at their next wait once they see the error word.
#include "step_kernel.cuh"

#include <algorithm>
#include <mutex>

namespace fx {
namespace {

constexpr unsigned long long kWaitNs = 2000000000ull;    // 2 s per wait
constexpr unsigned long long kPeerCheckNs = 1000000ull;  // look at the error word after 1 ms
constexpr int kConsumerWarps = kStepConsumers / 32;      // 15
constexpr int64_t kRingBytes = static_cast<int64_t>(kStepSlots) * kStepSlotBytes;  // 193,536
constexpr int kTileBars = 12;  // full / empty barrier pairs, tile k on pair k % 12 (more than the tiles in flight)
// Tiles in flight at most: as many as the bytes allow (<= 12) when the CTA's
// attention chunk spans two or more cache tiles, else 7 (the streaming then
// stays out of the way of the exchanges).  Measured on B200 (ms/token, fixed
// 7 x 27 KB slots -> this ring): 0.425 -> 0.403 at 8192, 0.403 -> 0.389 at
// 4096, 0.344 -> 0.342 at 128; 12 tiles at short contexts: 0.348 at 128.
constexpr int kRingAheadLong = kTileBars;
constexpr int kRingAheadShort = 7;
constexpr int kProducerWarp = kConsumerWarps;            // warp 15
constexpr int kRowBytes = kHidden * 4;                   // one 576-float row
constexpr int kStripBytes = kStepBlock * kStepStripRows * 4;  // one 2-D box (3072 B)
constexpr int kStripBoxes = kHidden / kStepStripRows;    // boxes per 576-row strip (3)
constexpr int kFeatureBlocks = kInter / kStepBlock;      // 384
constexpr int kAttnBlocks = kGroup * kHeadDim / kStepBlock;  // 48 per kv head
constexpr int kMaxChunks = 64;
constexpr int kBatchTiles = 4;                           // attention tiles held at once
constexpr int kBatchRows = kBatchTiles * kStepAttnRows + 4;  // + the new row, padded (220)
constexpr int kRowGroups = kConsumerWarps * 8;           // 4-lane score groups (120)
constexpr int kRowSlots = (kBatchTiles * kStepAttnRows + 1 + kRowGroups - 1) / kRowGroups;  // rows per group per batch (2)
constexpr int kPvSplits = kStepConsumers / (kHeadDim / 4);  // P.V row splits (30), two per warp
constexpr float kLog2e = 1.4426950408889634f;            // log2(e): scores kept in base-2 units
constexpr float kLn2 = 0.6931471805599453f;              // ln(2)
constexpr int kMaxOBlocks = 2;                           // needs >= 24 chunks per kv head
constexpr int kMaxFeatures = 12;                         // needs grid >= 128
// Tally words of the split-K sums: [7-bit contributor count | 7-bit count
// of contributors routed to the overflow word | 50-bit sum of biased
// fixed-point terms].  A contributor with |y| < 2^13 adds
// 2^57 + 2^42 + round(y * 2^29): the 2^42 bias keeps every term in (0, 2^43),
// so up to 127 terms never carry out of the sum.  A contributor with a
// larger (or non-finite) y adds y to the element's FP64 overflow word first,
// then 2^57 + 2^50 to the tally word with release semantics, so a reader that
// sees a non-zero overflow count and then fences reads the complete overflow
// word.  The count and the sum travel in one atomic word: a reader that sees
// the full count has the full sum.  Both counts fit 7 bits (at most 127
// contributors per replica word), so neither carries into the other.
constexpr int kTallyCountShift = 57;
constexpr int kTallyBadShift = 50;
constexpr unsigned long long kTallyOne = 1ull << kTallyCountShift;
constexpr unsigned long long kTallyBadOne = 1ull << kTallyBadShift;
constexpr unsigned long long kTallyValueMask = kTallyBadOne - 1;
constexpr unsigned long long kTallyCountMask = 0x7f;
constexpr long long kTallyBias = 1ll << 42;
constexpr float kTallyScale = 536870912.0f;                  // 2^29
constexpr double kTallyUnit = 1.862645149230957031e-09;      // 2^-29
constexpr float kTallyLimit = 8192.0f;                       // |y| < 2^13 in the fixed-point sum
constexpr int kTallyWords = 2 * kStepAccReplicas * kHidden;  // one layer: (o_proj, down) x replicas x 576
constexpr int kOverflowWords = 2 * kHidden;                  // one layer: (o_proj, down) x 576 FP64 overflow words

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

// 2-D tensor copy of one box at (x = column, y = row) (no multicast).  x is
// a multiple of 4 floats, so the box starts on a 16-byte boundary.
__device__ __forceinline__ void box_load(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
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

__device__ __forceinline__ void st_zero(unsigned long long* p) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], 0;" ::"l"(p) : "memory");
}

__device__ __forceinline__ void red_tally(unsigned long long* p, unsigned long long v) {
    asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Tally add that orders this thread's earlier writes (its overflow add) before it.
__device__ __forceinline__ void red_tally_release(unsigned long long* p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ double ld_overflow(const double* p) {
    double v;
    asm volatile("ld.relaxed.gpu.global.f64 %0, [%1];" : "=d"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t word_tag(unsigned long long v) { return static_cast<uint32_t>(v >> 32); }
__device__ __forceinline__ float word_value(unsigned long long v) {
    return __uint_as_float(static_cast<uint32_t>(v));
}

// Named barrier of the 15 consumer warps (the producer warp never joins it).
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 480;" ::: "memory"); }

__device__ __forceinline__ int64_t min64(int64_t x, int64_t y) { return x < y ? x : y; }

// A stamp packs the SM cycle counter (high 32 bits: precise durations
// within a CTA) with %globaltimer in ns (low 32 bits: the common clock that
// orders events across CTAs, coarse on some GPUs); both wrap after seconds.
#define STEP_MARK(event)                                                                                  \
    do {                                                                                                  \
        if (a.timeline != nullptr && threadIdx.x == 0)                                                     \
            a.timeline[static_cast<size_t>(blockIdx.x) * kStepTimelineEvents + (event)] =                  \
                (static_cast<unsigned long long>(static_cast<uint32_t>(clock64())) << 32) |                \
                static_cast<uint32_t>(global_timer());                                                     \
    } while (0)
#define LAYER_MARK(event) STEP_MARK(1 + kStepTimelinePerLayer * l + (event))

// ------------------------------------------------------------ shared state

// Phase B scratch: scores (then probabilities) of one batch, per-warp
// maxima, and the P.V partial sums of the row splits.
struct AttnScratch {
    alignas(16) float p[kGroup][kBatchRows];
    float wm[kConsumerWarps][kGroup];
    alignas(16) float o[kConsumerWarps][kGroup][kHeadDim];  // per warp (its two row splits summed)
    float l[kConsumerWarps][kGroup];
};

// The CTA's fixed share of every phase, derived from (grid, CTA, position).
struct Sched {
    int t0, t1;          // QKV row-pair tasks
    int replica;         // tally replica this CTA adds into (word offset)
    int f0, f1;          // MLP feature blocks (4 features each)
    int ob[kMaxOBlocks]; // attention-dim blocks (4 dims each) of kv head g
    int nob;
    int64_t v0, v1;      // vocab rows
    int g, c;            // attention kv head / chunk (g < 0: none)
    int64_t a0, a1;      // rows [a0, a1) of the valid length
    int64_t cached_end;  // rows [a0, cached_end) stream through the ring
    bool owns_new;       // the chunk holds row `pos` (read from the exchange)
    bool has_rows;
    int active;          // active chunks per kv head
    int n_att, n_lm, per_layer, total;
    int64_t pos, tok;
    uint32_t epoch;
};

// Kernel parameters read inside the layer loop, copied to shared memory at
// the start: the parameter block (~9 KB with the 60 tensor maps) does not
// stay in the SM's constant cache, and a miss there costs an L2 round trip.
struct HotParams {
    const float* input_norm[kLayers];
    const float* qkv[kLayers];
    const float* post_norm[kLayers];
    const float* gate_up[kLayers];
    float scale[kLayers];
    const float* key_cache;
    const float* value_cache;
    const float* final_norm;
    const float* lm_head;
    unsigned long long* x_qkv;
    unsigned long long* x_partial;
    int64_t capacity;
    float eps;
    int nch;
};

struct Shared {
    HotParams hp;
    Sched s;
    uint64_t full[kTileBars];
    uint64_t empty[kTileBars];
    uint32_t toff[kTileBars];   // ring byte offset of tile k at k % kTileBars (producer -> consumers)
    int64_t tend[kTileBars];    // producer bookkeeping: end of tile k in the ring's byte stream
    alignas(16) float hraw[kHidden];          // layer input h
    alignas(16) float mid[kHidden];           // h' (kept for the next layer's h)
    alignas(16) float xs[kHidden];            // normalised vector
    alignas(16) float wpost[kHidden];         // post-attention norm weight of the layer
    alignas(16) float qs[kGroup * kHeadDim];  // q of this CTA's kv head
    alignas(16) float knew[kHeadDim];
    alignas(16) float vnew[kHeadDim];
    alignas(16) float attn[kMaxOBlocks * kStepBlock];  // merged attention dims owned
    alignas(16) float act[kMaxFeatures];      // SwiGLU of the features owned
    float gate[kMaxFeatures];
    float up[kMaxFeatures];
    float rope_c[kHeadDim];                   // RoPE row of the step's position
    float rope_s[kHeadDim];
    float scratch[32];
    float cv[kConsumerWarps];
    long long ci[kConsumerWarps];
    float mm[kMaxOBlocks][kMaxChunks];               // phase M: m, l per (owned block's head, chunk)
    float ml[kMaxOBlocks][kMaxChunks];
    float mo[kMaxOBlocks * kStepBlock][kMaxChunks];  //          o[d] per (owned dim, chunk)
    AttnScratch att;
    volatile int abort;
    int is_last;
    int consumed;  // tiles released by the consumers
    int issued;    // tiles issued by the producer
};

constexpr size_t kRingOffset = (sizeof(Shared) + 127) / 128 * 128;



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
    s.replica = (cta % kStepAccReplicas) * kHidden;
    s.f0 = cta * kFeatureBlocks / G;
    s.f1 = (cta + 1) * kFeatureBlocks / G;
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
    s.nob = 0;
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
        for (int b = s.c; b < kAttnBlocks && s.nob < kMaxOBlocks; b += a.nch) s.ob[s.nob++] = b;
    }
    const int64_t cached = s.cached_end > s.a0 ? s.cached_end - s.a0 : 0;
    s.n_att = static_cast<int>((cached + kStepAttnRows - 1) / kStepAttnRows);
    s.per_layer = 1 + s.n_att + 4;  // A, attention, misc (norm + o strips), gate, up, down strips
    s.n_lm = s.v1 > s.v0 ? 1 + static_cast<int>((s.v1 - s.v0 + kStepLmRows - 1) / kStepLmRows) : 0;
    s.total = kLayers * s.per_layer + s.n_lm;
}

// Producer: bytes of tile k, then its copies.  Tiles of a layer, in
// consumption order: A = [input norm][row_a, row_b per QKV task];
// attention = [K rows][V rows]; misc = [post norm][o_proj strip per owned
// block, 576 x 4]; gate = [gate rows]; up = [up rows]; down = [down strip per
// feature block, 576 x 4].  LM head: [final norm], then 12-row vocab tiles.
enum class TileOp { kCount, kLoad };

__device__ uint32_t issue_tile(const StepArgs& a, const HotParams& hp, const Sched& s, int k, unsigned char* dst,
                               uint64_t* bar, TileOp op) {
    uint32_t off = 0;
    auto row_copy = [&](const float* src, uint32_t bytes) {
        if (op == TileOp::kLoad) bulk_load(dst + off, src, bytes, bar);
        off += bytes;
    };
    auto strip_copy = [&](const CUtensorMap* map, int x) {
        for (int b = 0; b < kStripBoxes; ++b) {
            if (op == TileOp::kLoad) box_load(dst + off, map, x, b * kStepStripRows, bar);
            off += kStripBytes;
        }
    };
    if (k < kLayers * s.per_layer) {
        const int l = k / s.per_layer;
        int sub = k % s.per_layer;
        const StepLayer& L = a.layer[l];  // only the tensor maps (their addresses) are used from here
        if (sub == 0) {
            row_copy(hp.input_norm[l], kRowBytes);
            for (int task = s.t0; task < s.t1; ++task) {
                int ra, rb, kind;
                task_rows(task, ra, rb, kind);
                row_copy(hp.qkv[l] + static_cast<int64_t>(ra) * kHidden, kRowBytes);
                row_copy(hp.qkv[l] + static_cast<int64_t>(rb) * kHidden, kRowBytes);
            }
            return off;
        }
        sub -= 1;
        if (sub < s.n_att) {
            const int64_t r0 = s.a0 + static_cast<int64_t>(sub) * kStepAttnRows;
            const int64_t n = min64(kStepAttnRows, s.cached_end - r0);
            const int64_t base = ((static_cast<int64_t>(l) * kKVHeads + s.g) * hp.capacity + r0) * kHeadDim;
            row_copy(hp.key_cache + base, static_cast<uint32_t>(n * kHeadDim * 4));
            row_copy(hp.value_cache + base, static_cast<uint32_t>(n * kHeadDim * 4));
            return off;
        }
        sub -= s.n_att;
        const int nf = (s.f1 - s.f0) * kStepBlock;
        if (sub == 0) {
            row_copy(hp.post_norm[l], kRowBytes);
            for (int j = 0; j < s.nob; ++j) strip_copy(&L.o_map, s.g * kGroup * kHeadDim + s.ob[j] * kStepBlock);
        } else if (sub == 1) {
            row_copy(hp.gate_up[l] + static_cast<int64_t>(s.f0) * kStepBlock * kHidden, nf * kRowBytes);
        } else if (sub == 2) {
            row_copy(hp.gate_up[l] + static_cast<int64_t>(kInter + s.f0 * kStepBlock) * kHidden, nf * kRowBytes);
        } else {
            for (int f = s.f0; f < s.f1; ++f) strip_copy(&L.down_map, f * kStepBlock);
        }
        return off;
    }
    const int j = k - kLayers * s.per_layer;
    if (j == 0) {
        row_copy(hp.final_norm, kRowBytes);
        return off;
    }
    const int64_t r0 = s.v0 + static_cast<int64_t>(j - 1) * kStepLmRows;
    const int64_t n = min64(kStepLmRows, s.v1 - r0);
    row_copy(hp.lm_head + r0 * kHidden, static_cast<uint32_t>(n * kRowBytes));
    return off;
}

__device__ __forceinline__ void fail(const StepArgs& a, Shared& sh) {
    sh.abort = 1;
    atomicOr(a.error, 2);
}

// Consumer-side bounded mbarrier wait; false when the wait gave up, another
// CTA reported a failure, or this CTA aborted.  Only consumer threads write
// sh.abort, and always before a consumer barrier after which every consumer
// reads it, so they leave together.
__device__ bool wait_bar(const StepArgs& a, Shared& sh, uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_timer();
    while (!mbar_try_wait(bar, parity)) {
        if (sh.abort) return false;
        const unsigned long long dt = global_timer() - t0;
        if (dt > kPeerCheckNs && ld_error(a.error) != 0) {
            sh.abort = 1;
            return false;
        }
        if (dt > kWaitNs) {
            fail(a, sh);
            return false;
        }
    }
    return true;
}

// Producer-side bounded wait for a free slot.  On expiry it only reports
// through the error word (the consumers see it in their own waits), since
// the producer is outside the consumers' barrier.
__device__ bool producer_wait(const StepArgs& a, Shared& sh, uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_timer();
    while (!mbar_try_wait(bar, parity)) {
        if (sh.abort) return false;
        if (global_timer() - t0 > kWaitNs) {
            atomicOr(a.error, 2);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ uint64_t* tile_full(Shared& sh, int k) { return &sh.full[k % kTileBars]; }
__device__ __forceinline__ uint64_t* tile_empty(Shared& sh, int k) { return &sh.empty[k % kTileBars]; }
__device__ __forceinline__ uint32_t tile_parity(int k) { return static_cast<uint32_t>(k / kTileBars) & 1u; }

// Tile k in the ring (its offset is published before its full barrier's arrival).
__device__ __forceinline__ const float* slot_ptr(const Shared& sh, unsigned char* ring, int k) {
    return reinterpret_cast<const float*>(ring + sh.toff[k % kTileBars]);
}

// Consumer side of tile k: wait until it landed; nullptr (uniformly) on abort.
__device__ const float* acquire(const StepArgs& a, Shared& sh, unsigned char* ring, int k) {
    wait_bar(a, sh, tile_full(sh, k), tile_parity(k));
    consumer_sync();
    if (sh.abort) return nullptr;
    return slot_ptr(sh, ring, k);
}

// Every consumer thread waits (bounded) until tiles k .. k + n - 1 landed,
// without a consumer barrier: the caller's next barrier makes an abort
// visible (sh.abort), and the caller reads sh.abort after it.
__device__ void wait_tiles(const StepArgs& a, Shared& sh, int k, int n) {
    for (int b = 0; b < n; ++b)
        if (!wait_bar(a, sh, tile_full(sh, k + b), tile_parity(k + b))) break;
}

// Tiles k .. k + n - 1 (one attention batch): wait until all landed; false (uniformly) on abort.
__device__ bool acquire_batch(const StepArgs& a, Shared& sh, int k, int n) {
    for (int b = 0; b < n; ++b)
        if (!wait_bar(a, sh, tile_full(sh, k + b), tile_parity(k + b))) break;
    consumer_sync();
    return !sh.abort;
}

__device__ void release_batch(Shared& sh, int k, int n) {
    consumer_sync();
    if (threadIdx.x == 0) {
        for (int b = 0; b < n; ++b) mbar_arrive(tile_empty(sh, k + b));
        sh.consumed = k + n;
    }
}

__device__ void release(Shared& sh, int k) {
    consumer_sync();
    if (threadIdx.x == 0) {
        mbar_arrive(tile_empty(sh, k));
        sh.consumed = k + 1;
    }
}

// Spin (bounded) until the word at p carries `tag`; returns the word.
__device__ unsigned long long poll_word(const StepArgs& a, Shared& sh, const unsigned long long* p,
                                        unsigned long long v, uint32_t tag) {
    const unsigned long long t0 = global_timer();
    while (word_tag(v) != tag) {
        // (no back-off: a 32 ns __nanosleep here cost 3 % of the step)
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

// Spin (bounded) until the N words at p[0..N-1] all carry `tag`; each round
// reloads only the stale ones, so they wait on one L2 round trip at a time
// together instead of one after another.
template <int N>
__device__ void poll_words(const StepArgs& a, Shared& sh, const unsigned long long* const (&p)[N],
                           unsigned long long (&v)[N], uint32_t tag) {
    auto stale = [&] {
        bool any = false;
#pragma unroll
        for (int j = 0; j < N; ++j) any = any || word_tag(v[j]) != tag;
        return any;
    };
    const unsigned long long t0 = global_timer();
    while (stale()) {
#pragma unroll
        for (int j = 0; j < N; ++j)
            if (word_tag(v[j]) != tag) v[j] = ld_word(p[j]);
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
}

// Phase B's inputs in one poll round and one barrier: q of kv group g (192
// words) and, for the CTA that owns the new row, that row's k and v (64 each).
__device__ bool poll_attention_inputs(const StepArgs& a, Shared& sh, const unsigned long long* qkv, int g,
                                      bool with_new, uint32_t tag) {
    constexpr int kQ = kGroup * kHeadDim;
    const int n = kQ + (with_new ? 2 * kHeadDim : 0);
    for (int i = threadIdx.x; i < n; i += kStepConsumers) {
        const unsigned long long* src;
        float* dst;
        if (i < kQ) {
            src = qkv + g * kQ + i;
            dst = sh.qs + i;
        } else if (i < kQ + kHeadDim) {
            src = qkv + kHidden + g * kHeadDim + (i - kQ);
            dst = sh.knew + (i - kQ);
        } else {
            src = qkv + kHidden + kKVHeads * kHeadDim + g * kHeadDim + (i - kQ - kHeadDim);
            dst = sh.vnew + (i - kQ - kHeadDim);
        }
        unsigned long long v = ld_word(src);
        if (word_tag(v) != tag) v = poll_word(a, sh, src, v, tag);
        *dst = word_value(v);
    }
    consumer_sync();
    return !sh.abort;
}

// Contributors per replica: CTA c adds into replica c % kStepAccReplicas.
__device__ __forceinline__ unsigned long long tally_expected(int G, int r) {
    return static_cast<unsigned long long>((G - r + kStepAccReplicas - 1) / kStepAccReplicas);
}

// dst[i] = base[i] + the split-K sum i, once every contributor's add has
// landed in every replica word (bounded polls; no fence needed: count and
// sum share the word).  Where contributors were out of the fixed-point range,
// their FP64 overflow word is added after an acquire fence.  The per-warp
// sums of squares of dst are left in sh.scratch for normalise() /
// norm_inverse(); with `norm_w`, also xg[i] = dst[i] * norm_w[i] (the RMSNorm
// weight applied, the 1 / rms factor left to the caller's dot products).
__device__ bool tally_read(const StepArgs& a, Shared& sh, const unsigned long long* acc, const double* overflow,
                           const float* base, float* dst, int G, const float* norm_w = nullptr,
                           float* xg = nullptr) {
    float ss = 0.0f;  // sum of squares of dst (per-warp partials left in scratch for the RMSNorm)
    for (int i = threadIdx.x; i < kHidden; i += kStepConsumers) {
        unsigned long long w[kStepAccReplicas];
        bool ready = true;
#pragma unroll
        for (int r = 0; r < kStepAccReplicas; ++r) {
            w[r] = ld_word(acc + r * kHidden + i);
            ready = ready && (w[r] >> kTallyCountShift) >= tally_expected(G, r);
        }
        if (!ready) {
            const unsigned long long t0 = global_timer();
            while (true) {
                ready = true;
#pragma unroll
                for (int r = 0; r < kStepAccReplicas; ++r) {
                    if ((w[r] >> kTallyCountShift) < tally_expected(G, r)) w[r] = ld_word(acc + r * kHidden + i);
                    ready = ready && (w[r] >> kTallyCountShift) >= tally_expected(G, r);
                }
                if (ready || sh.abort) break;
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
        }
        long long total = 0;
        unsigned long long routed = 0;  // contributors whose value went to the overflow word
#pragma unroll
        for (int r = 0; r < kStepAccReplicas; ++r) {
            const unsigned long long bad = (w[r] >> kTallyBadShift) & kTallyCountMask;
            routed += bad;
            total += static_cast<long long>(w[r] & kTallyValueMask) -
                     static_cast<long long>(tally_expected(G, r) - bad) * kTallyBias;
        }
        double sum = static_cast<double>(total) * kTallyUnit;
        if (routed != 0) {
            asm volatile("fence.acq_rel.gpu;" ::: "memory");
            sum += ld_overflow(overflow + i);
        }
        dst[i] = base[i] + static_cast<float>(sum);
        ss = fmaf(dst[i], dst[i], ss);
        if (xg != nullptr) xg[i] = dst[i] * norm_w[i];
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) sh.scratch[threadIdx.x >> 5] = ss;
    consumer_sync();
    return !sh.abort;
}

// xs = src * rsqrt(mean(src^2) + eps) * w (rmsnorm_cuda.cu:23-89); the
// per-warp sums of squares of src are already in sh.scratch (tally_read or
// the embedding gather wrote them before a consumer barrier).
__device__ void normalise(Shared& sh, const float* src, const float* w, float eps) {
    float ss = 0.0f;
#pragma unroll
    for (int q = 0; q < kConsumerWarps; ++q) ss += sh.scratch[q];
    const float inv = rsqrtf(ss / static_cast<float>(kHidden) + eps);
    for (int i = threadIdx.x; i < kHidden; i += kStepConsumers) sh.xs[i] = src[i] * inv * w[i];
    consumer_sync();
}

// 1 / rms of the vector whose per-warp sums of squares are in sh.scratch
// (after the barrier that published them).
__device__ __forceinline__ float norm_inverse(const Shared& sh, float eps) {
    float ss = 0.0f;
#pragma unroll
    for (int q = 0; q < kConsumerWarps; ++q) ss += sh.scratch[q];
    return rsqrtf(ss / static_cast<float>(kHidden) + eps);
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

// Split-K slice: y[r] = sum_j coef[j] * strip[j / 4][r][j % 4] for the 576
// rows r (blocks = 0: zeros), added into this CTA's replica of the tally;
// values outside the fixed-point range go through the FP64 overflow word.
__device__ void tally_products(const float* strips, const float* coef, int blocks, unsigned long long* acc,
                               double* overflow) {
    for (int r = threadIdx.x; r < kHidden; r += kStepConsumers) {
        float y = 0.0f;
        for (int b = 0; b < blocks; ++b) {
            const float4 w = reinterpret_cast<const float4*>(strips + static_cast<size_t>(b) * kHidden * kStepBlock)[r];
            const float4 c = reinterpret_cast<const float4*>(coef)[b];
            y = fmaf(w.x, c.x, y);
            y = fmaf(w.y, c.y, y);
            y = fmaf(w.z, c.z, y);
            y = fmaf(w.w, c.w, y);
        }
        if (fabsf(y) < kTallyLimit) {
            red_tally(acc + r, kTallyOne + static_cast<unsigned long long>(kTallyBias + __float2ll_rn(y * kTallyScale)));
        } else {
            atomicAdd(overflow + r, static_cast<double>(y));
            red_tally_release(acc + r, kTallyOne + kTallyBadOne);
        }
    }
}

__device__ __forceinline__ void argmax_take(float& bv, long long& bi, float v, long long i) {
    if (argmax_precedes(v, i, bv, bi)) {
        bv = v;
        bi = i;
    }
}

__device__ __forceinline__ size_t parity(int l) { return static_cast<size_t>(l & 1); }

// The step's output token to the host-mapped word of fx_decode_replay_host
// (system scope; the host reads it after the step has completed).
__device__ __forceinline__ void publish_host_token(const StepArgs& a, int64_t token) {
    if (a.host_out != nullptr)
        asm volatile("st.relaxed.sys.global.s64 [%0], %1;" ::"l"(a.host_out), "l"(static_cast<long long>(token))
                     : "memory");
}

// ------------------------------------------------------------------ kernel

__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const __grid_constant__ StepArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    Shared& sh = *reinterpret_cast<Shared*>(smem);
    unsigned char* ring = smem + kRingOffset;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, cta = blockIdx.x;

    if (*reinterpret_cast<volatile int*>(a.stop) != 0) {  // generation already ended on EOS (uniform)
        if (cta == 0 && tid == 0) publish_host_token(a, *a.token);  // the token a copy would return
        return;
    }
    // The schedule is uniform over the CTA and read throughout the step: it
    // lives in shared memory (as a per-thread struct it was spilled to local
    // memory, 64 KB per CTA, more than the L1 left beside the ring).
    if (tid == 0) make_sched(a, G, cta, sh.s);
    if (tid < kLayers) {
        const StepLayer& L = a.layer[tid];
        sh.hp.input_norm[tid] = L.input_norm;
        sh.hp.qkv[tid] = L.qkv;
        sh.hp.post_norm[tid] = L.post_norm;
        sh.hp.gate_up[tid] = L.gate_up;
        sh.hp.scale[tid] = L.scale;
    } else if (tid == 32) {
        sh.hp.key_cache = a.key_cache;
        sh.hp.value_cache = a.value_cache;
        sh.hp.final_norm = a.final_norm;
        sh.hp.lm_head = a.lm_head;
        sh.hp.x_qkv = a.x.qkv;
        sh.hp.x_partial = a.x.partial;
        sh.hp.capacity = a.capacity;
        sh.hp.eps = a.eps;
        sh.hp.nch = a.nch;
    }
    if (tid == 0) {
        for (int i = 0; i < kTileBars; ++i) {
            mbar_init(&sh.full[i], 1);
            mbar_init(&sh.empty[i], 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        sh.abort = 0;
        sh.consumed = 0;
        sh.issued = 0;
    }
    __syncthreads();
    const Sched& s = sh.s;
    if (s.pos < 0 || s.pos >= a.capacity) {  // uniform
        if (cta == 0 && tid == 0) {
            atomicOr(a.error, 1);
            publish_host_token(a, *a.token);
        }
        return;
    }
    if (cta == 0 && tid == 0) *a.length = s.pos + 1;
    STEP_MARK(0);

    if (warp == kProducerWarp) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            // The ring as a byte stream: tile k occupies [start, end) with
            // start = the stream position (moved to the next lap when the
            // tile would straddle the ring's end).  It may be written once the
            // tiles whose bytes it reuses (those ending after end - ring size)
            // are released, in order, and at most `ahead` tiles are in flight
            // (which also frees its barrier pair: tile k - kTileBars released).
            int64_t pos = 0, freed = 0;
            int next = 0;  // oldest tile whose release the producer has not yet seen
            const int ahead = s.n_att >= 2 ? kRingAheadLong : kRingAheadShort;
            bool ok = true;
            for (int k = 0; ok && k < s.total; ++k) {
                const uint32_t bytes = issue_tile(a, sh.hp, s, k, nullptr, nullptr, TileOp::kCount);
                const int64_t size = (static_cast<int64_t>(bytes) + 127) / 128 * 128;
                if (pos % kRingBytes + size > kRingBytes) pos += kRingBytes - pos % kRingBytes;
                const int64_t end = pos + size;
                while (next < k && (freed < end - kRingBytes || next <= k - ahead)) {
                    if (!producer_wait(a, sh, tile_empty(sh, next), tile_parity(next))) {
                        ok = false;
                        break;
                    }
                    freed = sh.tend[next % kTileBars];
                    ++next;
                }
                if (!ok) break;
                sh.toff[k % kTileBars] = static_cast<uint32_t>(pos % kRingBytes);
                sh.tend[k % kTileBars] = end;
                unsigned char* dst = ring + pos % kRingBytes;
                pos = end;
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive_expect_tx(tile_full(sh, k), bytes);
                issue_tile(a, sh.hp, s, k, dst, tile_full(sh, k), TileOp::kLoad);
                sh.issued = k + 1;
            }
        }
    } else {
        // --------------------------------------------------------- consumers
        const int half = lane >> 4, l16 = lane & 15;
        const int64_t cap = a.capacity;
        // This step's tallies: set (epoch & 1), [layer][o_proj | down][replica][576].
        unsigned long long* tallies = a.x.tally + static_cast<size_t>(s.epoch & 1u) * kLayers * kTallyWords;
        double* overflows = a.x.overflow + static_cast<size_t>(s.epoch & 1u) * kLayers * kOverflowWords;
        auto mid_tally = [&](int l) { return tallies + static_cast<size_t>(l) * kTallyWords; };
        auto down_tally = [&](int l) { return tallies + static_cast<size_t>(l) * kTallyWords + kTallyWords / 2; };
        auto mid_overflow = [&](int l) { return overflows + static_cast<size_t>(l) * kOverflowWords; };
        auto down_overflow = [&](int l) { return overflows + static_cast<size_t>(l) * kOverflowWords + kHidden; };
        // Zero the other set (tallies and overflow words) for the next step
        // (it was last read by the previous launch).
        {
            const uint32_t next = (s.epoch + 1u) & 1u;
            unsigned long long* words = a.x.tally + static_cast<size_t>(next) * kLayers * kTallyWords;
            size_t n = static_cast<size_t>(kLayers) * kTallyWords;
            for (size_t i = static_cast<size_t>(cta) * n / G + tid; i < static_cast<size_t>(cta + 1) * n / G;
                 i += kStepConsumers)
                st_zero(words + i);
            words = reinterpret_cast<unsigned long long*>(a.x.overflow + static_cast<size_t>(next) * kLayers * kOverflowWords);
            n = static_cast<size_t>(kLayers) * kOverflowWords;
            for (size_t i = static_cast<size_t>(cta) * n / G + tid; i < static_cast<size_t>(cta + 1) * n / G;
                 i += kStepConsumers)
                st_zero(words + i);
        }
        int k = 0;
        const int inject = *a.inject;
        for (int l = 0; l < kLayers; ++l) {
            const uint32_t tag = s.epoch * 64u + static_cast<uint32_t>(l) + 1u;
            if (inject == l + 1 && cta == 0) {
                // Test hook: CTA 0 reports a failure here (as if one of its
                // bounded waits had expired) and leaves; the other CTAs find
                // the error word within ~1 ms in their polls and drain.
                if (tid == 0) {
                    sh.abort = 1;
                    atomicOr(a.error, 2);
                }
                consumer_sync();
                goto done;
            }
            // ------------------------------------------------------ phase A
            // The tile with this layer's input-norm weights and QKV rows; the
            // barrier of the h read below also publishes this wait.  xs gets
            // h * norm weight, and the dot products take the 1 / rms factor.
            wait_tiles(a, sh, k, 1);
            const float* t = slot_ptr(sh, ring, k);
            if (l == 0) {
                const bool valid = s.tok >= 0 && s.tok < a.vocab;
                float ss = 0.0f;
                for (int i = tid; i < kHidden; i += kStepConsumers) {
                    sh.hraw[i] = valid ? __ldg(a.embedding + s.tok * kHidden + i) : 0.0f;
                    ss = fmaf(sh.hraw[i], sh.hraw[i], ss);
                    sh.xs[i] = sh.hraw[i] * t[i];
                }
                ss = warp_sum(ss);
                if (lane == 0) sh.scratch[warp] = ss;
                if (tid < kHeadDim) {
                    sh.rope_c[tid] = __ldg(a.cos_table + s.pos * kHeadDim + tid);
                    sh.rope_s[tid] = __ldg(a.sin_table + s.pos * kHeadDim + tid);
                }
                consumer_sync();
                if (sh.abort) goto done;
            } else if (!tally_read(a, sh, down_tally(l - 1), down_overflow(l - 1), sh.mid, sh.hraw, G, t, sh.xs)) {
                goto done;
            }
            LAYER_MARK(0);
            {
                const float inv = norm_inverse(sh, sh.hp.eps);
                if (warp < s.t1 - s.t0) {
                    int ra, rb, kind;
                    task_rows(s.t0 + warp, ra, rb, kind);
                    const float y = row_dot(t + kHidden * (1 + 2 * warp + half), sh.xs, l16) * inv;
                    const float ya = __shfl_sync(0xffffffffu, y, 0);
                    const float yb = __shfl_sync(0xffffffffu, y, 16);
                    float out = y;
                    const int row = half ? rb : ra;
                    if (kind == 2) {
                        if (l16 == 0) {
                            const int u = row - kHidden - kKVHeads * kHeadDim;
                            a.value_cache[((static_cast<int64_t>(l) * kKVHeads + u / kHeadDim) * cap + s.pos) *
                                              kHeadDim +
                                          u % kHeadDim] = y;
                        }
                    } else {
                        const int d = row % kHeadDim;
                        const float c = sh.rope_c[d];
                        const float sn = sh.rope_s[d];
                        out = half ? rope_value(yb, ya, c, sn, false) : rope_value(ya, yb, c, sn, true);
                        if (kind == 1 && l16 == 0) {
                            const int h = (row - kHidden) / kHeadDim;
                            a.key_cache[((static_cast<int64_t>(l) * kKVHeads + h) * cap + s.pos) * kHeadDim + d] = out;
                        }
                    }
                    // lanes 0..3 of each half publish the replicas
                    if (l16 < kStepReplicas)
                        st_word(sh.hp.x_qkv + (parity(l) * kStepReplicas + l16) * kQKV + row, tag, out);
                }
                release(sh, k++);
            }
            LAYER_MARK(1);

            // ------------------------------------------------------ phase B
            if (s.has_rows && s.a1 - s.a0 <= 32) {
                // A chunk of at most 32 rows (one cache tile at most): warp 0 does
                // it all -- lane r scores row r for the three heads, softmax within
                // the warp, P.V with each lane on two dims -- and publishes the
                // partial itself; the other warps wait at the barrier below (they
                // do not spin on phase M's polls meanwhile: spinning polls load the
                // L2 that every CTA's exchanges go through).
                if (warp == 0) {
                    const unsigned long long* qkv =
                        sh.hp.x_qkv + (parity(l) * kStepReplicas + cta % kStepReplicas) * kQKV;
                    // q of the kv head (192 words) and the new row's k, v (64 + 64):
                    // each lane's up to 10 words are loaded together and only the
                    // stale ones reloaded, one L2 round trip per round.
                    constexpr int kQ = kGroup * kHeadDim;
                    constexpr int kPer = (kQ + 2 * kHeadDim + 31) / 32;  // 10
                    const int nq = kQ + (s.owns_new ? 2 * kHeadDim : 0);
                    auto word_src = [&](int i) -> const unsigned long long* {
                        if (i < kQ) return qkv + s.g * kQ + i;
                        if (i < kQ + kHeadDim) return qkv + kHidden + s.g * kHeadDim + (i - kQ);
                        return qkv + kHidden + kKVHeads * kHeadDim + s.g * kHeadDim + (i - kQ - kHeadDim);
                    };
                    unsigned long long w[kPer];
#pragma unroll
                    for (int j = 0; j < kPer; ++j) {
                        const int i = lane + 32 * j;
                        w[j] = i < nq ? ld_word(word_src(i)) : (static_cast<unsigned long long>(tag) << 32);
                    }
                    {
                        const unsigned long long t0 = global_timer();
                        while (true) {
                            bool stale = false;
#pragma unroll
                            for (int j = 0; j < kPer; ++j) {
                                if (word_tag(w[j]) != tag) {
                                    w[j] = ld_word(word_src(lane + 32 * j));
                                    stale = true;
                                }
                            }
                            if (!stale || sh.abort) break;
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
                    }
#pragma unroll
                    for (int j = 0; j < kPer; ++j) {
                        const int i = lane + 32 * j;
                        if (i < kQ)
                            sh.qs[i] = word_value(w[j]);
                        else if (i < kQ + kHeadDim)
                            sh.knew[i - kQ] = word_value(w[j]);
                        else if (i < nq)
                            sh.vnew[i - kQ - kHeadDim] = word_value(w[j]);
                    }
                    __syncwarp();
                    LAYER_MARK(2);
                    if (s.n_att > 0) wait_bar(a, sh, tile_full(sh, k), tile_parity(k));
                    LAYER_MARK(3);
                    const int cached = static_cast<int>(s.cached_end - s.a0);  // rows in the tile (K, then V)
                    const int rows = static_cast<int>(s.a1 - s.a0);
                    const float* tile = slot_ptr(sh, ring, k);
                    const float scale2 = sh.hp.scale[l] * kLog2e;
                    const bool valid = lane < rows;
                    const float4* k4 = reinterpret_cast<const float4*>(lane < cached ? tile + lane * kHeadDim : sh.knew);
                    float d[kGroup] = {0.0f, 0.0f, 0.0f};
#pragma unroll 4
                    for (int j = 0; j < kHeadDim / 4; ++j) {
                        const int c = (j + lane) & (kHeadDim / 4 - 1);  // rotated: lanes spread over the banks
                        const float4 kv = k4[c];
#pragma unroll
                        for (int h = 0; h < kGroup; ++h) {
                            const float4 q = reinterpret_cast<const float4*>(sh.qs + h * kHeadDim)[c];
                            d[h] = fmaf(q.x, kv.x, d[h]);
                            d[h] = fmaf(q.y, kv.y, d[h]);
                            d[h] = fmaf(q.z, kv.z, d[h]);
                            d[h] = fmaf(q.w, kv.w, d[h]);
                        }
                    }
                    float m[kGroup], total[kGroup];
#pragma unroll
                    for (int h = 0; h < kGroup; ++h) {
                        const float sc = valid ? d[h] * scale2 : -INFINITY;
                        m[h] = warp_max(sc);  // row 0 is valid: finite
                        const float p = valid ? exp2f(sc - m[h]) : 0.0f;
                        total[h] = warp_sum(p);
                        if (valid) sh.att.p[h][lane] = p;
                    }
                    __syncwarp();
                    float2 o[kGroup];
#pragma unroll
                    for (int h = 0; h < kGroup; ++h) o[h] = make_float2(0.0f, 0.0f);
                    for (int r = 0; r < rows; ++r) {
                        const float2 v = reinterpret_cast<const float2*>(
                            r < cached ? tile + (cached + r) * kHeadDim : sh.vnew)[lane];
#pragma unroll
                        for (int h = 0; h < kGroup; ++h) {
                            const float p = sh.att.p[h][r];
                            o[h].x = fmaf(p, v.x, o[h].x);
                            o[h].y = fmaf(p, v.y, o[h].y);
                        }
                    }
                    __syncwarp();  // the warp is done with the tile
                    if (lane == 0 && s.n_att > 0) {
                        mbar_arrive(tile_empty(sh, k));
                        sh.consumed = k + 1;
                    }
                    LAYER_MARK(4);
                    const int nch = sh.hp.nch;
#pragma unroll
                    for (int h = 0; h < kGroup; ++h) {
                        unsigned long long* pw = sh.hp.x_partial +
                                                 parity(l) * (static_cast<size_t>(kQHeads) * nch * kStepPartial) +
                                                 ((static_cast<size_t>(s.g) * kGroup + h) * nch + s.c) * kStepPartial;
                        st_word(pw + 2 + 2 * lane, tag, o[h].x);
                        st_word(pw + 3 + 2 * lane, tag, o[h].y);
                        if (lane == 0) {
                            st_word(pw, tag, m[h] * kLn2);  // natural-log units
                            st_word(pw + 1, tag, total[h]);
                        }
                    }
                }
                k += s.n_att;
                consumer_sync();
            } else if (s.has_rows) {
                const unsigned long long* qkv = sh.hp.x_qkv + (parity(l) * kStepReplicas + cta % kStepReplicas) * kQKV;
                if (!poll_attention_inputs(a, sh, qkv, s.g, s.owns_new, tag)) goto done;
                LAYER_MARK(2);
                // Scores in base-2 units: s2 = (q . k) * scale * log2(e), so p = exp2(s2 - max).
                const float scale2 = sh.hp.scale[l] * kLog2e;
                // Score groups of 4 lanes; lane (gl, l4) of a warp covers the 16-byte
                // chunks l4 + 4 m of a row, visiting m = (j + gl) % 4 at step j so the
                // 32 lanes of one load hit 8 distinct bank groups.
                const int l4 = lane & 3, gl = lane >> 2, g4 = warp * 8 + gl;
                float4 qr[kGroup][4];
#pragma unroll
                for (int h = 0; h < kGroup; ++h)
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        qr[h][j] = reinterpret_cast<const float4*>(sh.qs + h * kHeadDim)[l4 + 4 * ((j + gl) & 3)];
                // P.V threads: (4-dim quad, row split), all 3 heads, so every V
                // row is read from shared memory once.
                const int pq = tid & 15, psplit = tid >> 4;
                float4 pacc[kGroup];
                float plsum[kGroup];
#pragma unroll
                for (int h = 0; h < kGroup; ++h) {
                    pacc[h] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    plsum[h] = 0.0f;
                }
                float mrun[kGroup];
#pragma unroll
                for (int h = 0; h < kGroup; ++h) mrun[h] = -INFINITY;
                // Batches of up to 4 cache tiles (every tile but the chunk's last
                // holds 54 rows); the last batch also takes the new row from the
                // exchange.  A running max rescales the earlier batches.
                int j = 0, last_batch = 0;
                do {
                    const int nb = min(kBatchTiles, s.n_att - j);
                    const int64_t r0 = s.a0 + static_cast<int64_t>(j) * kStepAttnRows;
                    const int cached = static_cast<int>(
                        max(static_cast<int64_t>(0), min64(static_cast<int64_t>(nb) * kStepAttnRows, s.cached_end - r0)));
                    const bool with_new = j + nb == s.n_att && s.owns_new;
                    const int rows = cached + (with_new ? 1 : 0);
                    // The first batch needs no barrier of its own (the poll's barrier
                    // precedes it; an abort is read after the score barrier below).
                    if (j == 0) {
                        wait_tiles(a, sh, k, nb);
                        LAYER_MARK(3);
                    } else if (!acquire_batch(a, sh, k, nb)) {
                        goto done;
                    }
                    auto tile_base = [&](int gi) {
                        return slot_ptr(sh, ring, k + gi / kStepAttnRows);
                    };
                    auto key_row = [&](int gi) -> const float* {
                        if (gi >= cached) return sh.knew;
                        return tile_base(gi) + (gi % kStepAttnRows) * kHeadDim;
                    };
                    // Scores of the batch's rows -> p (smem), per-warp maxima.
                    float mb[kGroup];
#pragma unroll
                    for (int h = 0; h < kGroup; ++h) mb[h] = -INFINITY;
#pragma unroll
                    for (int i = 0; i < kRowSlots; ++i) {
                        const int gi = g4 + kRowGroups * i;
                        if (warp * 8 + kRowGroups * i < rows) {  // warp-uniform: full-mask shuffles
                            const float4* k4 = reinterpret_cast<const float4*>(key_row(gi < rows ? gi : 0));
                            float d[kGroup] = {0.0f, 0.0f, 0.0f};
#pragma unroll
                            for (int jj = 0; jj < 4; ++jj) {
                                const float4 kv = k4[l4 + 4 * ((jj + gl) & 3)];
#pragma unroll
                                for (int h = 0; h < kGroup; ++h) {
                                    d[h] = fmaf(qr[h][jj].x, kv.x, d[h]);
                                    d[h] = fmaf(qr[h][jj].y, kv.y, d[h]);
                                    d[h] = fmaf(qr[h][jj].z, kv.z, d[h]);
                                    d[h] = fmaf(qr[h][jj].w, kv.w, d[h]);
                                }
                            }
#pragma unroll
                            for (int off = 1; off < 4; off <<= 1)
#pragma unroll
                                for (int h = 0; h < kGroup; ++h) d[h] += __shfl_xor_sync(0xffffffffu, d[h], off);
                            if (gi < rows) {
#pragma unroll
                                for (int h = 0; h < kGroup; ++h) {
                                    d[h] *= scale2;
                                    mb[h] = fmaxf(mb[h], d[h]);
                                }
                                if (l4 < kGroup) sh.att.p[l4][gi] = l4 == 0 ? d[0] : (l4 == 1 ? d[1] : d[2]);
                            }
                        }
                    }
#pragma unroll
                    for (int h = 0; h < kGroup; ++h) {
#pragma unroll
                        for (int off = 4; off < 32; off <<= 1) mb[h] = fmaxf(mb[h], __shfl_xor_sync(0xffffffffu, mb[h], off));
                        if (lane == 0) sh.att.wm[warp][h] = mb[h];
                    }
                    consumer_sync();
                    if (sh.abort) goto done;
                    // New running max (uniform over the CTA); rescale earlier batches.
                    float mnew[kGroup];
#pragma unroll
                    for (int h = 0; h < kGroup; ++h) {
                        float mx = lane < kConsumerWarps ? sh.att.wm[lane][h] : -INFINITY;
#pragma unroll
                        for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
                        mnew[h] = fmaxf(mrun[h], mx);
                    }
#pragma unroll
                    for (int h = 0; h < kGroup; ++h) {
                        const float f = exp2f(mrun[h] - mnew[h]);  // first batch: mrun = -inf -> 0
                        pacc[h].x *= f;
                        pacc[h].y *= f;
                        pacc[h].z *= f;
                        pacc[h].w *= f;
                        plsum[h] *= f;
                    }
#pragma unroll
                    for (int h = 0; h < kGroup; ++h) mrun[h] = mnew[h];
                    // p = exp2(s2 - max), in place.
#pragma unroll
                    for (int h = 0; h < kGroup; ++h)
                        for (int r = tid; r < rows; r += kStepConsumers) sh.att.p[h][r] = exp2f(sh.att.p[h][r] - mrun[h]);
                    consumer_sync();
                    // P.V: rows psplit, psplit + 30, ... of the batch, tile by tile.
                    {
                        float4 acc2[kGroup];
#pragma unroll
                        for (int h = 0; h < kGroup; ++h) acc2[h] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                        auto pv_row = [&](float4 (&acc)[kGroup], int row, const float4 v) {
#pragma unroll
                            for (int h = 0; h < kGroup; ++h) {
                                const float p = sh.att.p[h][row];
                                acc[h].x = fmaf(p, v.x, acc[h].x);
                                acc[h].y = fmaf(p, v.y, acc[h].y);
                                acc[h].z = fmaf(p, v.z, acc[h].z);
                                acc[h].w = fmaf(p, v.w, acc[h].w);
                                plsum[h] += p;
                            }
                        };
                        for (int b = 0; b < nb; ++b) {
                            const int base = b * kStepAttnRows;
                            const int n = min(kStepAttnRows, cached - base);
                            const float* vb = slot_ptr(sh, ring, k + b) + n * kHeadDim + pq * 4;
                            int rr = psplit - base % kPvSplits;
                            if (rr < 0) rr += kPvSplits;
                            for (; rr + kPvSplits < n; rr += 2 * kPvSplits) {  // two rows per trip
                                const float4 v0 = *reinterpret_cast<const float4*>(vb + rr * kHeadDim);
                                const float4 v1 = *reinterpret_cast<const float4*>(vb + (rr + kPvSplits) * kHeadDim);
                                pv_row(pacc, base + rr, v0);
                                pv_row(acc2, base + rr + kPvSplits, v1);
                            }
                            if (rr < n) pv_row(pacc, base + rr, *reinterpret_cast<const float4*>(vb + rr * kHeadDim));
                        }
                        if (with_new && cached % kPvSplits == psplit)
                            pv_row(pacc, cached, reinterpret_cast<const float4*>(sh.vnew)[pq]);
#pragma unroll
                        for (int h = 0; h < kGroup; ++h) {
                            pacc[h].x += acc2[h].x;
                            pacc[h].y += acc2[h].y;
                            pacc[h].z += acc2[h].z;
                            pacc[h].w += acc2[h].w;
                        }
                    }
                    if (j + nb < s.n_att) {
                        release_batch(sh, k, nb);  // the next batch needs the producer to move on
                        k += nb;
                    } else {
                        last_batch = nb;  // released at the combine barrier below
                    }
                    j += nb;
                } while (j < s.n_att);
                LAYER_MARK(4);
                // Sum the row splits: the warp's two halves by a shuffle, then the
                // 15 warps' sums.
#pragma unroll
                for (int h = 0; h < kGroup; ++h) {
                    pacc[h].x += __shfl_xor_sync(0xffffffffu, pacc[h].x, 16);
                    pacc[h].y += __shfl_xor_sync(0xffffffffu, pacc[h].y, 16);
                    pacc[h].z += __shfl_xor_sync(0xffffffffu, pacc[h].z, 16);
                    pacc[h].w += __shfl_xor_sync(0xffffffffu, pacc[h].w, 16);
                    plsum[h] += __shfl_xor_sync(0xffffffffu, plsum[h], 16);
                    if (lane < 16) reinterpret_cast<float4*>(sh.att.o[warp][h])[pq] = pacc[h];
                    if (lane == 0) sh.att.l[warp][h] = plsum[h];
                }
                consumer_sync();  // every thread is done with the last batch's tiles
                if (tid == 0) {
                    for (int b = 0; b < last_batch; ++b) mbar_arrive(tile_empty(sh, k + b));
                    sh.consumed = k + last_batch;
                }
                k += last_batch;
                if (tid < kGroup * kHeadDim) {
                    const int h = tid / kHeadDim, d = tid % kHeadDim;
                    const float mx = (h == 0 ? mrun[0] : (h == 1 ? mrun[1] : mrun[2])) * kLn2;  // natural-log units
                    float total = 0.0f, acc = 0.0f;
#pragma unroll
                    for (int w = 0; w < kConsumerWarps; ++w) {
                        total += sh.att.l[w][h];
                        acc += sh.att.o[w][h][d];
                    }
                    const int nch = sh.hp.nch;
                    unsigned long long* pw = sh.hp.x_partial + parity(l) * (static_cast<size_t>(kQHeads) * nch * kStepPartial) +
                                             ((static_cast<size_t>(s.g) * kGroup + h) * nch + s.c) * kStepPartial;
                    st_word(pw + 2 + d, tag, acc);
                    if (d == 0) {
                        st_word(pw, tag, mx);
                        st_word(pw + 1, tag, total);
                    }
                }
                // no barrier: phase M uses other shared arrays, and the next writes of
                // sh.att come after many barriers (next layer)
            }
            LAYER_MARK(5);

            // ------------------------------------------------------ phase M
            // Merge the owned attention dims over all chunks, then add their
            // o_proj products (a split-K slice) into the h' accumulator.
            {
                const int nd = s.nob * kStepBlock;
                if (nd > 0) {
                    const int nch = sh.hp.nch;
                    const unsigned long long* part = sh.hp.x_partial +
                                                     parity(l) * (static_cast<size_t>(kQHeads) * nch * kStepPartial) +
                                                     static_cast<size_t>(s.g) * kGroup * nch * kStepPartial;
                    // One poll item per thread: the o[d] word of each (owned dim,
                    // chunk), and the (m, l) pair of each (owned block, chunk) --
                    // polled once per block, not once per dim.  At most
                    // 5 * nob * active <= 480 items (nob = 2 needs nch < 48).
                    const int act = s.active, n_o = nd * act, n_ml = s.nob * act;
                    for (int it = tid; it < n_o + n_ml; it += kStepConsumers) {
                        if (it < n_o) {
                            const int q = it / act, cc = it % act;
                            const int j = s.ob[q / kStepBlock] * kStepBlock + q % kStepBlock;
                            const unsigned long long* p =
                                part + (static_cast<size_t>(j / kHeadDim) * nch + cc) * kStepPartial + 2 + j % kHeadDim;
                            unsigned long long v = ld_word(p);
                            if (word_tag(v) != tag) v = poll_word(a, sh, p, v, tag);
                            sh.mo[q][cc] = word_value(v);
                        } else {
                            const int b = (it - n_o) / act, cc = (it - n_o) % act;
                            const int h = s.ob[b] * kStepBlock / kHeadDim;
                            const unsigned long long* p = part + (static_cast<size_t>(h) * nch + cc) * kStepPartial;
                            const unsigned long long* const src[2] = {p, p + 1};
                            unsigned long long v[2] = {ld_word(src[0]), ld_word(src[1])};
                            poll_words<2>(a, sh, src, v, tag);
                            sh.mm[b][cc] = word_value(v[0]);
                            sh.ml[b][cc] = word_value(v[1]);
                        }
                    }
                    consumer_sync();
                    if (sh.abort) goto done;
                    LAYER_MARK(6);
                    if (warp < nd) {
                        const int b = warp / kStepBlock;
                        float mx = -INFINITY;
                        for (int cc = lane; cc < act; cc += 32) mx = fmaxf(mx, sh.mm[b][cc]);
                        mx = warp_max(mx);
                        float total = 0.0f, acc = 0.0f;
                        for (int cc = lane; cc < act; cc += 32) {
                            const float w = expf(sh.mm[b][cc] - mx);
                            total = fmaf(w, sh.ml[b][cc], total);
                            acc = fmaf(w, sh.mo[warp][cc], acc);
                        }
                        total = warp_sum(total);
                        acc = warp_sum(acc);
                        if (lane == 0) sh.attn[warp] = acc / total;
                    }
                }
                const float* t = acquire(a, sh, ring, k);
                if (t == nullptr) goto done;
                LAYER_MARK(7);
                for (int i = tid; i < kHidden; i += kStepConsumers) sh.wpost[i] = t[i];
                tally_products(t + kHidden, sh.attn, s.nob, mid_tally(l) + s.replica, mid_overflow(l));
                release(sh, k++);
            }
            LAYER_MARK(8);

            // ------------------------------------------------------ phase D
            // gate, up and down tiles together; the barrier of the h' read also
            // publishes these waits (xs = h' * post-norm weight).
            wait_tiles(a, sh, k, 3);
            if (!tally_read(a, sh, mid_tally(l), mid_overflow(l), sh.hraw, sh.mid, G, sh.wpost, sh.xs)) goto done;
            LAYER_MARK(9);
            {
                const int nf = (s.f1 - s.f0) * kStepBlock;
                const float inv = norm_inverse(sh, sh.hp.eps);
                // warp f: gate row f on lanes 0-15, up row f on lanes 16-31, SwiGLU on lane 0.
                if (warp < nf) {
                    const float y = row_dot(slot_ptr(sh, ring, k + half) + warp * kHidden, sh.xs, l16) * inv;
                    const float up = __shfl_sync(0xffffffffu, y, 16);
                    if (lane == 0) sh.act[warp] = swiglu(y, up);
                }
                consumer_sync();
                LAYER_MARK(10);
                tally_products(slot_ptr(sh, ring, k + 2), sh.act, s.f1 - s.f0, down_tally(l) + s.replica, down_overflow(l));
                release_batch(sh, k, 3);
                k += 3;
            }
            LAYER_MARK(11);
        }

        // ---------------------------------------------------------- LM head
        {
            STEP_MARK(1 + kStepTimelinePerLayer * kLayers);
            float bv = 0.0f;
            long long bi = -1;
            if (s.n_lm > 0) {
                if (!tally_read(a, sh, down_tally(kLayers - 1), down_overflow(kLayers - 1), sh.mid, sh.hraw, G)) goto done;
                wait_tiles(a, sh, k, 1);
                const float* t = slot_ptr(sh, ring, k);
                normalise(sh, sh.hraw, t, sh.hp.eps);
                if (sh.abort) goto done;
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
                    publish_host_token(a, selected);
                    const int64_t st = *a.step;
                    if (st >= 0 && st < cap) a.generated[st] = selected;
                    if (a.stop[1] != 0 && selected == static_cast<int64_t>(a.stop[1]) - 1) a.stop[0] = 1;
                    *a.step = st + 1;
                    *a.position = s.pos + 1;
                    a.sync[0] = 0u;
                    a.sync[1] = s.epoch + 1u;  // the next step's tags and counter base
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
            while (!mbar_try_wait(tile_full(sh, kk), tile_parity(kk)))
                if (global_timer() - t0 > kWaitNs) break;
        }
    }
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

fx_status encode_strip_map(CUtensorMap* map, const float* base, uint64_t columns, const char* what) {
    static std::once_flag once;
    static EncodeTiled encode = nullptr;
    static cudaError_t lookup = cudaSuccess;
    std::call_once(once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult found{};
        lookup = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &found);
        if (lookup == cudaSuccess && found == cudaDriverEntryPointSuccess) encode = reinterpret_cast<EncodeTiled>(fn);
    });
    if (encode == nullptr) {
        set_error("flux native decode: cuTensorMapEncodeTiled is unavailable from the driver");
        return FX_ERR_CUDA;
    }
    const cuuint64_t dims[2] = {columns, static_cast<cuuint64_t>(kHidden)};
    const cuuint64_t strides[1] = {columns * sizeof(float)};
    const cuuint32_t box[2] = {kStepBlock, kStepStripRows};
    const cuuint32_t element_strides[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box,
                              element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error(std::string("flux native decode: encoding the tensor map of ") + what + " failed (CUresult " +
                  std::to_string(static_cast<int>(r)) + ")");
        return FX_ERR_CUDA;
    }
    return FX_OK;
}

}  // namespace

size_t step_exchange_words(int nch) {
    auto up = [](size_t w) { return (w + 31) / 32 * 32; };  // 256-byte sections
    return up(2ull * kStepReplicas * kQKV) + up(2ull * kQHeads * nch * kStepPartial) +
           up(2ull * kLayers * kTallyWords) + up(2ull * kLayers * kOverflowWords);
}

StepExchange step_exchange_views(unsigned long long* base, int nch) {
    auto up = [](size_t w) { return (w + 31) / 32 * 32; };
    StepExchange x{};
    unsigned long long* p = base;
    x.qkv = p;
    p += up(2ull * kStepReplicas * kQKV);
    x.partial = p;
    p += up(2ull * kQHeads * nch * kStepPartial);
    x.tally = p;
    p += up(2ull * kLayers * kTallyWords);
    x.overflow = reinterpret_cast<double*>(p);
    return x;
}

fx_status encode_step_maps(const float* o_proj, const float* down, StepLayer* layer) {
    fx_status st = encode_strip_map(&layer->o_map, o_proj, kHidden, "o_proj");
    if (st != FX_OK) return st;
    return encode_strip_map(&layer->down_map, down, kInter, "the down projection");
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
    const fx_status raised = raise_smem_limit(reinterpret_cast<const void*>(decode_step_kernel), smem,
                                              "raising the step kernel's shared memory");
    if (raised != FX_OK) return raised;
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
        set_error("flux native decode: the persistent step needs a GPU with 128 to 384 SMs");
        return FX_ERR_INVALID;
    }
    *grid = sms;
    return FX_OK;
}

}  // namespace fx
