/*
 * flux_b200 -- C ABI of the B200 (sm_100a) Flux decode-loop library.
 *
 * Plain pointers and sizes only.  Every device pointer is a CUDA device
 * address on the runtime's device; every `stream` is a cudaStream_t passed as
 * `void*` (NULL = the legacy default stream).  Calls are asynchronous on that
 * stream unless stated otherwise.  A non-zero fx_status is an error whose
 * message is available from fx_last_error() on the calling thread.
 *
 * Each entry point names the reference interface it replaces (paths relative
 * to the Mahmood-Elahi/Flux checkout).
 */
#ifndef FLUX_B200_H
#define FLUX_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define FX_API __attribute__((visibility("default")))
#else
#define FX_API
#endif

typedef int32_t fx_status;

#define FX_OK 0
#define FX_ERR_INVALID 1   /* rejected argument (reference: cudaErrorInvalidValue / TORCH_CHECK) */
#define FX_ERR_CUDA 2      /* a CUDA runtime call failed */
#define FX_ERR_EXHAUSTED 3 /* fixed-capacity decode state is exhausted */
#define FX_ERR_STATE 4     /* call order violated (e.g. reuse without prefill or reset) */
#define FX_ERR_DEVICE 5    /* a kernel's own check or bounded wait reported failure */

/* Message of the last failing call on this thread ("" if none).  The
 * reference raises these messages as exceptions (TORCH_CHECK); an FFI caller
 * reads them here, and the Python layer raises them as RuntimeError. */
FX_API const char* fx_last_error(void);
/* Library version string (no counterpart in the reference). */
FX_API const char* fx_version(void);

/* ------------------------------------------------------------------------
 * Operators.  One entry per reference launcher; the torch.ops.flux.* surface
 * binds these.  Tensors are row-major unless strides are passed.
 * ---------------------------------------------------------------------- */

/* out[r, :] = x[r, :] * rsqrt(mean(x[r, :]^2) + eps) * w.
 * Replaces flux::rmsnorm_cuda_fp32 (csrc/rmsnorm/rmsnorm_cuda.h:12-19). */
FX_API fx_status fx_rmsnorm_f32(const float* input, const float* weight, float* output,
                         int64_t rows, int64_t width, float epsilon, void* stream);

/* residual_out = hidden + residual (exact); norm_out = rmsnorm(residual_out).
 * Replaces flux::residual_rmsnorm_cuda_fp32
 * (csrc/residual_rmsnorm/residual_rmsnorm_cuda.h:12-23). */
FX_API fx_status fx_residual_rmsnorm_f32(const float* hidden, const float* residual, const float* weight,
                                  float* norm_out, float* residual_out, int64_t rows, int64_t width,
                                  float epsilon, void* stream);

/* out[r, i] = silu(packed[r, i]) * packed[r, I + i], packed rows of width 2I.
 * Replaces flux::packed_swiglu_cuda_fp32 (csrc/packed_swiglu/packed_swiglu_cuda.h:9-15). */
FX_API fx_status fx_packed_swiglu_f32(const float* packed, float* output, int64_t rows,
                               int64_t intermediate, void* stream);

/* Row softmax over contiguous rows.
 * Replaces flux::softmax_cuda_fp32 (csrc/softmax/softmax_cuda.h:10-18). */
FX_API fx_status fx_softmax_f32(const float* input, float* output, int64_t rows, int64_t width, void* stream);

/* out = softmax(scores * scale + mask) over the last dim of contiguous
 * scores [B, H, Q, K]; mask has sizes/strides broadcastable to the scores.
 * Replaces flux::attention_score_softmax_cuda_fp32
 * (csrc/attention_score_softmax/attention_score_softmax_cuda.h:10-27). */
FX_API fx_status fx_attention_score_softmax_f32(const float* scores, const int64_t* sizes4, const float* mask,
                                         const int64_t* mask_sizes4, const int64_t* mask_strides4,
                                         float scale, float* output, void* stream);

/* Rotate-half RoPE of query [B, Hq, S, D] and key [B, Hk, S, D] (any
 * strides) with cos/sin [Rb, S, D] (Rb in {1, B}); contiguous outputs.
 * Products and sum are separately rounded (no FMA), matching transformers.
 * Replaces flux::rope_cuda_fp32 (csrc/rope/rope_cuda.h:10-28). */
FX_API fx_status fx_rope_f32(const float* query, const int64_t* query_strides4, const float* key,
                      const int64_t* key_strides4, const float* cos, const int64_t* cos_strides3,
                      const float* sin, const int64_t* sin_strides3, float* query_out, float* key_out,
                      int64_t batch, int64_t query_heads, int64_t key_heads, int64_t sequence,
                      int64_t head_dim, int64_t rope_batch, void* stream);

/* SmolLM2 packed QKV [960] -> RoPE(Q) into query_out [9, 64], RoPE(K) and V
 * into row *position of the compact caches [3, capacity, 64] (strides in
 * elements for [batch, head, seq, dim]).  If advance_length is non-NULL it
 * receives *position + 1 (the op form); position and advance_length may alias.
 * Replaces flux::packed_qkv_rope_cache_cuda_fp32 and the _at_position form
 * (csrc/packed_qkv_rope_cache/packed_qkv_rope_cache_cuda.h:30-62). */
FX_API fx_status fx_packed_qkv_rope_cache_f32(const float* packed_qkv, const int64_t* packed_strides3,
                                       const float* cos, const int64_t* cos_strides3, const float* sin,
                                       const int64_t* sin_strides3, float* key_cache,
                                       const int64_t* key_strides4, float* value_cache,
                                       const int64_t* value_strides4, int64_t capacity,
                                       const int64_t* position, int64_t* advance_length,
                                       float* query_out, void* stream);

/* Floats of split-K workspace fx_gqa_decode_attention_f32 needs:
 * batch * query_heads * ceil(capacity / 128) * (head_dim + 2), the layout of
 * the reference's workspace [B, Hq, chunks, D + 2]; 0 for non-positive sizes,
 * INT64_MAX when the product overflows (no workspace is large enough). */
FX_API int64_t fx_gqa_decode_attention_workspace_floats(int64_t batch, int64_t query_heads, int64_t capacity,
                                                 int64_t head_dim);

/* One-token grouped-query attention over the unexpanded cache.
 * query [B, Hq, 1, D], caches [B, Hkv, capacity, D] (strides in elements),
 * optional additive mask broadcastable to [B, Hq, 1, capacity], optional
 * device scalar cache_length (valid rows, clamped to [1, capacity]); output
 * contiguous [B, Hq, 1, D].  head_dim <= 256.  For SmolLM2's geometry over
 * contiguous caches, a workspace of at least
 * fx_gqa_decode_attention_workspace_floats(...) + batch * kv_heads floats
 * holds merge counters after the partials (zero them before the first call
 * with that workspace; every call leaves them zero): when the problem has at
 * most 512 chunk CTAs (batch * kv_heads * ceil(capacity / 128)) the merge
 * then runs in the chunk kernel, one launch instead of two.
 * Replaces flux::gqa_decode_attention_cuda_fp32
 * (csrc/gqa_decode_attention/gqa_decode_attention_cuda.h:10-30). */
FX_API fx_status fx_gqa_decode_attention_f32(const float* query, const int64_t* query_strides4,
                                      const float* key_cache, const int64_t* key_strides4,
                                      const float* value_cache, const int64_t* value_strides4,
                                      const float* mask, const int64_t* mask_sizes4,
                                      const int64_t* mask_strides4, const int64_t* cache_length,
                                      float* output, float* workspace, int64_t workspace_floats,
                                      float scale, int64_t batch, int64_t query_heads, int64_t kv_heads,
                                      int64_t capacity, int64_t head_dim, void* stream);

/* Allocation-free form of fx_gqa_decode_attention_f32 for callers that cannot
 * allocate device memory (a host that owns the whole device budget through its
 * own pool, or a plugin host that passes tensors but no allocator).  No
 * counterpart in the reference.  The split-K partials live in a file-scope
 * device array of fx_gqa_decode_attention_static_scratch_floats() floats
 * (1 MiB), resident on every device that loads the library until exit;
 * larger problems, and sizes beyond fx_gqa_decode_attention_f32's limits, are
 * rejected with FX_ERR_INVALID.  All calls on a device share the array (calls
 * that overlap on the GPU race).  The array's address belongs to a CUDA
 * context: the first call in each context (the primary context, or one the
 * host made current) looks it up and should come before any stream capture.
 * Calls no allocator. */
FX_API int64_t fx_gqa_decode_attention_static_scratch_floats(void);
FX_API fx_status fx_gqa_decode_attention_static_scratch_f32(
    const float* query, const int64_t* query_strides4, const float* key_cache, const int64_t* key_strides4,
    const float* value_cache, const int64_t* value_strides4, const float* mask, const int64_t* mask_sizes4,
    const int64_t* mask_strides4, const int64_t* cache_length, float* output, float scale, int64_t batch,
    int64_t query_heads, int64_t kv_heads, int64_t capacity, int64_t head_dim, void* stream);

/* out[i] = silu(W[i] . x) * (W[intermediate + i] . x), W [2I, width].
 * Replaces flux::packed_gate_up_swiglu_cuda_fp32
 * (csrc/packed_gate_up_gemv/packed_gate_up_gemv_cuda.h:8-12). */
FX_API fx_status fx_packed_gate_up_swiglu_f32(const float* input, const float* weight, float* output,
                                       int64_t intermediate, int64_t width, void* stream);

/* output[M, N] = input[M, K] . weight[N, K]^T (FP32 accumulate).
 * Replaces the cuBLASLt projection flux::cublaslt_linear_config_cuda_fp32
 * (csrc/cublaslt_linear/cublaslt_linear_cuda.h:20-33) and the prefill SGEMMs
 * (csrc/native_prefill_runtime/native_prefill_runtime_cuda.cu:280-302). */
FX_API fx_status fx_linear_f32(const float* input, const float* weight, float* output, int64_t m, int64_t k,
                        int64_t n, void* stream);

/* hi[i] = tf32(input[i]) and lo[i] = tf32(input[i] - hi[i]) (round to nearest,
 * ties away), n % 4 == 0, 16-byte aligned.  No counterpart in the reference:
 * the operand split of the 3xTF32 tensor-core projections below. */
FX_API fx_status fx_tf32_split_f32(const float* input, float* hi, float* lo, int64_t n, void* stream);

/* output[M, N] = input[M, K] . weight[N, K]^T (+ residual[M, N] when non-null)
 * on tcgen05 tensor cores with the 3xTF32 split (weight given as the hi / lo
 * halves from fx_tf32_split_f32; the input is split on chip), FP32
 * accumulation; K % 32 == 0, 16-byte aligned rows.  `error` is a device int
 * that gets bit 8 if an internal wait gave up (never expected).  Same
 * contract as fx_linear_f32 (csrc/cublaslt_linear/cublaslt_linear_cuda.h:20-33),
 * used by the batched and prefill projections.  M <= 64: one CTA per
 * 128 x 64 tile; M >= 2048 with N % 192 == 0: persistent CTA pairs (a
 * cluster launch of tcgen05 cta_group::2 MMAs); otherwise one persistent CTA
 * per SM over 128 x 128 tiles. */
FX_API fx_status fx_linear_3xtf32_f32(const float* input, const float* weight_hi, const float* weight_lo,
                               const float* residual, float* output, int64_t m, int64_t k, int64_t n,
                               int* error, void* stream);

/* *token = argmax(logits) with NaN as the maximum and the lowest index on ties.
 * Replaces flux::greedy_argmax_cuda_fp32
 * (csrc/greedy_generation/greedy_generation_cuda.h:9-14). */
FX_API fx_status fx_greedy_argmax_f32(const float* logits, int64_t vocab, int64_t* token, void* stream);

/* Greedy token plus the decode-state update: *token = argmax;
 * generated[*step] = token when *step < generated_capacity; ++*step;
 * *position = *attention_length.
 * Replaces flux::greedy_argmax_update_cuda_fp32
 * (csrc/greedy_generation/greedy_generation_cuda.h:16-26). */
FX_API fx_status fx_greedy_argmax_update_f32(const float* logits, int64_t vocab, int64_t* token,
                                      int64_t* generated, int64_t generated_capacity, int64_t* step,
                                      int64_t* position, const int64_t* attention_length, void* stream);

/* ------------------------------------------------------------------------
 * Whole-model batch-1 decode runtime.
 * Replaces flux::NativeSmolLM2Decode
 * (csrc/native_decode_runtime/native_decode_runtime.h:57-119).
 * Weights are borrowed device pointers that must outlive the runtime; the
 * caches, the stable token/logit/state buffers and the workspace are owned.
 * ---------------------------------------------------------------------- */

#define FX_SMOLLM2_LAYERS 30

typedef struct fx_model_desc {
    int32_t device;              /* CUDA device ordinal of every pointer */
    int64_t vocab;               /* rows of embedding / lm_head (> 0) */
    int64_t capacity;            /* cache rows; rope tables have this many rows */
    float epsilon;               /* RMSNorm epsilon shared by every norm (> 0) */
    const float* embedding;      /* [vocab, 576] */
    const float* final_norm;     /* [576] */
    const float* lm_head;        /* [vocab, 576]; may equal embedding (tied) */
    const float* rope_cos;       /* [capacity, 64] */
    const float* rope_sin;       /* [capacity, 64] */
    const float* input_norm[FX_SMOLLM2_LAYERS];   /* [576] */
    const float* packed_qkv[FX_SMOLLM2_LAYERS];   /* [960, 576]: q | k | v rows */
    const float* o_proj[FX_SMOLLM2_LAYERS];       /* [576, 576] */
    const float* post_norm[FX_SMOLLM2_LAYERS];    /* [576] */
    const float* gate_up[FX_SMOLLM2_LAYERS];      /* [3072, 576]: gate | up rows */
    const float* down[FX_SMOLLM2_LAYERS];         /* [576, 1536] */
    float attention_scale[FX_SMOLLM2_LAYERS];
} fx_model_desc;

typedef struct fx_decode fx_decode;

/* Stable device buffers of a decode runtime (addresses never change). */
typedef struct fx_decode_buffers {
    int64_t* input_token;        /* [1] next replay's token (argmax of the last step) */
    float* logits;               /* [vocab] */
    int64_t* generated_tokens;   /* [capacity] */
    int64_t* generation_step;    /* [1] */
    float* key_cache;            /* [30, 1, 3, capacity, 64] */
    float* value_cache;          /* [30, 1, 3, capacity, 64] */
    int64_t* position;           /* [1] cache row the next replay writes */
    int64_t* cache_length;       /* [1] valid rows after the last replay */
    float* workspace;            /* owned scratch */
    int64_t workspace_bytes;
    float* hidden_a;             /* [576] */
    float* hidden_b;             /* [576] */
    float* final_norm_output;    /* [576] */
    float* attention_workspace;  /* split-K partials */
    int64_t stable_buffer_bytes; /* token + logits + generated + step + position + length */
    uint64_t* timeline;          /* per-CTA stamps of the last step (SM cycle counter in the
                                    high 32 bits, %globaltimer ns in the low 32), or NULL
                                    (enabled by FLUX_B200_TIMELINE=1 at create) */
    int64_t timeline_ctas;
    int64_t timeline_events;     /* stamps per CTA */
} fx_decode_buffers;

/* Build the runtime, install the initial state and capture the step graph.
 * initial_token: device int64[1].  key_sources/value_sources: FX_SMOLLM2_LAYERS
 * device pointers to contiguous [3, source_rows, 64] (source_rows >= initial
 * position) or NULL when initial_position is 0.  Blocks until the graph is
 * captured.  Replaces the NativeSmolLM2Decode constructor
 * (csrc/native_decode_runtime/native_decode_runtime_cuda.cu:742-865). */
FX_API fx_status fx_decode_create(const fx_model_desc* model, const int64_t* initial_token,
                           const float* const* key_sources, const float* const* value_sources,
                           int64_t source_rows, int64_t initial_position, void* stream, fx_decode** out);

/* One step: optional device token copy, one graph launch; async.
 * FX_ERR_EXHAUSTED once capacity - start position replays were made.
 * Replaces NativeSmolLM2Decode::replay (native_decode_runtime_cuda.cu:907-931). */
FX_API fx_status fx_decode_replay(fx_decode* runtime, const int64_t* token, void* stream);

/* One step with HOST buffers, synchronous: copies *host_token in (skipped
 * when NULL), one graph launch, copies the sampled token out and returns once
 * *host_next holds it.  Both copies go through page-locked words owned by the
 * runtime, so any host pointer works and the copies stay asynchronous to the
 * launch.  Same capacity rule as fx_decode_replay.  The host-buffer form of
 * NativeSmolLM2Decode::replay followed by a read of the current token
 * (native_decode_runtime_cuda.cu:907-931), for hosts that keep tokens in host
 * memory (an FFI caller feeding tokens one at a time).  A device-side failure
 * of the step (a bounded wait that gave up) is reported, as for
 * fx_decode_replay, by the next fx_decode_read_state. */
FX_API fx_status fx_decode_replay_host(fx_decode* runtime, const int64_t* host_token, int64_t* host_next,
                                       void* stream);

/* `steps` chained greedy steps (graph launches), async.  FX_ERR_STATE when
 * called twice without a prefill or reset in between.
 * Replaces NativeSmolLM2Decode::generate_greedy (native_decode_runtime_cuda.cu:933-960). */
FX_API fx_status fx_decode_generate(fx_decode* runtime, int64_t steps, void* stream);

/* Synchronously restore a prefilled state (token, K/V rows [0, position)).
 * Replaces NativeSmolLM2Decode::reset (native_decode_runtime_cuda.cu:962-981). */
FX_API fx_status fx_decode_reset(fx_decode* runtime, const int64_t* token, const float* const* key_sources,
                          const float* const* value_sources, int64_t source_rows, int64_t position,
                          void* stream);

/* Install the state a prefill left in the owned cache: token, position and
 * length = `position`, generated[0] = token, step = 1.  Async.
 * Replaces NativeSmolLM2Decode::install_prefilled_state
 * (native_decode_runtime_cuda.cu:991-1027). */
FX_API fx_status fx_decode_install_prefill(fx_decode* runtime, const int64_t* token, int64_t position, void* stream);

/* Make `stream` wait for the runtime's last enqueued work.
 * Replaces NativeSmolLM2Decode::wait_for_prefill (native_decode_runtime_cuda.cu:983-989). */
FX_API fx_status fx_decode_wait(fx_decode* runtime, void* stream);

/* The runtime's stable device buffers (addresses never change).  Replaces
 * NativeSmolLM2Decode's tensor getters and addresses()
 * (native_decode_runtime_torch.cpp:61-70; buffers native_decode_runtime_cuda.cu:1162-1224). */
FX_API fx_status fx_decode_get_buffers(const fx_decode* runtime, fx_decode_buffers* out);

#define FX_STATE_POSITION 0
#define FX_STATE_CACHE_LENGTH 1
#define FX_STATE_GENERATION_STEP 2
/* Wait for pending work and read one device state scalar.
 * Replaces NativeSmolLM2Decode::position / cache_length / generation_step. */
FX_API fx_status fx_decode_read_state(fx_decode* runtime, int32_t which, int64_t* value);

typedef struct fx_decode_info {
    int64_t capacity;
    int64_t vocab;
    int64_t start_position;  /* position installed by create / reset / prefill */
    int64_t replay_count;    /* graph launches since then */
    int64_t kernels_per_step;/* kernel launches inside one step graph */
} fx_decode_info;
/* Host-side sizes and counters.  Replaces NativeSmolLM2Decode::capacity /
 * replay_count (native_decode_runtime_torch.cpp:73-79). */
FX_API fx_status fx_decode_get_info(const fx_decode* runtime, fx_decode_info* out);

/* Waits for pending work, then releases everything the runtime owns.
 * Replaces the runtime's destructor (native_decode_runtime_cuda.cu:867). */
FX_API void fx_decode_destroy(fx_decode* runtime);

/* ------------------------------------------------------------------------
 * Native prefill feeding an owned decode runtime.
 * Replaces flux::NativeSmolLM2Prefill
 * (csrc/native_prefill_runtime/native_prefill_runtime.h:14-60).
 * ---------------------------------------------------------------------- */

typedef struct fx_prefill fx_prefill;

typedef struct fx_prefill_buffers {
    float* prefill_logits;   /* [vocab] logits of the last prompt row */
    float* workspace;        /* prefill scratch */
    int64_t workspace_bytes;
    float* attention_output; /* [9, prompt, 64] */
    float* final_hidden;     /* [576] final-norm output of the last prompt row */
    int64_t* initial_token;  /* [1] argmax of prefill_logits */
} fx_prefill_buffers;

/* Allocate for a fixed prompt length, build the owned decode runtime (empty
 * cache) and run the first prefill of input_ids (device int64[prompt_length]).
 * Replaces the NativeSmolLM2Prefill constructor
 * (native_prefill_runtime_cuda.cu:355-445). */
FX_API fx_status fx_prefill_create(const fx_model_desc* model, const int64_t* input_ids, int64_t prompt_length,
                            void* stream, fx_prefill** out);

/* Re-run the fixed-shape prompt on `stream` and hand off to decode.
 * Replaces NativeSmolLM2Prefill::prefill (native_prefill_runtime_cuda.cu:540-551). */
FX_API fx_status fx_prefill_run(fx_prefill* runtime, const int64_t* input_ids, void* stream);

/* The owned decode runtime (borrowed; destroyed with the prefill runtime):
 * the prefill object's replay / generate_greedy / state getters go through it
 * (native_prefill_runtime_torch.cpp:24-41). */
FX_API fx_decode* fx_prefill_decode(fx_prefill* runtime);
/* Prefill-side stable buffers (prefill logits, final hidden state).  Replaces
 * NativeSmolLM2Prefill::logits / final_hidden (native_prefill_runtime_torch.cpp:26-30). */
FX_API fx_status fx_prefill_get_buffers(const fx_prefill* runtime, fx_prefill_buffers* out);
/* Replaces NativeSmolLM2Prefill::prompt_length (native_prefill_runtime_torch.cpp:38). */
FX_API int64_t fx_prefill_prompt_length(const fx_prefill* runtime);
/* Waits for pending work, then releases the prefill runtime and its decode
 * runtime.  Replaces the runtime's destructor (native_prefill_runtime_cuda.cu:447). */
FX_API void fx_prefill_destroy(fx_prefill* runtime);

/* ------------------------------------------------------------------------
 * Batched greedy decode: 1 to 64 independent sequences advanced together,
 * one CUDA-graph replay per step.  No counterpart in the reference (its
 * decode runtime and attention op are batch 1 only,
 * csrc/gqa_decode_attention/gqa_decode_attention_torch.cpp:35-36); it serves
 * the sequence-sharded batched configuration: each GPU holds its own
 * sequences and weights, nothing crosses GPUs.  Same weights descriptor as
 * the batch-1 runtime (borrowed); model->capacity is the cache capacity of
 * every sequence and the rope-table row count.
 * ---------------------------------------------------------------------- */

typedef struct fx_batch fx_batch;

typedef struct fx_batch_buffers {
    int64_t* tokens;             /* [B] input token of each sequence's next step */
    int64_t* positions;          /* [B] cache row each sequence's next step writes */
    float* logits;               /* [B, vocab] of the last step */
    int64_t* generated;          /* [B, generated_capacity] greedy tokens emitted per sequence */
    int64_t* step;               /* [1] steps since the last fx_batch_load */
    float* key_cache;            /* [30, B, 3, capacity, 64] */
    float* value_cache;          /* [30, B, 3, capacity, 64] */
    int64_t batch;
    int64_t capacity;
    int64_t generated_capacity;
    int64_t kernels_per_step;    /* launches in one step's graph */
} fx_batch_buffers;

/* Allocate caches and state for `batch` sequences and capture the step graph
 * (synchronous). */
FX_API fx_status fx_batch_create(const fx_model_desc* model, int64_t batch, int64_t generated_capacity,
                                 void* stream, fx_batch** out);
/* Install sequence `sequence`: rows [0, length) of every layer's K/V from
 * key_layers[l] / value_layers[l] ([3, source_rows, 64] each; may be NULL
 * when length == 0), next input token *token (device), position = length;
 * clears its generated row and resets the step counter. */
FX_API fx_status fx_batch_load(fx_batch* runtime, int64_t sequence, const int64_t* token,
                               const float* const* key_layers, const float* const* value_layers,
                               int64_t source_rows, int64_t length, void* stream);
/* Enqueue `steps` greedy steps for every sequence; FX_ERR_EXHAUSTED if a
 * sequence would pass the cache capacity. */
FX_API fx_status fx_batch_step(fx_batch* runtime, int64_t steps, void* stream);
/* Make `stream` wait for the runtime's enqueued work. */
FX_API fx_status fx_batch_wait(fx_batch* runtime, void* stream);
/* Wait for the runtime's work and report a device-side error
 * (FX_ERR_DEVICE: a position outside capacity, a bounded wait gave up). */
FX_API fx_status fx_batch_check(fx_batch* runtime);
FX_API fx_status fx_batch_get_buffers(const fx_batch* runtime, fx_batch_buffers* out);
FX_API void fx_batch_destroy(fx_batch* runtime);

#ifdef __cplusplus
/* EOS-aware greedy generation (the reference's generation is fixed-length,
 * README.md:220; its listed next step, README.md:391): once a step samples
 * `eos_token`, later replays leave every state buffer unchanged (the
 * persistent step returns at once), so fx_decode_generate(n) stops on device
 * and the generation step counter tells how many tokens were produced.  -1
 * disables it; create and reset disable it, prefill installs keep it. */
FX_API fx_status fx_decode_set_eos(fx_decode* runtime, int64_t eos_token);

/* Test hook (no counterpart in the reference): the next persistent decode
 * steps have CTA 0 report a failure at `layer` (0-29; -1 clears) as if one
 * of its bounded waits had expired.  The other CTAs find the error word in
 * their polls, drain their copies and return; fx_decode_read_state then
 * reports FX_ERR_DEVICE until fx_decode_reset.  No GPU fault is involved. */
FX_API fx_status fx_decode_inject_failure(fx_decode* runtime, int32_t layer);

}  /* extern "C" */
#endif

#endif /* FLUX_B200_H */
