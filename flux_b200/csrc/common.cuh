// Shared constants, error plumbing and warp/block helpers for flux_b200.
#pragma once

#include <utility>

#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>
#include <cstdio>
#include <string>

#include "flux_b200.h"

namespace fx {

// SmolLM2-135M geometry (fixed by the reference runtime:
// csrc/native_decode_runtime/native_decode_runtime_cuda.cu:29-37).
constexpr int kHidden = 576;
constexpr int kInter = 1536;
constexpr int kQHeads = 9;
constexpr int kKVHeads = 3;
constexpr int kGroup = kQHeads / kKVHeads;  // q heads per kv head
constexpr int kHeadDim = 64;
constexpr int kQKV = 960;
constexpr int kGateUp = 2 * kInter;
constexpr int kLayers = FX_SMOLLM2_LAYERS;

// ------------------------------------------------------------ error plumbing

// Thread-local message of the last failing C-ABI call (fx_last_error()).
void set_error(const std::string& message);
void clear_error();

// Formats "<what>: <cuda error string>" and records it; returns FX_ERR_CUDA.
fx_status cuda_failure(const char* what, cudaError_t error);

#define FX_CUDA_TRY(call, what)                                   \
    do {                                                          \
        cudaError_t fx_err_ = (call);                             \
        if (fx_err_ != cudaSuccess) return ::fx::cuda_failure((what), fx_err_); \
    } while (0)

#define FX_REQUIRE(cond, message)                                 \
    do {                                                          \
        if (!(cond)) {                                            \
            ::fx::set_error(message);                             \
            return FX_ERR_INVALID;                                \
        }                                                         \
    } while (0)

inline cudaStream_t as_stream(void* stream) { return static_cast<cudaStream_t>(stream); }

// Unique ID (cuCtxGetId) of the calling thread's current CUDA context; 0 when
// none is current yet.  A context created after cudaDeviceReset gets a new ID.
fx_status current_context_id(unsigned long long* id);

// Raise `kernel`'s dynamic shared-memory limit to `bytes` in the current
// context, once per (kernel, context, bytes): the attribute belongs to the
// context, so a process that drives several GPUs (or re-creates a context)
// sets it in each.  Thread-safe.
fx_status raise_smem_limit(const void* kernel, size_t bytes, const char* what);

// Device error word of a decode runtime; the prefill's kernels report into
// it (bit 8: a tensor-core projection's bounded wait gave up).
int* decode_error_word(fx_decode* runtime);

// Programmatic dependent launch.  A kernel launched with launch_dependent()
// is scheduled as the previous kernel in the stream retires its CTAs; it
// calls grid_dependency_wait() before touching anything that kernel produced
// (a no-op for an ordinary launch).  Kernels do not trigger their successors
// early: measured, an early trigger slowed the batched step.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Scheduling priority given to this thread's launch_dependent() launches
// (cudaLaunchAttributePriority, lower is more urgent; a captured launch keeps
// it as its graph node's priority), none by default.
constexpr int kNoLaunchPriority = 1 << 30;
inline int& launch_priority() {
    static thread_local int priority = kNoLaunchPriority;
    return priority;
}
struct LaunchPriorityScope {
    int saved;
    explicit LaunchPriorityScope(int priority) : saved(launch_priority()) { launch_priority() = priority; }
    ~LaunchPriorityScope() { launch_priority() = saved; }
};

template <typename... KArgs, typename... Args>
fx_status launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                           const char* what, Args&&... args) {
    cudaLaunchConfig_t config{};
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    cudaLaunchAttribute attributes[2]{};
    attributes[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attributes[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attributes;
    config.numAttrs = 1;
    if (launch_priority() != kNoLaunchPriority) {
        attributes[1].id = cudaLaunchAttributePriority;
        attributes[1].val.priority = launch_priority();
        config.numAttrs = 2;
    }
    FX_CUDA_TRY(cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...), what);
    return FX_OK;
}

// ----------------------------------------------------------- device helpers

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Sum within aligned groups of `Width` lanes (Width a power of two <= 32).
template <int Width>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int o = Width / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Sum within the aligned 8-lane group of the calling lane.  Only that group's
// lanes need to be active (the mask names exactly them), so row groups of a
// warp may diverge.
__device__ __forceinline__ float group8_sum(float v) {
    const unsigned mask = 0xFFu << ((threadIdx.x & 31) & 24);
    v += __shfl_xor_sync(mask, v, 4);
    v += __shfl_xor_sync(mask, v, 2);
    v += __shfl_xor_sync(mask, v, 1);
    return v;
}

// Block-wide sum; every thread gets the result.  `scratch` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* scratch) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int warps = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    v = lane < warps ? scratch[lane] : 0.0f;
    return warp_sum(v);
}

__device__ __forceinline__ float block_max(float v, float* scratch) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int warps = (blockDim.x + 31) >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    v = lane < warps ? scratch[lane] : -FLT_MAX;
    return warp_max(v);
}

// silu(g) * u with the reference's expression (packed_gate_up_gemv_cuda.cu:44).
__device__ __forceinline__ float swiglu(float g, float u) { return (g / (1.0f + expf(-g))) * u; }

// Rotate-half RoPE of one element with separately rounded products
// (packed_qkv_rope_cache_cuda.cu:19-49; transformers apply_rotary_pos_emb).
// `first_half` is true for dimension d < D/2, whose partner enters negated.
__device__ __forceinline__ float rope_value(float value, float partner, float c, float s, bool first_half) {
    const float signed_partner = first_half ? -partner : partner;
    return __fadd_rn(__fmul_rn(value, c), __fmul_rn(signed_partner, s));
}

// Greedy ordering: does (va, ia) precede (vb, ib)?  NaN ranks highest, then
// larger values, then the lower index (greedy_generation_cuda.cu:19-37 with
// torch.argmax's first-NaN rule).  `valid` flags let empty slots lose.
__device__ __forceinline__ bool argmax_precedes(float va, long long ia, float vb, long long ib) {
    if (ia < 0) return false;
    if (ib < 0) return true;
    const bool na = isnan(va), nb = isnan(vb);
    if (na != nb) return na;
    if (na) return ia < ib;
    return va > vb || (va == vb && ia < ib);
}

}  // namespace fx
