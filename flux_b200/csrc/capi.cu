// Error plumbing of the C ABI (fx_last_error, fx_version) and the per-context
// one-time set-up shared by every kernel launcher.
#include "common.cuh"

#include <cuda.h>

#include <mutex>
#include <set>
#include <string>
#include <tuple>

namespace fx {
namespace {
thread_local std::string g_last_error;
}  // namespace

void set_error(const std::string& message) { g_last_error = message; }
void clear_error() { g_last_error.clear(); }

fx_status cuda_failure(const char* what, cudaError_t error) {
    set_error(std::string(what) + " failed: " + cudaGetErrorString(error));
    return FX_ERR_CUDA;
}

namespace {
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);
}  // namespace

fx_status current_context_id(unsigned long long* id) {
    static std::once_flag once;
    static CtxGetCurrentFn get_current = nullptr;
    static CtxGetIdFn get_id = nullptr;
    std::call_once(once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult found{};
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &found) == cudaSuccess &&
            found == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
        fn = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &found) == cudaSuccess &&
            found == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<CtxGetIdFn>(fn);
    });
    if (get_current == nullptr || get_id == nullptr) {
        set_error("flux_b200: cuCtxGetCurrent / cuCtxGetId are unavailable from the driver");
        return FX_ERR_CUDA;
    }
    CUcontext context = nullptr;
    if (get_current(&context) != CUDA_SUCCESS) {
        set_error("flux_b200: cuCtxGetCurrent failed");
        return FX_ERR_CUDA;
    }
    *id = 0;
    if (context != nullptr && get_id(context, id) != CUDA_SUCCESS) {
        set_error("flux_b200: cuCtxGetId failed");
        return FX_ERR_CUDA;
    }
    return FX_OK;
}

fx_status raise_smem_limit(const void* kernel, size_t bytes, const char* what) {
    static std::mutex mutex;
    static std::set<std::tuple<const void*, unsigned long long, size_t>> done;
    unsigned long long id = 0;
    fx_status status = current_context_id(&id);
    if (status != FX_OK) return status;
    std::lock_guard<std::mutex> lock(mutex);
    if (id != 0 && done.count({kernel, id, bytes}) != 0) return FX_OK;
    FX_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)),
                what);
    if (id == 0) {  // the call made the device's primary context current
        status = current_context_id(&id);
        if (status != FX_OK) return status;
    }
    if (id != 0) done.insert({kernel, id, bytes});
    return FX_OK;
}

}  // namespace fx

extern "C" const char* fx_last_error(void) { return fx::g_last_error.c_str(); }

extern "C" const char* fx_version(void) { return "flux_b200 0.1 (sm_100a)"; }
