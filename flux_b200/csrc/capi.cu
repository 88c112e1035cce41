// Error plumbing of the C ABI (fx_last_error, fx_version).
#include "common.cuh"

#include <string>

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

}  // namespace fx

extern "C" const char* fx_last_error(void) { return fx::g_last_error.c_str(); }

extern "C" const char* fx_version(void) { return "flux_b200 0.1 (sm_100a)"; }
