// C-linkage shim over the reference's own C++ CPU kernels (test oracle only).
//
// oracle/Makefile compiles this file together with the reference sources
// where they lie (csrc/rmsnorm/rmsnorm.cpp, csrc/residual_rmsnorm/
// residual_rmsnorm.cpp, csrc/packed_swiglu/packed_swiglu.cpp) into
// oracle/_ref/libfluxref_cpu.so, so that ctypes can call them.  Exceptions
// thrown by the reference validation become a non-zero return code.
#include "rmsnorm.h"
#include "residual_rmsnorm.h"
#include "packed_swiglu.h"

#include <cstddef>
#include <exception>

extern "C" int fxref_rmsnorm_fp32(const float* input, const float* weight, float* output,
                                  std::size_t rows, std::size_t hidden, float epsilon) {
    try {
        flux::rmsnorm_fp32(input, weight, output, rows, hidden, epsilon);
    } catch (const std::exception&) {
        return 1;
    }
    return 0;
}

extern "C" int fxref_residual_rmsnorm_fp32(const float* hidden, const float* residual, const float* weight,
                                           float* norm_out, float* residual_out, std::size_t rows,
                                           std::size_t width, float epsilon) {
    try {
        flux::residual_rmsnorm_fp32(hidden, residual, weight, norm_out, residual_out, rows, width, epsilon);
    } catch (const std::exception&) {
        return 1;
    }
    return 0;
}

extern "C" int fxref_packed_swiglu_fp32(const float* packed, float* output, std::size_t rows,
                                        std::size_t intermediate) {
    try {
        flux::packed_swiglu_fp32(packed, output, rows, intermediate);
    } catch (const std::exception&) {
        return 1;
    }
    return 0;
}
