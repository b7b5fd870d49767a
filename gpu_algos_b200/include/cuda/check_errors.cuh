// cuda/check_errors.cuh -- abort on a failed CUDA (or C-ABI) call.
#pragma once

#include <cstdlib>
#include <iostream>

#include <cuda_runtime.h>

#include "glm_b200.h"

// Prints "[CUDA error <step>] <message> (<file>:<line>)" and exits with 1,
// like the reference's cuda_check_error (include/cuda/check_errors.cuh:25-32).
// Status codes of libglm_b200 (>= 1000) are printed with their own text.
#define cuda_check_error(cuda_err, step_name)                                                        \
    do {                                                                                             \
        const int glmb_status_ = static_cast<int>(cuda_err);                                         \
        if (glmb_status_ != 0) {                                                                     \
            const char* glmb_msg_ = glmb_status_ >= 1000                                             \
                                        ? glmb_status_string(glmb_status_)                           \
                                        : cudaGetErrorString(static_cast<cudaError_t>(glmb_status_)); \
            std::cerr << "[CUDA error " << step_name << "] " << glmb_msg_ << " (" << __FILE__ << ":"  \
                      << __LINE__ << ")" << std::endl;                                               \
            std::exit(1);                                                                            \
        }                                                                                            \
    } while (0)
