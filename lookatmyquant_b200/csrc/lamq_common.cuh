// Shared definitions for the lookatmyquant_b200 CUDA kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/lamq_b200.h"

namespace lamq {

// Records the first CUDA error of the calling thread's last API call, for lamq_last_error().
void set_error(const char *fmt, ...);

// Raises a kernel's dynamic shared-memory limit to `bytes` once per device (thread-safe; defined in api.cu).
cudaError_t smem_limit_once(const void *kernel, int bytes);
// The same, to the device's opt-in maximum: for kernels whose shared memory varies from call to call, so that a call
// on one host thread never lowers the limit under another thread's launch.
cudaError_t smem_limit_max_once(const void *kernel);

// Counts one kernel launch of this library (lamq_kernel_launches()).
void count_launch();

#define LAMQ_CHECK_LAUNCH(what)                                                         \
    do {                                                                                \
        cudaError_t _e = cudaGetLastError();                                            \
        if (_e != cudaSuccess) {                                                        \
            ::lamq::set_error("%s: %s", what, cudaGetErrorString(_e));                  \
            return LAMQ_ERR_CUDA;                                                       \
        }                                                                               \
        ::lamq::count_launch();                                                         \
    } while (0)

#define LAMQ_REQUIRE(cond, ...)                                                         \
    do {                                                                                \
        if (!(cond)) {                                                                  \
            ::lamq::set_error(__VA_ARGS__);                                             \
            return LAMQ_ERR_INVALID;                                                    \
        }                                                                               \
    } while (0)

// Round-to-nearest fp32 arithmetic that the compiler may not contract into a fused multiply-add: the trellis costs
// must round exactly as the reference's separate tensor ops do (a subtract, a square, an add).
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }

}  // namespace lamq
