// ABI version and per-thread error text for the lamq_b200 C ABI.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <mutex>
#include <set>
#include <utility>

#include "lamq_common.cuh"

namespace lamq {

static thread_local char g_error[512] = "";
static std::atomic<unsigned long long> g_launches{0};

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_error, sizeof(g_error), fmt, ap);
    va_end(ap);
}

cudaError_t smem_limit_once(const void *kernel, int bytes) {
    static std::mutex mu;
    static std::set<std::pair<const void *, int>> done;  // (kernel, device) pairs already raised
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    if (done.count({kernel, dev})) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done.insert({kernel, dev});
    return e;
}

cudaError_t smem_limit_max_once(const void *kernel) {
    int dev = 0, optin = 0;
    cudaFuncAttributes fa{};
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, kernel);
    if (e != cudaSuccess) return e;
    return smem_limit_once(kernel, optin - (int)fa.sharedSizeBytes);  // dynamic + static <= the opt-in maximum
}

}  // namespace lamq

extern "C" int lamq_abi_version(void) { return 4; }

extern "C" const char *lamq_last_error(void) { return lamq::g_error; }

extern "C" uint64_t lamq_kernel_launches(void) { return lamq::g_launches.load(std::memory_order_relaxed); }
