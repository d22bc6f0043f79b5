// Runtime helpers of libalb_cuda.so: status strings, device checks.
#include <cstdio>
#include <cstring>
#include <atomic>
#include <map>
#include <mutex>
#include <utility>

#include "alb_common.cuh"
#include "alb_internal.h"

static thread_local char g_last_error[512] = "";

void alb_set_last_cuda_error(cudaError_t e, const char * what) {
    snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}
void alb_set_last_error_msg(const char * msg) { snprintf(g_last_error, sizeof(g_last_error), "%s", msg); }

int alb_sm_count() {
    static std::atomic<int> count[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    int c = count[dev].load(std::memory_order_relaxed);
    if (c == 0) {
        cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
        if (c <= 0) c = 148;
        count[dev].store(c, std::memory_order_relaxed);
    }
    return c;
}

namespace alb {
// cudaFuncAttributeMaxDynamicSharedMemorySize is a per-device property of a
// kernel: remember, per (device, kernel), the largest value set so far, under a
// lock (several host threads may drive several devices in one process).
cudaError_t ensure_dynamic_smem(const void * func, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    static std::mutex mu;
    static std::map<std::pair<int, const void *>, size_t> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    size_t & cur = done[std::make_pair(dev, func)];
    if (cur >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) cur = bytes;
    return e;
}

int * device_error_ptr() {
    static int * ptrs[64] = {nullptr};
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(mu);
    if (!ptrs[dev]) {
        int * p = nullptr;
        if (cudaMalloc(&p, 64) != cudaSuccess) return nullptr;   // once per device, never on the hot path
        cudaMemset(p, 0, 64);
        cudaDeviceSynchronize();
        ptrs[dev] = p;
    }
    return ptrs[dev];
}
}  // namespace alb

extern "C" int alb_device_error(int clear) {
    int * p = alb::device_error_ptr();
    if (!p) return ALB_ERR_CUDA;
    int v = 0;
    if (cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return ALB_ERR_CUDA;
    if (clear) cudaMemset(p, 0, sizeof(int));
    return v;
}

extern "C" int alb_version(void) { return 100; }
extern "C" const char * alb_last_error(void) { return g_last_error; }

extern "C" int alb_device_check(int dev) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || dev < 0 || dev >= n) { alb_set_last_error_msg("no CUDA device"); return ALB_ERR_UNSUPPORTED; }
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0) {
        char buf[96];
        snprintf(buf, sizeof(buf), "device %d is sm_%d%d; this build targets sm_100a", dev, major, minor);
        alb_set_last_error_msg(buf);
        return ALB_ERR_UNSUPPORTED;
    }
    return ALB_OK;
}
