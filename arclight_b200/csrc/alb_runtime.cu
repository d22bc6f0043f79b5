// Runtime helpers of libalb_cuda.so: status strings, device checks.
#include <cstdio>
#include <cstring>
#include <mutex>

#include "alb_common.cuh"
#include "alb_internal.h"

static thread_local char g_last_error[512] = "";

void alb_set_last_cuda_error(cudaError_t e, const char * what) {
    snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}
void alb_set_last_error_msg(const char * msg) { snprintf(g_last_error, sizeof(g_last_error), "%s", msg); }

int alb_sm_count() {
    static int count[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (count[dev] == 0) {
        int c = 0;
        cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
        count[dev] = c > 0 ? c : 148;
    }
    return count[dev];
}

namespace alb {
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
