// alb_flash_attn_static: alb_flash_attn with its workspace in a fixed,
// file-scope device array instead of a caller-provided buffer, so the call
// allocates nothing (no cudaMalloc / cudaFree, no allocating library routine).
// It serves callers that cannot allocate device memory, such as an operator
// shim called from the reference's graph walk with only host scratch at hand.
//
// Limits and rules (also stated in include/alb_cuda.h):
//   * the workspace alb_flash_attn_workspace_bytes(...) of the call must fit
//     ALB_FLASH_ATTN_STATIC_BYTES (4 MiB) when the call's path uses one (the
//     split kernels); larger calls are rejected with ALB_ERR_INVALID before
//     anything is launched.  Prefill ubatches (T > 1, one split) use no
//     workspace and are never rejected for size;
//   * the array's address is looked up once per device and kept: a
//     cudaDeviceReset of that device afterwards is not supported;
//   * there is one such array per device, shared by every call on that
//     device: calls that overlap in time (other streams, other host threads)
//     race on it and must not be issued;
//   * the first call on a device looks the array up with cudaGetSymbolAddress
//     (that device current) and clears it once with cudaMemsetAsync on the
//     call's stream (the kernels keep no state in it between calls); make that
//     first call outside any stream capture.
#include <mutex>

#include "alb_common.cuh"
#include "alb_internal.h"

using namespace alb;

namespace {

constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_fa_static_ws[ALB_FLASH_ATTN_STATIC_BYTES];

std::mutex g_mu;
void * g_ws[kMaxDevices] = {};

// Address of this device's array, looked up and cleared on first use.
int static_workspace(void ** out, cudaStream_t stream) {
    int dev = -1;
    ALB_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) {
        alb_set_last_error_msg("alb_flash_attn_static: device ordinal out of range");
        return ALB_ERR_INVALID;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_ws[dev]) {
        void * p = nullptr;
        ALB_CUDA_TRY(cudaGetSymbolAddress(&p, g_fa_static_ws));
        ALB_CUDA_TRY(cudaMemsetAsync(p, 0, ALB_FLASH_ATTN_STATIC_BYTES, stream));
        g_ws[dev] = p;
    }
    *out = g_ws[dev];
    return ALB_OK;
}

}  // namespace

extern "C" int alb_flash_attn_static(const float * q, const uint16_t * k_cache, const uint16_t * v_cache, int64_t T,
                                     int32_t n_head, int32_t n_head_kv, int32_t pos0, float scale, int32_t splits,
                                     float * out, void * stream) {
    ALB_CHECK_ARG(q && k_cache && v_cache && out && T > 0 && T < 65536 && pos0 >= 0);
    ALB_CHECK_ARG(n_head > 0 && n_head_kv > 0 && n_head % n_head_kv == 0);
    const int G = n_head / n_head_kv;
    ALB_CHECK_ARG(G == 1 || G == 2 || G == 4 || G == 8);
    ALB_CHECK_ARG(splits >= 1 && splits <= 65535 && (int64_t)pos0 + T < (int64_t)1 << 30);
    const bool uses_ws = flash_attn_uses_ws(n_head, n_head_kv, (int)T, splits, (int)(pos0 + T));
    const size_t need = uses_ws ? flash_attn_ws_bytes(n_head, n_head_kv, (int)T, splits, (int)(pos0 + T)) : 0;
    if (need > ALB_FLASH_ATTN_STATIC_BYTES) {
        alb_set_last_error_msg("alb_flash_attn_static: workspace exceeds ALB_FLASH_ATTN_STATIC_BYTES");
        return ALB_ERR_INVALID;
    }
    void * ws = nullptr;
    const int rc = static_workspace(&ws, (cudaStream_t)stream);
    if (rc != ALB_OK) return rc;
    FlashArgs f;
    f.ncap = (int)(pos0 + T);
    f.q = q; f.kc = k_cache; f.vc = v_cache; f.Hq = n_head; f.Hkv = n_head_kv; f.T = (int)T;
    f.pos0 = pos0; f.scale = scale; f.S = splits; f.ws = (float *)ws; f.out = out; f.pdl = true;
    ALB_CUDA_TRY(launch_flash_attn(f, (cudaStream_t)stream));
    return ALB_OK;
}
