// fa_noalloc.cu -- acefa_flash_attn_ext_noalloc(): the attention operator for
// callers that cannot provide the engine any device memory at call time.
//
// Who needs it: hosts where every byte of device memory belongs to someone
// else's allocator (a ggml backend whose graph allocator has already planned
// all buffers, a plugin living inside a framework that forbids foreign
// allocations), threads that must never block (cudaMalloc may synchronise the
// whole device, which a real-time audio thread cannot afford), and builds that
// forbid runtime allocation once they have started.  They still pass Q, K, V,
// the mask and the output; what they cannot pass is the workspace that
// acefa_flash_attn_ext() asks for on the dense path (the mask-class table, the
// partial results of the last-wave key-range split, F16 copies of BF16 K/V;
// decode nodes need none).
//
// The scratch therefore lives in this file-scope device array.  Every GPU that
// loads libacefa.so holds it until the process exits.  All calls on a device
// share it and it keeps whatever the previous call left there; nothing in it has
// to start at zero, because each call's kernels write every class byte,
// partial slot and K/V copy before reading it.  Two calls whose kernels overlap on the GPU (different streams, or
// different host threads, without ordering between them) race on the array.
#include <mutex>

#include "fa_internal.h"

namespace acefa {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;

struct NoAllocDevice {
    void *ptr   = nullptr;  // device address of g_noalloc_scratch on this device
    bool  ready = false;
};
NoAllocDevice g_noalloc_dev[kNoAllocMaxDevices];
std::mutex    g_noalloc_mutex;

// Once per device, with that device current: the array's name is only a host
// stand-in, so fetch its real device address.  Retried on a later call if it
// failed.
int noalloc_scratch(void **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) {
        return ACEFA_ERR_CUDA;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    NoAllocDevice              &d = g_noalloc_dev[dev];
    if (!d.ready) {
        void       *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            return ACEFA_ERR_CUDA;
        }
        d.ptr   = p;
        d.ready = true;
    }
    *out = d.ptr;
    return ACEFA_OK;
}

}  // namespace
}  // namespace acefa

extern "C" ACEFA_API int acefa_flash_attn_ext_noalloc(const acefa_tensor *q, const acefa_tensor *k,
                                                      const acefa_tensor *v, const acefa_tensor *mask,
                                                      const acefa_tensor *sinks, const acefa_tensor *dst, float scale,
                                                      float max_bias, float logit_softcap, int prec, void *stream) {
    const int st = acefa_check(q, k, v, mask, sinks, dst);
    if (st != ACEFA_OK) {
        return st;
    }
    // Sized with the same limit the call below passes: the dense plan then
    // cuts its last-wave split (or drops it) to fit the fixed array, so only
    // operands whose smallest plan exceeds it are refused.
    const size_t need = acefa::workspace_bytes_within(q, k, v, mask, dst, acefa::kNoAllocScratchBytes);
    if (need == 0) {
        return ACEFA_ERR_DEVICE;  // operands are valid, so the device query failed
    }
    if (need > acefa::kNoAllocScratchBytes) {
        return ACEFA_ERR_NOALLOC_LIMIT;
    }
    void *scratch = nullptr;
    const int rc  = acefa::noalloc_scratch(&scratch);
    if (rc != ACEFA_OK) {
        return rc;
    }
    return acefa_flash_attn_ext(q, k, v, mask, sinks, dst, scale, max_bias, logit_softcap, prec, stream, scratch,
                                acefa::kNoAllocScratchBytes);
}
