// CUDA IPC through the C ABI: export / import / release of device buffers, so
// that the ranks of one node can map each other's output buffers and the
// attention kernels can store their rows straight into them
// (acefa_flash_attn_ext_mirrored).  Host code only.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <map>
#include <mutex>

#include "acefa.h"

static_assert(sizeof(cudaIpcMemHandle_t) == ACEFA_PEER_HANDLE_BYTES, "IPC handle size");

namespace {

std::mutex                  g_peer_mu;
std::map<uintptr_t, void *> g_peer_bases;  // imported address -> base of its mapping

using AddressRangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);

AddressRangeFn address_range_fn() {
    static AddressRangeFn fn = [] {
        void                            *p = nullptr;
        cudaDriverEntryPointQueryResult  q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            return reinterpret_cast<AddressRangeFn>(p);
        }
        return static_cast<AddressRangeFn>(nullptr);
    }();
    return fn;
}

}  // namespace

extern "C" {

ACEFA_API int acefa_peer_export(const void *ptr, void *handle, uint64_t *offset) {
    if (!ptr || !handle || !offset) {
        return ACEFA_ERR_NULL;
    }
    AddressRangeFn range = address_range_fn();
    if (!range) {
        return ACEFA_ERR_CUDA;
    }
    CUdeviceptr base = 0;
    size_t      size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
        return ACEFA_ERR_CUDA;
    }
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base)) != cudaSuccess) {
        cudaGetLastError();
        return ACEFA_ERR_CUDA;
    }
    std::memcpy(handle, &h, sizeof(h));
    *offset = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
    return ACEFA_OK;
}

ACEFA_API int acefa_peer_import(const void *handle, uint64_t offset, void **ptr) {
    if (!handle || !ptr) {
        return ACEFA_ERR_NULL;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void *base = nullptr;
    if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        return ACEFA_ERR_CUDA;
    }
    char *p = static_cast<char *>(base) + offset;
    {
        std::lock_guard<std::mutex> lk(g_peer_mu);
        g_peer_bases[reinterpret_cast<uintptr_t>(p)] = base;
    }
    *ptr = p;
    return ACEFA_OK;
}

ACEFA_API int acefa_peer_release(void *ptr) {
    if (!ptr) {
        return ACEFA_ERR_NULL;
    }
    void *base = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_peer_mu);
        auto                        it = g_peer_bases.find(reinterpret_cast<uintptr_t>(ptr));
        if (it == g_peer_bases.end()) {
            return ACEFA_ERR_NULL;
        }
        base = it->second;
        g_peer_bases.erase(it);
    }
    if (cudaIpcCloseMemHandle(base) != cudaSuccess) {
        cudaGetLastError();
        return ACEFA_ERR_CUDA;
    }
    return ACEFA_OK;
}

}  // extern "C"
