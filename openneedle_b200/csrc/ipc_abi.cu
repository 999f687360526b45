// CUDA IPC for device buffers shared between the ranks of one node (one
// process per GPU): a rank exports a buffer (handle + offset inside its
// allocation), the other ranks import it and get a pointer they can write
// over NVLink.  Used to fuse the all-gather of an N-sharded GEMM into the
// GEMM's epilogue (needle2_sdot_multiply_gather_device).  No counterpart in
// the reference, which runs on one host.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstring>
#include <map>
#include <mutex>

#include "common.cuh"
#include "needle2_b200.h"

namespace {

PFN_cuMemGetAddressRange_v3020 address_range_fn() {
    static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
    });
    return fn;
}

std::mutex g_imports_mu;
std::map<void *, void *> g_imports;   // imported pointer (base + offset) -> mapped base

}  // namespace

extern "C" {

int needle2_b200_ipc_export(const void *ptr, void *handle, unsigned long long *offset) {
    nb200::clear_error();
    if (!ptr || !handle || !offset) { nb200::set_error("null argument"); return -1; }
    auto fn = address_range_fn();
    if (!fn) { nb200::set_error("cuMemGetAddressRange is not available from the driver"); return -1; }
    CUdeviceptr base = 0;
    size_t size = 0;
    if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
        nb200::set_error("pointer is not device memory of this process");
        return -1;
    }
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
    if (e != cudaSuccess) {
        nb200::set_error(std::string("cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
        return -1;
    }
    std::memcpy(handle, &h, sizeof(h));
    *offset = reinterpret_cast<CUdeviceptr>(ptr) - base;
    return 0;
}

int needle2_b200_ipc_import(const void *handle, unsigned long long offset, void **ptr) {
    nb200::clear_error();
    if (!handle || !ptr) { nb200::set_error("null argument"); return -1; }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void *base = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        nb200::set_error(std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
        return -1;
    }
    *ptr = static_cast<char *>(base) + offset;
    std::lock_guard<std::mutex> lock(g_imports_mu);
    g_imports[*ptr] = base;
    return 0;
}

int needle2_b200_ipc_close(void *ptr) {
    nb200::clear_error();
    void *base = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_imports_mu);
        auto it = g_imports.find(ptr);
        if (it == g_imports.end()) { nb200::set_error("pointer was not imported"); return -1; }
        base = it->second;
        g_imports.erase(it);
    }
    const cudaError_t e = cudaIpcCloseMemHandle(base);
    if (e != cudaSuccess) {
        nb200::set_error(std::string("cudaIpcCloseMemHandle: ") + cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

}  // extern "C"
