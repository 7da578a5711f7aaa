// cm_ipc.cu -- device buffers of one process made writable by the kernels of
// another (one process per GPU; CUDA IPC over NVLink / NVSwitch).
//
// The batch-sharded drivers gather a step's outputs on one GPU.  Instead of a
// separate collective after the kernels, the root exports its full-size output
// buffers and every other rank opens them: the rank's own kernels (MatMul GEMM
// epilogue, VectorOP, Pooling) then write their shard straight into the root's
// memory with ordinary stores, so each output word crosses NVLink once, while
// the kernel that computes it runs, and no SM time is spent on a copy.  Only
// plain stores reach the peer's memory: no TMA (bulk or tensor) copy and no
// library kernel is given a peer address.  Alternatively a rank computes into
// its own memory and pushes each finished output with cm_copy_async (one
// cudaMemcpyAsync, a copy engine over NVLink) while its next output computes.
#include <cuda.h>

#include <cstring>
#include <map>
#include <mutex>

#include "cm_common.cuh"

namespace cm {
namespace {

typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range_fn() {
    static AddressRangeFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (AddressRangeFn)p;
    }
    return fn;
}

// Allocations opened in this process: base address -> (handle, opens), so that one
// allocation exported for several buffers is mapped once and unmapped with its last close.
struct Opened {
    cudaIpcMemHandle_t handle;
    int refs;
};
std::mutex g_ipc_mu;
std::map<uintptr_t, Opened> g_opened;          // by mapped base
std::multimap<uintptr_t, uintptr_t> g_open_ptrs;    // returned pointer -> mapped base (one entry per open)

}  // namespace
}  // namespace cm

using namespace cm;

extern "C" int cm_ipc_export(const void* dev_ptr, cm_ipc_handle_t* handle) {
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    if (!dev_ptr || !handle) return set_error(CM_EINVAL, "cm_ipc_export: null argument");
    AddressRangeFn range = address_range_fn();
    if (!range) return set_error(CM_ECUDA, "cm_ipc_export: cuMemGetAddressRange is not available");
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, (CUdeviceptr)(uintptr_t)dev_ptr) != CUDA_SUCCESS)
        return set_error(CM_EINVAL, "cm_ipc_export: %p is not device memory of this process", dev_ptr);
    cudaIpcMemHandle_t mh;
    cudaError_t e = cudaIpcGetMemHandle(&mh, (void*)(uintptr_t)base);
    if (e != cudaSuccess) return cuda_error(e, "cudaIpcGetMemHandle");
    static_assert(sizeof(mh) <= sizeof(handle->handle), "IPC handle size");
    memset(handle, 0, sizeof(*handle));
    memcpy(handle->handle, &mh, sizeof(mh));
    handle->offset = (uint64_t)((uintptr_t)dev_ptr - (uintptr_t)base);
    handle->device = cx->device;
    return CM_OK;
}

extern "C" int cm_ipc_open(const cm_ipc_handle_t* handle, void** dev_ptr) {
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    if (!handle || !dev_ptr) return set_error(CM_EINVAL, "cm_ipc_open: null argument");
    cudaIpcMemHandle_t mh;
    memcpy(&mh, handle->handle, sizeof(mh));
    std::lock_guard<std::mutex> lk(g_ipc_mu);
    uintptr_t base = 0;
    for (auto& kv : g_opened)
        if (!memcmp(&kv.second.handle, &mh, sizeof(mh))) base = kv.first;
    if (!base) {
        void* p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, mh, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return cuda_error(e, "cudaIpcOpenMemHandle");
        base = (uintptr_t)p;
        g_opened[base] = Opened{mh, 0};
    }
    g_opened[base].refs++;
    void* p = (void*)(base + handle->offset);
    *dev_ptr = p;
    g_open_ptrs.emplace((uintptr_t)p, base);
    return CM_OK;
}

extern "C" int cm_ipc_close(void* dev_ptr) {
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(g_ipc_mu);
    auto it = g_open_ptrs.find((uintptr_t)dev_ptr);
    if (it == g_open_ptrs.end()) return set_error(CM_EINVAL, "cm_ipc_close: %p was not opened by cm_ipc_open", dev_ptr);
    const uintptr_t base = it->second;
    g_open_ptrs.erase(it);
    auto& o = g_opened[base];
    if (--o.refs == 0) {
        g_opened.erase(base);
        cudaError_t e = cudaIpcCloseMemHandle((void*)base);
        if (e != cudaSuccess) return cuda_error(e, "cudaIpcCloseMemHandle");
    }
    return CM_OK;
}

extern "C" int cm_copy_async(void* dst, const void* src, size_t bytes, cm_stream_t stream) {
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    if (bytes == 0) return CM_OK;
    if (!dst || !src) return set_error(CM_EINVAL, "cm_copy_async: null pointer");
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, (cudaStream_t)stream);
    return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_copy_async");
}
