// Peer-memory plumbing for the multi-GPU output gather (one process per GPU): CUDA IPC export
// and import of a device buffer, and an asynchronous device-to-device copy.  A rank that holds
// a shard of the output pushes it with one copy straight into its slice of the gathering
// rank's buffer: a peer copy over NVLink run by the copy engines, ordered on the caller's stream
// after the kernels that produced the shard.  The reference has no multi-GPU path.
#include <cstdint>
#include <cstring>
#include <mutex>

#include <cuda.h>

#include "scx.h"
#include "scx_internal.h"

namespace {

typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

// cuMemGetAddressRange through the runtime's driver entry point (no libcuda link): the base of
// the allocation that contains a pointer (a caching allocator hands out pointers inside larger
// allocations, and an IPC handle names a whole allocation).
AddressRangeFn address_range() {
    static std::once_flag once;
    static AddressRangeFn fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<AddressRangeFn>(p);
    });
    return fn;
}

}  // namespace

extern "C" {

int scx_ipc_handle_bytes(void) { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }

int scx_ipc_export(const void* dev_ptr, void* handle_out, unsigned long long* offset_out) {
    if (!dev_ptr || !handle_out || !offset_out) return cudaErrorInvalidValue;
    AddressRangeFn fn = address_range();
    if (fn == nullptr) return cudaErrorNotSupported;
    CUdeviceptr base = 0;
    size_t size = 0;
    if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) return cudaErrorInvalidValue;
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
    if (e != cudaSuccess) return e;
    std::memcpy(handle_out, &h, sizeof(h));
    *offset_out = static_cast<unsigned long long>(reinterpret_cast<uintptr_t>(dev_ptr) - static_cast<uintptr_t>(base));
    return cudaSuccess;
}

int scx_ipc_import(const void* handle, void** base_out) {
    if (!handle || !base_out) return cudaErrorInvalidValue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    return cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess);
}

int scx_ipc_close(void* base) {
    if (!base) return cudaErrorInvalidValue;
    return cudaIpcCloseMemHandle(base);
}

int scx_copy_async(void* dst, const void* src, size_t bytes, scx_stream_t stream) {
    if (bytes == 0) return cudaSuccess;
    if (!dst || !src) return cudaErrorInvalidValue;
    return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
