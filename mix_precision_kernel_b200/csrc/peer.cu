// Cross-process sharing of device buffers for the fused all-gather (CUDA IPC),
// and the checks that every pointer the gather kernels store through is mapped
// for the current GPU and large enough.
//
// Export: the allocation that contains a pointer (driver cuMemGetAddressRange)
// gets a cudaIpcMemHandle; the pointer's offset and the allocation's size travel
// with it.  Import: the handle is opened with the importing process's own device
// current and cudaIpcMemLazyEnablePeerAccess, so the mapping belongs to that
// device's context and peer access to the owner is enabled -- a kernel on this GPU
// may then store through it.  Imported ranges are recorded; store targets are
// accepted only inside a recorded range imported on the current device or inside
// an allocation of the current device.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>
#include <vector>

#include "mpk.h"
#include "mpk_internal.h"

namespace mpk {

namespace {

typedef CUresult (*PFN_getAddressRange)(CUdeviceptr*, size_t*, CUdeviceptr);

struct Imported {
    uintptr_t base;
    size_t size;
    int device;
    int refs;
    unsigned char handle[sizeof(cudaIpcMemHandle_t)];
};

std::mutex g_peer_mu;   // guards g_imported
std::mutex g_range_mu;  // guards g_range_fn
std::vector<Imported> g_imported;
PFN_getAddressRange g_range_fn = nullptr;

int address_range(const void* ptr, uintptr_t* base, size_t* size)
{
    {
        std::lock_guard<std::mutex> lk(g_range_mu);
        if (!g_range_fn) {
            void* f = nullptr;
            cudaDriverEntryPointQueryResult q;
            cudaError_t e = cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &f, 12000, cudaEnableDefault, &q);
            if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !f) {
                set_last_error("cuMemGetAddressRange entry point unavailable");
                return MPK_ERR_DRIVER;
            }
            g_range_fn = reinterpret_cast<PFN_getAddressRange>(f);
        }
    }
    CUdeviceptr b = 0;
    size_t s = 0;
    const CUresult r = g_range_fn(&b, &s, reinterpret_cast<CUdeviceptr>(ptr));
    if (r != CUDA_SUCCESS) {
        set_last_error("cuMemGetAddressRange failed (CUresult %d): not a device allocation", (int)r);
        return MPK_ERR_INVALID_VALUE;
    }
    *base = (uintptr_t)b;
    *size = s;
    return MPK_SUCCESS;
}

}  // namespace

int check_store_target(const void* ptr, size_t bytes, const char* what)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        set_last_error("no current device");
        return MPK_ERR_INVALID_VALUE;
    }
    const uintptr_t p = reinterpret_cast<uintptr_t>(ptr);
    {
        std::lock_guard<std::mutex> lk(g_peer_mu);
        for (const Imported& im : g_imported) {
            if (p >= im.base && p < im.base + im.size) {
                if (im.device != dev) {
                    set_last_error("%s was imported on device %d, not the current device %d", what, im.device, dev);
                    return MPK_ERR_INVALID_VALUE;
                }
                if (bytes > im.base + im.size - p) {
                    set_last_error("%s: %zu bytes do not fit in the imported buffer", what, bytes);
                    return MPK_ERR_INVALID_VALUE;
                }
                return MPK_SUCCESS;
            }
        }
    }
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, ptr) != cudaSuccess) {
        cudaGetLastError();
        set_last_error("%s is not a device pointer", what);
        return MPK_ERR_INVALID_VALUE;
    }
    if (attr.type != cudaMemoryTypeDevice || attr.device != dev) {
        set_last_error("%s is not memory of the current device %d (import other GPUs' buffers with "
                       "mpk_ipc_import)", what, dev);
        return MPK_ERR_INVALID_VALUE;
    }
    uintptr_t base = 0;
    size_t size = 0;
    if (int rc = address_range(ptr, &base, &size)) return rc;
    if (bytes > base + size - p) {
        set_last_error("%s: %zu bytes do not fit in its allocation", what, bytes);
        return MPK_ERR_INVALID_VALUE;
    }
    return MPK_SUCCESS;
}

}  // namespace mpk

using namespace mpk;

extern "C" {

int mpk_ipc_export(const void* dev_ptr, void* handle, uint64_t* offset, uint64_t* alloc_bytes)
{
    if (!dev_ptr || !handle || !offset || !alloc_bytes) {
        set_last_error("null argument");
        return MPK_ERR_INVALID_VALUE;
    }
    uintptr_t base = 0;
    size_t size = 0;
    if (int rc = address_range(dev_ptr, &base, &size)) return rc;
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
    if (e != cudaSuccess) {
        set_last_error("cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
        return (int)e;
    }
    std::memcpy(handle, &h, sizeof(h));
    *offset = reinterpret_cast<uintptr_t>(dev_ptr) - base;
    *alloc_bytes = size;
    return MPK_SUCCESS;
}

int mpk_ipc_import(const void* handle, uint64_t offset, uint64_t alloc_bytes, void** dev_ptr)
{
    if (!handle || !dev_ptr || offset >= alloc_bytes) {
        set_last_error("bad import arguments");
        return MPK_ERR_INVALID_VALUE;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        set_last_error("cudaGetDevice: %s", cudaGetErrorString(e));
        return (int)e;
    }
    std::lock_guard<std::mutex> lk(g_peer_mu);
    for (Imported& im : g_imported) {
        if (im.device == dev && std::memcmp(im.handle, handle, sizeof(im.handle)) == 0) {
            ++im.refs;
            *dev_ptr = reinterpret_cast<void*>(im.base + offset);
            return MPK_SUCCESS;
        }
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        set_last_error("cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
        return (int)e;
    }
    // The recorded size bounds every later store check, so it is the mapping's real
    // size, and a caller's size larger than that is refused.
    uintptr_t mbase = 0;
    size_t msize = 0;
    if (int rc = address_range(base, &mbase, &msize)) {
        cudaIpcCloseMemHandle(base);
        return rc;
    }
    if (mbase != reinterpret_cast<uintptr_t>(base) || alloc_bytes > msize) {
        cudaIpcCloseMemHandle(base);
        set_last_error("imported allocation is %zu bytes, not the %llu the exporter described", msize,
                       (unsigned long long)alloc_bytes);
        return MPK_ERR_INVALID_VALUE;
    }
    Imported im;
    im.base = reinterpret_cast<uintptr_t>(base);
    im.size = msize;
    im.device = dev;
    im.refs = 1;
    std::memcpy(im.handle, handle, sizeof(im.handle));
    g_imported.push_back(im);
    *dev_ptr = reinterpret_cast<void*>(im.base + offset);
    return MPK_SUCCESS;
}

int mpk_ipc_close(void* dev_ptr)
{
    const uintptr_t p = reinterpret_cast<uintptr_t>(dev_ptr);
    std::lock_guard<std::mutex> lk(g_peer_mu);
    for (size_t i = 0; i < g_imported.size(); ++i) {
        Imported& im = g_imported[i];
        if (p >= im.base && p < im.base + im.size) {
            if (--im.refs > 0) return MPK_SUCCESS;
            const cudaError_t e = cudaIpcCloseMemHandle(reinterpret_cast<void*>(im.base));
            g_imported.erase(g_imported.begin() + (long)i);
            if (e != cudaSuccess) {
                set_last_error("cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
                return (int)e;
            }
            return MPK_SUCCESS;
        }
    }
    set_last_error("pointer was not imported with mpk_ipc_import");
    return MPK_ERR_INVALID_VALUE;
}

}  // extern "C"
