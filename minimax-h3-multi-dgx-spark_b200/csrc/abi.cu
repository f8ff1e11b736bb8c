// Error reporting, the device status word and CUDA IPC plumbing of libh3b.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <cuda.h>

#include "common.cuh"

namespace h3b {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

int cuda_error(cudaError_t e, const char* what) {
    return set_error(H3B_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

// One status word per device; kernels record the first error code here.
__device__ int g_status_word;

int device_status(DeviceStatus* out) {
    constexpr int kMaxDevices = 64;
    static int* cached[kMaxDevices] = {};
    int dev = 0;
    H3B_CUDA_TRY(cudaGetDevice(&dev));
    if (dev >= 0 && dev < kMaxDevices && cached[dev]) {
        out->word = cached[dev];
        return H3B_OK;
    }
    void* p = nullptr;
    H3B_CUDA_TRY(cudaGetSymbolAddress(&p, g_status_word));
    out->word = static_cast<int*>(p);
    if (dev >= 0 && dev < kMaxDevices) cached[dev] = out->word;
    return H3B_OK;
}

}  // namespace h3b

using namespace h3b;

extern "C" int h3b_abi_version(void) { return H3B_ABI_VERSION; }

extern "C" const char* h3b_last_error(void) { return g_last_error; }

extern "C" int h3b_status_get(int* status_out, void* stream) {
    H3B_REQUIRE(status_out != nullptr, "h3b_status_get: status_out is NULL");
    DeviceStatus ds;
    if (int rc = device_status(&ds)) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    H3B_CUDA_TRY(cudaStreamSynchronize(s));
    H3B_CUDA_TRY(cudaMemcpy(status_out, ds.word, sizeof(int), cudaMemcpyDeviceToHost));
    return H3B_OK;
}

extern "C" int h3b_status_clear(void* stream) {
    DeviceStatus ds;
    if (int rc = device_status(&ds)) return rc;
    H3B_CUDA_TRY(cudaMemsetAsync(ds.word, 0, sizeof(int), static_cast<cudaStream_t>(stream)));
    return H3B_OK;
}

// ---------------------------------------------------------------------------
// CUDA IPC.  The driver's cuMemGetAddressRange is fetched through the runtime
// (cudaGetDriverEntryPoint) so the library has no link-time dependency on
// libcuda and loads on hosts without a GPU driver.

typedef CUresult (*PFN_getAddressRange)(CUdeviceptr*, size_t*, CUdeviceptr);

static PFN_getAddressRange address_range_fn() {
    static PFN_getAddressRange fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_getAddressRange>(p);
    }
    return fn;
}

extern "C" int h3b_ipc_handle(const void* dev_ptr, void* handle_out, int64_t* offset_out) {
    H3B_REQUIRE(dev_ptr && handle_out && offset_out, "h3b_ipc_handle: NULL argument");
    PFN_getAddressRange range = address_range_fn();
    if (!range) return set_error(H3B_ERR_CUDA, "h3b_ipc_handle: cuMemGetAddressRange unavailable");
    CUdeviceptr base = 0;
    size_t size = 0;
    CUresult r = range(&base, &size, (CUdeviceptr)(uintptr_t)dev_ptr);
    if (r != CUDA_SUCCESS) return set_error(H3B_ERR_CUDA, "h3b_ipc_handle: cuMemGetAddressRange failed (%d)", (int)r);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, (void*)(uintptr_t)base);
    if (e != cudaSuccess)
        return set_error(H3B_ERR_CUDA,
                         "h3b_ipc_handle: cudaIpcGetMemHandle failed: %s (allocations from expandable segments "
                         "or cuMemCreate cannot be shared this way)",
                         cudaGetErrorString(e));
    memcpy(handle_out, &h, sizeof(h));
    *offset_out = (int64_t)((uintptr_t)dev_ptr - (uintptr_t)base);
    return H3B_OK;
}

extern "C" int h3b_ipc_open(const void* handle, int64_t offset, void** dev_ptr_out, void** base_out) {
    H3B_REQUIRE(handle && dev_ptr_out && base_out && offset >= 0, "h3b_ipc_open: bad argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    H3B_CUDA_TRY(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
    *base_out = base;
    *dev_ptr_out = static_cast<char*>(base) + offset;
    return H3B_OK;
}

extern "C" int h3b_ipc_close(void* base) {
    H3B_REQUIRE(base != nullptr, "h3b_ipc_close: NULL base");
    H3B_CUDA_TRY(cudaIpcCloseMemHandle(base));
    return H3B_OK;
}
