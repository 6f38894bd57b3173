// zq_noalloc.cu -- zq_matmul_noalloc: the quantized matmul for callers that
// cannot allocate device memory.
//
// Some hosts own all device memory and forbid cudaMalloc on their call path:
// plugin hosts whose plugin interface hands over only input and output
// buffers, pool-based allocators whose accounting breaks on raw allocations,
// and latency-critical loops where an allocation would synchronise the
// device.  Such a caller cannot hand zq_matmul a workspace either.  This
// entry point instead uses a scratch array compiled into the library
// (kNoAllocScratchBytes of device memory, held by every GPU that loads the
// library until the process exits) and allocates nothing itself.
//
// Set-up: the first call on each device looks up the array's device address
// with cudaGetSymbolAddress while that device is current (the array's name is
// only a host-side stand-in in host code).  That first call may load the
// library's device code and so should come before any stream capture.  The
// address is cached for the life of the process: after a cudaDeviceReset() on
// a device it no longer names the array, and this entry point must not be
// called on that device again.
//
// Sharing: every call on a device uses the same array, which keeps the last
// call's contents.  The kernels overwrite every scratch byte they read (codes,
// row scales and, for INT4 prefill, the expanded weight codes), so nothing
// needs clearing between calls.  Calls that may overlap on the GPU (different
// streams without ordering between them) race on the array; serialise them.
#include "zq.h"
#include "zq_kernels.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

namespace {

constexpr size_t kNoAllocScratchBytes = ZQ_NOALLOC_SCRATCH_BYTES;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

}  // namespace

extern "C" zq_status zq_matmul_noalloc(const zq_weight* w, const float* x, size_t m, const float* bias, float* y,
                                       void* stream) {
    if (!w) return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: weights are empty");
    if (m == 0) return ZQ_OK;
    const size_t need = zq_matmul_workspace_bytes(w, m);
    if (need > kNoAllocScratchBytes) {
        char buf[200];
        std::snprintf(buf, sizeof buf,
                      "zyron_b200: zq_matmul_noalloc needs %zu bytes of scratch for m=%zu, more than its fixed "
                      "%zu-byte array; use zq_matmul with a workspace",
                      need, m, kNoAllocScratchBytes);
        return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, buf);
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return zq::set_error(ZQ_ERR_CUDA, "zyron_b200: cudaGetDevice failed");
    if (dev < 0 || dev >= kMaxDevices) return zq::set_error(ZQ_ERR_CUDA, "zyron_b200: device ordinal out of range");
    void* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_scratch_ptr[dev]) {
            void* p = nullptr;
            e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (e != cudaSuccess) {
                char buf[160];
                std::snprintf(buf, sizeof buf, "zyron_b200: cudaGetSymbolAddress(scratch) failed: %s",
                              cudaGetErrorString(e));
                return zq::set_error(ZQ_ERR_CUDA, buf);
            }
            g_scratch_ptr[dev] = p;
        }
        scratch = g_scratch_ptr[dev];
    }
    return zq::matmul_with_scratch(w, x, m, bias, y, scratch, kNoAllocScratchBytes, stream);
}
