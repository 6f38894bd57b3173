// zq_api.cu -- the C ABI (include/zq.h) over the B200 kernels.
//
// Host-side responsibilities: argument validation with the reference's
// messages, device weight objects in the panel layout, .zyq parsing /
// writing, tensor-map creation for the tcgen05 GEMM, kernel dispatch and the
// device error word.  No entry point falls back to the CPU.
#include "zq.h"
#include "zq_common.cuh"
#include "zq_internal.h"
#include "zq_kernels.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <atomic>
#include <cstring>
#include <limits>
#include <mutex>
#include <string>
#include <vector>

// Error word written by bounded device waits (see mbar_wait_bounded).  One
// per device; the host reads and clears it in zq_device_error().
__device__ uint32_t g_zq_device_error = 0;

namespace {

constexpr uint32_t kZyqMagic = 0x315A5951u;  // "QYZ1" (quantization.cpp:20)
constexpr uint32_t kZyqVersion = 1;          // quantization.cpp:21

thread_local std::string t_last_error;

zq_status fail(zq_status s, const std::string& msg) {
    t_last_error = msg;
    return s;
}

zq_status cuda_fail(cudaError_t e, const char* what) {
    std::string m = "zyron_b200: CUDA error in ";
    m += what;
    m += ": ";
    m += cudaGetErrorName(e);
    m += " (";
    m += cudaGetErrorString(e);
    m += ")";
    return fail(ZQ_ERR_CUDA, m);
}

#define ZQ_CUDA(call)                                         \
    do {                                                      \
        cudaError_t _e = (call);                              \
        if (_e != cudaSuccess) return cuda_fail(_e, #call);   \
    } while (0)

cudaStream_t as_stream(void* s) { return s ? static_cast<cudaStream_t>(s) : cudaStreamPerThread; }

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

bool mul_overflows(size_t a, size_t b) { return a != 0 && b > std::numeric_limits<size_t>::max() / a; }

size_t ref_payload_bytes(int type, size_t K, size_t N) {
    const size_t e = K * N;
    return type == ZQ_TYPE_INT8 ? e : (e + 1) / 2;
}

size_t col_bytes(const zq_weight* w) { return w->type == ZQ_TYPE_INT8 ? (size_t)w->Kp : (size_t)w->Kp / 2; }

// ---- driver entry point for tensor-map encoding (no libcuda link) ---------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

zq_status get_encoder() {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!g_encode) return fail(ZQ_ERR_CUDA, "zyron_b200: cuTensorMapEncodeTiled is unavailable");
    return ZQ_OK;
}

// 2D K-major int8 map: rows x Kp bytes, box 128 bytes x box_rows, 128 B swizzle.
zq_status encode_kmajor(CUtensorMap* map, const void* base, size_t rows, int Kp, int box_rows) {
    zq_status s = get_encoder();
    if (s != ZQ_OK) return s;
    cuuint64_t dims[2] = {(cuuint64_t)Kp, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)Kp};
    cuuint32_t box[2] = {128u, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1u, 1u};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char buf[160];
        std::snprintf(buf, sizeof buf, "zyron_b200: cuTensorMapEncodeTiled failed (%d) rows=%zu Kp=%d box=%d",
                      (int)r, rows, Kp, box_rows);
        return fail(ZQ_ERR_CUDA, buf);
    }
    return ZQ_OK;
}

// ---- device error word ----------------------------------------------------
std::mutex g_err_mu;
uint32_t* g_err_ptr[64] = {nullptr};
std::vector<std::pair<void*, void*>> g_ipc_bases;  // imported pointer -> mapped allocation base

zq_status device_error_ptr(uint32_t** out) {
    int dev = 0;
    ZQ_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(ZQ_ERR_CUDA, "zyron_b200: device ordinal out of range");
    std::lock_guard<std::mutex> lk(g_err_mu);
    if (!g_err_ptr[dev]) {
        void* p = nullptr;
        ZQ_CUDA(cudaGetSymbolAddress(&p, g_zq_device_error));
        g_err_ptr[dev] = static_cast<uint32_t*>(p);
    }
    *out = g_err_ptr[dev];
    return ZQ_OK;
}

zq_status check_dims(size_t rows, size_t cols) {
    if (rows == 0 || cols == 0) return fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: weights are empty");
    if (mul_overflows(rows, cols)) return fail(ZQ_ERR_OVERFLOW, "ZYRON quantization: matrix size overflow");
    if (rows > (size_t)std::numeric_limits<int>::max() - 64 || cols > (size_t)std::numeric_limits<int>::max())
        return fail(ZQ_ERR_OVERFLOW, "zyron_b200: matrix dimension exceeds 2^31-1");
    return ZQ_OK;
}

zq_status new_weight(int type, size_t K, size_t N, zq_weight** out) {
    auto* w = new (std::nothrow) zq_weight;
    if (!w) return fail(ZQ_ERR_RUNTIME, "zyron_b200: out of host memory");
    w->type = type;
    w->K = K;
    w->N = N;
    w->Kp = zq::padded_k(type, (int)K);
    cudaGetDevice(&w->device);
    w->panel_bytes = N * col_bytes(w);
    cudaError_t e = cudaMalloc(&w->panel, w->panel_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&w->scales, N * sizeof(float));
    if (e != cudaSuccess) {
        cudaFree(w->panel);
        cudaFree(w->scales);
        delete w;
        return cuda_fail(e, "cudaMalloc(weight)");
    }
    *out = w;
    return ZQ_OK;
}

// Upload reference-layout payload into an allocated panel.
zq_status upload_payload(zq_weight* w, const void* payload, cudaStream_t st) {
    const size_t K = w->K, N = w->N;
    ZQ_CUDA(cudaMemsetAsync(w->panel, 0, w->panel_bytes, st));
    if (w->type == ZQ_TYPE_INT8) {
        ZQ_CUDA(cudaMemcpy2DAsync(w->panel, (size_t)w->Kp, payload, K, K, N, cudaMemcpyHostToDevice, st));
    } else {
        // the reference's nibble stream, rearranged into the panel layout
        const size_t bytes = ref_payload_bytes(w->type, K, N);
        uint8_t* tmp = nullptr;
        ZQ_CUDA(cudaMalloc(&tmp, bytes));
        cudaError_t e = cudaMemcpyAsync(tmp, payload, bytes, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = zq::launch_repack_int4(tmp, (int)K, (int)N, w->Kp, w->panel, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        cudaFree(tmp);
        if (e != cudaSuccess) return cuda_fail(e, "int4 repack upload");
    }
    return ZQ_OK;
}

zq_status download_payload(const zq_weight* w, void* payload, cudaStream_t st) {
    const size_t K = w->K, N = w->N;
    if (w->type == ZQ_TYPE_INT8) {
        ZQ_CUDA(cudaMemcpy2DAsync(payload, K, w->panel, (size_t)w->Kp, K, N, cudaMemcpyDeviceToHost, st));
    } else {
        // the panel layout, rearranged into the reference's nibble stream
        const size_t bytes = ref_payload_bytes(w->type, K, N);
        uint8_t* tmp = nullptr;
        ZQ_CUDA(cudaMalloc(&tmp, bytes));
        cudaError_t e = zq::launch_unpack_panel_int4(w->panel, (int)K, (int)N, w->Kp, tmp, st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(payload, tmp, bytes, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        cudaFree(tmp);
        if (e != cudaSuccess) return cuda_fail(e, "int4 download");
        return ZQ_OK;
    }
    ZQ_CUDA(cudaStreamSynchronize(st));
    return ZQ_OK;
}

// Packed INT4 panel [N][Kp/2] bytes, box 64 bytes (128 codes) x box_rows
// columns, unswizzled: the decode kernel and the GEMMs unpack it in shared
// memory.
zq_status encode_packed_int4(CUtensorMap* map, const void* base, size_t cols, int Kp, int box_rows = 128) {
    zq_status s = get_encoder();
    if (s != ZQ_OK) return s;
    cuuint64_t dims[2] = {(cuuint64_t)(Kp / 2), (cuuint64_t)cols};
    cuuint64_t strides[1] = {(cuuint64_t)(Kp / 2)};
    cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1u, 1u};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char buf[160];
        std::snprintf(buf, sizeof buf, "zyron_b200: cuTensorMapEncodeTiled failed (%d) cols=%zu Kp=%d (packed)",
                      (int)r, cols, Kp);
        return fail(ZQ_ERR_CUDA, buf);
    }
    return ZQ_OK;
}

// 3-D view of a K-major [rows][Kp] panel (Kp a multiple of 128 codes) for
// the decode kernel: (bytes within a k-block row, rows, k-block), box
// kblock_bytes x box_rows x zq::skinny_kgroup().  INT8 panels and activation
// codes: 128 bytes per k-block row, 128-byte swizzle; packed INT4 panels: 64
// bytes, unswizzled (the kernel unpacks them).
zq_status encode_decode_view(CUtensorMap* map, const void* base, size_t rows, int Kp, int kblock_bytes,
                             int box_rows) {
    zq_status s = get_encoder();
    if (s != ZQ_OK) return s;
    if (Kp % 128 != 0) return fail(ZQ_ERR_RUNTIME, "zyron_b200: decode view needs whole 128-code k-blocks");
    const int row_bytes = kblock_bytes == 128 ? Kp : Kp / 2;
    cuuint64_t dims[3] = {(cuuint64_t)kblock_bytes, (cuuint64_t)rows, (cuuint64_t)(Kp / 128)};
    cuuint64_t strides[2] = {(cuuint64_t)row_bytes, (cuuint64_t)kblock_bytes};
    cuuint32_t box[3] = {(cuuint32_t)kblock_bytes, (cuuint32_t)box_rows, (cuuint32_t)zq::skinny_kgroup()};
    cuuint32_t estr[3] = {1u, 1u, 1u};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE,
                          kblock_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char buf[160];
        std::snprintf(buf, sizeof buf, "zyron_b200: cuTensorMapEncodeTiled failed (%d) rows=%zu Kp=%d (decode view)",
                      (int)r, rows, Kp);
        return fail(ZQ_ERR_CUDA, buf);
    }
    return ZQ_OK;
}

int tile_index(int block_n) {
    return block_n == zq::kPairBlockN ? 3 : (block_n == 256 ? 2 : (block_n == 128 ? 1 : 0));
}

// Rows of the weight box one CTA loads: the 2-SM kernel splits its 256 tile
// columns between the two CTAs of a pair.
int box_rows_b(int block_n) { return block_n == zq::kPairBlockN ? 128 : block_n; }

// Per-thread device buffers and copy streams of zq_matmul_host.
constexpr int kHostChunks = 8;
struct HostStaging {
    int device = -1;
    cudaStream_t h2d = nullptr, d2h = nullptr;
    cudaEvent_t in_done[kHostChunks] = {}, mm_done[kHostChunks] = {}, out_done = nullptr;
    bool streams_ready = false;
    void* x = nullptr;
    size_t x_cap = 0;
    void* y = nullptr;
    size_t y_cap = 0;
    void* b = nullptr;
    size_t b_cap = 0;
    void* ws = nullptr;
    size_t ws_cap = 0;
    ~HostStaging() {
        cudaFree(x);
        cudaFree(y);
        cudaFree(b);
        cudaFree(ws);
        if (streams_ready) {
            cudaStreamDestroy(h2d);
            cudaStreamDestroy(d2h);
            for (int i = 0; i < kHostChunks; ++i) {
                cudaEventDestroy(in_done[i]);
                cudaEventDestroy(mm_done[i]);
            }
            cudaEventDestroy(out_done);
        }
    }
    cudaError_t init_streams() {
        if (streams_ready) return cudaSuccess;
        cudaError_t e = cudaStreamCreateWithFlags(&h2d, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&d2h, cudaStreamNonBlocking);
        for (int i = 0; i < kHostChunks && e == cudaSuccess; ++i) {
            e = cudaEventCreateWithFlags(&in_done[i], cudaEventDisableTiming);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&mm_done[i], cudaEventDisableTiming);
        }
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&out_done, cudaEventDisableTiming);
        if (e == cudaSuccess) streams_ready = true;
        return e;
    }
};
thread_local HostStaging t_staging;

cudaError_t ensure(void*& p, size_t& cap, size_t need) {
    if (cap >= need) return cudaSuccess;
    cudaFree(p);
    p = nullptr;
    cap = 0;
    cudaError_t e = cudaMalloc(&p, need);
    if (e == cudaSuccess) cap = need;
    return e;
}

}  // namespace

extern "C" {

const char* zq_last_error(void) { return t_last_error.c_str(); }

int zq_abi_version(void) { return ZQ_ABI_VERSION; }

zq_status zq_weight_create(int type, size_t rows, size_t cols, const float* scales_host, const void* payload_host,
                           size_t payload_bytes, void* stream, zq_weight** out) {
    if (!out) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null output handle");
    *out = nullptr;
    if (type != ZQ_TYPE_INT8 && type != ZQ_TYPE_INT4)
        return fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: unsupported type");
    zq_status s = check_dims(rows, cols);
    if (s != ZQ_OK) return s;
    if (!scales_host || !payload_host) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null scales or payload");
    if (payload_bytes != ref_payload_bytes(type, rows, cols))
        return fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: invalid payload size");
    zq_weight* w = nullptr;
    s = new_weight(type, rows, cols, &w);
    if (s != ZQ_OK) return s;
    cudaStream_t st = as_stream(stream);
    s = upload_payload(w, payload_host, st);
    if (s == ZQ_OK) {
        cudaError_t e = cudaMemcpyAsync(w->scales, scales_host, cols * sizeof(float), cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) s = cuda_fail(e, "weight upload");
    }
    if (s != ZQ_OK) {
        zq_weight_destroy(w);
        return s;
    }
    *out = w;
    return ZQ_OK;
}

zq_status zq_weight_quantize(const float* w_dev, size_t rows, size_t cols, int type, void* stream, zq_weight** out) {
    if (!out) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null output handle");
    *out = nullptr;
    if (type != ZQ_TYPE_INT8 && type != ZQ_TYPE_INT4)
        return fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: unsupported type");
    zq_status s = check_dims(rows, cols);
    if (s != ZQ_OK) return s;
    if (!w_dev) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null weights");
    zq_weight* w = nullptr;
    s = new_weight(type, rows, cols, &w);
    if (s != ZQ_OK) return s;
    cudaStream_t st = as_stream(stream);
    uint32_t* tmp = nullptr;
    cudaError_t e = cudaMalloc(&tmp, cols * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemsetAsync(w->panel, 0, w->panel_bytes, st);
    if (e == cudaSuccess)
        e = zq::launch_quantize_weights(w_dev, (int)rows, (int)cols, w->Kp, type, tmp, w->scales, w->panel, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    cudaFree(tmp);
    if (e != cudaSuccess) {
        zq_weight_destroy(w);
        return cuda_fail(e, "device quantize");
    }
    *out = w;
    return ZQ_OK;
}

zq_status zq_weight_quantize_host(const float* w_host, size_t rows, size_t cols, int type, void* stream,
                                  zq_weight** out) {
    if (!out) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null output handle");
    *out = nullptr;
    if (type != ZQ_TYPE_INT8 && type != ZQ_TYPE_INT4)
        return fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: unsupported type");
    zq_status s = check_dims(rows, cols);
    if (s != ZQ_OK) return s;
    if (!w_host) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null weights");
    float* tmp = nullptr;
    cudaStream_t st = as_stream(stream);
    ZQ_CUDA(cudaMalloc(&tmp, rows * cols * sizeof(float)));
    cudaError_t e = cudaMemcpyAsync(tmp, w_host, rows * cols * sizeof(float), cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) {
        cudaFree(tmp);
        return cuda_fail(e, "weight copy");
    }
    s = zq_weight_quantize(tmp, rows, cols, type, stream, out);
    cudaFree(tmp);
    return s;
}

zq_status zq_weight_load_zyq(const void* bytes, size_t len, size_t* consumed, void* stream, zq_weight** out) {
    if (!out) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null output handle");
    *out = nullptr;
    zq::ZyqRecord rec;
    zq_status s = zq::parse_zyq(bytes, len, &rec);
    if (s != ZQ_OK) return s;
    s = zq_weight_create(rec.type, rec.rows, rec.cols, rec.scales.data(), rec.payload, rec.payload_bytes, stream, out);
    if (s == ZQ_OK && consumed) *consumed = rec.consumed;
    return s;
}

zq_status zq_weight_info(const zq_weight* w, int* type, size_t* rows, size_t* cols, size_t* payload_bytes,
                         int* device) {
    if (!w) return fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: weights are empty");
    if (type) *type = w->type;
    if (rows) *rows = w->K;
    if (cols) *cols = w->N;
    if (payload_bytes) *payload_bytes = ref_payload_bytes(w->type, w->K, w->N);
    if (device) *device = w->device;
    return ZQ_OK;
}

zq_status zq_weight_download(const zq_weight* w, float* scales_host, void* payload_host, void* stream) {
    if (!w) return fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: weights are empty");
    cudaStream_t st = as_stream(stream);
    if (scales_host) ZQ_CUDA(cudaMemcpyAsync(scales_host, w->scales, w->N * sizeof(float), cudaMemcpyDeviceToHost, st));
    if (payload_host) {
        zq_status s = download_payload(w, payload_host, st);
        if (s != ZQ_OK) return s;
    }
    ZQ_CUDA(cudaStreamSynchronize(st));
    return ZQ_OK;
}

zq_status zq_weight_save_zyq(const zq_weight* w, void* buf, size_t cap, size_t* len, void* stream) {
    if (!w) return fail(ZQ_ERR_RUNTIME, "ZYRON quantization: cannot save empty matrix");
    const size_t pay = ref_payload_bytes(w->type, w->K, w->N);
    const size_t total = 4 * 3 + 8 * 3 + w->N * sizeof(float) + 8 + pay;
    if (len) *len = total;
    if (!buf) return ZQ_OK;
    if (cap < total) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: buffer too small");
    uint8_t* p = static_cast<uint8_t*>(buf);
    const uint32_t h32[3] = {kZyqMagic, kZyqVersion, (uint32_t)w->type};
    const uint64_t h64[3] = {(uint64_t)w->K, (uint64_t)w->N, (uint64_t)w->N};
    std::memcpy(p, h32, 12);
    std::memcpy(p + 12, h64, 24);
    float* scales = reinterpret_cast<float*>(p + 36);
    const uint64_t pay64 = pay;
    uint8_t* pay_at = p + 36 + w->N * sizeof(float);
    std::memcpy(pay_at, &pay64, 8);
    // scales may be unaligned inside the caller's buffer: go through a copy
    std::vector<float> sc(w->N);
    zq_status s = zq_weight_download(w, sc.data(), pay_at + 8, stream);
    if (s != ZQ_OK) return s;
    std::memcpy(scales, sc.data(), w->N * sizeof(float));
    return ZQ_OK;
}

zq_status zq_weight_slice_cols(const zq_weight* w, size_t col_begin, size_t col_end, void* stream, zq_weight** out) {
    if (!out) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null output handle");
    *out = nullptr;
    if (!w) return fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: weights are empty");
    if (col_begin >= col_end || col_end > w->N)
        return fail(ZQ_ERR_OUT_OF_RANGE, "zyron_b200: column slice out of range");
    zq_weight* r = nullptr;
    zq_status s = new_weight(w->type, w->K, col_end - col_begin, &r);
    if (s != ZQ_OK) return s;
    cudaStream_t st = as_stream(stream);
    const size_t cb = col_bytes(w);
    cudaError_t e = cudaMemcpyAsync(r->panel, w->panel + col_begin * cb, r->panel_bytes, cudaMemcpyDefault, st);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(r->scales, w->scales + col_begin, r->N * sizeof(float), cudaMemcpyDefault, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        zq_weight_destroy(r);
        return cuda_fail(e, "column slice");
    }
    *out = r;
    return ZQ_OK;
}

zq_status zq_weight_destroy(zq_weight* w) {
    if (!w) return ZQ_OK;
    int cur = 0;
    cudaGetDevice(&cur);
    if (cur != w->device) cudaSetDevice(w->device);
    cudaFree(w->panel);
    cudaFree(w->scales);
    if (cur != w->device) cudaSetDevice(cur);
    delete w;
    return ZQ_OK;
}

size_t zq_matmul_workspace_bytes(const zq_weight* w, size_t m) {
    if (!w || m == 0) return 0;
    size_t b = align256(m * (size_t)w->Kp) + align256(m * sizeof(float));
    // scratch: decode counters and partial sums (m <= 16); the GEMMs need
    // none (INT4 weights are unpacked in shared memory)
    size_t scratch = 0;
    if (m <= (size_t)zq::kSkinnyMaxRows) scratch = zq::skinny_scratch_bytes((int)w->N, (int)m);
    return b + scratch;
}

zq_status zq_quantize_rows(const float* x, size_t m, size_t k, int8_t* q, size_t ldq, float* row_scale,
                           void* stream) {
    if (m == 0) return ZQ_OK;
    if (k == 0) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: k must be > 0");
    if (ldq < k) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: ldq must be >= k");
    if (!x || !q || !row_scale) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null pointer");
    if (m > (size_t)std::numeric_limits<int>::max() || ldq > (size_t)std::numeric_limits<int>::max() - 64)
        return fail(ZQ_ERR_OVERFLOW, "zyron_b200: dimension exceeds 2^31-1");
    ZQ_CUDA(zq::launch_quantize_rows(x, (int)m, (int)k, (int)ldq, q, row_scale, as_stream(stream)));
    return ZQ_OK;
}

size_t zq_weight_padded_k(const zq_weight* w) { return w ? (size_t)w->Kp : 0; }

}  // extern "C"

namespace {

zq_status validate_matmul(const zq_weight* w, size_t m, const void* in, const float* y, const void* workspace,
                          size_t workspace_bytes) {
    if (!in || !y) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null input or output");
    if (m > (size_t)std::numeric_limits<int>::max())
        return fail(ZQ_ERR_OVERFLOW, "zyron_b200: row count exceeds 2^31-1");
    const size_t need = zq_matmul_workspace_bytes(w, m);
    if (!workspace || workspace_bytes < need) {
        char buf[128];
        std::snprintf(buf, sizeof buf, "zyron_b200: workspace too small (%zu < %zu bytes)", workspace_bytes, need);
        return fail(ZQ_ERR_INVALID_ARGUMENT, buf);
    }
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
        return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: workspace must be 256-byte aligned");
    int dev = 0;
    ZQ_CUDA(cudaGetDevice(&dev));
    if (dev != w->device) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: weight lives on another device");
    return ZQ_OK;
}

// Dot + epilogue on activation codes q [m][Kp] (row stride Kp) and row
// scales rs.  `scratch` is where INT4 weights are expanded for the GEMM.
zq::OutDesc single_output(float* y, size_t N) {
    zq::OutDesc o{};
    o.base[0] = y;
    o.count = 1;
    o.ldy = (long long)N;
    o.col_offset = 0;
    o.vec = ((N & 3) == 0) && ((reinterpret_cast<uintptr_t>(y) & 15u) == 0);
    return o;
}

// Dot + epilogue on activation codes q [m][Kp] (row stride Kp) and row
// scales rs; the GEMM path writes through `out` (several destinations when
// gathering), the GEMV path to out.base[0] with row stride N.
// Whether a plain-output matmul with M rows runs the dp4a GEMV (the weight's
// ZQ_OPT_DECODE_KERNEL option).  Default: the GEMV for 1-4 rows, where the
// weight stream alone sets the time and it has the least fixed cost per
// launch; the tensor cores above that, where dp4a and shared-memory reads of
// the activation rows limit the GEMV.
bool use_gemv(const zq_weight* w, int M) {
    const int decode = w->opt_decode.load(std::memory_order_relaxed);
    const bool fits = M <= zq::kGemvMaxRows && zq::gemv_smem_bytes(M, w->Kp) <= 200 * 1024;
    return fits && (decode == ZQ_DECODE_CUDA_CORE || (decode == ZQ_DECODE_AUTO && M <= 4));
}

// Failure-path testing of the decode kernel's bounded waits
// (zq_test_decode_wait_timeout); absent in every other call.
struct WaitTest {
    int wait_extra;
    uint64_t limit_ns;
};

zq_status run_codes_out(const zq_weight* w, const int8_t* codes, const float* rs, size_t m, const float* bias,
                        const zq::OutDesc& out, uint8_t* scratch, cudaStream_t st, bool pdl,
                        const WaitTest* test = nullptr);

zq_status run_codes(const zq_weight* w, const int8_t* codes, const float* rs, size_t m, const float* bias, float* y,
                    uint8_t* scratch, cudaStream_t st, bool pdl, const WaitTest* test = nullptr) {
    return run_codes_out(w, codes, rs, m, bias, single_output(y, w->N), scratch, st, pdl, test);
}

zq_status run_codes_out(const zq_weight* w, const int8_t* codes, const float* rs, size_t m, const float* bias,
                        const zq::OutDesc& out, uint8_t* scratch, cudaStream_t st, bool pdl, const WaitTest* test) {
    float* y = out.base[0];
    uint32_t* err = nullptr;
    zq_status s = device_error_ptr(&err);
    if (s != ZQ_OK) return s;
    const int M = (int)m, N = (int)w->N, Kp = w->Kp;
    const int reserved = w->opt_reserved_sms.load(std::memory_order_relaxed);
    const bool plain = out.count == 1 && out.ldy == (long long)N && out.col_offset == 0;
    if (plain && !test && use_gemv(w, M)) {
        zq::GemvArgs a{w->type, w->panel, N, Kp, w->scales, codes, rs, bias, y, M};
        a.reserved_sms = reserved;
        ZQ_CUDA(zq::launch_gemv(a, st, pdl));
        return ZQ_OK;
    }
    if (plain && M <= zq::kSkinnyMaxRows) {
        // Tensor-core decode kernel.  Its counters must be zero when it
        // starts: the quantizer of this call cleared them (pdl: it ran just
        // before), otherwise a zeroing kernel does.
        int* counters = reinterpret_cast<int*>(scratch);
        int* partials = reinterpret_cast<int*>(scratch + align256((size_t)zq::skinny_counter_words(N) * sizeof(int)));
        if (!pdl) ZQ_CUDA(zq::launch_zero_words(counters, zq::skinny_counter_words(N), st));
        CUtensorMap tmap_x;
        s = encode_decode_view(&tmap_x, codes, m, Kp, 128, 16);
        if (s != ZQ_OK) return s;
        const CUtensorMap* tmap_w = nullptr;
        {
            zq_weight* mw = const_cast<zq_weight*>(w);
            std::lock_guard<std::mutex> lk(mw->mu);
            if (!mw->tmap_dec_ready) {
                s = encode_decode_view(&mw->tmap_dec, w->panel, w->N, Kp, w->type == ZQ_TYPE_INT8 ? 128 : 64,
                                       zq::skinny_block_n());
                if (s != ZQ_OK) return s;
                mw->tmap_dec_ready = true;
            }
            tmap_w = &mw->tmap_dec;
        }
        zq::SkinnyArgs a{w->type, tmap_w, &tmap_x, M, N, Kp, rs, w->scales, bias, y, counters, partials, err};
        a.reserved_sms = reserved;
        if (test) {
            a.wait_extra = test->wait_extra;
            a.peer_limit_ns = test->limit_ns;
        }
        ZQ_CUDA(zq::launch_skinny(a, st, true));
        return ZQ_OK;
    }
    int bn = zq::gemm_block_n(M, N);
    if (w->type == ZQ_TYPE_INT4 && bn == 256) bn = 128;  // INT4 tiles: 128 columns or the 2-SM pair
    CUtensorMap tmap_a;
    s = encode_kmajor(&tmap_a, codes, m, Kp, 128);
    if (s != ZQ_OK) return s;
    const CUtensorMap* tmap_b = nullptr;
    {
        zq_weight* mw = const_cast<zq_weight*>(w);
        std::lock_guard<std::mutex> lk(mw->mu);
        const int ti = tile_index(bn);
        if (w->type == ZQ_TYPE_INT8) {
            if (!mw->tmap_ready[ti]) {
                s = encode_kmajor(&mw->tmap_b[ti], w->panel, w->N, Kp, box_rows_b(bn));
                if (s != ZQ_OK) return s;
                mw->tmap_ready[ti] = true;
            }
            tmap_b = &mw->tmap_b[ti];
        } else {
            // packed panel; the GEMM unpacks each box in shared memory
            if (!mw->tmap_p_ready[ti]) {
                s = encode_packed_int4(&mw->tmap_p[ti], w->panel, w->N, Kp, box_rows_b(bn));
                if (s != ZQ_OK) return s;
                mw->tmap_p_ready[ti] = true;
            }
            tmap_b = &mw->tmap_p[ti];
        }
    }
    (void)scratch;
    zq::GemmArgs g{&tmap_a, tmap_b, M, N, Kp, bn, rs, w->scales, bias, out, err,
                   w->opt_group_m.load(std::memory_order_relaxed)};
    g.reserved_sms = reserved;
    g.w4 = w->type == ZQ_TYPE_INT4;
    ZQ_CUDA(zq::launch_gemm(g, st, pdl));
    return ZQ_OK;
}

// Quantizer + dot/epilogue with all scratch in `ws` (already validated:
// 256-byte aligned, zq_matmul_workspace_bytes(w, m) bytes).
zq_status matmul_in_workspace_out(const zq_weight* w, const float* x, size_t m, const float* bias,
                                  const zq::OutDesc& out, uint8_t* ws, cudaStream_t st) {
    const bool plain = out.count == 1 && out.ldy == (long long)w->N && out.col_offset == 0;
    if (plain && m <= 4 && use_gemv(w, (int)m)) {
        // one launch: the GEMV quantizes the rows itself (same codes and
        // scales as the standalone quantizer)
        zq::GemvArgs a{w->type, w->panel, (int)w->N, w->Kp, w->scales, nullptr, nullptr, bias, out.base[0], (int)m};
        a.x = x;
        a.K = (int)w->K;
        a.reserved_sms = w->opt_reserved_sms.load(std::memory_order_relaxed);
        ZQ_CUDA(zq::launch_gemv(a, st, true));
        return ZQ_OK;
    }
    int8_t* codes = reinterpret_cast<int8_t*>(ws);
    float* rs = reinterpret_cast<float*>(ws + align256(m * (size_t)w->Kp));
    uint8_t* scratch = ws + align256(m * (size_t)w->Kp) + align256(m * sizeof(float));
    // m <= 16: the decode kernel's counters sit at the start of the scratch
    // and the quantizer clears them.
    int* counters = m <= (size_t)zq::kSkinnyMaxRows ? reinterpret_cast<int*>(scratch) : nullptr;
    const int n_counters = counters ? zq::skinny_counter_words((int)w->N) : 0;
    ZQ_CUDA(zq::launch_quantize_rows(x, (int)m, (int)w->K, w->Kp, codes, rs, st, counters, n_counters));
    return run_codes_out(w, codes, rs, m, bias, out, scratch, st, true);
}

zq_status matmul_in_workspace(const zq_weight* w, const float* x, size_t m, const float* bias, float* y,
                              uint8_t* ws, cudaStream_t st) {
    return matmul_in_workspace_out(w, x, m, bias, single_output(y, w->N), ws, st);
}

}  // namespace

namespace zq {

zq_status matmul_with_scratch(const zq_weight* w, const float* x, size_t m, const float* bias, float* y,
                              void* scratch, size_t scratch_bytes, void* stream) {
    if (!w) return fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: weights are empty");
    if (m == 0) return ZQ_OK;
    zq_status s = validate_matmul(w, m, x, y, scratch, scratch_bytes);
    if (s != ZQ_OK) return s;
    return matmul_in_workspace(w, x, m, bias, y, static_cast<uint8_t*>(scratch), as_stream(stream));
}

zq_status set_error(zq_status s, const char* msg) { return fail(s, msg); }

zq_status device_error_word(uint32_t** out) { return device_error_ptr(out); }

zq_status parse_zyq(const void* bytes, size_t len, ZyqRecord* rec) {
    const uint8_t* p = static_cast<const uint8_t*>(bytes);
    size_t off = 0;
    auto read = [&](void* dst, size_t n) -> bool {
        if (!p || off > len || len - off < n) return false;
        std::memcpy(dst, p + off, n);
        off += n;
        return true;
    };
    const char* corrupted = "ZYRON quantization: corrupted file";
    uint32_t magic = 0, version = 0, type = 0;
    uint64_t rows = 0, cols = 0, scale_count = 0, payload = 0;
    // quantization.cpp:270-272 (short-circuit: the version is read only when
    // the magic matches)
    if (!read(&magic, 4)) return fail(ZQ_ERR_RUNTIME, corrupted);
    if (magic != kZyqMagic) return fail(ZQ_ERR_RUNTIME, "ZYRON quantization: unsupported format");
    if (!read(&version, 4)) return fail(ZQ_ERR_RUNTIME, corrupted);
    if (version != kZyqVersion) return fail(ZQ_ERR_RUNTIME, "ZYRON quantization: unsupported format");
    // 275-279
    if (!read(&type, 4)) return fail(ZQ_ERR_RUNTIME, corrupted);
    if (type != ZQ_TYPE_INT8 && type != ZQ_TYPE_INT4) return fail(ZQ_ERR_RUNTIME, "ZYRON quantization: invalid type");
    // 280-289
    if (!read(&rows, 8) || !read(&cols, 8)) return fail(ZQ_ERR_RUNTIME, corrupted);
    if (rows == 0 || cols == 0) return fail(ZQ_ERR_RUNTIME, "ZYRON quantization: invalid matrix dimensions");
    if (mul_overflows((size_t)rows, (size_t)cols)) return fail(ZQ_ERR_OVERFLOW, "ZYRON quantization: matrix size overflow");
    // 291-297
    if (!read(&scale_count, 8)) return fail(ZQ_ERR_RUNTIME, corrupted);
    if (scale_count != cols) return fail(ZQ_ERR_RUNTIME, "ZYRON quantization: invalid scale count");
    if (mul_overflows((size_t)cols, sizeof(float)) || len - off < cols * sizeof(float))
        return fail(ZQ_ERR_RUNTIME, corrupted);
    rec->scales.resize((size_t)cols);
    read(rec->scales.data(), cols * sizeof(float));
    for (float sc : rec->scales)
        if (!(sc > 0.0f) || !std::isfinite(sc)) return fail(ZQ_ERR_RUNTIME, "ZYRON quantization: invalid scale");
    // 299-309
    if (!read(&payload, 8)) return fail(ZQ_ERR_RUNTIME, corrupted);
    const size_t expected = ref_payload_bytes((int)type, (size_t)rows, (size_t)cols);
    if (payload != expected) return fail(ZQ_ERR_RUNTIME, "ZYRON quantization: invalid payload size");
    if (len - off < expected) return fail(ZQ_ERR_RUNTIME, corrupted);
    rec->type = (int)type;
    rec->rows = (size_t)rows;
    rec->cols = (size_t)cols;
    rec->payload = p + off;
    rec->payload_bytes = expected;
    rec->consumed = off + expected;
    return ZQ_OK;
}

zq_status concat_cols(zq_weight* const* parts, int n, void* stream, zq_weight** out) {
    *out = nullptr;
    if (n < 1) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: nothing to concatenate");
    size_t N = 0;
    for (int i = 0; i < n; ++i) {
        if (!parts[i] || parts[i]->type != parts[0]->type || parts[i]->K != parts[0]->K)
            return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: column concatenation needs equal type and rows");
        N += parts[i]->N;
    }
    zq_weight* r = nullptr;
    zq_status s = new_weight(parts[0]->type, parts[0]->K, N, &r);
    if (s != ZQ_OK) return s;
    cudaStream_t st = as_stream(stream);
    size_t col = 0;
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < n && e == cudaSuccess; ++i) {
        e = cudaMemcpyAsync(r->panel + col * col_bytes(r), parts[i]->panel, parts[i]->panel_bytes, cudaMemcpyDefault, st);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(r->scales + col, parts[i]->scales, parts[i]->N * sizeof(float), cudaMemcpyDefault, st);
        col += parts[i]->N;
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        zq_weight_destroy(r);
        return cuda_fail(e, "column concatenation");
    }
    *out = r;
    return ZQ_OK;
}

zq_status cuda_error(cudaError_t e, const char* what) { return cuda_fail(e, what); }

}  // namespace zq

extern "C" {

zq_status zq_matmul(const zq_weight* w, const float* x, size_t m, const float* bias, float* y, void* workspace,
                    size_t workspace_bytes, void* stream) {
    return zq::matmul_with_scratch(w, x, m, bias, y, workspace, workspace_bytes, stream);
}

zq_status zq_matmul_multi(const zq_weight* w, const float* x, size_t m, const float* bias, float* const* dsts,
                          int n_dst, size_t ldy, size_t col_offset, void* workspace, size_t workspace_bytes,
                          void* stream) {
    if (!w) return fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: weights are empty");
    if (m == 0) return ZQ_OK;
    if (!dsts || n_dst < 1 || n_dst > zq::kMaxOutputs)
        return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: zq_matmul_multi needs 1 to 8 destinations");
    if (m <= (size_t)zq::kGemvMaxRows)
        return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: zq_matmul_multi needs m > 8 (tensor-core path)");
    if (ldy < w->N || col_offset > ldy - w->N)
        return fail(ZQ_ERR_OUT_OF_RANGE, "zyron_b200: output columns exceed the destination row stride");
    zq::OutDesc out{};
    out.count = n_dst;
    out.ldy = (long long)ldy;
    out.col_offset = (long long)col_offset;
    out.vec = (ldy % 4 == 0) && (col_offset % 4 == 0) && (w->N % 4 == 0);
    for (int i = 0; i < n_dst; ++i) {
        if (!dsts[i]) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null destination");
        out.base[i] = dsts[i];
        if (reinterpret_cast<uintptr_t>(dsts[i]) & 15u) out.vec = 0;
    }
    zq_status s = validate_matmul(w, m, x, out.base[0], workspace, workspace_bytes);
    if (s != ZQ_OK) return s;
    if (out.vec && n_dst > 1) {
        // every destination 16-byte aligned at the column offset, pitch a
        // multiple of 16 bytes: the epilogue can store with TMA
        s = get_encoder();
        if (s != ZQ_OK) return s;
        for (int i = 0; i < n_dst; ++i) {
            cuuint64_t dims[2] = {(cuuint64_t)w->N, (cuuint64_t)m};
            cuuint64_t strides[1] = {(cuuint64_t)(ldy * sizeof(float))};
            cuuint32_t box[2] = {32u, 32u};
            cuuint32_t estr[2] = {1u, 1u};
            CUresult r = g_encode(&out.map[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, dsts[i] + col_offset, dims, strides,
                                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            if (r != CUDA_SUCCESS) return fail(ZQ_ERR_CUDA, "zyron_b200: cuTensorMapEncodeTiled failed (output view)");
        }
        out.tma = 1;
    }
    return matmul_in_workspace_out(w, x, m, bias, out, static_cast<uint8_t*>(workspace), as_stream(stream));
}

zq_status zq_matmul_codes(const zq_weight* w, const int8_t* q, const float* row_scale, size_t m, const float* bias,
                          float* y, void* workspace, size_t workspace_bytes, void* stream) {
    if (!w) return fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: weights are empty");
    if (m == 0) return ZQ_OK;
    if (!row_scale) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null row scales");
    zq_status s = validate_matmul(w, m, q, y, workspace, workspace_bytes);
    if (s != ZQ_OK) return s;
    if ((reinterpret_cast<uintptr_t>(q) & 15u) != 0)
        return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: codes must be 16-byte aligned");
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    uint8_t* scratch = ws + align256(m * (size_t)w->Kp) + align256(m * sizeof(float));
    return run_codes(w, q, row_scale, m, bias, y, scratch, as_stream(stream), false);
}

zq_status zq_matmul_host(const zq_weight* w, const float* x_host, size_t m, const float* bias_host, float* y_host,
                         void* stream) {
    if (!w) return fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: weights are empty");
    if (m == 0) return ZQ_OK;
    if (!x_host || !y_host) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null input or output");
    if (mul_overflows(m, w->K) || mul_overflows(m, w->N))
        return fail(ZQ_ERR_OVERFLOW, "ZYRON quantization: matrix size overflow");
    HostStaging& h = t_staging;
    int dev = 0;
    ZQ_CUDA(cudaGetDevice(&dev));
    if (h.device != dev) {
        h.~HostStaging();
        new (&h) HostStaging();
        h.device = dev;
    }
    cudaStream_t st = as_stream(stream);
    const size_t xb = m * w->K * sizeof(float), yb = m * w->N * sizeof(float);
    // Large calls run in row chunks on three streams: copy-in of chunk i+1
    // and copy-out of chunk i-1 overlap the matmul of chunk i (host buffers
    // must be pinned for the copies to overlap).
    size_t chunks = xb / (32u << 20);
    if (chunks < 1) chunks = 1;
    if (chunks > (size_t)kHostChunks) chunks = kHostChunks;
    if (chunks > m) chunks = m;
    const size_t rows_per = (m + chunks - 1) / chunks;
    chunks = (m + rows_per - 1) / rows_per;
    const size_t wsb = zq_matmul_workspace_bytes(w, rows_per);
    ZQ_CUDA(ensure(h.x, h.x_cap, xb));
    ZQ_CUDA(ensure(h.y, h.y_cap, yb));
    ZQ_CUDA(ensure(h.ws, h.ws_cap, wsb));
    float* bdev = nullptr;
    if (bias_host) {
        ZQ_CUDA(ensure(h.b, h.b_cap, w->N * sizeof(float)));
        bdev = static_cast<float*>(h.b);
        ZQ_CUDA(cudaMemcpyAsync(bdev, bias_host, w->N * sizeof(float), cudaMemcpyHostToDevice, st));
    }
    if (chunks == 1) {
        ZQ_CUDA(cudaMemcpyAsync(h.x, x_host, xb, cudaMemcpyHostToDevice, st));
        zq_status s = zq_matmul(w, static_cast<const float*>(h.x), m, bdev, static_cast<float*>(h.y), h.ws, h.ws_cap,
                                stream);
        if (s != ZQ_OK) return s;
        ZQ_CUDA(cudaMemcpyAsync(y_host, h.y, yb, cudaMemcpyDeviceToHost, st));
    } else {
        ZQ_CUDA(h.init_streams());
        // copies must not start before earlier work on the caller's stream
        ZQ_CUDA(cudaEventRecord(h.out_done, st));
        ZQ_CUDA(cudaStreamWaitEvent(h.h2d, h.out_done, 0));
        ZQ_CUDA(cudaStreamWaitEvent(h.d2h, h.out_done, 0));
        const size_t K = w->K, N = w->N;
        for (size_t c = 0; c < chunks; ++c) {
            const size_t r0 = c * rows_per;
            const size_t rows = (m - r0) < rows_per ? (m - r0) : rows_per;
            const float* xh = x_host + r0 * K;
            float* xd = static_cast<float*>(h.x) + r0 * K;
            float* yd = static_cast<float*>(h.y) + r0 * N;
            ZQ_CUDA(cudaMemcpyAsync(xd, xh, rows * K * sizeof(float), cudaMemcpyHostToDevice, h.h2d));
            ZQ_CUDA(cudaEventRecord(h.in_done[c], h.h2d));
            ZQ_CUDA(cudaStreamWaitEvent(st, h.in_done[c], 0));
            zq_status s = zq_matmul(w, xd, rows, bdev, yd, h.ws, h.ws_cap, stream);
            if (s != ZQ_OK) return s;
            ZQ_CUDA(cudaEventRecord(h.mm_done[c], st));
            ZQ_CUDA(cudaStreamWaitEvent(h.d2h, h.mm_done[c], 0));
            ZQ_CUDA(cudaMemcpyAsync(y_host + r0 * N, yd, rows * N * sizeof(float), cudaMemcpyDeviceToHost, h.d2h));
        }
        ZQ_CUDA(cudaEventRecord(h.out_done, h.d2h));
        ZQ_CUDA(cudaStreamWaitEvent(st, h.out_done, 0));
    }
    uint32_t code = 0;
    return zq_device_error(stream, &code);
}

zq_status zq_dequantize(const zq_weight* w, float* out, void* stream) {
    if (!w) return fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: weights are empty");
    if (!out) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null output");
    ZQ_CUDA(zq::launch_dequantize(w->panel, w->type, (int)w->K, (int)w->N, w->Kp, w->scales, out, as_stream(stream)));
    return ZQ_OK;
}

zq_status zq_dequantize_host(const zq_weight* w, float* out_host, void* stream) {
    if (!w) return fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: weights are empty");
    if (!out_host) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null output");
    cudaStream_t st = as_stream(stream);
    const size_t bytes = w->K * w->N * sizeof(float);
    float* tmp = nullptr;
    ZQ_CUDA(cudaMalloc(&tmp, bytes));
    cudaError_t e = zq::launch_dequantize(w->panel, w->type, (int)w->K, (int)w->N, w->Kp, w->scales, tmp, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out_host, tmp, bytes, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    cudaFree(tmp);
    if (e != cudaSuccess) return cuda_fail(e, "dequantize to host");
    return ZQ_OK;
}

zq_status zq_weight_set_option(zq_weight* w, int option, int value, int* previous) {
    if (!w) return fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: weights are empty");
    std::atomic<int>* slot = nullptr;
    switch (option) {
        case ZQ_OPT_DECODE_KERNEL:
            if (value < ZQ_DECODE_AUTO || value > ZQ_DECODE_CUDA_CORE)
                return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: unknown decode kernel");
            slot = &w->opt_decode;
            break;
        case ZQ_OPT_RESERVED_SMS:
            if (value < 0) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: reserved SM count must be >= 0");
            slot = &w->opt_reserved_sms;
            break;
        case ZQ_OPT_GEMM_GROUP_M:
            if (value < 0) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: GEMM group size must be >= 0");
            slot = &w->opt_group_m;
            break;
        default:
            return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: unknown weight option");
    }
    const int old = slot->exchange(value);
    if (previous) *previous = old;
    return ZQ_OK;
}

zq_status zq_test_decode_wait_timeout(const zq_weight* w, const int8_t* q, const float* row_scale, size_t m,
                                      float* y, void* workspace, size_t workspace_bytes, uint64_t limit_ns,
                                      void* stream) {
    if (!w) return fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: weights are empty");
    if (m == 0 || m > (size_t)zq::kSkinnyMaxRows)
        return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: the decode kernel takes 1 to 16 rows");
    if (!row_scale) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null row scales");
    if (limit_ns < 100000ull || limit_ns > 1000000000ull)
        return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: limit_ns must be within [1e5, 1e9]");
    zq_status s = validate_matmul(w, m, q, y, workspace, workspace_bytes);
    if (s != ZQ_OK) return s;
    if ((reinterpret_cast<uintptr_t>(q) & 15u) != 0)
        return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: codes must be 16-byte aligned");
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    uint8_t* scratch = ws + align256(m * (size_t)w->Kp) + align256(m * sizeof(float));
    const WaitTest t{1, limit_ns};
    return run_codes(w, q, row_scale, m, nullptr, y, scratch, as_stream(stream), false, &t);
}

zq_status zq_ipc_export(const void* dev_ptr, zq_ipc_handle* out) {
    if (!dev_ptr || !out) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null argument");
    static_assert(sizeof(cudaIpcMemHandle_t) <= sizeof(out->handle), "IPC handle size");
    PFN_cuMemGetAddressRange_v3020 range = nullptr;
    {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &fn, 3020, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
    }
    if (!range) return fail(ZQ_ERR_CUDA, "zyron_b200: cuMemGetAddressRange is unavailable");
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
        return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: pointer is not a device allocation");
    cudaIpcMemHandle_t h;
    ZQ_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
    std::memset(out, 0, sizeof *out);
    std::memcpy(out->handle, &h, sizeof h);
    out->offset = (uint64_t)(reinterpret_cast<uintptr_t>(dev_ptr) - (uintptr_t)base);
    cudaPointerAttributes attr;
    ZQ_CUDA(cudaPointerGetAttributes(&attr, dev_ptr));
    out->device = attr.device;
    return ZQ_OK;
}

zq_status zq_ipc_import(const zq_ipc_handle* h, void** dev_ptr) {
    if (!h || !dev_ptr) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null argument");
    cudaIpcMemHandle_t ih;
    std::memcpy(&ih, h->handle, sizeof ih);
    void* base = nullptr;
    // opened while the accessing device is current: the lazy flag enables
    // that device's peer access to the exporting device
    ZQ_CUDA(cudaIpcOpenMemHandle(&base, ih, cudaIpcMemLazyEnablePeerAccess));
    *dev_ptr = static_cast<uint8_t*>(base) + h->offset;
    std::lock_guard<std::mutex> lk(g_err_mu);
    g_ipc_bases.emplace_back(*dev_ptr, base);
    return ZQ_OK;
}

zq_status zq_ipc_close(void* dev_ptr) {
    void* base = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_err_mu);
        for (auto it = g_ipc_bases.begin(); it != g_ipc_bases.end(); ++it)
            if (it->first == dev_ptr) {
                base = it->second;
                g_ipc_bases.erase(it);
                break;
            }
    }
    if (!base) return fail(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: pointer was not imported");
    ZQ_CUDA(cudaIpcCloseMemHandle(base));
    return ZQ_OK;
}

zq_status zq_device_error(void* stream, uint32_t* code) {
    ZQ_CUDA(cudaStreamSynchronize(as_stream(stream)));
    uint32_t* p = nullptr;
    zq_status s = device_error_ptr(&p);
    if (s != ZQ_OK) return s;
    uint32_t v = 0;
    ZQ_CUDA(cudaMemcpy(&v, p, sizeof v, cudaMemcpyDeviceToHost));
    if (code) *code = v;
    if (v != 0) {
        const uint32_t zero = 0;
        ZQ_CUDA(cudaMemcpy(p, &zero, sizeof zero, cudaMemcpyHostToDevice));
        char buf[96];
        std::snprintf(buf, sizeof buf, "zyron_b200: device wait timed out (code %u)", v);
        return fail(ZQ_ERR_DEVICE_TIMEOUT, buf);
    }
    return ZQ_OK;
}

}  // extern "C"
