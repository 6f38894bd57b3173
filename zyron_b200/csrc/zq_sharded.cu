// zq_sharded.cu -- the column-sharded matmul joined by one NCCL all-gather,
// as a C entry point taking an NCCL communicator, plus the communicator
// helpers a C or C++ host needs to make one.
//
// A weight's columns are quantized independently (one scale per column,
// src/quantization/quantization.cpp:141-159) and stored contiguously
// (quantization.cpp:155), so rank r of W ranks owns the contiguous columns
// [begin_r, end_r) of the full N-column weight (zq_shard_range: the first
// N % W ranks one column wider).  Every rank quantizes the same activations,
// so codes and row scales agree bit for bit without an exchange (the row
// quantizer, quantization.cpp:202-212, reads x only).  Each rank computes its
// block with the ordinary matmul into a send buffer padded to the widest
// shard, one ncclAllGather concatenates the blocks, and join_columns_kernel
// writes them into the row-major [M, N] output.  The result is bit-identical
// to the single-GPU matmul.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2).  A process that has
// already loaded NCCL (PyTorch does at import) shares that library, so
// communicators it created work here; a process that never calls these entry
// points needs no NCCL.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "zq.h"
#include "zq_internal.h"
#include "zq_kernels.h"

namespace {

struct NcclApi {
    bool ok = false;
    char why[256] = {0};
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_count)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*comm_user_rank)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

template <typename F>
bool resolve(void* h, const char* name, F& fn, NcclApi& api) {
    fn = reinterpret_cast<F>(dlsym(h, name));
    if (!fn) std::snprintf(api.why, sizeof api.why, "zyron_b200: libnccl.so.2 has no %s", name);
    return fn != nullptr;
}

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) {
            std::snprintf(api.why, sizeof api.why, "zyron_b200: cannot load libnccl.so.2 (%s)", dlerror());
            return;
        }
        api.ok = resolve(h, "ncclGetUniqueId", api.get_unique_id, api) &&
                 resolve(h, "ncclCommInitRank", api.comm_init_rank, api) &&
                 resolve(h, "ncclCommDestroy", api.comm_destroy, api) &&
                 resolve(h, "ncclCommCount", api.comm_count, api) &&
                 resolve(h, "ncclCommUserRank", api.comm_user_rank, api) &&
                 resolve(h, "ncclAllGather", api.all_gather, api) &&
                 resolve(h, "ncclGetErrorString", api.error_string, api);
    });
    return api;
}

zq_status nccl_fail(ncclResult_t r, const char* what) {
    char buf[256];
    std::snprintf(buf, sizeof buf, "zyron_b200: %s failed: %s", what, nccl().error_string(r));
    return zq::set_error(ZQ_ERR_RUNTIME, buf);
}

#define ZQ_NCCL_API_OR_FAIL()                                             \
    do {                                                                  \
        if (!nccl().ok) return zq::set_error(ZQ_ERR_RUNTIME, nccl().why); \
    } while (0)

inline size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

// Column split shared by the host and join_columns_kernel: base columns per
// rank, and the first `extra` ranks one more.
__host__ __device__ inline void shard_of(long long n, int world, int rank, long long& begin, long long& width) {
    const long long base = n / world, extra = n % world;
    width = base + (rank < extra ? 1 : 0);
    begin = rank < extra ? rank * (base + 1) : extra * (base + 1) + (rank - extra) * base;
}

// y[row][c] = block of the rank owning column c, row `row`.  recv holds
// `world` blocks of m x wmax floats; block r is [m][width_r] row-major at
// its start.  Threads own columns (the owning rank is found once per
// thread) and stride over rows, so loads and stores stay coalesced within a
// rank's columns.
__global__ void join_columns_kernel(const float* __restrict__ recv, float* __restrict__ y, int m, int n, int world,
                                    long long wmax) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= n) return;
    const long long base = n / world, extra = n % world;
    const long long wide = extra * (base + 1);
    const int r = c < wide ? (int)(c / (base + 1)) : (int)(extra + (c - wide) / base);
    long long begin, width;
    shard_of(n, world, r, begin, width);
    const float* blk = recv + (long long)r * m * wmax + (c - begin);
    for (int row = blockIdx.y; row < m; row += gridDim.y)
        y[(long long)row * n + c] = __ldg(blk + (long long)row * width);
}

}  // namespace

extern "C" {

zq_status zq_shard_range(size_t n_cols, int world, int rank, size_t* begin, size_t* end) {
    if (!begin || !end) return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null output");
    if (world < 1 || rank < 0 || rank >= world)
        return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: rank outside [0, world)");
    if (n_cols < (size_t)world) return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: fewer columns than ranks");
    long long b, w;
    shard_of((long long)n_cols, world, rank, b, w);
    *begin = (size_t)b;
    *end = (size_t)(b + w);
    return ZQ_OK;
}

zq_status zq_nccl_get_unique_id(void* id_out) {
    ZQ_NCCL_API_OR_FAIL();
    if (!id_out) return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null id buffer");
    static_assert(sizeof(ncclUniqueId) == ZQ_NCCL_UNIQUE_ID_BYTES, "NCCL unique id size");
    ncclUniqueId id;
    const ncclResult_t r = nccl().get_unique_id(&id);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    std::memcpy(id_out, &id, sizeof id);
    return ZQ_OK;
}

zq_status zq_nccl_comm_init(int nranks, const void* id, int rank, void** comm) {
    ZQ_NCCL_API_OR_FAIL();
    if (!id || !comm) return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null id or communicator");
    if (nranks < 1 || rank < 0 || rank >= nranks)
        return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: rank outside [0, nranks)");
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof uid);
    ncclComm_t c = nullptr;
    const ncclResult_t r = nccl().comm_init_rank(&c, nranks, uid, rank);
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
    *comm = c;
    return ZQ_OK;
}

zq_status zq_nccl_comm_destroy(void* comm) {
    if (!comm) return ZQ_OK;
    ZQ_NCCL_API_OR_FAIL();
    const ncclResult_t r = nccl().comm_destroy(static_cast<ncclComm_t>(comm));
    return r == ncclSuccess ? ZQ_OK : nccl_fail(r, "ncclCommDestroy");
}

size_t zq_matmul_sharded_workspace_bytes(const zq_weight* shard, size_t m, size_t n_cols, int world) {
    if (!shard || m == 0 || world < 1 || n_cols < (size_t)world) return 0;
    const size_t wmax = (n_cols + world - 1) / world;
    return align256(zq_matmul_workspace_bytes(shard, m)) + align256(m * wmax * sizeof(float)) +
           align256((size_t)world * m * wmax * sizeof(float));
}

zq_status zq_matmul_sharded(const zq_weight* shard, const float* x, size_t m, const float* bias_shard, float* y,
                            size_t n_cols, void* nccl_comm, void* workspace, size_t workspace_bytes, void* stream) {
    if (!shard) return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: weights are empty");
    if (m == 0) return ZQ_OK;
    if (!nccl_comm) return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null NCCL communicator");
    if (!x || !y) return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null input or output");
    ZQ_NCCL_API_OR_FAIL();
    ncclComm_t comm = static_cast<ncclComm_t>(nccl_comm);
    int world = 0, rank = 0;
    ncclResult_t r = nccl().comm_count(comm, &world);
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommCount");
    r = nccl().comm_user_rank(comm, &rank);
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommUserRank");
    if (n_cols < (size_t)world || n_cols > (size_t)0x7fffffff || m > (size_t)0x7fffffff)
        return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: column count must lie in [world, 2^31)");
    int type = 0;
    size_t rows = 0, cols = 0;
    zq_status s = zq_weight_info(shard, &type, &rows, &cols, nullptr, nullptr);
    if (s != ZQ_OK) return s;
    size_t begin = 0, end = 0;
    s = zq_shard_range(n_cols, world, rank, &begin, &end);
    if (s != ZQ_OK) return s;
    if (cols != end - begin) {
        char buf[200];
        std::snprintf(buf, sizeof buf, "zyron_b200: rank %d holds %zu columns, its shard of %zu is [%zu, %zu)", rank,
                      cols, n_cols, begin, end);
        return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, buf);
    }
    const size_t need = zq_matmul_sharded_workspace_bytes(shard, m, n_cols, world);
    if (!workspace || workspace_bytes < need) {
        char buf[160];
        std::snprintf(buf, sizeof buf, "zyron_b200: workspace too small (%zu < %zu bytes)", workspace_bytes, need);
        return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, buf);
    }
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
        return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: workspace must be 256-byte aligned");
    const size_t wmax = (n_cols + world - 1) / world;
    const size_t mm_bytes = align256(zq_matmul_workspace_bytes(shard, m));
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    float* send = reinterpret_cast<float*>(ws + mm_bytes);
    float* recv = reinterpret_cast<float*>(ws + mm_bytes + align256(m * wmax * sizeof(float)));
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    // this rank's block, [m][cols] row-major at the start of the send buffer
    s = zq_matmul(shard, x, m, bias_shard, send, ws, mm_bytes, stream);
    if (s != ZQ_OK) return s;
    r = nccl().all_gather(send, recv, m * wmax, ncclFloat32, comm, st);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather");
    const dim3 block(256);
    const dim3 grid((unsigned)((n_cols + 255) / 256), (unsigned)(m < 64 ? m : 64));
    join_columns_kernel<<<grid, block, 0, st>>>(recv, y, (int)m, (int)n_cols, world, (long long)wmax);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return zq::cuda_error(e, "join_columns_kernel");
    return ZQ_OK;
}

}  // extern "C"
