// zq_kernels.h -- internal launcher interface between the C ABI (zq_api.cu)
// and the kernels.  Not installed; the public interface is include/zq.h.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "zq.h"

namespace zq {

constexpr int kGemvMaxRows = 8;
// GemmArgs::block_n value selecting the 2-SM (cluster pair) 256 x 256 tile kernel.
constexpr int kPairBlockN = 512;

// Codes per column on the device, rounded up so every column starts on a
// 16-byte boundary (INT8: 16 codes, INT4: 32 codes).
inline int padded_k(int type, int K) { return type == 1 ? (K + 15) / 16 * 16 : (K + 31) / 32 * 32; }

struct GemvArgs {
    int type;
    const uint8_t* panel;
    int N;
    int Kp;
    const float* col_scale;
    const int8_t* q;
    const float* row_scale;
    const float* bias;
    float* y;
    int M;
};

// Where the GEMM epilogue writes: element (row, col) of the matmul goes to
// base[d][row * ldy + col_offset + col] for every d < count.  count > 1 means
// the other bases are peer GPUs' buffers mapped into this process.
constexpr int kMaxOutputs = 8;
struct OutDesc {
    float* base[kMaxOutputs];
    int count;
    int vec;  // ldy, col_offset and every base allow 16-byte stores
    long long ldy;
    long long col_offset;
};

struct GemmArgs {
    const CUtensorMap* tmap_a;
    const CUtensorMap* tmap_b;
    int M, N, Kp;
    int block_n;
    const float* row_scale;
    const float* col_scale;
    const float* bias;
    OutDesc out;
    uint32_t* err;
    int group_m;  // tile-order group size in M-tiles (0 = all M-tiles)
};

cudaError_t launch_quantize_rows(const float* x, int M, int K, int Kp, int8_t* q, float* row_scale,
                                 cudaStream_t stream);
cudaError_t launch_repack_int4(const uint8_t* src, int K, int N, int Kp, uint8_t* dst, cudaStream_t stream);
cudaError_t launch_unpack_panel_int4(const uint8_t* panel, int K, int N, int Kp, uint8_t* dst,
                                     cudaStream_t stream);
cudaError_t launch_quantize_weights(const float* w, int K, int N, int Kp, int type, uint32_t* absmax_tmp,
                                    float* scales, uint8_t* panel, cudaStream_t stream);
cudaError_t launch_dequantize(const uint8_t* panel, int type, int K, int N, int Kp, const float* scales,
                              float* out, cudaStream_t stream);
cudaError_t launch_expand_int4(const uint8_t* panel4, int N, int Kp, int8_t* panel8, cudaStream_t stream);

size_t gemv_smem_bytes(int M, int Kp);
cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t stream, bool pdl);

int gemm_block_n(int M, int N);

// Multiprocessors of the current device available to the persistent kernels
// (device count cached per device, minus the reserved count).
int sm_count();
int set_reserved_sms(int sms);

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) at most once per kernel
// (keyed by the kernel's address) and size: host-side launch overhead matters
// for microsecond kernels.
cudaError_t ensure_smem_attr_ptr(const void* kern, size_t bytes);
template <class K>
cudaError_t ensure_smem_attr(K kern, size_t bytes) {
    return ensure_smem_attr_ptr(reinterpret_cast<const void*>(kern), bytes);
}

// zq_matmul with caller-supplied scratch (validated here: 256-byte aligned and
// at least zq_matmul_workspace_bytes(w, m) bytes).  Defined in zq_api.cu.
zq_status matmul_with_scratch(const zq_weight* w, const float* x, size_t m, const float* bias, float* y,
                              void* scratch, size_t scratch_bytes, void* stream);
// Records `msg` as the calling thread's last error and returns `s`.
zq_status set_error(zq_status s, const char* msg);
cudaError_t launch_gemm(const GemmArgs& a, cudaStream_t stream, bool pdl);

}  // namespace zq
