// zq_kernels.h -- internal launcher interface between the C ABI (zq_api.cu)
// and the kernels.  Not installed; the public interface is include/zq.h.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "zq.h"

namespace zq {

// Launches `kern` with programmatic dependent launch: it may start while the
// kernel before it on the stream is still running, once that kernel has
// executed griddepcontrol.launch_dependents (or at its end if it never does).
// Every kernel launched this way reads only immutable data (weight panels,
// scales) before its griddepcontrol.wait, and reads or writes everything else
// after it; the wait returns when the kernels before it have completed and
// their memory is visible.
template <class... Params, class... Args>
cudaError_t launch_pdl_kernel(void (*kern)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<Params>(args)...);
}

constexpr int kGemvMaxRows = 8;
// GemmArgs::block_n value selecting the 2-SM (cluster pair) 256 x 256 tile kernel.
constexpr int kPairBlockN = 512;

// Codes per column on the device, rounded up to whole 128-code k-blocks (the
// padding codes are zero): every column starts on a 16-byte boundary, and the
// decode kernel's 3-D TMA boxes, several k-blocks deep, never cross from one
// column into the next.
inline int padded_k(int type, int K) {
    (void)type;
    return (K + 127) / 128 * 128;
}

struct GemvArgs {
    int type;
    const uint8_t* panel;
    int N;
    int Kp;
    const float* col_scale;
    const int8_t* q;          // activation codes [M][Kp] and
    const float* row_scale;   // row scales [M], or null when x is given
    const float* bias;
    float* y;
    int M;
    const float* x = nullptr; // fp32 activations [M][K], quantized inside the kernel (M <= 4)
    int K = 0;
    int reserved_sms = 0;     // SMs left out of the grid
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
    // Several destinations with vec: 2-D fp32 views [M][N] of each
    // destination from its column offset (row pitch ldy), 32 x 32 boxes with
    // the 128-byte swizzle; the gathering epilogue stores whole 32 x 32
    // blocks with TMA through them.
    int tma;
    CUtensorMap map[kMaxOutputs];
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
    int reserved_sms = 0;  // SMs left out of the persistent grid
    // INT4 weights: tmap_b covers the packed panel [N][Kp/2] (box 64 bytes x
    // BN or 128 rows, unswizzled) and the kernel unpacks in shared memory.
    bool w4 = false;
};

// `zero` (n_zero ints, may be NULL) is cleared by the same launch: the
// decode kernel's counters, so that zeroing them costs no launch of its own.
cudaError_t launch_quantize_rows(const float* x, int M, int K, int Kp, int8_t* q, float* row_scale,
                                 cudaStream_t stream, int* zero = nullptr, int n_zero = 0);
cudaError_t launch_repack_int4(const uint8_t* src, int K, int N, int Kp, uint8_t* dst, cudaStream_t stream);
cudaError_t launch_unpack_panel_int4(const uint8_t* panel, int K, int N, int Kp, uint8_t* dst,
                                     cudaStream_t stream);
cudaError_t launch_quantize_weights(const float* w, int K, int N, int Kp, int type, uint32_t* absmax_tmp,
                                    float* scales, uint8_t* panel, cudaStream_t stream);
cudaError_t launch_dequantize(const uint8_t* panel, int type, int K, int N, int Kp, const float* scales,
                              float* out, cudaStream_t stream);

size_t gemv_smem_bytes(int M, int Kp);
cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t stream, bool pdl);

// Decode-sized matmul on tensor cores (zq_skinny_sm100.cu), M <= 16.
constexpr int kSkinnyMaxRows = 16;
constexpr int kSkinnyMaxCtas = 256;
struct SkinnyArgs {
    int type;
    const CUtensorMap* tmap_w;  // 3-D panel view (k-block row bytes, N, Kp/128), box x 64 columns x skinny_kgroup()
    const CUtensorMap* tmap_x;  // 3-D view of the codes [M][Kp], box 128 B x 16 rows x skinny_kgroup(), swizzled
    int M, N, Kp;
    const float* row_scale;
    const float* col_scale;
    const float* bias;
    float* y;
    int* counters;  // skinny_counter_words(N), zero when the kernel starts
    int* partials;  // kSkinnyMaxCtas * 2 * M * skinny_block_n()
    uint32_t* err;
    // Failure-path testing only (0 otherwise): a split block's finisher waits
    // for wait_extra more partial sums than exist, giving up after
    // peer_limit_ns (0: the default 4 s).
    int wait_extra = 0;
    uint64_t peer_limit_ns = 0;
    int reserved_sms = 0;  // SMs left out of the grid
};
// Weight columns per decode tile and the tiles of N columns.
int skinny_block_n();
// k-blocks per decode iteration (the depth of its 3-D TMA boxes).
int skinny_kgroup();
int skinny_blocks(int N);
// Arrival and publication counters of the split blocks (8 per block).
int skinny_counter_words(int N);
// Scratch of one decode launch: counters, then partial sums (256-byte aligned).
size_t skinny_scratch_bytes(int N, int M);
cudaError_t launch_zero_words(int* p, int n, cudaStream_t stream);
cudaError_t launch_skinny(const SkinnyArgs& a, cudaStream_t stream, bool pdl);

int gemm_block_n(int M, int N);

// Multiprocessors of the current device available to the persistent kernels
// (device count cached per device, minus `reserved`, at least 2).
int sm_count(int reserved = 0);

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
