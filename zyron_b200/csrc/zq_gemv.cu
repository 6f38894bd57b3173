// zq_gemv.cu -- decode-sized quantized matmul (M = 1..8 activation rows).
//
// Computes, for every output column n and activation row m,
//   acc[m][n] = sum_k q_a[m][k] * q_w[n][k]         (exact int32)
//   y[m][n]   = float(acc) * s_row[m] * s_col[n] (+ bias[n])
// which is quantization::matmul's dot and epilogue (src/quantization/
// quantization.cpp:215-232) plus QuantizedLinear's bias pass
// (src/quantization/quantized_linear.cpp:44-48).
//
// HBM-bound design: every weight byte is read exactly once with 128-bit
// L1-bypassing loads.  One warp owns one column at a time (columns are
// contiguous in the panel layout), the activation codes of all M rows sit in
// shared memory, dp4a does four int8 MACs per instruction and a warp-shuffle
// tree reduces the 32 lane partials.  The kernel is launched with
// programmatic dependent launch behind the activation quantizer: it starts
// prefetching weights into L2 while the quantizer finishes, then waits on
// griddepcontrol before touching the codes.
#include "zq_common.cuh"
#include "zq_dot.cuh"
#include "zq_kernels.h"

namespace zq {

namespace {

constexpr int kGemvThreads = 256;

// One group of kCols columns for one warp: dp4a over all chunks (kUnroll
// 16-byte loads per lane per column in flight), warp-shuffle reduction, exact
// epilogue.
// kUnroll: 16-byte weight chunks in flight per lane per column.
template <int kType, int kM, int kCols, int kUnroll>
__device__ __forceinline__ void gemv_group(int g, const uint8_t* __restrict__ panel,
                                           int N, int Kp, size_t col_bytes, int chunks, const int8_t* __restrict__ sq,
                                           const float* __restrict__ col_scale, const float (&srow)[kM],
                                           const float* __restrict__ bias, float* __restrict__ y, int M, int lane) {
    const int col0 = g * kCols;
    int acc[kCols][kM];
#pragma unroll
    for (int c = 0; c < kCols; ++c)
#pragma unroll
        for (int m = 0; m < kM; ++m) acc[c][m] = 0;

    for (int base = lane; base < chunks; base += 32 * kUnroll) {
        uint4 w[kCols][kUnroll];
#pragma unroll
        for (int c = 0; c < kCols; ++c) {
            const uint8_t* wc = panel + (size_t)min(col0 + c, N - 1) * col_bytes;
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int ch = base + 32 * u;
                w[c][u] = ch < chunks ? ld_stream_u4(wc + (size_t)ch * 16) : make_uint4(0, 0, 0, 0);
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int ch = base + 32 * u;
            if (ch < chunks) {
#pragma unroll
                for (int c = 0; c < kCols; ++c) {
                    if (kType == kInt8)
                        dot16_int8<kM>(w[c][u], sq, Kp, ch * 16, acc[c]);
                    else
                        dot16_int4<kM>(w[c][u], sq, Kp, ch * 32, acc[c]);
                }
            }
        }
    }

#pragma unroll
    for (int c = 0; c < kCols; ++c) {
#pragma unroll
        for (int m = 0; m < kM; ++m) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[c][m] += __shfl_xor_sync(0xffffffffu, acc[c][m], o);
        }
        const int col = col0 + c;
        if (col < N) {
            const float sc = __ldg(col_scale + col);
            const float b = bias ? __ldg(bias + col) : 0.0f;
#pragma unroll
            for (int m = 0; m < kM; ++m) {
                if (lane == m && m < M) {
                    y[(size_t)m * N + col] = bias ? zq_epilogue_bias(acc[c][m], srow[m], sc, b)
                                                  : zq_epilogue(acc[c][m], srow[m], sc);
                }
            }
        }
    }
}

// kCols columns per warp iteration: each shared-memory activation read feeds
// kCols columns' dp4a (M >= 4 is dp4a/LDS-heavy; M <= 2 is purely HBM-bound).
template <int kType, int kM, int kCols, int kUnroll>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const uint8_t* __restrict__ panel, int N, int Kp,
                                                            const float* __restrict__ col_scale,
                                                            const int8_t* __restrict__ q,
                                                            const float* __restrict__ row_scale,
                                                            const float* __restrict__ bias, float* __restrict__ y,
                                                            int M) {
    extern __shared__ __align__(16) int8_t sq[];  // [kM][Kp]
    const int lane = threadIdx.x & 31;
    const int warp_global = (blockIdx.x * kGemvThreads + threadIdx.x) >> 5;
    const int warps_total = (gridDim.x * kGemvThreads) >> 5;
    const size_t col_bytes = kType == kInt8 ? (size_t)Kp : (size_t)(Kp >> 1);
    const int groups = (N + kCols - 1) / kCols;

    const int chunks = (int)(col_bytes >> 4);  // 16-byte chunks per column
    // Warm L2 with this warp's first columns while the quantizer finishes.
    if (warp_global < groups) {
        for (int c = 0; c < kCols; ++c) {
            const int col = warp_global * kCols + c;
            if (col >= N) break;
            const uint8_t* c0 = panel + (size_t)col * col_bytes;
            for (size_t off = (size_t)lane * 128; off < col_bytes; off += 32 * 128)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(c0 + off));
        }
    }
    pdl_wait_primary();

    // Stage the activation codes (rows >= M are zero).
    {
        const uint32_t* q4 = reinterpret_cast<const uint32_t*>(q);
        uint32_t* s4 = reinterpret_cast<uint32_t*>(sq);
        const int words = Kp >> 2;
        for (int i = threadIdx.x; i < kM * words; i += kGemvThreads) {
            const int m = i / words;
            const int wi = i - m * words;
            if (kType == kInt8) {
                s4[i] = m < M ? q4[(size_t)m * words + wi] : 0u;
            } else {
                // two source words (8 codes) -> even/odd split
                if ((wi & 1) == 0) {
                    uint32_t a = 0, b = 0;
                    if (m < M) {
                        a = q4[(size_t)m * words + wi];
                        b = q4[(size_t)m * words + wi + 1];
                    }
                    s4[i] = __byte_perm(a, b, 0x6420);
                    s4[i + 1] = __byte_perm(a, b, 0x7531);
                }
            }
        }
    }
    __syncthreads();

    float srow[kM];
#pragma unroll
    for (int m = 0; m < kM; ++m) srow[m] = m < M ? row_scale[m] : 0.0f;

    for (int g = warp_global; g < groups; g += warps_total)
        gemv_group<kType, kM, kCols, kUnroll>(g, panel, N, Kp, col_bytes, chunks, sq, col_scale, srow, bias, y, M, lane);
}

// Four chunks per lane: with at most 64 resident warps per SM, eight per
// lane (one round for a 4096-code column) measured slower (fewer warps).
template <int kType, int kM, int kCols, int kUnroll = 4>
cudaError_t launch_gemv_t(const GemvArgs& a, cudaStream_t stream, bool pdl) {
    const size_t smem = (size_t)kM * a.Kp;
    auto kern = gemv_kernel<kType, kM, kCols, kUnroll>;
    cudaError_t e = ensure_smem_attr(kern, smem);
    if (e != cudaSuccess) return e;
    const int sms = sm_count();
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kGemvThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    // As many resident warps as occupancy allows: under load the HBM needs
    // many loads in flight per SM, and warps are what carry them.
    const int groups = (a.N + kCols - 1) / kCols;
    const int needed = (groups + kGemvThreads / 32 - 1) / (kGemvThreads / 32);
    const int blocks = sms * per_sm < needed ? sms * per_sm : needed;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a.panel, a.N, a.Kp, a.col_scale, a.q, a.row_scale, a.bias, a.y,
                              a.M);
}

template <int kType>
cudaError_t dispatch_m(const GemvArgs& a, cudaStream_t stream, bool pdl) {
    switch (a.M) {
        case 1: return launch_gemv_t<kType, 1, 1>(a, stream, pdl);
        case 2: return launch_gemv_t<kType, 2, 1>(a, stream, pdl);
        case 3:
        case 4: return launch_gemv_t<kType, 4, 2>(a, stream, pdl);
        default: return launch_gemv_t<kType, 8, 2>(a, stream, pdl);
    }
}

}  // namespace

size_t gemv_smem_bytes(int M, int Kp) {
    const int mm = M <= 2 ? M : (M <= 4 ? 4 : 8);
    return (size_t)mm * Kp;
}

cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t stream, bool pdl) {
    if (a.M < 1 || a.M > kGemvMaxRows) return cudaErrorInvalidValue;
    return a.type == kInt8 ? dispatch_m<kInt8>(a, stream, pdl) : dispatch_m<kInt4>(a, stream, pdl);
}

}  // namespace zq
