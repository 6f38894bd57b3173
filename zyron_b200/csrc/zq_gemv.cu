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
constexpr int kUnroll = 4;  // 16-byte weight chunks in flight per lane

template <int kType, int kM>
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

    // Warm L2 with this warp's first column while the quantizer finishes.
    if (warp_global < N) {
        const uint8_t* c0 = panel + (size_t)warp_global * col_bytes;
        for (size_t off = (size_t)lane * 128; off < col_bytes; off += 32 * 128)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(c0 + off));
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

    for (int col = warp_global; col < N; col += warps_total) {
        const uint8_t* wc = panel + (size_t)col * col_bytes;
        int acc[kM];
#pragma unroll
        for (int m = 0; m < kM; ++m) acc[m] = 0;

        const int chunks = (int)(col_bytes >> 4);  // 16-byte chunks in the column
        int c = lane;
        for (; c + 32 * (kUnroll - 1) < chunks; c += 32 * kUnroll) {
            uint4 w[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) w[u] = ld_stream_u4(wc + (size_t)(c + 32 * u) * 16);
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                if (kType == kInt8)
                    dot16_int8<kM>(w[u], sq, Kp, (c + 32 * u) * 16, acc);
                else
                    dot16_int4<kM>(w[u], sq, Kp, (c + 32 * u) * 32, acc);
            }
        }
        for (; c < chunks; c += 32) {
            const uint4 w = ld_stream_u4(wc + (size_t)c * 16);
            if (kType == kInt8)
                dot16_int8<kM>(w, sq, Kp, c * 16, acc);
            else
                dot16_int4<kM>(w, sq, Kp, c * 32, acc);
        }

#pragma unroll
        for (int m = 0; m < kM; ++m) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
        }
        const float sc = __ldg(col_scale + col);
        const float b = bias ? __ldg(bias + col) : 0.0f;
#pragma unroll
        for (int m = 0; m < kM; ++m) {
            if (lane == m && m < M) {
                y[(size_t)m * N + col] = bias ? zq_epilogue_bias(acc[m], srow[m], sc, b)
                                              : zq_epilogue(acc[m], srow[m], sc);
            }
        }
    }
}

template <int kType, int kM>
cudaError_t launch_gemv_t(const GemvArgs& a, cudaStream_t stream, bool pdl) {
    const size_t smem = (size_t)kM * a.Kp;
    auto kern = gemv_kernel<kType, kM>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0, per_sm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kGemvThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const int warps_needed = a.N;
    int blocks = sms * per_sm;
    const int blocks_needed = (warps_needed + (kGemvThreads / 32) - 1) / (kGemvThreads / 32);
    if (blocks > blocks_needed) blocks = blocks_needed;

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
        case 1: return launch_gemv_t<kType, 1>(a, stream, pdl);
        case 2: return launch_gemv_t<kType, 2>(a, stream, pdl);
        case 3:
        case 4: return launch_gemv_t<kType, 4>(a, stream, pdl);
        default: return launch_gemv_t<kType, 8>(a, stream, pdl);
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
