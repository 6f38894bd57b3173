// zq_quant.cu -- activation quantizer, weight layout kernels and dequantize.
//
// Device weight layout ("panel" layout).  The reference stores a K x N weight
// column-major, element (row k, col n) at linear index n*K + k, INT4 as two
// codes per byte with the low nibble holding the even linear index
// (src/quantization/quantization.cpp:52-67, 155).  On the device every column
// starts on a 16-byte boundary and is zero-padded to Kp codes:
//   INT8: codes[n * Kp + k]                       Kp = roundup(K, 16)
//   INT4: Kp/2 bytes per column, Kp = roundup(K, 32), codes in groups of
//         eight: byte 4g + j holds code 8g + j (low nibble) and 8g + j + 4
//         (high nibble), so a 32-bit word unpacks into codes in k order
//         without byte shuffles (panel_int4_byte, panel_int4_shift)
// Zero codes contribute nothing to an integer dot product, so padding never
// changes a result; it gives every TMA tensor map 16-byte strides and every
// GEMV lane aligned 128-bit loads.
#include "zq_common.cuh"
#include "zq_kernels.h"

#include <cstdint>

namespace zq {

// ---------------------------------------------------------------------------
// Per-row dynamic activation quantizer (quantization.cpp:202-212).
// One warp per row: pass 1 reduces |x| with fmaxf (NaN skipped, like
// std::max), pass 2 writes codes; the [K, Kp) tail is zero-filled.
// ---------------------------------------------------------------------------
// Block 0 also clears `zero[0, n_zero)` (see launch_quantize_rows).
__device__ __forceinline__ void clear_words(int* zero, int n_zero) {
    if (blockIdx.x == 0)
        for (int i = threadIdx.x; i < n_zero; i += blockDim.x) zero[i] = 0;
}

template <bool kVec>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const float* __restrict__ x, int M, int K,
                                                            int Kp, int8_t* __restrict__ q,
                                                            float* __restrict__ row_scale, int* zero, int n_zero) {
    pdl_launch_dependents();
    pdl_wait_primary();  // x may come from, and q / counters be read by, the kernels before
    clear_words(zero, n_zero);
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= M) return;
    const float* xr = x + (size_t)warp * K;
    int8_t* qr = q + (size_t)warp * Kp;

    float m = 0.0f;
    if (kVec) {
        const float4* x4 = reinterpret_cast<const float4*>(xr);
        for (int i = lane; i < (K >> 2); i += 32) {
            const float4 v = __ldg(x4 + i);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
    } else {
        for (int i = lane; i < K; i += 32) m = fmaxf(m, fabsf(__ldg(xr + i)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float s = zq_scale_from_absmax(m, 127.0f);
    if (lane == 0) row_scale[warp] = s;
    const float rcp = zq_quant_rcp(s);

    if (kVec) {
        const float4* x4 = reinterpret_cast<const float4*>(xr);
        uint32_t* q4 = reinterpret_cast<uint32_t*>(qr);
        for (int i = lane; i < (K >> 2); i += 32) {
            const float4 v = __ldg(x4 + i);
            const uint32_t b0 = (uint32_t)(uint8_t)(int8_t)zq_quantize_value_rcp(v.x, s, rcp, 127);
            const uint32_t b1 = (uint32_t)(uint8_t)(int8_t)zq_quantize_value_rcp(v.y, s, rcp, 127);
            const uint32_t b2 = (uint32_t)(uint8_t)(int8_t)zq_quantize_value_rcp(v.z, s, rcp, 127);
            const uint32_t b3 = (uint32_t)(uint8_t)(int8_t)zq_quantize_value_rcp(v.w, s, rcp, 127);
            q4[i] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
        }
        for (int i = (K >> 2) + lane; i < (Kp >> 2); i += 32) q4[i] = 0u;
    } else {
        for (int i = lane; i < K; i += 32) qr[i] = (int8_t)zq_quantize_value_rcp(__ldg(xr + i), s, rcp, 127);
        for (int i = K + lane; i < Kp; i += 32) qr[i] = 0;
    }
}

// Register-resident variant: a row is held by kWarpsPerRow warps, each lane
// keeping up to kVec float4 in registers, so x is read from memory exactly
// once (absmax and codes come from the same registers).  Used when K is a
// multiple of 4 and K/4 <= 32 * kWarpsPerRow * kVec.
template <int kWarpsPerRow, int kVec>
__global__ void __launch_bounds__(256) quantize_rows_reg_kernel(const float* __restrict__ x, int M, int K, int Kp,
                                                                int8_t* __restrict__ q,
                                                                float* __restrict__ row_scale, int* zero,
                                                                int n_zero) {
    pdl_launch_dependents();
    pdl_wait_primary();  // x may come from, and q / counters be read by, the kernels before
    clear_words(zero, n_zero);
    constexpr int kRowsPerBlock = 8 / kWarpsPerRow;
    constexpr int kT = 32 * kWarpsPerRow;
    __shared__ float part[8];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * kRowsPerBlock + warp / kWarpsPerRow;
    const int t = (warp % kWarpsPerRow) * 32 + lane;
    const int k4 = K >> 2;
    float4 v[kVec];
    float m = 0.0f;
    if (row < M) {
        const float4* x4 = reinterpret_cast<const float4*>(x + (size_t)row * K);
#pragma unroll
        for (int i = 0; i < kVec; ++i) {
            const int idx = t + i * kT;
            v[i] = idx < k4 ? __ldg(x4 + idx) : make_float4(0.f, 0.f, 0.f, 0.f);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (kWarpsPerRow > 1) {
        if (lane == 0) part[warp] = m;
        __syncthreads();
        const int first = (warp / kWarpsPerRow) * kWarpsPerRow;
#pragma unroll
        for (int w = 0; w < kWarpsPerRow; ++w) m = fmaxf(m, part[first + w]);
    }
    if (row >= M) return;
    const float s = zq_scale_from_absmax(m, 127.0f);
    if (t == 0) row_scale[row] = s;
    const float rcp = zq_quant_rcp(s);
    uint32_t* q4 = reinterpret_cast<uint32_t*>(q + (size_t)row * Kp);
#pragma unroll
    for (int i = 0; i < kVec; ++i) {
        const int idx = t + i * kT;
        if (idx < k4) {
            const uint32_t b0 = (uint32_t)(uint8_t)(int8_t)zq_quantize_value_rcp(v[i].x, s, rcp, 127);
            const uint32_t b1 = (uint32_t)(uint8_t)(int8_t)zq_quantize_value_rcp(v[i].y, s, rcp, 127);
            const uint32_t b2 = (uint32_t)(uint8_t)(int8_t)zq_quantize_value_rcp(v[i].z, s, rcp, 127);
            const uint32_t b3 = (uint32_t)(uint8_t)(int8_t)zq_quantize_value_rcp(v[i].w, s, rcp, 127);
            q4[idx] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
        }
    }
    for (int i = k4 + t; i < (Kp >> 2); i += kT) q4[i] = 0u;
}

cudaError_t launch_quantize_rows(const float* x, int M, int K, int Kp, int8_t* q, float* row_scale,
                                 cudaStream_t stream, int* zero, int n_zero) {
    if (M <= 0) return cudaSuccess;
    const bool aligned = (K % 4 == 0) && (Kp % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) &&
                         ((reinterpret_cast<uintptr_t>(q) & 3u) == 0);
    const int k4 = K / 4;
    if (aligned && k4 <= 2048) {
        int wpr = 1;
        while (wpr < 8 && k4 > 32 * wpr * 8) wpr *= 2;
        const int rows_per_block = 8 / wpr;
        const dim3 grid((M + rows_per_block - 1) / rows_per_block);
        switch (wpr) {
            case 1: return launch_pdl_kernel(quantize_rows_reg_kernel<1, 8>, grid, dim3(256), 0, stream, x, M, K, Kp, q,
                                             row_scale, zero, n_zero);
            case 2: return launch_pdl_kernel(quantize_rows_reg_kernel<2, 8>, grid, dim3(256), 0, stream, x, M, K, Kp, q,
                                             row_scale, zero, n_zero);
            case 4: return launch_pdl_kernel(quantize_rows_reg_kernel<4, 8>, grid, dim3(256), 0, stream, x, M, K, Kp, q,
                                             row_scale, zero, n_zero);
            default: return launch_pdl_kernel(quantize_rows_reg_kernel<8, 8>, grid, dim3(256), 0, stream, x, M, K,
                                              Kp, q, row_scale, zero, n_zero);
        }
    }
    const int rows_per_block = 8;
    const dim3 grid((M + rows_per_block - 1) / rows_per_block);
    const bool vec = (K % 4 == 0) && (Kp % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) &&
                     ((reinterpret_cast<uintptr_t>(q) & 3u) == 0);
    if (vec)
        return launch_pdl_kernel(quantize_rows_kernel<true>, grid, dim3(256), 0, stream, x, M, K, Kp, q, row_scale,
                                 zero, n_zero);
    return launch_pdl_kernel(quantize_rows_kernel<false>, grid, dim3(256), 0, stream, x, M, K, Kp, q, row_scale, zero,
                             n_zero);
}

// ---------------------------------------------------------------------------
// INT4 repack: reference nibble stream (column c at nibble c*K, low nibble =
// even linear index) -> panel layout.  One thread per output byte.
// ---------------------------------------------------------------------------
__global__ void repack_int4_kernel(const uint8_t* __restrict__ src, int K, int N, int Kp,
                                   uint8_t* __restrict__ dst) {
    const int bytes_per_col = Kp >> 1;
    const size_t total = (size_t)N * bytes_per_col;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t c = i / bytes_per_col;
        const int j = (int)(i - c * bytes_per_col);
        uint32_t out = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int k = ((j >> 2) << 3) + (j & 3) + 4 * h;  // panel byte j: codes k (low) and k + 4 (high)
            if (k < K) {
                const size_t lin = c * (size_t)K + k;
                const uint8_t b = src[lin >> 1];
                const uint32_t nib = (lin & 1u) ? (b >> 4) : (b & 0x0Fu);
                out |= nib << (4 * h);
            }
        }
        dst[i] = (uint8_t)out;
    }
}

cudaError_t launch_repack_int4(const uint8_t* src, int K, int N, int Kp, uint8_t* dst, cudaStream_t stream) {
    const size_t total = (size_t)N * (Kp >> 1);
    const int threads = 256;
    const int blocks = (int)((total + threads - 1) / threads < 148 * 16 ? (total + threads - 1) / threads
                                                                         : 148 * 16);
    repack_int4_kernel<<<blocks, threads, 0, stream>>>(src, K, N, Kp, dst);
    return cudaGetLastError();
}

// Panel layout -> reference payload (for save / download); one thread per
// output byte of the reference stream.
__global__ void unpack_panel_int4_kernel(const uint8_t* __restrict__ panel, int K, int N, int Kp,
                                         uint8_t* __restrict__ dst) {
    const size_t nibbles = (size_t)K * N;
    const size_t total = (nibbles + 1) / 2;
    const int bpc = Kp >> 1;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        uint32_t out = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const size_t lin = 2 * i + h;
            if (lin < nibbles) {
                const size_t c = lin / K;
                const int k = (int)(lin - c * K);
                const uint8_t b = panel[c * bpc + panel_int4_byte(k)];
                out |= (uint32_t)((b >> panel_int4_shift(k)) & 0x0Fu) << (4 * h);
            }
        }
        dst[i] = (uint8_t)out;
    }
}

cudaError_t launch_unpack_panel_int4(const uint8_t* panel, int K, int N, int Kp, uint8_t* dst,
                                     cudaStream_t stream) {
    const size_t total = ((size_t)K * N + 1) / 2;
    const int threads = 256;
    const size_t want = (total + threads - 1) / threads;
    const int blocks = (int)(want < 148 * 16 ? want : 148 * 16);
    unpack_panel_int4_kernel<<<blocks > 0 ? blocks : 1, threads, 0, stream>>>(panel, K, N, Kp, dst);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Weight quantization on the device (quantize(): quantization.cpp:121-162).
// w is fp32 row-major [K][N].
//   pass 1: per-column absmax; threads own columns (coalesced along N), the
//           grid's y dimension splits K and partial maxima meet in an
//           atomicMax on the non-negative float bit pattern.
//   pass 2: scale = absmax / limit, codes written transposed into the panel
//           layout through a 32 x 32 shared-memory tile.
// ---------------------------------------------------------------------------
__global__ void column_absmax_kernel(const float* __restrict__ w, int K, int N, int rows_per_block,
                                     uint32_t* __restrict__ absmax_bits) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    const int k0 = blockIdx.y * rows_per_block;
    const int k1 = min(K, k0 + rows_per_block);
    float m = 0.0f;
    for (int k = k0; k < k1; ++k) m = fmaxf(m, fabsf(__ldg(w + (size_t)k * N + n)));
    atomicMax(absmax_bits + n, __float_as_uint(m));
}

__global__ void column_scale_kernel(const uint32_t* __restrict__ absmax_bits, int N, float limit,
                                    float* __restrict__ scales) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n < N) scales[n] = zq_scale_from_absmax(__uint_as_float(absmax_bits[n]), limit);
}

template <int kType>
__global__ void __launch_bounds__(256) quantize_panel_kernel(const float* __restrict__ w, int K, int N,
                                                             int Kp, const float* __restrict__ scales,
                                                             uint8_t* __restrict__ panel) {
    // tile: 32 columns (n) x 128 rows (k); threads (32, 8).  Reads are rows
    // of 32 consecutive floats; each column's 128 codes go out as one
    // 128-byte (INT8) or 64-byte (INT4) segment.
    __shared__ int8_t tile[32][128 + 4];
    const int n0 = blockIdx.x * 32;
    const int k0 = blockIdx.y * 128;
    const int tx = threadIdx.x, ty = threadIdx.y;
    const int limit = kType == kInt8 ? 127 : 7;
    const int n = n0 + tx;
    const float s = n < N ? scales[n] : 1.0f;
    const float rcp = zq_quant_rcp(s);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int k = k0 + ty + 8 * j;
        int8_t v = 0;
        if (n < N && k < K) v = (int8_t)zq_quantize_value_rcp(__ldg(w + (size_t)k * N + n), s, rcp, limit);
        tile[tx][ty + 8 * j] = v;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int c = ty + 8 * j;
        const int nn = n0 + c;
        const int k = k0 + 4 * tx;  // codes k .. k+3 of column nn
        if (nn >= N || k >= Kp) continue;
        const uint32_t c0 = (uint8_t)tile[c][4 * tx], c1 = (uint8_t)tile[c][4 * tx + 1];
        const uint32_t c2 = (uint8_t)tile[c][4 * tx + 2], c3 = (uint8_t)tile[c][4 * tx + 3];
        if (kType == kInt8) {
            *reinterpret_cast<uint32_t*>(panel + (size_t)nn * Kp + k) = c0 | (c1 << 8) | (c2 << 16) | (c3 << 24);
        } else if ((tx & 1) == 0) {
            // codes k .. k+7 of the group: byte j holds codes k+j (low) and
            // k+j+4 (high nibble)
            const int8_t* t = &tile[c][4 * tx];
            uint32_t word = 0;
#pragma unroll
            for (int b = 0; b < 4; ++b)
                word |= ((uint32_t)((uint8_t)t[b] & 0x0Fu) | ((uint32_t)((uint8_t)t[b + 4] & 0x0Fu) << 4)) << (8 * b);
            *reinterpret_cast<uint32_t*>(panel + (size_t)nn * (Kp >> 1) + (k >> 1)) = word;
        }
    }
}

cudaError_t launch_quantize_weights(const float* w, int K, int N, int Kp, int type, uint32_t* absmax_tmp,
                                    float* scales, uint8_t* panel, cudaStream_t stream) {
    cudaError_t e = cudaMemsetAsync(absmax_tmp, 0, sizeof(uint32_t) * (size_t)N, stream);
    if (e != cudaSuccess) return e;
    const int rows_per_block = 256;
    dim3 g1((N + 127) / 128, (K + rows_per_block - 1) / rows_per_block);
    column_absmax_kernel<<<g1, 128, 0, stream>>>(w, K, N, rows_per_block, absmax_tmp);
    column_scale_kernel<<<(N + 255) / 256, 256, 0, stream>>>(absmax_tmp, N, type == kInt8 ? 127.0f : 7.0f,
                                                            scales);
    dim3 g2((N + 31) / 32, (Kp + 127) / 128);
    if (type == kInt8)
        quantize_panel_kernel<kInt8><<<g2, dim3(32, 8), 0, stream>>>(w, K, N, Kp, scales, panel);
    else
        quantize_panel_kernel<kInt4><<<g2, dim3(32, 8), 0, stream>>>(w, K, N, Kp, scales, panel);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// dequantize() (quantization.cpp:164-175): out[k][n] = float(code(n,k)) * s_n,
// fp32 row-major [K][N].  32 x 32 tile transpose; reads the panel along k,
// writes out along n.
// ---------------------------------------------------------------------------
template <int kType>
__global__ void __launch_bounds__(256) dequantize_kernel(const uint8_t* __restrict__ panel, int K, int N,
                                                         int Kp, const float* __restrict__ scales,
                                                         float* __restrict__ out) {
    __shared__ int8_t tile[32][64 + 4];  // [n][k]
    const int n0 = blockIdx.x * 32;
    const int k0 = blockIdx.y * 64;
    const int tx = threadIdx.x, ty = threadIdx.y;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int c = ty + 8 * j;
        const int nn = n0 + c;
        const int k = k0 + 2 * tx;
        int8_t a = 0, b = 0;
        if (nn < N && k < Kp) {
            if (kType == kInt8) {
                const uint16_t pair = *reinterpret_cast<const uint16_t*>(panel + (size_t)nn * Kp + k);
                a = (int8_t)(pair & 0xFF);
                b = (int8_t)(pair >> 8);
            } else {
                const uint8_t* col = panel + (size_t)nn * (Kp >> 1);
                const int lo = (col[panel_int4_byte(k)] >> panel_int4_shift(k)) & 0x0F;
                const int hi = (col[panel_int4_byte(k + 1)] >> panel_int4_shift(k + 1)) & 0x0F;
                a = (int8_t)(lo < 8 ? lo : lo - 16);
                b = (int8_t)(hi < 8 ? hi : hi - 16);
            }
        }
        tile[c][2 * tx] = a;
        tile[c][2 * tx + 1] = b;
    }
    __syncthreads();
    const int n = n0 + tx;
    if (n >= N) return;
    const float s = scales[n];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int k = k0 + ty + 8 * j;
        if (k < K) out[(size_t)k * N + n] = x86_mul((float)tile[tx][ty + 8 * j], s);
    }
}

cudaError_t launch_dequantize(const uint8_t* panel, int type, int K, int N, int Kp, const float* scales,
                              float* out, cudaStream_t stream) {
    dim3 g((N + 31) / 32, (K + 63) / 64);
    if (type == kInt8)
        dequantize_kernel<kInt8><<<g, dim3(32, 8), 0, stream>>>(panel, K, N, Kp, scales, out);
    else
        dequantize_kernel<kInt4><<<g, dim3(32, 8), 0, stream>>>(panel, K, N, Kp, scales, out);
    return cudaGetLastError();
}

}  // namespace zq
