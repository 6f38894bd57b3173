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
template <int kType, int kM, int kCols, int kUnroll, bool kX16>
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
                        dot16_int4<kM, kX16>(w[c][u], sq, Kp, ch * 32, acc[c]);
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
            if (kX16) acc[c][m] >>= 4;  // the codes entered as 16 x the code
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

// One activation row quantized in a single read (the fused INT8 kernel at M = 1):
// the absmax pass keeps the fp32 row in shared memory (xs, Kp floats after
// the codes) and the codes are made from there, so x is read once -- the
// general path reads it twice, for the absmax and for the codes, two L2
// round trips before the first dot.  Same arithmetic as that path.
template <int kThreads>
__device__ __forceinline__ void quantize_row_staged(const float* __restrict__ x, int K, int Kp, int8_t* sq,
                                                    float& srow) {
    __shared__ float redm1[kThreads / 32];
    const int tid = threadIdx.x, lane = tid & 31;
    const int kgroups = Kp >> 3;
    float4* xs4 = reinterpret_cast<float4*>(sq + Kp);  // Kp is a multiple of 128: 16-byte aligned
    const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (K & 3) == 0;
    float mx = 0.0f;
    for (int gi = tid; gi < kgroups; gi += kThreads) {
        const int k0 = gi * 8;
        float4 lo, hi;
        if (vec && k0 + 8 <= K) {
            lo = __ldg(reinterpret_cast<const float4*>(x + k0));
            hi = __ldg(reinterpret_cast<const float4*>(x + k0) + 1);
        } else {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = k0 + j < K ? __ldg(x + k0 + j) : 0.0f;
            lo = make_float4(v[0], v[1], v[2], v[3]);
            hi = make_float4(v[4], v[5], v[6], v[7]);
        }
        // NaN skipped by fmaxf, as std::max does
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(lo.x), fabsf(lo.y)), fmaxf(fabsf(lo.z), fabsf(lo.w))));
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(hi.x), fabsf(hi.y)), fmaxf(fabsf(hi.z), fabsf(hi.w))));
        xs4[2 * gi] = lo;
        xs4[2 * gi + 1] = hi;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) redm1[tid >> 5] = mx;
    __syncthreads();
    float t = redm1[0];
#pragma unroll
    for (int w = 1; w < kThreads / 32; ++w) t = fmaxf(t, redm1[w]);
    const float sm = zq_scale_from_absmax(t, 127.0f);
    const float rcp = zq_quant_rcp(sm);
    uint32_t* s4 = reinterpret_cast<uint32_t*>(sq);
    for (int gi = tid; gi < kgroups; gi += kThreads) {  // this thread's own groups: no barrier needed
        const float4 lo = xs4[2 * gi], hi = xs4[2 * gi + 1];
        const float v[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
        uint32_t c[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) c[j] = (uint32_t)(uint8_t)(int8_t)zq_quantize_value_rcp(v[j], sm, rcp, 127);
        s4[2 * gi] = c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24);
        s4[2 * gi + 1] = c[4] | (c[5] << 8) | (c[6] << 16) | (c[7] << 24);
    }
    srow = sm;
}

// kCols columns per warp iteration: each shared-memory activation read feeds
// kCols columns' dp4a (M >= 4 is dp4a/LDS-heavy; M <= 2 is purely HBM-bound).
// kFused: the activation rows arrive as fp32 `x` [M][K] and every block
// quantizes them itself with the standalone quantizer's arithmetic
// (quantization.cpp:202-212: fmaxf absmax, absmax / 127 correctly rounded,
// round half away from zero), so a decode matmul is a single launch.
template <int kType, int kM, int kCols, int kUnroll, bool kFused, int kThreads, bool kX16>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const uint8_t* __restrict__ panel, int N, int Kp,
                                                            const float* __restrict__ col_scale,
                                                            const int8_t* __restrict__ q,
                                                            const float* __restrict__ row_scale,
                                                            const float* __restrict__ bias, float* __restrict__ y,
                                                            int M, const float* __restrict__ x, int K) {
    extern __shared__ __align__(16) int8_t sq[];  // [kM][Kp]
    const int lane = threadIdx.x & 31;
    const int warp_global = (blockIdx.x * kThreads + threadIdx.x) >> 5;
    const int warps_total = (gridDim.x * kThreads) >> 5;
    const size_t col_bytes = kType == kInt8 ? (size_t)Kp : (size_t)(Kp >> 1);
    const int groups = (N + kCols - 1) / kCols;

    const int chunks = (int)(col_bytes >> 4);  // 16-byte chunks per column
    // No griddepcontrol.launch_dependents: a dependent launched early (at
    // the start, or at each warp's last column) put its blocks and L2
    // prefetches beside this grid's stream and measured slower (N = 11008,
    // K = 4096, M = 1: INT8 8.0 -> 10.8 / 9.5 us, INT4 7.3 -> 7.9 / 7.8 us);
    // the next kernel starts when this grid ends.
    // Warm L2 with this warp's first column group while the kernel before
    // (the quantizer, or the previous matmul) finishes.  Prefetching a
    // second group measured slower.
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

    float srow[kM];
    if constexpr (kFused && kM == 1 && kType == kInt8) {  // INT4 measured 0.1 us slower this way
        quantize_row_staged<kThreads>(x, K, Kp, sq, srow[0]);
    } else if constexpr (kFused) {
        // Per-row absmax (NaN skipped by fmaxf, as std::max does).  When the
        // rows start on 16-byte boundaries they are read as float4, two
        // loads in flight per thread.
        __shared__ float redm[kThreads / 32][kM];
        const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (K & 3) == 0;
        float mx[kM];
#pragma unroll
        for (int m = 0; m < kM; ++m) {
            mx[m] = 0.0f;
            if (m < M) {
                const float* xr = x + (size_t)m * K;
                if (vec) {
                    const float4* x4 = reinterpret_cast<const float4*>(xr);
                    const int K4 = K >> 2;
                    for (int b = threadIdx.x; b < K4; b += 2 * kThreads) {
                        float4 v[2];
#pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            const int i = b + u * kThreads;
                            v[u] = i < K4 ? __ldg(x4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
                        }
#pragma unroll
                        for (int u = 0; u < 2; ++u)
                            mx[m] = fmaxf(mx[m], fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)),
                                                       fmaxf(fabsf(v[u].z), fabsf(v[u].w))));
                    }
                } else {
                    for (int i = threadIdx.x; i < K; i += kThreads) mx[m] = fmaxf(mx[m], fabsf(__ldg(xr + i)));
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx[m] = fmaxf(mx[m], __shfl_xor_sync(0xffffffffu, mx[m], o));
            if (lane == 0) redm[threadIdx.x >> 5][m] = mx[m];
        }
        __syncthreads();
#pragma unroll
        for (int m = 0; m < kM; ++m) {
            float t = redm[0][m];
#pragma unroll
            for (int w = 1; w < kThreads / 32; ++w) t = fmaxf(t, redm[w][m]);
            srow[m] = m < M ? zq_scale_from_absmax(t, 127.0f) : 0.0f;
        }
        // codes into shared memory in k order, 8 per step
        uint32_t* s4 = reinterpret_cast<uint32_t*>(sq);
        const int kgroups = Kp >> 3;
        for (int gi = threadIdx.x; gi < kM * kgroups; gi += kThreads) {
            const int m = gi / kgroups, k0 = (gi - m * kgroups) * 8;
            float sm = 0.0f;
#pragma unroll
            for (int mm = 0; mm < kM; ++mm)
                if (mm == m) sm = srow[mm];
            float v[8];
            const float* xk = x + (size_t)m * K + k0;
            if (m < M && vec && k0 + 8 <= K) {
                const float4 lo = __ldg(reinterpret_cast<const float4*>(xk));
                const float4 hi = __ldg(reinterpret_cast<const float4*>(xk) + 1);
                v[0] = lo.x; v[1] = lo.y; v[2] = lo.z; v[3] = lo.w;
                v[4] = hi.x; v[5] = hi.y; v[6] = hi.z; v[7] = hi.w;
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = (m < M && k0 + j < K) ? __ldg(xk + j) : 0.0f;
            }
            uint32_t c[8];
            const float rcp = zq_quant_rcp(sm);
#pragma unroll
            for (int j = 0; j < 8; ++j) c[j] = (uint32_t)(uint8_t)(int8_t)zq_quantize_value_rcp(v[j], sm, rcp, 127);
            s4[2 * gi] = c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24);
            s4[2 * gi + 1] = c[4] | (c[5] << 8) | (c[6] << 16) | (c[7] << 24);
        }
    } else {
    // Stage the activation codes (rows >= M are zero).
    {
        const uint32_t* q4 = reinterpret_cast<const uint32_t*>(q);
        uint32_t* s4 = reinterpret_cast<uint32_t*>(sq);
        const int words = Kp >> 2;
        for (int i = threadIdx.x; i < kM * words; i += kThreads) {
            const int m = i / words;
            const int wi = i - m * words;
            s4[i] = m < M ? q4[(size_t)m * words + wi] : 0u;
        }
    }
#pragma unroll
    for (int m = 0; m < kM; ++m) srow[m] = m < M ? row_scale[m] : 0.0f;
    }
    __syncthreads();

    for (int g = warp_global; g < groups; g += warps_total)
        gemv_group<kType, kM, kCols, kUnroll, kX16>(g, panel, N, Kp, col_bytes, chunks, sq, col_scale, srow, bias, y, M,
                                                    lane);
}

// Four chunks per lane: with at most 64 resident warps per SM, eight per
// lane (one round for a 4096-code column) measured slower (fewer warps).
template <int kType, int kM, int kCols, int kUnroll = 4, bool kFused = false>
cudaError_t launch_gemv_t(const GemvArgs& a, cudaStream_t stream, bool pdl);

// INT4 codes are unpacked as 16 x the code (three operations per eight
// codes instead of nine) whenever the dot then fits in int32.
template <int kType, int kM, int kCols, int kUnroll, bool kFused, bool kX16>
cudaError_t launch_gemv_x(const GemvArgs& a, cudaStream_t stream, bool pdl) {
    // The fused variant runs 512-thread blocks, so each SM reads and
    // quantizes the activation rows half as often as with 256 (512 keeps the
    // register budget of the 256-thread variants: no spills, same occupancy).
    constexpr int kThreads = kFused ? 512 : kGemvThreads;
    // codes [kM][Kp]; the fused one-row kernel also stages the fp32 row
    const size_t smem = (size_t)kM * a.Kp + (kFused && kM == 1 && kType == kInt8 ? 4 * (size_t)a.Kp : 0);
    auto kern = gemv_kernel<kType, kM, kCols, kUnroll, kFused, kThreads, kX16>;
    cudaError_t e = ensure_smem_attr(kern, smem);
    if (e != cudaSuccess) return e;
    const int sms = sm_count(a.reserved_sms);
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    // As many resident warps as occupancy allows: under load the HBM needs
    // many loads in flight, and warps carry them.  The fused kernel also
    // prefetches each warp's first columns during its prologue, and the INT4
    // kernel is issue-bound, so both keep every resident warp.  The staged
    // INT8 kernel is a pure weight stream, where the last round is the cost:
    // it takes the fewest rounds the resident warps allow, then just enough
    // warps for that many (rounded up to whole SMs), so that nearly every warp
    // streams the same number of columns (N = 11008, M = 1: 8.85 -> 8.41 us).
    const int groups = (a.N + kCols - 1) / kCols;
    const int wpb = kThreads / 32;
    const int max_blocks = sms * per_sm;
    const int needed = (groups + wpb - 1) / wpb;
    int blocks = max_blocks < needed ? max_blocks : needed;
    if (kType == kInt8 && !kFused && needed > max_blocks) {
        const int max_warps = max_blocks * wpb;
        const int rounds = (groups + max_warps - 1) / max_warps;
        const int warps = (groups + rounds - 1) / rounds;
        const int even = ((warps + wpb - 1) / wpb + sms - 1) / sms * sms;
        blocks = even < max_blocks ? even : max_blocks;
    }

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    // Always a programmatic dependent launch: the kernel reads only the
    // weight panel before griddepcontrol.wait.
    (void)pdl;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a.panel, a.N, a.Kp, a.col_scale, a.q, a.row_scale, a.bias, a.y,
                              a.M, a.x, a.K);
}

template <int kType, int kM, int kCols, int kUnroll, bool kFused>
cudaError_t launch_gemv_t(const GemvArgs& a, cudaStream_t stream, bool pdl) {
    if constexpr (kType == kInt4) {
        if (int4_x16_fits(a.Kp)) return launch_gemv_x<kType, kM, kCols, kUnroll, kFused, true>(a, stream, pdl);
    }
    return launch_gemv_x<kType, kM, kCols, kUnroll, kFused, false>(a, stream, pdl);
}

template <int kType>
cudaError_t dispatch_m(const GemvArgs& a, cudaStream_t stream, bool pdl) {
    if (a.x) {  // quantizer fused, up to 4 rows
        switch (a.M) {
            // INT4, one row: two columns per warp halve the blocks that each
            // quantize the row (N = 11008, K = 4096: call 9.4 -> 8.4 us; INT8
            // and the staged INT4 kernel measured slower that way)
            case 1:
                return kType == kInt4 ? launch_gemv_t<kType, 1, 2, 4, true>(a, stream, pdl)
                                      : launch_gemv_t<kType, 1, 1, 4, true>(a, stream, pdl);
            case 2: return launch_gemv_t<kType, 2, 1, 4, true>(a, stream, pdl);
            default: return launch_gemv_t<kType, 4, 2, 4, true>(a, stream, pdl);
        }
    }
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
    // one row: the fused kernel also stages the fp32 row (4 Kp bytes)
    return (size_t)mm * Kp + (M == 1 ? 4 * (size_t)Kp : 0);
}

cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t stream, bool pdl) {
    if (a.M < 1 || a.M > kGemvMaxRows || (a.x && a.M > 4)) return cudaErrorInvalidValue;
    return a.type == kInt8 ? dispatch_m<kInt8>(a, stream, pdl) : dispatch_m<kInt4>(a, stream, pdl);
}

}  // namespace zq
