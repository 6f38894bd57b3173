// zq_skinny_sm100.cu -- decode-sized quantized matmul (M <= 16 activation
// rows) on 5th-generation tensor cores (tcgen05, sm_100a).
//
// Computes, for every activation row m and output column n,
//   acc[m][n] = sum_k q_a[m][k] * q_w[n][k]            (exact int32)
//   y[m][n]   = float(acc) * s_row[m] * s_col[n] (+ bias[n])
// which is quantization::matmul's dot and epilogue (src/quantization/
// quantization.cpp:215-232) plus QuantizedLinear's bias pass
// (src/quantization/quantized_linear.cpp:44-48).
//
// With a handful of activation rows the weight stream is the whole cost, so
// the job is to read every weight byte from HBM exactly once, at full
// bandwidth, on every SM until the end.  The MMA operands are swapped with
// respect to the prefill GEMM: A is a block of 128 weight columns (the panel
// [N][Kp] is K-major, so 128 columns are a 128-row K-major tile), B is the
// activation codes, whose TMA box of 16 rows is zero-filled past row M, and
// the TMEM accumulator is acc transposed (128 lanes = columns, 16 columns =
// activation rows).  tcgen05.mma.kind::i8 M=128 N=16 K=32 takes 32 cycles
// per 16 KiB k-block, far below the HBM time of the same bytes.
//
// Work split (stream-K): the (column block, k-block) iterations are cut into
// equal contiguous ranges, one per CTA and one CTA per SM, so every SM
// streams the same number of weight bytes whatever N and K are.  A column
// block whose k-range spans several CTAs is finished by the one that
// completes its share last: every sharer writes its int32 partial sums to
// the workspace and then counts its share done; the CTA whose count
// completes the block adds the others' sums to its own (integer addition,
// exact in any order) and applies the epilogue.  No CTA ever waits for
// another.  (Choosing the finisher by arrival instead left CTAs waiting up to
// 10 us for a CTA that shares the block from the middle of its range.)  The
// counters are zeroed by the kernel launched just before this one (the
// activation quantizer, or a zeroing kernel).
//
// INT4 weights arrive as packed [128 columns][64 bytes] tiles; four unpack
// warps sign-extend each into the 128-byte-swizzled int8 tile the MMA reads.
//
// Warps: 0 TMA producer; 1 TMEM allocator + MMA issuer; 2-5 epilogue;
// 6-9 (INT4 only) unpack.  Every mbarrier wait is bounded.
#include "zq_common.cuh"
#include "zq_kernels.h"
#include "zq_tcgen05.cuh"

#include <cuda.h>

namespace zq {

namespace {

constexpr int kSkBlockN = 128;  // weight columns per tile (MMA M)
constexpr int kSkRows = 16;     // activation rows per MMA (MMA N); rows >= M are zeros
constexpr int kSkKBlock = 128;  // codes per k-block (one 128-byte swizzle row of int8)
constexpr int kSkUmmaK = 32;

template <int kType>
struct SkCfg;
template <>
struct SkCfg<kInt8> {
    static constexpr int kStages = 8;
    static constexpr int kThreads = 192;
    static constexpr int kWBytes = kSkBlockN * kSkKBlock;  // swizzled int8, read by the MMA
    static constexpr int kXBytes = kSkRows * kSkKBlock;
    static constexpr int kStageBytes = kWBytes + kXBytes;  // 18 KiB
};
template <>
struct SkCfg<kInt4> {
    static constexpr int kStages = 6;
    static constexpr int kThreads = 192 + 32 * kStages;  // one unpack warp per stage
    static constexpr int kWBytes = kSkBlockN * kSkKBlock / 2;  // packed, row-major [128][64]
    static constexpr int kXBytes = kSkRows * kSkKBlock;
    static constexpr int kConvBytes = kSkBlockN * kSkKBlock;  // unpacked int8, swizzled
    static constexpr int kStageBytes = kWBytes + kXBytes + kConvBytes;  // 26 KiB
};

template <int kType>
constexpr int sk_smem_bytes() {
    using C = SkCfg<kType>;
    return 1024 /*alignment slack*/ + C::kStages * C::kStageBytes + 8 * (3 * C::kStages + 5) + 16;
}

// CTA g owns iterations [g*T/G, (g+1)*T/G); iteration t is k-block t % KB of
// column block t / KB.
__device__ __forceinline__ long long sk_start(int g, long long T, int G) { return (long long)g * T / G; }
// The CTA whose range holds iteration t: the largest g with g*T/G <= t.
__device__ __forceinline__ int sk_owner(long long t, long long T, int G) {
    return (int)(((t + 1) * (long long)G - 1) / T);
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Waits until *p >= target, bounded like every wait in this library: after
// `limit_ns` it records `code` in *err and returns false.
__device__ __forceinline__ bool wait_count_bounded(const int* p, int target, uint32_t* err, uint32_t code,
                                                   uint64_t limit_ns = 4000000000ull) {
    if (ld_acquire_gpu(p) >= target) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        __nanosleep(32);
        if (ld_acquire_gpu(p) >= target) return true;
        if (*(volatile uint32_t*)err != kDevErrNone) return false;
        if (global_timer_ns() - t0 > limit_ns) {
            atomicCAS(err, kDevErrNone, code);
            return false;
        }
    }
}

template <int kType>
__global__ void __launch_bounds__(SkCfg<kType>::kThreads, 1)
    skinny_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x, int M,
                  int N, int KB, long long T, const float* __restrict__ row_scale,
                  const float* __restrict__ col_scale, const float* __restrict__ bias, float* __restrict__ y,
                  int* __restrict__ counters, int* __restrict__ partials, uint32_t* __restrict__ err,
                  int wait_extra, unsigned long long peer_limit_ns, int x16) {
    using C = SkCfg<kType>;
    constexpr int S = C::kStages;
    constexpr uint32_t kTmemCols = 32;  // two 16-column accumulators
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * C::kStageBytes);
    uint64_t* full = bars;           // TMA -> MMA (INT8) or -> unpack (INT4)
    uint64_t* conv_full = bars + S;  // unpack -> MMA (INT4)
    uint64_t* empty = bars + 2 * S;  // MMA -> TMA
    uint64_t* tfull = bars + 3 * S;
    uint64_t* tempty = bars + 3 * S + 2;
    uint64_t* mma_done = bars + 3 * S + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * S + 5);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int G = gridDim.x;
    const int g = blockIdx.x;
    const long long it0 = sk_start(g, T, G);
    const long long it1 = sk_start(g + 1, T, G);
    // The next kernel on the stream may launch now (it reads nothing of ours
    // before its griddepcontrol.wait) and take over the SMs as this grid's
    // CTAs finish.
    pdl_launch_dependents();

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&conv_full[s], 1);  // the stage's unpack warp
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 128);
        }
        mbar_init(mma_done, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmap_w);
        tma_prefetch_desc(&tmap_x);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // The weight tiles of the first stages do not depend on the
            // kernel before this one: start streaming them while it finishes,
            // and add the activation tiles once its codes are visible.
            const int pre = (int)((it1 - it0) < S ? (it1 - it0) : S);
            for (int i = 0; i < pre; ++i) {
                const long long t = it0 + i;
                const int b = (int)(t / KB), kb = (int)(t % KB);
                mbar_arrive_expect_tx(&full[i], C::kWBytes + C::kXBytes);
                tma_load_2d(smem + i * C::kStageBytes, &tmap_w, &full[i], kType == kInt8 ? kb * 128 : kb * 64,
                            b * kSkBlockN);
            }
            pdl_wait_primary();
            for (int i = 0; i < pre; ++i) {
                const int kb = (int)((it0 + i) % KB);
                tma_load_2d(smem + i * C::kStageBytes + C::kWBytes, &tmap_x, &full[i], kb * kSkKBlock, 0);
            }
            int stage = pre == S ? 0 : pre;
            uint32_t phase = pre == S ? 1u : 0u;
            uint32_t last_phase[S];
            bool issued[S];
#pragma unroll
            for (int s = 0; s < S; ++s) issued[s] = s < pre, last_phase[s] = 0;
            for (long long t = it0 + pre; t < it1; ++t) {
                if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, err, kDevErrTimeoutProducer)) break;
                const int b = (int)(t / KB), kb = (int)(t % KB);
                uint8_t* st = smem + stage * C::kStageBytes;
                mbar_arrive_expect_tx(&full[stage], C::kWBytes + C::kXBytes);
                tma_load_2d(st, &tmap_w, &full[stage], kType == kInt8 ? kb * 128 : kb * 64, b * kSkBlockN);
                tma_load_2d(st + C::kWBytes, &tmap_x, &full[stage], kb * kSkKBlock, 0);
                issued[stage] = true;
                last_phase[stage] = phase;
                if (++stage == S) stage = 0, phase ^= 1u;
            }
            // Every copy this thread issued lands before the CTA may exit.
            for (int s = 0; s < S; ++s)
                if (issued[s]) mbar_drain_bounded(&full[s], last_phase[s], err, kDevErrTimeoutDrain);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(kSkBlockN, kSkRows);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            long long t = it0;
            while (t < it1 && ok) {
                const int b = (int)(t / KB);
                const long long seg0 = t;
                const long long seg1 = it1 < (long long)(b + 1) * KB ? it1 : (long long)(b + 1) * KB;
                if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1u, err, kDevErrTimeoutMma)) break;
                tmem_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * kSkRows);
                for (; t < seg1; ++t) {
                    uint64_t* ready = kType == kInt8 ? &full[stage] : &conv_full[stage];
                    if (!mbar_wait_bounded(ready, phase, err, kDevErrTimeoutMma)) {
                        ok = false;
                        break;
                    }
                    tmem_fence_after();
                    const uint32_t base = smem_u32(smem + stage * C::kStageBytes);
                    const uint32_t sa = kType == kInt8 ? base : base + C::kWBytes + C::kXBytes;
                    const uint32_t sb = base + C::kWBytes;
#pragma unroll
                    for (int kk = 0; kk < kSkKBlock / kSkUmmaK; ++kk)
                        umma_i8(d, make_sw128_desc(sa + kk * kSkUmmaK), make_sw128_desc(sb + kk * kSkUmmaK), idesc,
                                (t > seg0 || kk > 0) ? 1u : 0u);
                    umma_commit(&empty[stage]);
                    if (++stage == S) stage = 0, phase ^= 1u;
                }
                if (!ok) break;
                umma_commit(&tfull[acc]);
                if (++acc == 2) acc = 0, acc_phase ^= 1u;
            }
            // All MMAs issued by this thread complete before TMEM is freed.
            umma_commit(mma_done);
            mbar_drain_bounded(mma_done, 0, err, kDevErrTimeoutDrain);
        }
    } else if (warp < 6) {
        // Epilogue: warp w reads TMEM lanes (w % 4) * 32 .. +31, i.e. 32
        // columns of the block, all 16 activation rows per thread.
        const int q = warp & 3;
        const int col_local = q * 32 + lane;
        // Row scales and counters are written by the kernel before this one;
        // read them only through L2 (this SM's L1 may hold older lines).
        pdl_wait_primary();
        float sr[kSkRows];
#pragma unroll
        for (int m = 0; m < kSkRows; ++m) sr[m] = m < M ? __ldcg(row_scale + m) : 0.0f;
        const int first_b = (int)(it0 / KB);
        int acc = 0;
        uint32_t acc_phase = 0;
        long long t = it0;
        while (t < it1) {
            const int b = (int)(t / KB);
            const long long bk0 = (long long)b * KB, bk1 = bk0 + KB;
            const bool whole = t == bk0 && it1 >= bk1;
            t = it1 < bk1 ? it1 : bk1;
            if (!mbar_wait_bounded(&tfull[acc], acc_phase, err, kDevErrTimeoutEpilogue)) break;
            tmem_fence_after();
            uint32_t r[kSkRows];
            tmem_ld_32x32b_x16(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * kSkRows), r);
            tmem_ld_wait();
            tmem_fence_before();
            mbar_arrive(&tempty[acc]);
            if (++acc == 2) acc = 0, acc_phase ^= 1u;

            if (!whole) {
                // A block shared with other CTAs: publish this CTA's exact
                // int32 share, then count it; the CTA whose count completes
                // the block adds the others' shares to its own and writes the
                // output.  Nobody waits: the block is finished by whichever
                // CTA finishes its share last.
                const int slot = b == first_b ? 0 : 1;
                int* mine = partials + (size_t)(g * 2 + slot) * M * kSkBlockN + col_local;
#pragma unroll
                for (int m = 0; m < kSkRows; ++m)
                    if (m < M) mine[(size_t)m * kSkBlockN] = (int)r[m];
                __threadfence();
                __syncwarp();
                int* done = counters + b * 8 + q;
                const int g0 = sk_owner(bk0, T, G), g1 = sk_owner(bk1 - 1, T, G);
                int prior = 0;
                if (lane == 0) prior = atomicAdd(done, 1);
                prior = __shfl_sync(0xffffffffu, prior, 0);
                if (prior != g1 - g0) continue;  // another CTA's share is still running
                if (wait_extra > 0) {
                    // failure-path test only: wait for shares that do not exist
                    int fine = 1;
                    if (lane == 0)
                        fine = wait_count_bounded(done, g1 - g0 + 1 + wait_extra, err, kDevErrTimeoutPeer,
                                                  peer_limit_ns)
                                   ? 1
                                   : 0;
                    if (__shfl_sync(0xffffffffu, fine, 0) == 0) continue;
                }
                __threadfence();  // the other shares were published before their counts
                for (int h = g0; h <= g1; ++h) {
                    if (h == g) continue;
                    const int hs = sk_start(h, T, G) / KB == b ? 0 : 1;
                    const int* p = partials + (size_t)(h * 2 + hs) * M * kSkBlockN + col_local;
#pragma unroll
                    for (int m = 0; m < kSkRows; ++m)
                        if (m < M) r[m] += (uint32_t)__ldcg(p + (size_t)m * kSkBlockN);
                }
            }
            if (x16) {
#pragma unroll
                for (int m = 0; m < kSkRows; ++m) r[m] = (uint32_t)((int32_t)r[m] >> 4);  // 16 x the dot, exactly
            }
            const int n = b * kSkBlockN + col_local;
            if (n < N) {
                const float sc = __ldg(col_scale + n);
                if (bias) {
                    const float bv = __ldcg(bias + n);
#pragma unroll
                    for (int m = 0; m < kSkRows; ++m)
                        if (m < M) y[(size_t)m * N + n] = zq_epilogue_bias((int32_t)r[m], sr[m], sc, bv);
                } else {
#pragma unroll
                    for (int m = 0; m < kSkRows; ++m)
                        if (m < M) y[(size_t)m * N + n] = zq_epilogue((int32_t)r[m], sr[m], sc);
                }
            }
        }
    } else if constexpr (kType == kInt4) {
        // Unpack: warp 6 + s owns stage s and turns its packed [128][64 B]
        // tile into the swizzled int8 [128][128 B] tile at every phase.  Lane
        // i takes 16-byte chunks i, i + 32, ...: row = chunk / 4, codes
        // 32 * (chunk % 4) .. +31 (in k order: the panel layout), which land in
        // the row's logical 16-byte chunks 2c and 2c+1, stored at physical
        // chunk (logical ^ row % 8) -- the 128-byte swizzle.  One warp per
        // stage: the generic-to-async proxy fence before each release then
        // overlaps across stages (four warps sharing every stage paid it
        // stage after stage, slower than the weight stream).  With x16 the
        // codes enter as 16 x the code and the epilogue shifts the sums back.
        const int u = warp - 6;
        uint32_t phase = 0;
        for (long long t = it0 + u; t < it1; t += S) {
            if (!mbar_wait_bounded(&full[u], phase, err, kDevErrTimeoutMma)) break;
            const uint8_t* raw = smem + u * C::kStageBytes;
            uint8_t* conv = smem + u * C::kStageBytes + C::kWBytes + C::kXBytes;
#pragma unroll 4
            for (int j = 0; j < 16; ++j) {
                const int idx = lane + 32 * j;
                const int row = idx >> 2, c = idx & 3;
                const uint4 v = *reinterpret_cast<const uint4*>(raw + idx * 16);
                uint4 lo, hi;
                if (x16)
                    zq_expand_int4x32_x16(v, lo, hi);
                else
                    zq_expand_int4x32(v, lo, hi);
                uint8_t* rp = conv + row * 128;
                const int sw = row & 7;
                *reinterpret_cast<uint4*>(rp + (((2 * c) ^ sw) << 4)) = lo;
                *reinterpret_cast<uint4*>(rp + (((2 * c + 1) ^ sw) << 4)) = hi;
            }
            // generic-proxy writes become visible to the tensor core's reads
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&conv_full[u]);
            phase ^= 1u;
        }
    }

    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                     : "memory");
    }
}

__global__ void zero_words_kernel(int* __restrict__ p, int n) {
    pdl_launch_dependents();
    pdl_wait_primary();  // the kernel before may still use the counters
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) p[i] = 0;
}

template <int kType>
cudaError_t launch_skinny_t(const SkinnyArgs& a, cudaStream_t stream, bool pdl) {
    auto kern = skinny_kernel<kType>;
    constexpr int smem = sk_smem_bytes<kType>();
    cudaError_t e = ensure_smem_attr(kern, smem);
    if (e != cudaSuccess) return e;
    const int KB = (a.Kp + kSkKBlock - 1) / kSkKBlock;
    const long long T = (long long)skinny_blocks(a.N) * KB;
    long long G = sm_count(a.reserved_sms);
    if (G > kSkinnyMaxCtas) G = kSkinnyMaxCtas;
    if (G > T) G = T;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)G);
    cfg.blockDim = dim3(SkCfg<kType>::kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, *a.tmap_w, *a.tmap_x, a.M, a.N, KB, T, a.row_scale, a.col_scale, a.bias,
                              a.y, a.counters, a.partials, a.err, a.wait_extra,
                              (unsigned long long)(a.peer_limit_ns ? a.peer_limit_ns : 4000000000ull),
                              (kType == kInt4 && int4_x16_fits(a.Kp)) ? 1 : 0);
}

}  // namespace

int skinny_blocks(int N) { return (N + kSkBlockN - 1) / kSkBlockN; }

int skinny_counter_words(int N) { return skinny_blocks(N) * 8; }

size_t skinny_scratch_bytes(int N, int M) {
    const size_t t = ((size_t)skinny_counter_words(N) * sizeof(int) + 255) / 256 * 256;
    const size_t p = ((size_t)kSkinnyMaxCtas * 2 * M * kSkBlockN * sizeof(int) + 255) / 256 * 256;
    return t + p;
}

cudaError_t launch_zero_words(int* p, int n, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const int threads = 256;
    int blocks = (n + threads - 1) / threads;
    if (blocks > 148) blocks = 148;
    return launch_pdl_kernel(zero_words_kernel, dim3(blocks), dim3(threads), 0, stream, p, n);
}

cudaError_t launch_skinny(const SkinnyArgs& a, cudaStream_t stream, bool pdl) {
    if (a.M < 1 || a.M > kSkinnyMaxRows) return cudaErrorInvalidValue;
    return a.type == kInt8 ? launch_skinny_t<kInt8>(a, stream, pdl) : launch_skinny_t<kInt4>(a, stream, pdl);
}

}  // namespace zq
