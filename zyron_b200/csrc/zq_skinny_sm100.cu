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
// respect to the prefill GEMM: A is a block of 64 weight columns (the panel
// [N][Kp] is K-major, so 64 columns are a 64-row K-major tile), B is the
// activation codes, whose TMA box of 16 rows is zero-filled past row M, and
// the TMEM accumulator is acc transposed (64 columns in lanes 0-15 of each
// 32-lane quarter, 16 TMEM columns = activation rows).
//
// One iteration is four k-blocks of one column block: a single 3-D TMA box
// of [4 k-blocks][64 columns][128 B] (32 KiB of INT8 weights).  Streaming a
// 45 MB panel in back-to-back launches measured flat at about 4.4 TB/s for
// 16-64 KiB per copy instruction, whether the box is one k-block of 128
// columns, four k-blocks of 64 or a contiguous bulk copy, the same as plain
// 16-byte loads with no ring; 8 KiB copies were much slower (2.4 TB/s for
// one k-block of 64 columns), so small copies cost per instruction, not per
// 128-byte row piece of the box.  MMAs that accumulate
// into one TMEM accumulator run one after another (about 130 ns each for
// M=64 N=16 K=32), which would make a single chain slower than the weight
// stream; so the four K=32 slices of each k-block go to four accumulators
// (independent chains) that the epilogue adds up.
//
// Work split (stream-K): the (column block, k-block) iterations are cut into
// equal contiguous ranges, one per CTA and one CTA per SM, so every SM
// streams the same number of weight bytes whatever N and K are.  A column
// block whose k-range spans several CTAs ("shared") needs one CTA to add the
// others' int32 sums (exact in any order) and apply the epilogue.  Under a
// saturated memory system each global round trip costs about a microsecond,
// so that exchange must not sit at the end of the kernel:
//   * every CTA streams its shared pieces first (the shorter one first) and
//     its whole blocks last, so the last thing most CTAs do needs no
//     exchange at all;
//   * the finisher of a shared block is the sharer whose share ends latest in
//     that order (every CTA computes the same choice).  Its epilogue warps
//     wait for the others' shares while its own MMAs still run, and add them
//     when its own accumulator lands;
//   * the other sharers publish their sums and count them (release), never
//     waiting.  A finisher whose partners are not done within a short
//     patience (their SMs taken by other work, say) publishes and counts its
//     own share as well; the share that completes the count then finishes
//     the block.  No CTA waits long for another.
// With 64-column blocks the blocks outnumber the SMs for N >= 9472, and then
// no CTA lies inside a single shared block, so every shared block has one
// early and one late share.  The counters are zeroed by the kernel launched
// just before this one (the activation quantizer, or a zeroing kernel).
//
// INT4 weights arrive as packed [4][64 columns][64 bytes] boxes; two unpack
// warps per ring stage sign-extend them into the 128-byte-swizzled int8
// tiles the MMA reads.
//
// Warps: 0 TMA producer; 1 TMEM allocator + MMA issuer; 2-5 epilogue;
// 6.. (INT4 only) unpack, two per stage.  Every mbarrier wait is bounded.
#include "zq_common.cuh"
#include "zq_kernels.h"
#include "zq_tcgen05.cuh"

#include <cuda.h>

namespace zq {

namespace {

constexpr int kSkBlockN = 64;   // weight columns per tile (MMA M)
constexpr int kSkRows = 16;     // activation rows per MMA (MMA N); rows >= M are zeros
constexpr int kSkKBlock = 128;  // codes per k-block (one 128-byte swizzle row of int8)
constexpr int kSkUmmaK = 32;
constexpr int kSkChains = kSkKBlock / kSkUmmaK;  // accumulators per block, one per K=32 slice
constexpr int kSkKGroup = 4;  // k-blocks per iteration (one TMA box)
// How long a finisher waits for its partners' shares before it counts its own
// share instead (normally they are done well before it needs them).
constexpr uint64_t kSkPatienceNs = 20000;

template <int kType>
struct SkCfg;
// Both rings take more than half of an SM's shared memory: with two CTAs
// fitting on one SM the block scheduler may stack the grid's CTAs two to an
// SM and leave others idle (a 100 KiB ring measured twice as slow).
template <>
struct SkCfg<kInt8> {
    static constexpr int kStages = 5;
    static constexpr int kThreads = 192;
    static constexpr int kWSub = kSkBlockN * kSkKBlock;      // one k-block, swizzled int8 (8 KiB)
    static constexpr int kWBytes = kWSub * kSkKGroup;         // 32 KiB
    static constexpr int kXSub = kSkRows * kSkKBlock;         // 2 KiB
    static constexpr int kXBytes = kXSub * kSkKGroup;         // 8 KiB
    static constexpr int kStageBytes = kWBytes + kXBytes;     // 40 KiB
};
template <>
struct SkCfg<kInt4> {
    static constexpr int kStages = 3;
    static constexpr int kUnpackWarps = 2 * kStages;  // two per stage, two k-blocks each
    static constexpr int kThreads = 192 + 32 * kUnpackWarps;
    static constexpr int kPSub = kSkBlockN * kSkKBlock / 2;   // one k-block, packed [64][64 B] (4 KiB)
    static constexpr int kWBytes = kPSub * kSkKGroup;         // 16 KiB
    static constexpr int kXSub = kSkRows * kSkKBlock;
    static constexpr int kXBytes = kXSub * kSkKGroup;         // 8 KiB
    static constexpr int kWSub = kSkBlockN * kSkKBlock;       // one k-block unpacked, swizzled (8 KiB)
    static constexpr int kConvBytes = kWSub * kSkKGroup;      // 32 KiB
    static constexpr int kStageBytes = kWBytes + kXBytes + kConvBytes;  // 56 KiB
};

template <int kType>
constexpr int sk_smem_bytes() {
    using C = SkCfg<kType>;
    return 1024 /*alignment slack*/ + C::kStages * C::kStageBytes + 8 * (3 * C::kStages + 5) + 16;
}
static_assert(2 * sk_smem_bytes<kInt8>() > 228 * 1024 && 2 * sk_smem_bytes<kInt4>() > 228 * 1024,
              "one decode CTA per SM");
static_assert(sk_smem_bytes<kInt8>() <= 227 * 1024 && sk_smem_bytes<kInt4>() <= 227 * 1024, "fits one SM");

// CTA g owns iterations [g*T/G, (g+1)*T/G); iteration t is k-group t % KG
// (k-blocks 4 (t % KG) .. +3) of column block t / KG.
__device__ __forceinline__ long long sk_start(int g, long long T, int G) { return (long long)g * T / G; }
// The CTA whose range holds iteration t: the largest g with g*T/G <= t.
__device__ __forceinline__ int sk_owner(long long t, long long T, int G) {
    return (int)(((t + 1) * (long long)G - 1) / T);
}

// The order in which a CTA streams its range: the pieces of the blocks it
// shares with other CTAs (at most two, the shorter first), then its whole
// blocks (one contiguous run).  Each piece is a contiguous run of
// iterations.
struct SkPlan {
    long long lo[3], hi[3];
    int n;
    long long len;
};

__device__ __forceinline__ SkPlan sk_plan(int g, long long T, int G, int KG) {
    SkPlan p;
    p.n = 0;
    const long long a = sk_start(g, T, G), b = sk_start(g + 1, T, G);
    p.len = b - a;
    if (a >= b) return p;
    const long long bf = a / KG, bl = (b - 1) / KG;
    if (bf == bl) {
        p.lo[0] = a, p.hi[0] = b, p.n = 1;
        return p;
    }
    const bool first_shared = a != bf * KG;
    const bool last_shared = b != (bl + 1) * KG;
    long long slo[2], shi[2];
    int ns = 0;
    if (first_shared) slo[ns] = a, shi[ns] = (bf + 1) * KG, ++ns;
    if (last_shared) slo[ns] = bl * KG, shi[ns] = b, ++ns;
    if (ns == 2 && shi[1] - slo[1] < shi[0] - slo[0]) {
        const long long l = slo[0], h = shi[0];
        slo[0] = slo[1], shi[0] = shi[1], slo[1] = l, shi[1] = h;
    }
    const long long w0 = first_shared ? (bf + 1) * KG : a;
    const long long w1 = last_shared ? bl * KG : b;
    if (ns == 0) {
        p.lo[0] = w0, p.hi[0] = w1, p.n = 1;
    } else if (ns == 1) {
        p.lo[0] = slo[0], p.hi[0] = shi[0], p.n = 1;
        if (w0 < w1) p.lo[1] = w0, p.hi[1] = w1, p.n = 2;
    } else {
        p.lo[0] = slo[0], p.hi[0] = shi[0], p.lo[1] = slo[1], p.hi[1] = shi[1], p.n = 2;
        if (w0 < w1) p.lo[2] = w0, p.hi[2] = w1, p.n = 3;
    }
    return p;
}

// The i-th iteration this CTA streams.
__device__ __forceinline__ long long sk_t_at(const SkPlan& p, long long i) {
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        if (j >= p.n) break;
        const long long l = p.hi[j] - p.lo[j];
        if (i < l) return p.lo[j] + i;
        i -= l;
    }
    return -1;
}

// Position (iterations streamed) at which CTA h completes its share of block
// `blk`.
__device__ __forceinline__ long long sk_share_end(int h, long long T, int G, int KG, long long blk) {
    const SkPlan p = sk_plan(h, T, G, KG);
    const long long bk0 = blk * KG, bk1 = bk0 + KG;
    long long before = 0;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        if (j >= p.n) break;
        if (p.lo[j] < bk1 && p.hi[j] > bk0) return before + ((p.hi[j] < bk1 ? p.hi[j] : bk1) - p.lo[j]);
        before += p.hi[j] - p.lo[j];
    }
    return -1;
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

__device__ __forceinline__ int atom_add_relaxed_gpu(int* p, int v) {
    int old;
    asm volatile("atom.relaxed.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Whole warp: waits until *p >= target for at most `patience_ns`; every lane
// reads with acquire semantics, so its later loads see what the writers
// published before counting.
__device__ __forceinline__ bool warp_poll_count(const int* p, int target, uint64_t patience_ns) {
    const uint64_t t0 = global_timer_ns();
    while (true) {
        const int v = ld_acquire_gpu(p);
        if (__all_sync(0xffffffffu, v >= target)) return true;
        const int give_up = global_timer_ns() - t0 > patience_ns ? 1 : 0;
        if (__shfl_sync(0xffffffffu, give_up, 0)) return false;
        __nanosleep(64);
    }
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
                  int N, int KG, long long T, const float* __restrict__ row_scale,
                  const float* __restrict__ col_scale, const float* __restrict__ bias, float* __restrict__ y,
                  int* __restrict__ counters, int* __restrict__ partials, uint32_t* __restrict__ err,
                  int wait_extra, unsigned long long peer_limit_ns, int x16) {
    using C = SkCfg<kType>;
    constexpr int S = C::kStages;
    constexpr uint32_t kTmemCols = 2 * kSkChains * kSkRows;  // two buffers of four 16-column accumulators
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
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
    const SkPlan plan = sk_plan(g, T, G, KG);
    // The next kernel on the stream may launch now (it reads nothing of ours
    // before its griddepcontrol.wait) and take over the SMs as this grid's
    // CTAs finish.
    pdl_launch_dependents();

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&conv_full[s], 2);  // the stage's two unpack warps (INT4)
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
            // Both maps are 3-D: (bytes within a k-block row, rows,
            // k-block); a box is kSkKGroup k-blocks of 64 weight columns or
            // of the 16 activation rows.
            const int pre = (int)(plan.len < S ? plan.len : S);
            for (int i = 0; i < pre; ++i) {
                const long long t = sk_t_at(plan, i);
                const int b = (int)(t / KG), kg = (int)(t % KG);
                mbar_arrive_expect_tx(&full[i], C::kWBytes + C::kXBytes);
                tma_load_3d(smem + i * C::kStageBytes, &tmap_w, &full[i], 0, b * kSkBlockN, kg * kSkKGroup);
            }
            pdl_wait_primary();
            for (int i = 0; i < pre; ++i) {
                const int kg = (int)(sk_t_at(plan, i) % KG);
                tma_load_3d(smem + i * C::kStageBytes + C::kWBytes, &tmap_x, &full[i], 0, 0, kg * kSkKGroup);
            }
            int stage = pre == S ? 0 : pre;
            uint32_t phase = pre == S ? 1u : 0u;
            uint32_t last_phase[S];
            bool issued[S];
#pragma unroll
            for (int s = 0; s < S; ++s) issued[s] = s < pre, last_phase[s] = 0;
            for (long long i = pre; i < plan.len; ++i) {
                if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, err, kDevErrTimeoutProducer)) break;
                const long long t = sk_t_at(plan, i);
                const int b = (int)(t / KG), kg = (int)(t % KG);
                uint8_t* st = smem + stage * C::kStageBytes;
                mbar_arrive_expect_tx(&full[stage], C::kWBytes + C::kXBytes);
                tma_load_3d(st, &tmap_w, &full[stage], 0, b * kSkBlockN, kg * kSkKGroup);
                tma_load_3d(st + C::kWBytes, &tmap_x, &full[stage], 0, 0, kg * kSkKGroup);
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
            long long i = 0;
            while (i < plan.len && ok) {
                const long long b = sk_t_at(plan, i) / KG;
                if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1u, err, kDevErrTimeoutMma)) break;
                tmem_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * kSkChains * kSkRows);
                bool first = true;
                for (; i < plan.len; ++i) {
                    if (sk_t_at(plan, i) / KG != b) break;
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
                    for (int j = 0; j < kSkKGroup; ++j) {
#pragma unroll
                        for (int kk = 0; kk < kSkChains; ++kk)
                            umma_i8(d + (uint32_t)(kk * kSkRows), make_sw128_desc(sa + j * C::kWSub + kk * kSkUmmaK),
                                    make_sw128_desc(sb + j * C::kXSub + kk * kSkUmmaK), idesc,
                                    (first && j == 0) ? 0u : 1u);
                    }
                    first = false;
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
        // Epilogue: warp w reads TMEM lanes (w % 4) * 32 .. +31, whose first
        // 16 hold columns (w % 4) * 16 .. +15 of the block (the M=64 data
        // path layout), all 16 activation rows per thread.
        const int q = warp & 3;
        const int col_local = q * 16 + (lane & 15);
        const bool owner_lane = lane < 16;
        // Row scales and counters are written by the kernel before this one;
        // read them only through L2 (this SM's L1 may hold older lines).
        pdl_wait_primary();
        float sr[kSkRows];
#pragma unroll
        for (int m = 0; m < kSkRows; ++m) sr[m] = m < M ? __ldcg(row_scale + m) : 0.0f;
        const int first_b = (int)(it0 / KG);
        int acc = 0;
        uint32_t acc_phase = 0;
        long long i = 0;
        while (i < plan.len) {
            const long long b = sk_t_at(plan, i) / KG;
            const long long bk0 = b * KG, bk1 = bk0 + KG;
            const long long s0 = it0 > bk0 ? it0 : bk0, s1 = it1 < bk1 ? it1 : bk1;
            i += s1 - s0;
            const bool whole = s0 == bk0 && s1 == bk1;
            int g0 = g, g1 = g;
            bool have_others = false;
            uint32_t others[kSkRows];
#pragma unroll
            for (int m = 0; m < kSkRows; ++m) others[m] = 0u;
            int* done = counters + b * 8 + q;
            if (!whole) {
                g0 = sk_owner(bk0, T, G), g1 = sk_owner(bk1 - 1, T, G);
                int fin = g0;
                long long latest = -1;
                for (int h = g0; h <= g1; ++h) {
                    const long long e = sk_share_end(h, T, G, KG, b);
                    if (e > latest) latest = e, fin = h;
                }
                if (fin == g && wait_extra == 0 && warp_poll_count(done, g1 - g0, kSkPatienceNs)) {
                    // Every other share is published: add them up while this
                    // CTA's own MMAs finish.
                    have_others = true;
                    for (int h = g0; h <= g1; ++h) {
                        if (h == g) continue;
                        const int hs = sk_start(h, T, G) / KG == b ? 0 : 1;
                        const int* p = partials + (size_t)(h * 2 + hs) * M * kSkBlockN + col_local;
#pragma unroll
                        for (int m = 0; m < kSkRows; ++m)
                            if (m < M) others[m] += (uint32_t)__ldcg(p + (size_t)m * kSkBlockN);
                    }
                }
            }
            if (!mbar_wait_bounded(&tfull[acc], acc_phase, err, kDevErrTimeoutEpilogue)) break;
            tmem_fence_after();
            uint32_t r[kSkRows];
            {
                const uint32_t ta = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * kSkChains * kSkRows);
                uint32_t r1[kSkRows];
                tmem_ld_32x32b_x16(ta, r);
                tmem_ld_32x32b_x16(ta + kSkRows, r1);
                tmem_ld_wait();
#pragma unroll
                for (int c = 2; c < kSkChains; ++c) {
#pragma unroll
                    for (int m = 0; m < kSkRows; ++m) r[m] += r1[m];  // exact int32 (mod 2^32)
                    tmem_ld_32x32b_x16(ta + c * kSkRows, r1);
                    tmem_ld_wait();
                }
#pragma unroll
                for (int m = 0; m < kSkRows; ++m) r[m] += r1[m];
            }
            tmem_fence_before();
            mbar_arrive(&tempty[acc]);
            if (++acc == 2) acc = 0, acc_phase ^= 1u;

            if (!whole) {
                if (have_others) {
#pragma unroll
                    for (int m = 0; m < kSkRows; ++m) r[m] += others[m];
                } else {
                    // Publish this CTA's exact int32 share and count it; the
                    // share that completes the count (all g1 - g0 + 1 of them)
                    // adds the others and writes the output.
                    const int slot = b == first_b ? 0 : 1;
                    int* mine = partials + (size_t)(g * 2 + slot) * M * kSkBlockN + col_local;
                    if (owner_lane) {
#pragma unroll
                        for (int m = 0; m < kSkRows; ++m)
                            if (m < M) mine[(size_t)m * kSkBlockN] = (int)r[m];
                    }
                    __syncwarp();
                    int prior = 0;
                    if (lane == 0) {
                        fence_acq_rel_gpu();  // the warp's stores, before the count
                        prior = atom_add_relaxed_gpu(done, 1);
                    }
                    prior = __shfl_sync(0xffffffffu, prior, 0);
                    if (prior != g1 - g0) continue;  // another share is still running
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
                    fence_acq_rel_gpu();  // the other shares were published before their counts
                    for (int h = g0; h <= g1; ++h) {
                        if (h == g) continue;
                        const int hs = sk_start(h, T, G) / KG == b ? 0 : 1;
                        const int* p = partials + (size_t)(h * 2 + hs) * M * kSkBlockN + col_local;
#pragma unroll
                        for (int m = 0; m < kSkRows; ++m)
                            if (m < M) r[m] += (uint32_t)__ldcg(p + (size_t)m * kSkBlockN);
                    }
                }
            }
            if (x16) {
#pragma unroll
                for (int m = 0; m < kSkRows; ++m) r[m] = (uint32_t)((int32_t)r[m] >> 4);  // 16 x the dot, exactly
            }
            const int n = (int)(b * kSkBlockN) + col_local;
            if (owner_lane && n < N) {
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
        // Unpack: warps 6 + 2s and 7 + 2s own stage s, each two of its four
        // k-blocks: every packed [64][64 B] k-block becomes the swizzled
        // int8 [64][128 B] tile the MMA reads.  Lane i takes 16-byte chunks
        // i, i + 32, ...: row = chunk / 4, codes 32 * (chunk % 4) .. +31 (in
        // k order: the panel layout), which land in the row's logical
        // 16-byte chunks 2c and 2c+1, stored at physical chunk
        // (logical ^ row % 8) -- the 128-byte swizzle.  Stages are owned,
        // not shared round-robin: the generic-to-async proxy fence before
        // each release then overlaps across warps.  With x16 the codes enter
        // as 16 x the code and the epilogue shifts the sums back.
        const int u = warp - 6;
        const int st = u >> 1, half = u & 1;
        uint32_t phase = 0;
        for (long long i = st; i < plan.len; i += S) {
            if (!mbar_wait_bounded(&full[st], phase, err, kDevErrTimeoutMma)) break;
#pragma unroll
            for (int jj = 0; jj < kSkKGroup / 2; ++jj) {
                const int kblk = half * (kSkKGroup / 2) + jj;
                const uint8_t* raw = smem + st * C::kStageBytes + kblk * C::kPSub;
                uint8_t* conv = smem + st * C::kStageBytes + C::kWBytes + C::kXBytes + kblk * C::kWSub;
#pragma unroll 4
                for (int j = 0; j < kSkBlockN * 4 / 32; ++j) {
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
            }
            // generic-proxy writes become visible to the tensor core's reads
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&conv_full[st]);
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
    const int KG = (KB + kSkKGroup - 1) / kSkKGroup;  // k-blocks past KB are zero-filled boxes
    const long long T = (long long)skinny_blocks(a.N) * KG;
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
    return cudaLaunchKernelEx(&cfg, kern, *a.tmap_w, *a.tmap_x, a.M, a.N, KG, T, a.row_scale, a.col_scale, a.bias,
                              a.y, a.counters, a.partials, a.err, a.wait_extra,
                              (unsigned long long)(a.peer_limit_ns ? a.peer_limit_ns : 4000000000ull),
                              (kType == kInt4 && int4_x16_fits(a.Kp)) ? 1 : 0);
}

}  // namespace

int skinny_block_n() { return kSkBlockN; }

int skinny_kgroup() { return kSkKGroup; }

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
