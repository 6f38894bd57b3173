// zq_gemm_sm100.cu -- prefill-sized quantized matmul on 5th-generation tensor
// cores (tcgen05, sm_100a).
//
// Computes y[m][n] = float(acc) * s_row[m] * s_col[n] (+ bias[n]) with
// acc[m][n] = sum_k q_a[m][k] * q_w[n][k] in exact int32, i.e. the dot and
// epilogue of quantization::matmul (src/quantization/quantization.cpp:
// 215-232) and QuantizedLinear's bias pass (quantized_linear.cpp:44-48).
//
// Both operands are K-major int8: the activation codes are row-major [M][Kp]
// and the weight panel is column-major [N][Kp] (one contiguous K-run per
// output column, exactly the reference's column-major storage).  So A and B
// load with the same kind of 2D TMA box and feed tcgen05.mma.kind::i8 without
// any transpose.
//
// Structure (one CTA per SM, persistent over 128 x BN output tiles):
//   warp 0      TMA producer: A box 128x128 B and B box BNx128 B per k-block,
//               128-byte swizzle, STAGES-deep ring of shared-memory buffers.
//   warp 1      TMEM allocator + MMA issuer: one thread issues
//               tcgen05.mma.cta_group::1.kind::i8 (M=128, N=BN, K=32) four
//               times per k-block into an int32 TMEM accumulator and commits
//               to the stage's "empty" barrier.
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns at a time, exact
//               fp32 rescale (+ bias), 128-bit global stores.
// Two TMEM accumulators (2 x BN columns) let the epilogue of tile i overlap
// the main loop of tile i+1.
//
// INT4 weights (kW4) stay packed in HBM and in the TMA copy.  The A boxes
// keep their own ring, as deep as the INT8 kernel's; k-block i's packed
// BNx64-byte B box goes to slot i % S (S = 4, or 5 in the 2-SM kernel without
// output staging), which also holds its unpacked 128-byte-swizzled
// BNx128-byte int8 tile.  Four more warps per slot (warps 6, 7, ...) own the
// slots: they unpack slot u's box for k-blocks u, u + S, ...,
// release the packed box to the producer and the tile to the MMA, which
// reads it with the stage's A box and frees it with a second commit.  Every
// release of a tile needs a generic-to-async proxy fence; with slots owned
// by warps, four slots' fences run at once instead of one k-block's after
// another (one group of warps taking every k-block in turn ran the tensor
// pipe at 40 %).  Each barrier has one waiting role that takes all its
// phases in order, so no parity wait can match an older phase.  The weight
// bytes crossing HBM and L2 are the packed ones; nothing is expanded in
// global memory.
//
// Every mbarrier wait is bounded (see
// mbar_wait_bounded): on timeout the kernel records an error code, drains its
// own in-flight copies and MMAs, frees TMEM and returns.
#include "zq_common.cuh"
#include "zq_kernels.h"
#include "zq_tcgen05.cuh"

#include <cuda.h>

#include <atomic>
#include <mutex>
#include <unordered_map>

namespace zq {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 128;  // bytes == int8 codes per k-block (one 128 B swizzle row)
constexpr int kUmmaK = 32;
constexpr int kThreads = 192;
constexpr int kEpilogueThreads = 128;
constexpr int kUnpackThreads = 512;  // warps 6..21 of an INT4-weight kernel (two per slot: 0.95x)
constexpr int kUnpackWarps = kUnpackThreads / 32;
constexpr int kSlots = 4;              // packed + unpacked B tiles of an INT4-weight kernel
constexpr int kSlotWarps = kUnpackWarps / kSlots;  // unpack warps per slot
template <bool kW4>
constexpr int threads_for() { return kW4 ? kThreads + kUnpackThreads : kThreads; }
// The 2-SM kernel's INT4 slots: four unpack warps each; the gathering kernel
// keeps four slots beside its epilogue staging, the plain one takes one more
// (8192 x 8192 x 16384: 2273 TOPS against 2057 with four).
constexpr int kPairSlotsGather = 4, kPairSlotsPlain = 5;
template <bool kW4, bool kGather>
constexpr int pair_slots() { return kW4 ? (kGather ? kPairSlotsGather : kPairSlotsPlain) : kSlots; }
template <bool kW4, bool kGather>
constexpr int pair_threads() { return kW4 ? kThreads + 32 * kSlotWarps * pair_slots<kW4, kGather>() : kThreads; }

// An accumulator word: the int32 dot, or (INT4 weights unpacked as 16 x the
// code, see unpack_stage) 16 x the dot, shifted back exactly.
__device__ __forceinline__ int32_t acc_of(uint32_t r, int shift) { return (int32_t)r >> shift; }

// Epilogue staging: each epilogue warp turns its 32 rows x 32 columns of
// accumulators around in shared memory so that global stores are 128-byte
// row segments (coalesced in HBM, large packets over NVLink).
constexpr int kEpiPitch = 32;  // floats per staged row; float4 slots XOR-swizzled by row
constexpr int kEpiBlockFloats = 32 * kEpiPitch;      // one staged 32 x 32 block (4 KiB)
constexpr int kEpiBytes = 4 * 2 * kEpiBlockFloats * 4;  // two blocks per epilogue warp

// TMA store of one staged 32 x 32 fp32 block (128-byte swizzle, the staging
// layout) through an output view, in a bulk group of this thread.
__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
                 "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// At most one bulk group of this thread still reading shared memory.
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
// Every bulk group of this thread complete (its global writes performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Ring stage: [A 128x128 | B BNx128 int8, swizzled] (INT8) or [A] (INT4);
// INT4 adds kSlots slots of [unpacked B BNx128, swizzled | packed B BNx64].
template <int BN, int STAGES, bool kW4>
struct Smem {
    static constexpr int kABytes = kBM * kBK;
    static constexpr int kBBytes = BN * kBK;
    static constexpr int kPBytes = BN * kBK / 2;
    static constexpr int kStageBytes = kABytes + (kW4 ? 0 : kBBytes);  // = TMA bytes per stage
    static constexpr int kSlotOffset = STAGES * kStageBytes;
    static constexpr int kSlotBytes = kBBytes + kPBytes;
    static constexpr int kSlotsBytes = kW4 ? kSlots * kSlotBytes : 0;
    // rounded to 1 KiB: the staging area after it takes 128-byte-swizzled TMA stores
    static constexpr int kBarrierBytes = (8 * (2 * STAGES + 4 * kSlots + 6) + 16 + 1023) / 1024 * 1024;
    // staging area last: it is only allocated when the output has peers
    static constexpr int kTotal = 1024 /*alignment slack*/ + kSlotOffset + kSlotsBytes + kBarrierBytes;
    static_assert(kTotal + kEpiBytes <= 227 * 1024, "shared memory of the gathering kernel");
};

// Unpack of one stage's packed INT4 tile (rows x 64 bytes of the panel
// layout, unswizzled) into the 128-byte-swizzled int8 tile (rows x 128 bytes)
// the MMA reads, by the unpack threads: 16-byte chunk i of the packed tile is row
// i / 4, codes 32 (i % 4) .. +31, which land in the row's logical 16-byte
// chunks 2 (i % 4) and 2 (i % 4) + 1, stored at physical chunk
// (logical ^ row % 8).  Eight consecutive threads cover two rows:
// conflict-free 16-byte reads and writes.
//
// scaled: the codes enter as 16 x the code (zq_expand_int4x32_x16: three
// operations per eight codes instead of nine); the MMA then accumulates
// exactly 16 x the dot, which the epilogue shifts back.  The caller uses it
// while int4_x16_fits(Kp).
template <int kRows>
__device__ __forceinline__ void unpack_stage(const uint8_t* __restrict__ packed, uint8_t* __restrict__ conv, int tid,
                                             bool scaled) {
    constexpr int kT = 32 * kSlotWarps;  // threads unpacking one slot; a multiple of 32
    static_assert(kT % 32 == 0, "");
    // Chunk tid + kT j: row tid / 4 + (kT / 4) j, column tid % 4; kT / 4 is
    // a multiple of 8, so the row's swizzle (row % 8) is the same for all j.
    const int c = tid & 3, sw = (tid >> 2) & 7;
    const uint8_t* src = packed + tid * 16;
    uint8_t* dlo = conv + (tid >> 2) * 128 + (((2 * c) ^ sw) << 4);
    uint8_t* dhi = conv + (tid >> 2) * 128 + (((2 * c + 1) ^ sw) << 4);
#pragma unroll
    for (int j = 0; j < kRows * 4 / kT; ++j) {
        const uint4 v = *reinterpret_cast<const uint4*>(src + kT * 16 * j);
        uint4 lo, hi;
        if (scaled)
            zq_expand_int4x32_x16(v, lo, hi);
        else
            zq_expand_int4x32(v, lo, hi);
        *reinterpret_cast<uint4*>(dlo + (kT / 4) * 128 * j) = lo;
        *reinterpret_cast<uint4*>(dhi + (kT / 4) * 128 * j) = hi;
    }
    // generic-proxy writes become visible to the tensor core's reads
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}



// Several destinations (other GPUs' outputs over NVLink: the all-gather
// fused into the matmul).  The warp's 32 x 32 block (lane = row row0+lane,
// registers = columns n0 .. n0+31) is rescaled, turned around in the warp's
// shared-memory stage (float4 slots XOR-swizzled by row: conflict-free
// 16-byte writes and reads) and stored so that each store instruction writes
// four rows x 128 contiguous bytes to every destination -- large NVLink
// packets instead of 16-byte ones.  Ragged blocks store element by element.
//
// With output views (out.tma) a full block leaves by TMA instead: lane 0
// stores the staged block through every destination's view and commits one
// bulk group (returns true); the caller alternates between two staging
// blocks, and the wait before staging keeps at most one group reading.
__device__ __forceinline__ bool store_block(const uint32_t (&r)[32], float* __restrict__ stage, int row0, int lane,
                                            int M, int n0, int N, float sr, const float* __restrict__ col_scale,
                                            const float* __restrict__ bias, const OutDesc& out, int shift) {
    const int row = row0 + lane;
    if (out.vec && n0 + 32 <= N) {
        if (out.tma) {
            if (lane == 0) bulk_wait_read_1();  // this staging block's previous group has been read
            __syncwarp();
        }
        const float4* cs4 = reinterpret_cast<const float4*>(col_scale + n0);
        const float4* b4 = bias ? reinterpret_cast<const float4*>(bias + n0) : nullptr;
        float4 o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float4 s4 = __ldg(cs4 + j);
            if (b4) {
                const float4 b = __ldg(b4 + j);
                o[j].x = zq_epilogue_bias(acc_of(r[4 * j + 0], shift), sr, s4.x, b.x);
                o[j].y = zq_epilogue_bias(acc_of(r[4 * j + 1], shift), sr, s4.y, b.y);
                o[j].z = zq_epilogue_bias(acc_of(r[4 * j + 2], shift), sr, s4.z, b.z);
                o[j].w = zq_epilogue_bias(acc_of(r[4 * j + 3], shift), sr, s4.w, b.w);
            } else {
                o[j].x = zq_epilogue(acc_of(r[4 * j + 0], shift), sr, s4.x);
                o[j].y = zq_epilogue(acc_of(r[4 * j + 1], shift), sr, s4.y);
                o[j].z = zq_epilogue(acc_of(r[4 * j + 2], shift), sr, s4.z);
                o[j].w = zq_epilogue(acc_of(r[4 * j + 3], shift), sr, s4.w);
            }
        }
        float4* st4 = reinterpret_cast<float4*>(stage);
#pragma unroll
        for (int j = 0; j < 8; ++j) st4[lane * 8 + (j ^ (lane & 7))] = o[j];
        if (out.tma) {
            // generic-proxy writes become visible to the TMA unit's reads
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                for (int d = 0; d < out.count; ++d) tma_store_2d(&out.map[d], stage, n0, row0);
                bulk_commit();
            }
            return true;
        }
        __syncwarp();
        const int sub = lane >> 3;  // row within a group of four
        const int q = lane & 7;     // column quad
#pragma unroll
        for (int it = 0; it < 8; ++it) {
            const int rl = it * 4 + sub;
            const int grow = row0 + rl;
            const float4 v = st4[rl * 8 + (q ^ (rl & 7))];
            if (grow < M) {
                const size_t off = (size_t)grow * (size_t)out.ldy + (size_t)out.col_offset + n0 + 4 * q;
                for (int d = 0; d < out.count; ++d) *reinterpret_cast<float4*>(out.base[d] + off) = v;
            }
        }
        __syncwarp();  // the staging area is reused by the next block
        return false;
    }
    if (row >= M) return false;
    const size_t base_off = (size_t)row * (size_t)out.ldy + (size_t)out.col_offset;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const int n = n0 + j;
        if (n < N) {
            const float sc = __ldg(col_scale + n);
            const float val =
                bias ? zq_epilogue_bias(acc_of(r[j], shift), sr, sc, __ldg(bias + n)) : zq_epilogue(acc_of(r[j], shift), sr, sc);
            for (int d = 0; d < out.count; ++d) out.base[d][base_off + n] = val;
        }
    }
    return false;
}

// One destination (the plain matmul): each thread rescales its row of the
// tile 32 columns at a time and writes them as 128 contiguous bytes
// (eight 16-byte stores; L2 merges the lines before they reach HBM).
template <int BN>
__device__ __forceinline__ void store_tile_rows(uint32_t taddr, int row, bool row_ok, int nbase, int N, float sr,
                                                const float* __restrict__ col_scale,
                                                const float* __restrict__ bias, float* __restrict__ y, bool vec_ok,
                                                int shift) {
    float* yrow = y + (size_t)(row_ok ? row : 0) * N;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + c * 32, r);
        tmem_ld_wait();
        const int n0 = nbase + c * 32;
        if (!row_ok || n0 >= N) continue;
        const float4* cs4 = reinterpret_cast<const float4*>(col_scale + n0);
        if (vec_ok && n0 + 32 <= N) {
            const float4* b4 = bias ? reinterpret_cast<const float4*>(bias + n0) : nullptr;
            float4* dst = reinterpret_cast<float4*>(yrow + n0);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 s = __ldg(cs4 + j);
                float4 o;
                if (b4) {
                    const float4 b = __ldg(b4 + j);
                    o.x = zq_epilogue_bias(acc_of(r[4 * j + 0], shift), sr, s.x, b.x);
                    o.y = zq_epilogue_bias(acc_of(r[4 * j + 1], shift), sr, s.y, b.y);
                    o.z = zq_epilogue_bias(acc_of(r[4 * j + 2], shift), sr, s.z, b.z);
                    o.w = zq_epilogue_bias(acc_of(r[4 * j + 3], shift), sr, s.w, b.w);
                } else {
                    o.x = zq_epilogue(acc_of(r[4 * j + 0], shift), sr, s.x);
                    o.y = zq_epilogue(acc_of(r[4 * j + 1], shift), sr, s.y);
                    o.z = zq_epilogue(acc_of(r[4 * j + 2], shift), sr, s.z);
                    o.w = zq_epilogue(acc_of(r[4 * j + 3], shift), sr, s.w);
                }
                dst[j] = o;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int n = n0 + j;
                if (n < N) {
                    const float sc = __ldg(col_scale + n);
                    yrow[n] = bias ? zq_epilogue_bias(acc_of(r[j], shift), sr, sc, __ldg(bias + n))
                                   : zq_epilogue(acc_of(r[j], shift), sr, sc);
                }
            }
        }
    }
}

// Tile order: groups of `group_m` M-tiles; inside a group the M-tile index
// runs fastest, then the N-tile.  The CTAs running at the same time then
// share a few A panels (activation rows) and B panels (weight columns) in L2.
__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int group_m, int& mt, int& nt) {
    const int per_group = group_m * n_tiles;
    const int g = t / per_group;
    const int first_m = g * group_m;
    const int gm = min(m_tiles - first_m, group_m);
    const int r = t - g * per_group;
    mt = first_m + r % gm;
    nt = r / gm;
}

// kGather: the output goes to several GPUs' buffers (the all-gather fused
// into the matmul).  A separate instantiation keeps the single-destination
// epilogue lean: the gather path's staging roughly doubles the epilogue
// warps' registers and costs the plain matmul about 8 % when compiled in.
template <int BN, int STAGES, bool kGather, bool kW4>
__global__ void __launch_bounds__(threads_for<kW4>(), 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   int M, int N, int Kp, const float* __restrict__ row_scale,
                   const float* __restrict__ col_scale, const float* __restrict__ bias,
                   const __grid_constant__ OutDesc out, uint32_t* __restrict__ err, int group_m, int shift) {
    using S = Smem<BN, STAGES, kW4>;
    constexpr uint32_t kTmemCols = 2 * BN;  // power of two >= 32 for BN in {64,128,256}
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
    uint8_t* stage_base = smem;
    uint8_t* slot_base = smem + S::kSlotOffset;  // INT4: [unpacked | packed] B tiles
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kSlotOffset + S::kSlotsBytes);
    float* epi_stage = reinterpret_cast<float*>(smem + S::kSlotOffset + S::kSlotsBytes + S::kBarrierBytes);
    uint64_t* full = bars;
    uint64_t* empty = bars + STAGES;
    uint64_t* tfull = bars + 2 * STAGES;
    uint64_t* tempty = bars + 2 * STAGES + 2;
    uint64_t* mma_done = bars + 2 * STAGES + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
    // INT4 slots: packed box landed (TMA) / read (unpack warps); unpacked
    // tile ready (unpack warps) / read (MMA commit)
    uint64_t* full_p = bars + 2 * STAGES + 6;
    uint64_t* p_empty = full_p + kSlots;
    uint64_t* conv_full = full_p + 2 * kSlots;
    uint64_t* conv_empty = full_p + 3 * kSlots;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int m_tiles = (M + kBM - 1) / kBM;
    const int n_tiles = (N + BN - 1) / BN;
    const int num_tiles = m_tiles * n_tiles;
    const int k_blocks = (Kp + kBK - 1) / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        if (kW4)
            for (int c = 0; c < kSlots; ++c) {
                mbar_init(&full_p[c], 1);
                mbar_init(&p_empty[c], kSlotWarps);
                mbar_init(&conv_full[c], kSlotWarps);
                mbar_init(&conv_empty[c], 1);
            }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], kEpilogueThreads);
        }
        mbar_init(mma_done, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
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

    // The activation codes and row scales come from the quantizer launched
    // just before this grid (programmatic dependent launch).
    pdl_wait_primary();

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int slot = 0;  // INT4: slot of this k-block's packed box
            uint32_t pphase = 0;
            int issued[STAGES];
            uint32_t last_phase[STAGES];
            int p_issued[kSlots];
            uint32_t p_last[kSlots];
#pragma unroll
            for (int s = 0; s < STAGES; ++s) issued[s] = 0, last_phase[s] = 0;
#pragma unroll
            for (int s = 0; s < kSlots; ++s) p_issued[s] = 0, p_last[s] = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                int mt, nt;
                tile_coords(t, m_tiles, n_tiles, group_m, mt, nt);
                for (int kb = 0; kb < k_blocks; ++kb) {
                    if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, err, kDevErrTimeoutProducer) ||
                        (kW4 && !mbar_wait_bounded(&p_empty[slot], pphase ^ 1u, err, kDevErrTimeoutProducer))) {
                        ok = false;
                        break;
                    }
                    uint8_t* sa = stage_base + stage * S::kStageBytes;
                    mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
                    tma_load_2d(sa, &tmap_a, &full[stage], kb * kBK, mt * kBM);
                    if (kW4) {
                        mbar_arrive_expect_tx(&full_p[slot], S::kPBytes);
                        tma_load_2d(slot_base + slot * S::kSlotBytes + S::kBBytes, &tmap_b, &full_p[slot],
                                    kb * (kBK / 2), nt * BN);
                        p_issued[slot] = 1;
                        p_last[slot] = pphase;
                        if (++slot == kSlots) slot = 0, pphase ^= 1u;
                    } else {
                        tma_load_2d(sa + S::kABytes, &tmap_b, &full[stage], kb * kBK, nt * BN);
                    }
                    issued[stage] = 1;
                    last_phase[stage] = phase;
                    if (++stage == STAGES) stage = 0, phase ^= 1u;
                }
            }
            // Drain: every copy this thread issued must land before the CTA
            // can exit (on the normal path these waits return at once).
            for (int s = 0; s < STAGES; ++s)
                if (issued[s]) mbar_drain_bounded(&full[s], last_phase[s], err, kDevErrTimeoutDrain);
            for (int s = 0; s < kSlots; ++s)
                if (p_issued[s]) mbar_drain_bounded(&full_p[s], p_last[s], err, kDevErrTimeoutDrain);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(kBM, BN);
            int stage = 0;
            uint32_t phase = 0;
            int slot = 0;  // INT4: slot of this k-block's unpacked tile
            uint32_t cphase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1u, err, kDevErrTimeoutMma)) break;
                tmem_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * BN);
                for (int kb = 0; kb < k_blocks; ++kb) {
                    if (!mbar_wait_bounded(&full[stage], phase, err, kDevErrTimeoutMma) ||
                        (kW4 && !mbar_wait_bounded(&conv_full[slot], cphase, err, kDevErrTimeoutMma))) {
                        ok = false;
                        break;
                    }
                    tmem_fence_after();
                    const uint32_t sa = smem_u32(stage_base + stage * S::kStageBytes);
                    const uint32_t sb = kW4 ? smem_u32(slot_base + slot * S::kSlotBytes) : sa + S::kABytes;
#pragma unroll
                    for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
                        umma_i8(d, make_sw128_desc(sa + kk * kUmmaK), make_sw128_desc(sb + kk * kUmmaK), idesc,
                                (kb > 0 || kk > 0) ? 1u : 0u);
                    }
                    umma_commit(&empty[stage]);
                    if (kW4) {
                        umma_commit(&conv_empty[slot]);
                        if (++slot == kSlots) slot = 0, cphase ^= 1u;
                    }
                    if (++stage == STAGES) stage = 0, phase ^= 1u;
                }
                if (!ok) break;
                umma_commit(&tfull[acc]);
                if (++acc == 2) acc = 0, acc_phase ^= 1u;
            }
            // All MMAs issued by this thread complete before TMEM is freed.
            umma_commit(mma_done);
            mbar_drain_bounded(mma_done, 0, err, kDevErrTimeoutDrain);
        }
    } else if (kW4 && warp >= 6) {
        // Unpack warps 6 + 4u .. 9 + 4u own slot u: k-blocks u, u + 4, ...
        const int u = (warp - 6) / kSlotWarps;  // the slot's warps are consecutive: different sub-partitions
        const int tid = ((warp - 6) % kSlotWarps) * 32 + lane;  // within the slot's warps
        uint8_t* conv = slot_base + u * S::kSlotBytes;
        uint32_t ph = 0;
        const long long total =
            (long long)((num_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x) * k_blocks;
        for (long long it = u; it < total; it += kSlots) {
            if (!mbar_wait_bounded(&full_p[u], ph, err, kDevErrTimeoutMma) ||
                !mbar_wait_bounded(&conv_empty[u], ph ^ 1u, err, kDevErrTimeoutMma))
                break;
            unpack_stage<BN>(conv + S::kBBytes, conv, tid, shift != 0);
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&p_empty[u]);
                mbar_arrive(&conv_full[u]);
            }
            ph ^= 1u;
        }
    } else {
        // Epilogue warps 2..5 own TMEM lane quarters (warp % 4) * 32.
        const int quarter = warp & 3;
        int acc = 0;
        uint32_t acc_phase = 0;
        const bool vec1 = out.vec != 0;
        int nb = 0;  // bulk groups this warp committed (gathering epilogue, output views)
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            int mt, nt;
            tile_coords(t, m_tiles, n_tiles, group_m, mt, nt);
            if (!mbar_wait_bounded(&tfull[acc], acc_phase, err, kDevErrTimeoutEpilogue)) break;
            tmem_fence_after();
            const int row0 = mt * kBM + quarter * 32;
            const int row = row0 + lane;
            const float sr = row < M ? __ldg(row_scale + row) : 0.0f;
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
            if constexpr (!kGather) {
                store_tile_rows<BN>(taddr, row, row < M, nt * BN, N, sr, col_scale, bias, out.base[0], vec1, shift);
            } else {
                float* stage = epi_stage + quarter * 2 * kEpiBlockFloats;  // this warp's two staging blocks
#pragma unroll 1
                for (int c = 0; c < BN / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(taddr + c * 32, r);
                    tmem_ld_wait();
                    const int n0 = nt * BN + c * 32;
                    if (row0 < M && n0 < N &&
                        store_block(r, stage + (nb & 1) * kEpiBlockFloats, row0, lane, M, n0, N, sr, col_scale, bias,
                                    out, shift))
                        ++nb;
                }
            }
            tmem_fence_before();
            mbar_arrive(&tempty[acc]);
            if (++acc == 2) acc = 0, acc_phase ^= 1u;
        }
    }

    if (kGather && warp >= 2 && lane == 0) bulk_wait_all();  // this thread's TMA stores complete
    if (kGather && warp >= 2) __threadfence_system();  // peer stores performed before the grid ends
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                     : "memory");
    }
}

// Anything but one dense [M, N] output (several destinations, a row pitch
// wider than N, a column offset) takes the staged general epilogue.
bool general_output(const GemmArgs& a) {
    return a.out.count != 1 || a.out.ldy != (long long)a.N || a.out.col_offset != 0;
}

template <int BN, int STAGES, bool kW4>
cudaError_t launch_gemm_t(const GemmArgs& a, cudaStream_t stream, bool pdl) {
    using S = Smem<BN, STAGES, kW4>;
    const bool gather = general_output(a);
    auto kern = gather ? gemm_i8_kernel<BN, STAGES, true, kW4> : gemm_i8_kernel<BN, STAGES, false, kW4>;
    const int smem = S::kTotal + (gather ? kEpiBytes : 0);
    cudaError_t e = ensure_smem_attr(kern, smem);
    if (e != cudaSuccess) return e;
    const int sms = sm_count(a.reserved_sms);
    const int tiles = ((a.M + kBM - 1) / kBM) * ((a.N + BN - 1) / BN);
    const int grid = tiles < sms ? tiles : sms;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads_for<kW4>());
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const int m_tiles = (a.M + kBM - 1) / kBM;
    int group_m = a.group_m > 0 ? a.group_m : m_tiles;
    if (group_m > m_tiles) group_m = m_tiles;
    // INT4: codes unpacked as 16 x the code while 16 x Kp products fit in an
    // int32 accumulator even for the extreme codes -128 and -8 (16 x 128 x 8
    // x 131040 < 2^31), exact sign extension beyond
    const int shift = kW4 && int4_x16_fits(a.Kp) ? 4 : 0;
    return cudaLaunchKernelEx(&cfg, kern, *a.tmap_a, *a.tmap_b, a.M, a.N, a.Kp, a.row_scale, a.col_scale, a.bias,
                              a.out, a.err, group_m, shift);
}


// ===========================================================================
// 2-SM variant for large problems: a cluster of two CTAs on two SMs computes
// a 256 x 256 output tile with tcgen05.mma.cta_group::2 (M = 256).  Each CTA
// loads its own 128 activation rows and its own half (128 weight columns) of
// the tile's B operand, so an SM fills 32 KiB of shared memory per k-block
// instead of 48 KiB and six stages fit -- more bytes in flight against L2 and
// DRAM latency, a third less L2 -> SM traffic.  The even CTA (leader) issues
// the MMAs; its commits arrive on both CTAs' barriers (CTA mask 0b11).  Each
// CTA's accumulator rows live in its own TMEM, so the epilogue is unchanged.
//
// INT4 weights: the A boxes keep the pair's ring on the leader's barriers;
// each CTA lands its packed 128x64-byte B box in slot i % 4 on its own
// barrier, its slot-owning unpack warps write the swizzled int8 tile next to
// it and arrive on the leader's `conv_full` barrier across the cluster; the
// leader's MMA issuer waits there for both CTAs' tiles, and its commits free
// the tile (`conv_empty`) in both CTAs.
// ===========================================================================
template <bool kW4, bool kGather>
struct Smem2 {
    static constexpr int kSlotsN = pair_slots<kW4, kGather>();
    static constexpr int kStages = 6;
    static constexpr int kABytes = 128 * kBK;  // this CTA's 128 rows of A
    static constexpr int kBBytes = 128 * kBK;  // this CTA's 128 rows (columns of W) of B, int8 swizzled
    static constexpr int kPBytes = 128 * kBK / 2;  // packed INT4 B box
    static constexpr int kStageBytes = kABytes + (kW4 ? 0 : kBBytes);  // = TMA bytes per stage and CTA
    static constexpr int kSlotOffset = kStages * kStageBytes;
    static constexpr int kSlotBytes = kBBytes + kPBytes;
    static constexpr int kSlotsBytes = kW4 ? kSlotsN * kSlotBytes : 0;
    static constexpr int kBarrierBytes = (8 * (2 * kStages + 4 * kSlotsN + 6) + 16 + 1023) / 1024 * 1024;
    static constexpr int kTotal = 1024 + kSlotOffset + kSlotsBytes + kBarrierBytes;
    static_assert(kTotal + (kGather ? kEpiBytes : 0) <= 227 * 1024, "shared memory of the 2-SM kernel");
};


__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// TMA load whose completion bytes count on the pair leader's barrier.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const void* tmap, uint64_t* bar_local, int x, int y) {
    const uint32_t bar = smem_u32(bar_local) & 0xFEFFFFFFu;  // peer bit cleared: the leader's copy of `bar`
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void umma_i8_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Completion of this thread's MMAs arrives on `bar` in both CTAs of the pair.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"((uint16_t)0x3)
        : "memory");
}

template <bool kGather, bool kW4>
__global__ void __launch_bounds__((pair_threads<kW4, kGather>()), 1)
    gemm_i8_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                        int M, int N, int Kp, const float* __restrict__ row_scale,
                        const float* __restrict__ col_scale, const float* __restrict__ bias,
                        const __grid_constant__ OutDesc out, uint32_t* __restrict__ err, int group_m, int shift) {
    using S = Smem2<kW4, kGather>;
    constexpr int kPS = S::kSlotsN;
    constexpr int kStages2 = S::kStages;
    constexpr uint32_t kTmemCols = 512;  // two 256-column accumulators
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
    uint8_t* stage_base = smem;
    uint8_t* slot_base = smem + S::kSlotOffset;  // INT4: [unpacked | packed] B tiles
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kSlotOffset + S::kSlotsBytes);
    float* epi_stage = reinterpret_cast<float*>(smem + S::kSlotOffset + S::kSlotsBytes + S::kBarrierBytes);
    uint64_t* full = bars;                       // INT8: leader's copy used; INT4: each CTA's own
    uint64_t* empty = bars + kStages2;           // both copies used
    uint64_t* tfull = bars + 2 * kStages2;       // both copies used
    uint64_t* tempty = bars + 2 * kStages2 + 2;  // leader's copy used
    uint64_t* mma_done = bars + 2 * kStages2 + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages2 + 5);
    // INT4 slots: packed box landed (own TMA) / read (own unpack warps);
    // unpacked tiles ready (leader's copy, both CTAs' unpack warps) / read
    // (MMA commit, both copies)
    uint64_t* full_p = bars + 2 * kStages2 + 6;
    uint64_t* p_empty = full_p + kPS;
    uint64_t* conv_full = full_p + 2 * kPS;
    uint64_t* conv_empty = full_p + 3 * kPS;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int m_tiles = (M + 255) / 256;
    const int n_tiles = (N + 255) / 256;
    const int num_tiles = m_tiles * n_tiles;
    const int k_blocks = (Kp + kBK - 1) / kBK;
    const int cluster = blockIdx.x >> 1;
    const int clusters = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages2; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        if (kW4)
            for (int c = 0; c < kPS; ++c) {
                mbar_init(&full_p[c], 1);
                mbar_init(&p_empty[c], kSlotWarps);
                mbar_init(&conv_full[c], 2 * kSlotWarps);  // both CTAs' slot warps
                mbar_init(&conv_empty[c], 1);
            }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 2 * kEpilogueThreads);  // both CTAs' epilogue threads
        }
        mbar_init(mma_done, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tmem_fence_before();
    cluster_sync_all();  // barriers initialised and TMEM allocated in both CTAs
    tmem_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait_primary();

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int slot = 0;  // INT4: slot of this k-block's packed box
            uint32_t pphase = 0;
            int issued[kStages2];
            uint32_t last_phase[kStages2];
            int p_issued[kPS];
            uint32_t p_last[kPS];
#pragma unroll
            for (int s = 0; s < kStages2; ++s) issued[s] = 0, last_phase[s] = 0;
#pragma unroll
            for (int s = 0; s < kPS; ++s) p_issued[s] = 0, p_last[s] = 0;
            bool ok = true;
            for (int t = cluster; t < num_tiles && ok; t += clusters) {
                int mt, nt;
                tile_coords(t, m_tiles, n_tiles, group_m, mt, nt);
                for (int kb = 0; kb < k_blocks; ++kb) {
                    if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, err, kDevErrTimeoutProducer) ||
                        (kW4 && !mbar_wait_bounded(&p_empty[slot], pphase ^ 1u, err, kDevErrTimeoutProducer))) {
                        ok = false;
                        break;
                    }
                    uint8_t* sa = stage_base + stage * S::kStageBytes;
                    // the leader expects both CTAs' A (and INT8 B) bytes on its barrier
                    if (leader) mbar_arrive_expect_tx(&full[stage], 2 * S::kStageBytes);
                    tma_load_2d_pair(sa, &tmap_a, &full[stage], kb * kBK, mt * 256 + (int)rank * 128);
                    if (kW4) {
                        // own barrier: this CTA's unpack warps wait for it
                        mbar_arrive_expect_tx(&full_p[slot], S::kPBytes);
                        tma_load_2d(slot_base + slot * S::kSlotBytes + S::kBBytes, &tmap_b, &full_p[slot],
                                    kb * (kBK / 2), nt * 256 + (int)rank * 128);
                        p_issued[slot] = 1;
                        p_last[slot] = pphase;
                        if (++slot == kPS) slot = 0, pphase ^= 1u;
                    } else {
                        tma_load_2d_pair(sa + S::kABytes, &tmap_b, &full[stage], kb * kBK,
                                         nt * 256 + (int)rank * 128);
                    }
                    issued[stage] = 1;
                    last_phase[stage] = phase;
                    if (++stage == kStages2) stage = 0, phase ^= 1u;
                }
            }
            // Drain: the leader can see every copy of the pair complete on its
            // full barriers; the peer's copies land before the leader's MMAs
            // release the stage (empty), so the peer waits on empty instead.
            // Packed INT4 boxes land on each CTA's own barriers.
            for (int s = 0; s < kStages2; ++s) {
                if (!issued[s]) continue;
                if (leader)
                    mbar_drain_bounded(&full[s], last_phase[s], err, kDevErrTimeoutDrain);
                else
                    mbar_drain_bounded(&empty[s], last_phase[s], err, kDevErrTimeoutDrain);
            }
            for (int s = 0; s < kPS; ++s)
                if (p_issued[s]) mbar_drain_bounded(&full_p[s], p_last[s], err, kDevErrTimeoutDrain);
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = idesc_i8(256, 256);
            int stage = 0;
            uint32_t phase = 0;
            int slot = 0;  // INT4: slot of this k-block's unpacked tiles
            uint32_t cphase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int t = cluster; t < num_tiles && ok; t += clusters) {
                if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1u, err, kDevErrTimeoutMma)) break;
                tmem_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * 256);
                for (int kb = 0; kb < k_blocks; ++kb) {
                    if (!mbar_wait_bounded(&full[stage], phase, err, kDevErrTimeoutMma) ||
                        (kW4 && !mbar_wait_bounded_cluster(&conv_full[slot], cphase, err, kDevErrTimeoutMma))) {
                        ok = false;
                        break;
                    }
                    tmem_fence_after();
                    const uint32_t sa = smem_u32(stage_base + stage * S::kStageBytes);
                    const uint32_t sb = kW4 ? smem_u32(slot_base + slot * S::kSlotBytes) : sa + S::kABytes;
#pragma unroll
                    for (int kk = 0; kk < kBK / kUmmaK; ++kk)
                        umma_i8_pair(d, make_sw128_desc(sa + kk * kUmmaK), make_sw128_desc(sb + kk * kUmmaK), idesc,
                                     (kb > 0 || kk > 0) ? 1u : 0u);
                    umma_commit_pair(&empty[stage]);
                    if (kW4) {
                        umma_commit_pair(&conv_empty[slot]);
                        if (++slot == kPS) slot = 0, cphase ^= 1u;
                    }
                    if (++stage == kStages2) stage = 0, phase ^= 1u;
                }
                if (!ok) break;
                umma_commit_pair(&tfull[acc]);
                if (++acc == 2) acc = 0, acc_phase ^= 1u;
            }
            umma_commit_pair(mma_done);
            mbar_drain_bounded(mma_done, 0, err, kDevErrTimeoutDrain);
        } else if (lane == 0) {
            // peer: its TMEM is written by the leader's MMAs; wait for them to
            // finish before the final barrier frees TMEM
            mbar_drain_bounded(mma_done, 0, err, kDevErrTimeoutDrain);
        }
    } else if (kW4 && warp >= 6) {
        // Unpack warps 6 + 4u .. 9 + 4u (both CTAs) own slot u: this CTA's
        // tiles of k-blocks u, u + 4, ..., announced on the leader's barrier.
        const int u = (warp - 6) / kSlotWarps;  // the slot's warps are consecutive: different sub-partitions
        const int tid = ((warp - 6) % kSlotWarps) * 32 + lane;  // within the slot's warps
        uint8_t* conv = slot_base + u * S::kSlotBytes;
        const uint32_t conv_leader = map_to_rank(&conv_full[u], 0);
        uint32_t ph = 0;
        const long long total = (long long)((num_tiles - cluster + clusters - 1) / clusters) * k_blocks;
        for (long long it = u; it < total; it += kPS) {
            if (!mbar_wait_bounded(&full_p[u], ph, err, kDevErrTimeoutMma) ||
                !mbar_wait_bounded(&conv_empty[u], ph ^ 1u, err, kDevErrTimeoutMma))
                break;
            unpack_stage<128>(conv + S::kBBytes, conv, tid, shift != 0);
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&p_empty[u]);
                mbar_arrive_cluster(conv_leader);
            }
            ph ^= 1u;
        }
    } else {
        const int quarter = warp & 3;
        const uint32_t tempty_leader = map_to_rank(&tempty[0], 0);
        int acc = 0;
        uint32_t acc_phase = 0;
        const bool vec1 = out.vec != 0;
        int nb = 0;  // bulk groups this warp committed (gathering epilogue, output views)
        for (int t = cluster; t < num_tiles; t += clusters) {
            int mt, nt;
            tile_coords(t, m_tiles, n_tiles, group_m, mt, nt);
            if (!mbar_wait_bounded(&tfull[acc], acc_phase, err, kDevErrTimeoutEpilogue)) break;
            tmem_fence_after();
            const int row0 = mt * 256 + (int)rank * 128 + quarter * 32;
            const int row = row0 + lane;
            const float sr = row < M ? __ldg(row_scale + row) : 0.0f;
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * 256);
            if constexpr (!kGather) {
                store_tile_rows<256>(taddr, row, row < M, nt * 256, N, sr, col_scale, bias, out.base[0], vec1, shift);
            } else {
                float* stage = epi_stage + quarter * 2 * kEpiBlockFloats;  // this warp's two staging blocks
#pragma unroll 1
                for (int c = 0; c < 256 / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(taddr + c * 32, r);
                    tmem_ld_wait();
                    const int n0 = nt * 256 + c * 32;
                    if (row0 < M && n0 < N &&
                        store_block(r, stage + (nb & 1) * kEpiBlockFloats, row0, lane, M, n0, N, sr, col_scale, bias,
                                    out, shift))
                        ++nb;
                }
            }
            tmem_fence_before();
            mbar_arrive_cluster(tempty_leader + (uint32_t)(acc * sizeof(uint64_t)));
            if (++acc == 2) acc = 0, acc_phase ^= 1u;
        }
    }

    if (kGather && warp >= 2 && lane == 0) bulk_wait_all();  // this thread's TMA stores complete
    if (kGather && warp >= 2) __threadfence_system();  // peer stores performed before the grid ends
    tmem_fence_before();
    cluster_sync_all();  // no CTA leaves while its peer may still signal its barriers
    tmem_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                     : "memory");
    }
}

template <bool kW4>
cudaError_t launch_gemm_pair(const GemmArgs& a, cudaStream_t stream, bool pdl) {
    const bool gather = general_output(a);
    auto kern = gather ? gemm_i8_pair_kernel<true, kW4> : gemm_i8_pair_kernel<false, kW4>;
    const int smem = gather ? Smem2<kW4, true>::kTotal + kEpiBytes : Smem2<kW4, false>::kTotal;
    cudaError_t e = ensure_smem_attr(kern, smem);
    if (e != cudaSuccess) return e;
    const int sms = sm_count(a.reserved_sms);
    const int tiles = ((a.M + 255) / 256) * ((a.N + 255) / 256);
    int clusters = sms / 2;
    if (clusters < 1) clusters = 1;
    if (clusters > tiles) clusters = tiles;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters);
    cfg.blockDim = dim3(gather ? pair_threads<kW4, true>() : pair_threads<kW4, false>());
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const int m_tiles = (a.M + 255) / 256;
    int group_m = a.group_m > 0 ? (a.group_m + 1) / 2 : m_tiles;  // group size in 256-row tiles
    if (group_m > m_tiles) group_m = m_tiles;
    if (group_m < 1) group_m = 1;
    // INT4: codes unpacked as 16 x the code while 16 x Kp products fit in an
    // int32 accumulator even for the extreme codes -128 and -8 (16 x 128 x 8
    // x 131040 < 2^31), exact sign extension beyond
    const int shift = kW4 && int4_x16_fits(a.Kp) ? 4 : 0;
    return cudaLaunchKernelEx(&cfg, kern, *a.tmap_a, *a.tmap_b, a.M, a.N, a.Kp, a.row_scale, a.col_scale, a.bias,
                              a.out, a.err, group_m, shift);
}

}  // namespace

cudaError_t ensure_smem_attr_ptr(const void* kern, size_t bytes) {
    static std::mutex mu;
    static std::unordered_map<const void*, size_t> done;
    std::lock_guard<std::mutex> lk(mu);
    auto it = done.find(kern);
    if (it != done.end() && it->second >= bytes) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) done[kern] = bytes;
    return e;
}

int sm_count(int reserved) {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    int sms = 148;
    if (dev >= 0 && dev < 64) {
        if (!cached[dev]) {
            int n = 0;
            cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
            cached[dev] = n > 0 ? n : 148;
        }
        sms = cached[dev];
    }
    const int avail = sms - (reserved > 0 ? reserved : 0);
    return avail >= 2 ? avail : 2;
}

int gemm_block_n(int M, int N) {
    // 2-SM 256 x 256 tiles when there are at least two per SM pair;
    // otherwise wide 1-SM tiles when there are enough of them to fill the
    // GPU, and narrower tiles to spread small problems over more SMs.
    const long pair_tiles = (long)((M + 255) / 256) * ((N + 255) / 256);
    if (pair_tiles >= 148) return kPairBlockN;
    const long tiles256 = (long)((M + kBM - 1) / kBM) * ((N + 255) / 256);
    if (tiles256 >= 148) return 256;
    const long tiles128 = (long)((M + kBM - 1) / kBM) * ((N + 127) / 128);
    if (tiles128 >= 148) return 128;
    return 64;
}

cudaError_t launch_gemm(const GemmArgs& a, cudaStream_t stream, bool pdl) {
    if (a.w4) {
        // INT4: 16 KiB A stages plus four 24 / 12 KiB slots; a 256-column
        // tile's slots would leave too shallow an A ring
        if (a.block_n == kPairBlockN) return launch_gemm_pair<true>(a, stream, pdl);
        switch (a.block_n) {
            case 128: return launch_gemm_t<128, 6, true>(a, stream, pdl);
            case 64: return launch_gemm_t<64, 8, true>(a, stream, pdl);
            default: return cudaErrorInvalidValue;
        }
    }
    if (a.block_n == kPairBlockN) return launch_gemm_pair<false>(a, stream, pdl);
    switch (a.block_n) {
        case 256: return launch_gemm_t<256, 4, false>(a, stream, pdl);
        case 128: return launch_gemm_t<128, 6, false>(a, stream, pdl);
        case 64: return launch_gemm_t<64, 8, false>(a, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace zq
