// zq_common.cuh -- shared device helpers for the B200 quantized matmul path.
//
// Exact-arithmetic rules (the reference computes on an x86-64 CPU in IEEE
// fp32; see src/quantization/quantization.cpp:45-50, 202-212, 231-232):
//   * divisions use __fdiv_rn (correctly rounded, no fast-math),
//   * lround() is round-half-away-from-zero -> roundf(),
//   * the epilogue float(acc) * s_row * s_col (+ bias) is three separately
//     rounded operations -> __int2float_rn / __fmul_rn / __fadd_rn, never an
//     FMA.
// The library is compiled without --use_fast_math and with denormals kept.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace zq {

// Weight types; numerically identical to zyron::quantization::Type
// (include/zyron/quantization/quantization.hpp:13-16).
enum : int { kInt8 = 1, kInt4 = 2 };

// Device-side error codes written into the per-device error word when a
// bounded wait gives up.  The host reads and clears it with
// zq_device_error().
enum : uint32_t {
    kDevErrNone = 0,
    kDevErrTimeoutProducer = 1,
    kDevErrTimeoutMma = 2,
    kDevErrTimeoutEpilogue = 3,
    kDevErrTimeoutDrain = 4,
    kDevErrTimeoutPeer = 5,  // a CTA waited for another CTA's partial sums
};

// ---------------------------------------------------------------------------
// Exact scalar arithmetic shared by every kernel
// ---------------------------------------------------------------------------

// Row / column scale: absmax / limit when absmax > 0, else 1.0
// (quantization.cpp:147-148, 209).
__device__ __forceinline__ float zq_scale_from_absmax(float absmax, float limit) {
    return absmax > 0.0f ? __fdiv_rn(absmax, limit) : 1.0f;
}

// quantize_value (quantization.cpp:45-50).  A NaN quotient follows the x86-64
// lround() result (LONG_MIN), which the clamp maps to -limit.
__device__ __forceinline__ int zq_quantize_value(float v, float scale, int limit) {
    if (!(scale > 0.0f) || isinf(scale)) return 0;  // scale <= 0, NaN or inf
    const float t = __fdiv_rn(v, scale);
    if (isnan(t)) return -limit;
    const float r = roundf(t);  // half away from zero, exact for |t| < 2^23
    if (r >= (float)limit) return limit;
    if (r <= (float)-limit) return -limit;
    return (int)r;
}

// The row's reciprocal for zq_quantize_value_rcp: 1 / scale rounded to
// nearest, or 0 when zq_quantize_value returns 0 for every value of the row.
__device__ __forceinline__ float zq_quant_rcp(float scale) {
    return (!(scale > 0.0f) || isinf(scale)) ? 0.0f : __frcp_rn(scale);
}

// zq_quantize_value(v, scale, limit) with one multiply in the common case.
// y = v * rcp (rcp = 1/scale rounded) is within |q| * (2^-23 + 2^-48) of the
// exact quotient q = v / scale, and the correctly rounded quotient within
// |q| * 2^-24 of q: for |q| <= 128 the two lie within 2.3e-5 of each other.
// So rounding y half away from zero gives the same integer whenever y is
// more than 1e-4 from a half-integer and below the clamp; every other value
// (near a tie, at or past the clamp, NaN, inf, or rcp == 0) takes the exact
// division.
__device__ __forceinline__ int zq_quantize_value_rcp(float v, float scale, float rcp, int limit) {
    const float y = __fmul_rn(v, rcp);
    const float ay = fabsf(y);
    if (rcp != 0.0f && ay < (float)limit + 0.4f) {  // false for NaN
        const float f = ay - floorf(ay);             // exact: ay < 2^23
        if (fabsf(f - 0.5f) > 1.0e-4f) return (int)roundf(y);
    }
    return zq_quantize_value(v, scale, limit);
}

// NaN bit patterns of the reference's x86-64 SSE arithmetic: an invalid
// operation (0 * inf, inf - inf) yields the "default NaN" 0xFFC00000, and a
// NaN operand propagates its own payload, quieted (the first operand's when
// both are NaN).  The GPU's canonical NaN differs, so every place where the
// reference can produce a NaN restates this rule to stay bit-identical.
constexpr uint32_t kX86DefaultNaN = 0xFFC00000u;

__device__ __forceinline__ float x86_mul(float a, float b) {
    const float r = __fmul_rn(a, b);
    if (!isnan(r)) return r;
    if (isnan(a)) return __uint_as_float(__float_as_uint(a) | 0x00400000u);
    if (isnan(b)) return __uint_as_float(__float_as_uint(b) | 0x00400000u);
    return __uint_as_float(kX86DefaultNaN);
}

__device__ __forceinline__ float x86_add(float a, float b) {
    const float r = __fadd_rn(a, b);
    if (!isnan(r)) return r;
    if (isnan(a)) return __uint_as_float(__float_as_uint(a) | 0x00400000u);
    if (isnan(b)) return __uint_as_float(__float_as_uint(b) | 0x00400000u);
    return __uint_as_float(kX86DefaultNaN);
}

// y = float(acc) * s_row * s_col, evaluated left to right (quantization.cpp:231-232).
__device__ __forceinline__ float zq_epilogue(int32_t acc, float s_row, float s_col) {
    return x86_mul(x86_mul(__int2float_rn(acc), s_row), s_col);
}

// + bias as the separate pass of QuantizedLinear::forward (quantized_linear.cpp:44-48).
__device__ __forceinline__ float zq_epilogue_bias(int32_t acc, float s_row, float s_col, float b) {
    return x86_add(zq_epilogue(acc, s_row, s_col), b);
}

// Device INT4 panel layout: a column's codes in groups of eight (four
// bytes); byte j of group g holds code 8g + j in its low nibble and code
// 8g + j + 4 in its high nibble.  A 32-bit word of the panel therefore holds
// codes 0..3 of its group in its low nibbles and codes 4..7 in its high
// nibbles, both in k order, so unpacking needs no byte shuffles.
__host__ __device__ __forceinline__ int panel_int4_byte(int k) { return ((k >> 3) << 2) | (k & 3); }
__host__ __device__ __forceinline__ int panel_int4_shift(int k) { return k & 4; }  // 0: low nibble, 4: high

// 8 codes of a panel word -> int8 codes: k 0..3 in `lo4`, 4..7 in `hi4`,
// sign-extended (v | ((v & 8) * 0x1E) per byte sets the high nibble to 0xF
// for negatives).
__device__ __forceinline__ void zq_unpack_int4x8(uint32_t w, uint32_t& lo4, uint32_t& hi4) {
    const uint32_t lo = w & 0x0F0F0F0Fu;
    const uint32_t hi = (w >> 4) & 0x0F0F0F0Fu;
    lo4 = lo | ((lo & 0x08080808u) * 0x1Eu);
    hi4 = hi | ((hi & 0x08080808u) * 0x1Eu);
}

// The same as 16 x the codes: a nibble moved to the top of its byte, read as
// int8, is exactly 16 times its signed value.  Three operations instead of
// nine; a dot over such codes is 16 times the dot (exact while it fits in
// int32), so callers shift it back by 4.
__device__ __forceinline__ void zq_unpack_int4x8_x16(uint32_t w, uint32_t& lo4, uint32_t& hi4) {
    lo4 = (w << 4) & 0xF0F0F0F0u;
    hi4 = w & 0xF0F0F0F0u;
}

// 32 codes (16 panel bytes) -> int8 codes in k order: 0..15 in `lo`, 16..31
// in `hi`.
__device__ __forceinline__ void zq_expand_int4x32(const uint4& w, uint4& lo, uint4& hi) {
    zq_unpack_int4x8(w.x, lo.x, lo.y);
    zq_unpack_int4x8(w.y, lo.z, lo.w);
    zq_unpack_int4x8(w.z, hi.x, hi.y);
    zq_unpack_int4x8(w.w, hi.z, hi.w);
}
__device__ __forceinline__ void zq_expand_int4x32_x16(const uint4& w, uint4& lo, uint4& hi) {
    zq_unpack_int4x8_x16(w.x, lo.x, lo.y);
    zq_unpack_int4x8_x16(w.y, lo.z, lo.w);
    zq_unpack_int4x8_x16(w.z, hi.x, hi.y);
    zq_unpack_int4x8_x16(w.w, hi.z, hi.w);
}

// A dot over codes unpacked as 16 x the code fits in int32 when
// 16 x 128 x 8 x Kp does (the extreme codes -128 and -8 included): Kp < 2^17.
__host__ __device__ __forceinline__ bool int4_x16_fits(int Kp) { return Kp < (1 << 17); }

// ---------------------------------------------------------------------------
// PTX wrappers (sm_100a)
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// The first 1024-byte-aligned byte (in the shared window) of a dynamic
// shared-memory array.  Pure arithmetic on the array pointer: an integer round
// trip would hide its address space from the compiler and turn every access
// through the result into a generic load or store.
__device__ __forceinline__ uint8_t* smem_align1024(uint8_t* raw) {
    return raw + ((1024u - (smem_u32(raw) & 1023u)) & 1023u);
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
            smem_u32(bar)),
        "r"(bytes)
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: gives up after `limit_ns` of wall time on the GPU's global
// timer, records `code` in *err and returns false.  No wait in this library
// can spin forever.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t* err,
                                                  uint32_t code, uint64_t limit_ns = 4000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    uint32_t spins = 0;
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((++spins & 255u) == 0u) {
            if (*(volatile uint32_t*)err != kDevErrNone) return false;  // someone else failed
            if (global_timer_ns() - t0 > limit_ns) {
                atomicCAS(err, kDevErrNone, code);
                return false;
            }
        }
    }
}

// mbar_wait_bounded for a barrier that threads of other CTAs of the cluster
// arrive on (release at cluster scope): acquire at cluster scope, so their
// shared-memory writes before the arrival are visible after the wait.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_bounded_cluster(uint64_t* bar, uint32_t parity, uint32_t* err,
                                                          uint32_t code, uint64_t limit_ns = 4000000000ull) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    uint32_t spins = 0;
    while (true) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((++spins & 255u) == 0u) {
            if (*(volatile uint32_t*)err != kDevErrNone) return false;  // someone else failed
            if (global_timer_ns() - t0 > limit_ns) {
                atomicCAS(err, kDevErrNone, code);
                return false;
            }
        }
    }
}

// Bounded wait for this CTA's own copies or MMAs before it exits (the drain
// after a loop ended, normally or on an error).  Unlike mbar_wait_bounded it
// does not give up when another CTA has recorded an error: whatever this CTA
// issued must land before its shared memory and TMEM are released.  It still
// gives up after `limit_ns`, recording `code`.
__device__ __forceinline__ bool mbar_drain_bounded(uint64_t* bar, uint32_t parity, uint32_t* err, uint32_t code,
                                                   uint64_t limit_ns = 4000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    uint32_t spins = 0;
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((++spins & 255u) == 0u && global_timer_ns() - t0 > limit_ns) {
            atomicCAS(err, kDevErrNone, code);
            return false;
        }
    }
}

// TMA 2D tiled load into shared memory, completion on an mbarrier.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// TMA 3D tiled load (x innermost), completion on an mbarrier.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, uint64_t* bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// Programmatic dependent launch controls (no-ops when launched without the
// attribute).
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_primary() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// 128-bit streaming load that bypasses L1 allocation (weights are read once).
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

}  // namespace zq
