/*
 * zq_oracle.c -- CPU restatement of ZYRON's quantized matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA path is
 * compared against; it is never linked into the product library and nothing
 * under zyron_b200/ may call it.  Only tests/, the smoke check and the
 * bench's cpu_baseline leg load it.
 *
 * Every function restates one piece of the reference (ZYRON) algorithm and
 * cites the file:line it follows.  Parity is pinned by running the compiled
 * reference itself (oracle/_ref, built by oracle/Makefile from the
 * reference's own sources) against this restatement on the golden inputs in
 * tests/golden/ (see tests/golden/make_golden.py).
 *
 * Layout conventions (same as the reference):
 *   activations x : fp32 row-major [M][K]
 *   weights      : logical [K rows][N cols]; stored column-major, element
 *                  (row r, col c) at linear index c*K + r
 *                  (src/quantization/quantization.cpp:155)
 *   INT4 payload : two codes per byte, low nibble = even linear index
 *                  (src/quantization/quantization.cpp:59-67)
 *   outputs y    : fp32 row-major [M][N]
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>
#include <stdlib.h>
#include <string.h>

#define ZO_INT8 1
#define ZO_INT4 2

/* quantization.cpp:45-50.  lroundf rounds half away from zero; a NaN
 * quotient converts to LONG_MIN on x86-64 glibc, which the clamp maps to
 * -limit.  The same libm call is used here so the oracle inherits that
 * platform behaviour exactly. */
int8_t zo_quantize_value(float value, float scale, int limit) {
    if (scale <= 0.0f || !isfinite(scale)) return 0;
    long r = lroundf(value / scale);
    if (r < -limit) r = -limit;
    if (r > limit) r = limit;
    return (int8_t)r;
}

/* quantization.cpp:52-57 */
int8_t zo_unpack_int4(uint8_t packed, int high) {
    uint8_t nib = high ? (uint8_t)(packed >> 4) : (uint8_t)(packed & 0x0Fu);
    return (int8_t)(nib < 8u ? (int)nib : (int)nib - 16);
}

/* quantization.cpp:59-67 */
static void zo_pack_int4(uint8_t* dst, size_t index, int8_t value) {
    size_t b = index >> 1;
    uint8_t nib = (uint8_t)value & 0x0Fu;
    if ((index & 1u) == 0u) dst[b] = (uint8_t)((dst[b] & 0xF0u) | nib);
    else dst[b] = (uint8_t)((dst[b] & 0x0Fu) | (uint8_t)(nib << 4));
}

/* Weight code at (col, row); quantization.cpp:89-97 without the bounds check. */
int8_t zo_weight_code(int type, const void* payload, size_t K, size_t col, size_t row) {
    size_t lin = col * K + row;
    if (type == ZO_INT8) return ((const int8_t*)payload)[lin];
    return zo_unpack_int4(((const uint8_t*)payload)[lin >> 1], (int)(lin & 1u));
}

/* Payload bytes for a K x N matrix: quantization.cpp:137-138, 300. */
size_t zo_payload_bytes(int type, size_t K, size_t N) {
    size_t e = K * N;
    return type == ZO_INT8 ? e : (e + 1) / 2;
}

/* quantize(): quantization.cpp:121-162.  w is row-major [K][N] fp32.
 * Writes scales[N] and the column-major payload (INT4 payload must be
 * zero-initialised by the caller, as quantization.cpp:138 assigns 0). */
void zo_quantize_weights(const float* w, size_t K, size_t N, int type,
                         void* payload, float* scales) {
    const float limitf = type == ZO_INT8 ? 127.0f : 7.0f;
    const int limit = type == ZO_INT8 ? 127 : 7;
    if (type == ZO_INT4) memset(payload, 0, zo_payload_bytes(type, K, N));
    for (size_t c = 0; c < N; ++c) {
        float max_abs = 0.0f;
        for (size_t r = 0; r < K; ++r) {
            float a = fabsf(w[r * N + c]);
            /* std::max(max_abs, a) returns max_abs when a is NaN */
            if (max_abs < a) max_abs = a;
        }
        float s = max_abs > 0.0f ? max_abs / limitf : 1.0f;
        scales[c] = s;
        for (size_t r = 0; r < K; ++r) {
            int8_t q = zo_quantize_value(w[r * N + c], s, limit);
            size_t lin = c * K + r;
            if (type == ZO_INT8) ((int8_t*)payload)[lin] = q;
            else zo_pack_int4((uint8_t*)payload, lin, q);
        }
    }
}

/* Per-row dynamic activation quantizer: quantization.cpp:203-212. */
void zo_quantize_rows(const float* x, size_t M, size_t K, int8_t* q, float* row_scale) {
    for (size_t m = 0; m < M; ++m) {
        const float* xr = x + m * K;
        float max_abs = 0.0f;
        for (size_t k = 0; k < K; ++k) {
            float a = fabsf(xr[k]);
            if (max_abs < a) max_abs = a;
        }
        float s = max_abs > 0.0f ? max_abs / 127.0f : 1.0f;
        row_scale[m] = s;
        for (size_t k = 0; k < K; ++k) q[m * K + k] = zo_quantize_value(xr[k], s, 127);
    }
}

/* Integer dot + epilogue: quantization.cpp:215-232.  acc (optional, may be
 * NULL) receives the int32 accumulators [M][N].  The epilogue is
 * float(acc) * s_row * s_col evaluated left to right (231-232), each product
 * rounded to fp32.  When bias is non-NULL it is added as a separate rounded
 * fp32 add, as QuantizedLinear::forward does (quantized_linear.cpp:44-48). */
void zo_matmul_codes(const int8_t* q, const float* row_scale, size_t M, size_t K,
                     int type, const void* payload, const float* col_scale, size_t N,
                     const float* bias, int32_t* acc, float* y) {
    /* Column-outer loop: the column's codes (INT4 unpacked once, as value()
     * would return them) are reused for every row.  Integer sums are exact,
     * so the loop order does not change any result. */
    int8_t* col = (int8_t*)malloc(K ? K : 1);
    for (size_t c = 0; c < N; ++c) {
        const int8_t* wc;
        if (type == ZO_INT8) {
            wc = (const int8_t*)payload + c * K;
        } else {
            for (size_t k = 0; k < K; ++k) col[k] = zo_weight_code(type, payload, K, c, k);
            wc = col;
        }
        for (size_t m = 0; m < M; ++m) {
            const int8_t* qr = q + m * K;
            int32_t a = 0;
            for (size_t k = 0; k < K; ++k) a += (int32_t)qr[k] * (int32_t)wc[k];
            if (acc) acc[m * N + c] = a;
            volatile float t = (float)a * row_scale[m];
            volatile float v = t * col_scale[c];
            if (bias) v = v + bias[c];
            y[m * N + c] = v;
        }
    }
    free(col);
}

/* matmul(): quantization.cpp:177-238 (row quant then dot + epilogue).
 * q_scratch holds M*K codes, s_scratch M row scales. */
void zo_matmul(const float* x, size_t M, size_t K, int type, const void* payload,
               const float* col_scale, size_t N, const float* bias,
               int8_t* q_scratch, float* s_scratch, int32_t* acc, float* y) {
    zo_quantize_rows(x, M, K, q_scratch, s_scratch);
    zo_matmul_codes(q_scratch, s_scratch, M, K, type, payload, col_scale, N, bias, acc, y);
}

/* dequantize(): quantization.cpp:164-175.  out is row-major [K][N]. */
void zo_dequantize(int type, const void* payload, const float* col_scale,
                   size_t K, size_t N, float* out) {
    for (size_t c = 0; c < N; ++c)
        for (size_t r = 0; r < K; ++r)
            out[r * N + c] = (float)zo_weight_code(type, payload, K, c, r) * col_scale[c];
}
