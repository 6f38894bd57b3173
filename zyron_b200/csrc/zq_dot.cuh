// zq_dot.cuh -- 16-byte weight chunk x shared-memory activation codes dot
// products (dp4a), shared by the decode GEMV and the language-model kernels.
#pragma once

#include "zq_common.cuh"

namespace zq {

template <int kM>
__device__ __forceinline__ void dot16_int8(const uint4 w, const int8_t* __restrict__ sq, int Kp, int koff,
                                           int (&acc)[kM]) {
#pragma unroll
    for (int m = 0; m < kM; ++m) {
        const uint4 a = *reinterpret_cast<const uint4*>(sq + m * Kp + koff);
        acc[m] = __dp4a((int)w.x, (int)a.x, acc[m]);
        acc[m] = __dp4a((int)w.y, (int)a.y, acc[m]);
        acc[m] = __dp4a((int)w.z, (int)a.z, acc[m]);
        acc[m] = __dp4a((int)w.w, (int)a.w, acc[m]);
    }
}

// 16 packed bytes = 32 INT4 codes covering k = kcode .. kcode+31.  Shared
// activations for INT4 are stored "even/odd split" per group of 8 codes:
// [k0 k2 k4 k6 | k1 k3 k5 k7], matching the nibble unpack order.
template <int kM>
__device__ __forceinline__ void dot16_int4(const uint4 w, const int8_t* __restrict__ sq, int Kp, int kcode,
                                           int (&acc)[kM]) {
    uint32_t ev[4], od[4];
    zq_unpack_int4x8(w.x, ev[0], od[0]);
    zq_unpack_int4x8(w.y, ev[1], od[1]);
    zq_unpack_int4x8(w.z, ev[2], od[2]);
    zq_unpack_int4x8(w.w, ev[3], od[3]);
#pragma unroll
    for (int m = 0; m < kM; ++m) {
        const uint4 a0 = *reinterpret_cast<const uint4*>(sq + m * Kp + kcode);
        const uint4 a1 = *reinterpret_cast<const uint4*>(sq + m * Kp + kcode + 16);
        int s = acc[m];
        s = __dp4a((int)ev[0], (int)a0.x, s);
        s = __dp4a((int)od[0], (int)a0.y, s);
        s = __dp4a((int)ev[1], (int)a0.z, s);
        s = __dp4a((int)od[1], (int)a0.w, s);
        s = __dp4a((int)ev[2], (int)a1.x, s);
        s = __dp4a((int)od[2], (int)a1.y, s);
        s = __dp4a((int)ev[3], (int)a1.z, s);
        s = __dp4a((int)od[3], (int)a1.w, s);
        acc[m] = s;
    }
}

}  // namespace zq
