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

// 16 panel bytes = 32 INT4 codes covering k = kcode .. kcode+31 (the panel
// layout keeps them in k order, see panel_int4_byte), against activation
// codes in k order.  kX16: the codes are unpacked as 16 x the code (three
// operations per eight codes) and the dot is 16 times the true one; the
// caller shifts the finished sum right by 4 (exact; int4_x16_fits(Kp)).
template <int kM, bool kX16 = false>
__device__ __forceinline__ void dot16_int4(const uint4 w, const int8_t* __restrict__ sq, int Kp, int kcode,
                                           int (&acc)[kM]) {
    uint4 lo, hi;
    if (kX16)
        zq_expand_int4x32_x16(w, lo, hi);
    else
        zq_expand_int4x32(w, lo, hi);
#pragma unroll
    for (int m = 0; m < kM; ++m) {
        const uint4 a0 = *reinterpret_cast<const uint4*>(sq + m * Kp + kcode);
        const uint4 a1 = *reinterpret_cast<const uint4*>(sq + m * Kp + kcode + 16);
        int s = acc[m];
        s = __dp4a((int)lo.x, (int)a0.x, s);
        s = __dp4a((int)lo.y, (int)a0.y, s);
        s = __dp4a((int)lo.z, (int)a0.z, s);
        s = __dp4a((int)lo.w, (int)a0.w, s);
        s = __dp4a((int)hi.x, (int)a1.x, s);
        s = __dp4a((int)hi.y, (int)a1.y, s);
        s = __dp4a((int)hi.z, (int)a1.z, s);
        s = __dp4a((int)hi.w, (int)a1.w, s);
        acc[m] = s;
    }
}

}  // namespace zq
