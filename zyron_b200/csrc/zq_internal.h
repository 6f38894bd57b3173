// zq_internal.h -- library-internal types shared by the C ABI translation
// units (zq_api.cu, zq_lm.cu).  Not installed.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <mutex>
#include <vector>

#include "zq.h"

struct zq_weight {
    int type = 0;
    size_t K = 0, N = 0;
    int Kp = 0;
    int device = 0;
    uint8_t* panel = nullptr;  // [N][Kp] int8 or [N][Kp/2] packed int4
    float* scales = nullptr;   // [N]
    size_t panel_bytes = 0;
    // Tensor maps over the INT8 panel, one per GEMM tile shape (64/128/256
    // columns, and the 2-SM pair tile); the decode kernel reads 64-column
    // boxes.
    std::mutex mu;
    CUtensorMap tmap_b[4];
    bool tmap_ready[4] = {false, false, false, false};
    // INT4: tensor maps over the packed panel per tile shape (the kernels
    // unpack in shared memory).
    CUtensorMap tmap_p[4];
    bool tmap_p_ready[4] = {false, false, false, false};
    // The decode kernel's 3-D view of the panel: boxes of several k-blocks
    // of 64 columns.
    CUtensorMap tmap_dec;
    bool tmap_dec_ready = false;
    // Options of this weight's matmuls (zq_weight_set_option).
    std::atomic<int> opt_decode{ZQ_DECODE_AUTO};
    std::atomic<int> opt_reserved_sms{0};
    std::atomic<int> opt_group_m{32};
};

namespace zq {

// One parsed .zyq record (quantization.cpp:269-311), still on the host.
struct ZyqRecord {
    int type = 0;
    size_t rows = 0, cols = 0;
    std::vector<float> scales;
    const uint8_t* payload = nullptr;  // points into the parsed buffer
    size_t payload_bytes = 0;
    size_t consumed = 0;               // bytes of the whole record
};

// Validates one .zyq record with the reference's checks and messages; no
// device work.
zq_status parse_zyq(const void* bytes, size_t len, ZyqRecord* rec);

// New weight whose columns are the columns of parts[0..n) in order (same
// type and rows).  Columns are independent, so this is exact.
zq_status concat_cols(zq_weight* const* parts, int n, void* stream, zq_weight** out);

// Records a CUDA failure as the calling thread's last error.
zq_status cuda_error(cudaError_t e, const char* what);

// The current device's error word, where bounded device waits record a
// timeout (read and cleared by zq_device_error).
zq_status device_error_word(uint32_t** out);

}  // namespace zq
