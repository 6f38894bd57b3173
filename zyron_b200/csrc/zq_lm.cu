// zq_lm.cu -- device-resident decode loop of ZYRON's QuantizedLanguageModel.
//
// The reference (src/model/quantized_language_model.cpp) recomputes the whole
// prefix on the host for every generated token (generate_batch 503-547 ->
// forward 468-494 -> forward_block 412-461) and runs each QuantizedLinear
// through quantization::matmul.  Here weights, the KV cache and all
// activations stay in HBM and one decode step is a fixed chain of kernels
// that reads the position and token from device memory, so a step is
// captured once as a CUDA graph and replayed for every position:
//
//   embed            token_lookup (271-282) [+ sinusoidal PE (488-490)]
//   per block        norm1 -> q|k|v QuantizedLinear (one fused matmul over the
//                    concatenated columns) -> RoPE + KV-cache append + causal
//                    GQA attention for the new row (421-451) -> out_proj +
//                    residual (453-454) -> norm2 -> ff_up + GELU -> ff_down +
//                    residual (456-460)
//   head             final RMS norm (492) -> lm_head (493) -> greedy argmax
//                    (sample_next 82-174 with top_k = 1)
//
// Kernels are chained with programmatic dependent launch, so several later
// kernels of the chain can already be resident on an SM while earlier ones
// run.  griddepcontrol.wait makes the producer's writes visible in L2, but an
// SM's L1 may still hold lines another resident kernel loaded before those
// writes; every read of data produced by another kernel (activations,
// position state, tokens, KV cache, logits) therefore goes through L2 only
// (ld.global.cg).  Constant data (weights, norms, RoPE tables) may use L1.
//
// Every QuantizedLinear keeps the reference's quantized arithmetic exactly:
// the row of activations is quantized per row (absmax / 127, round half away
// from zero), dotted in int32 against the INT8/INT4 column codes and rescaled
// as float(acc) * s_row * s_col + bias.  The fp32 parts (norm reductions,
// softmax, tanh-GELU, attention sums) follow the reference's formulas with a
// parallel reduction order, so logits agree within a tolerance rather than
// bit for bit, and an int8 code can flip where a value sits on a rounding
// boundary.
#include "zq.h"
#include "zq_common.cuh"
#include "zq_dot.cuh"
#include "zq_internal.h"
#include "zq_kernels.h"

#include <cmath>
#include <cstdio>
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <random>
#include <string>
#include <vector>

namespace zq {

// zq_sample.cpp: validate_generation_config and sample_next on the host.
zq_status check_generation_config(const zq_generation_config* c);
std::size_t sample_row(std::mt19937& rng, const float* logits, std::size_t vocab, const int64_t* history,
                       std::size_t len, const zq_generation_config& cfg);

namespace lm {

constexpr int kThreads = 256;
constexpr int kMaxHeadDim = 128;
constexpr int kAttnChunk = 64;  // positions per attention block

// Position state in device memory: the step kernels read it, the argmax
// kernel advances it, so one captured step serves every position.
struct State {
    int pos;         // position whose logits this step computes
    int prompt_len;  // positions < prompt_len - 1 are prefill (no logits needed)
    int pad[2];
};

enum Prologue { kProNone = 0, kProRms = 1, kProLayer = 2, kProMerge = 3 };
enum Epilogue { kEpiStore = 0, kEpiGelu = 1, kEpiResidual = 2, kEpiLogits = 3 };

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide reductions (all threads get the result).  `sh` holds >= 32 floats.
template <int kN>
__device__ float block_sum(float v, float* sh) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    float t = (threadIdx.x < kN / 32) ? sh[threadIdx.x] : 0.0f;
    if (w == 0) t = warp_sum(t);
    if (threadIdx.x == 0) sh[0] = t;
    __syncthreads();
    return sh[0];
}
template <int kN>
__device__ float block_max(float v, float* sh) {
    v = warp_max(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    float t = (threadIdx.x < kN / 32) ? sh[threadIdx.x] : -INFINITY;
    if (w == 0) t = warp_max(t);
    if (threadIdx.x == 0) sh[0] = t;
    __syncthreads();
    return sh[0];
}

// tanh-approximation GELU as the reference evaluates it (gelu 321-331):
// 0.5f * x * (1 + tanh(kInvSqrt2Pi * (x + kC * x^3))), each operation rounded.
__device__ __forceinline__ float gelu_ref(float x) {
    const float kC = 0.044715f;
    const float kInvSqrt2Pi = 0.7978845608028654f;
    const float x3 = __fmul_rn(__fmul_rn(x, x), x);
    const float inner = __fmul_rn(kInvSqrt2Pi, __fadd_rn(x, __fmul_rn(kC, x3)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

// Greedy choice as one comparable 64-bit key: the logit's bits made
// order-preserving (-0 counted as +0), then the complement of the column, so
// the larger key is the larger logit and, on ties, the lower token id.
__device__ __forceinline__ unsigned long long argmax_key(float v, int col) {
    uint32_t b = __float_as_uint(v);
    if ((b & 0x7fffffffu) == 0u) b = 0u;
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (unsigned long long)(0xffffffffu - (uint32_t)col);
}
__device__ __forceinline__ int token_from_key(unsigned long long key, int nan, int V) {
    if (nan || key == 0ull) return 0;
    const uint32_t hi = (uint32_t)(key >> 32);
    const float best = __uint_as_float((hi & 0x80000000u) ? (hi ^ 0x80000000u) : ~hi);
    const int idx = (int)(0xffffffffu - (uint32_t)key);
    return (isinf(best) || idx >= V) ? 0 : idx;
}

// ---------------------------------------------------------------------------
// token_lookup (271-282): h[j] = float(code(j, token)) * scale[j]; the
// embedding is quantized with vocab rows and hidden columns, so a token's
// vector is one code from each hidden column.  Optional sinusoidal PE add.
// ---------------------------------------------------------------------------
__global__ void embed_kernel(const uint8_t* __restrict__ panel, int type, int Kp, const float* __restrict__ scales,
                             int hidden, const int32_t* __restrict__ tokens, const State* __restrict__ st,
                             const float* __restrict__ pe, float* __restrict__ h) {
    pdl_launch_dependents();
    pdl_wait_primary();
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= hidden) return;
    const int pos = __ldcg(&st->pos);
    const int tok = __ldcg(tokens + pos);
    int code;
    if (type == kInt8) {
        code = (int8_t)panel[(size_t)j * Kp + tok];
    } else {
        const uint8_t b = panel[(size_t)j * (Kp >> 1) + panel_int4_byte(tok)];
        const int nib = (b >> panel_int4_shift(tok)) & 0x0F;
        code = nib < 8 ? nib : nib - 16;
    }
    float v = x86_mul((float)code, scales[j]);
    if (pe) v = x86_add(v, pe[(size_t)pos * hidden + j]);
    h[j] = v;
}

// ---------------------------------------------------------------------------
// The row prologue of every decode linear: xs[0, K) holds the activation row
// (fp32, shared memory, [K, Kp) zero).  Optional RMSNorm / LayerNorm (norm
// 284-319) in place, then the per-row activation quantizer
// (quantization.cpp:202-212) into qs, codes in k order (the INT4 panel
// layout unpacks into k order too).
// Returns the row scale.  Every thread of the block calls it.
// ---------------------------------------------------------------------------
// One-barrier block reductions for the row prologue: the r-th reduction of a
// row writes its warp partials to red[32 r ..] (at most three per row, and
// the row ends with a barrier), and every thread adds them in one order.
template <int kNT>
__device__ __forceinline__ float row_sum(float v, float* red, int r) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) red[32 * r + (threadIdx.x >> 5)] = v;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < kNT / 32; ++w) t = __fadd_rn(t, red[32 * r + w]);
    return t;
}
template <int kNT>
__device__ __forceinline__ float row_max(float v, float* red, int r) {
    v = warp_max(v);
    if ((threadIdx.x & 31) == 0) red[32 * r + (threadIdx.x >> 5)] = v;
    __syncthreads();
    float t = red[32 * r];
#pragma unroll
    for (int w = 1; w < kNT / 32; ++w) t = fmaxf(t, red[32 * r + w]);
    return t;
}

// Copies the activation row x[0, K) into xs (zero up to Kp) with every
// thread's loads issued before its first store: a row of a few thousand
// floats then costs one L2 round trip instead of one per strided element.
template <int kNT>
__device__ __forceinline__ void load_row(const float* __restrict__ x, int K, int Kp, float* xs) {
    constexpr int kBatch = 8;
    for (int i0 = 0; i0 < Kp; i0 += kBatch * kNT) {
        float v[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int i = i0 + threadIdx.x + u * kNT;
            v[u] = i < K ? __ldcg(x + i) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int i = i0 + threadIdx.x + u * kNT;
            if (i < Kp) xs[i] = v[u];
        }
    }
}

// Norm weights held in registers: element tid + kNT k for k < kNormRegs
// (the rest of a longer row is read from global memory).
constexpr int kNormRegs = 4;

// `red` holds 96 floats; nwr / nbr hold this thread's norm weights and
// LayerNorm biases (loaded before the kernel's dependency wait).
template <int kNT>
__device__ float quantize_row(float* xs, int8_t* qs, int K, int Kp, int type, int pro, const float* __restrict__ nw,
                              const float* __restrict__ nb, const float (&nwr)[kNormRegs],
                              const float (&nbr)[kNormRegs], float eps, float* red) {
    if (pro == kProRms) {
        float ss = 0.0f;
        for (int i = threadIdx.x; i < K; i += kNT) ss = __fadd_rn(ss, __fmul_rn(xs[i], xs[i]));
        ss = row_sum<kNT>(ss, red, 0);
        const float var = __fdiv_rn(ss, (float)K);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
        for (int k = 0; k < kNormRegs; ++k) {
            const int i = threadIdx.x + kNT * k;
            if (i < K) xs[i] = __fmul_rn(__fmul_rn(xs[i], inv), nwr[k]);
        }
        for (int i = threadIdx.x + kNT * kNormRegs; i < K; i += kNT) xs[i] = __fmul_rn(__fmul_rn(xs[i], inv), nw[i]);
        __syncthreads();
    } else if (pro == kProLayer) {
        float sm = 0.0f;
        for (int i = threadIdx.x; i < K; i += kNT) sm = __fadd_rn(sm, xs[i]);
        sm = row_sum<kNT>(sm, red, 0);
        const float mean = __fdiv_rn(sm, (float)K);
        float ss = 0.0f;
        for (int i = threadIdx.x; i < K; i += kNT) {
            const float c = __fsub_rn(xs[i], mean);
            ss = __fadd_rn(ss, __fmul_rn(c, c));
        }
        ss = row_sum<kNT>(ss, red, 1);
        const float var = __fdiv_rn(ss, (float)K);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
        for (int k = 0; k < kNormRegs; ++k) {
            const int i = threadIdx.x + kNT * k;
            if (i < K) xs[i] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xs[i], mean), inv), nwr[k]), nbr[k]);
        }
        for (int i = threadIdx.x + kNT * kNormRegs; i < K; i += kNT)
            xs[i] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xs[i], mean), inv), nw[i]), nb[i]);
        __syncthreads();
    }
    float m = 0.0f;
    for (int i = threadIdx.x; i < K; i += kNT) m = fmaxf(m, fabsf(xs[i]));
    m = row_max<kNT>(m, red, 2);
    const float s = zq_scale_from_absmax(m, 127.0f);
    const float rcp = zq_quant_rcp(s);
    for (int i = threadIdx.x; i < Kp; i += kNT) {
        const int8_t code = i < K ? (int8_t)zq_quantize_value_rcp(xs[i], s, rcp, 127) : (int8_t)0;
        qs[i] = code;
    }
    __syncthreads();
    return s;
}

// Attention chunk partials for the merge prologue: part[head][chunk][130]
// holds each 64-position chunk's softmax maximum m, sum l and context c.
struct MergeArgs {
    const float* part;
    int heads, hd, n_chunks_max;
};

// The lm_head's greedy choice: every block folds its columns into one
// order-preserving key (argmax_key), stored in its own slot (no contended
// atomics across thousands of blocks), and raises a shared flag on a NaN;
// next_token_kernel reduces the slots and clears the flag.
struct ArgmaxArgs {
    unsigned long long* slots;  // [lm_head blocks]
    int* nan;
};

// The context row of the newest position from its chunks' partials:
// ctx = (sum_c c_c e^(m_c - M)) / (sum_c l_c e^(m_c - M)), M = max_c m_c, per
// head, into xs[0, heads * hd).  `mls` holds 2 * heads * nchunk floats and
// `invl` heads floats of shared memory.  Ends with a barrier.
template <int kNT>
__device__ void merge_rows(const MergeArgs& a, int nchunk, float* xs, float* mls, float* invl) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t stride = kMaxHeadDim + 2;
    const int H = a.heads * a.hd;
    // Contexts of up to 768 positions, rows of up to 3 kNT: this thread's
    // chunk contexts are loaded with the (m, l) pairs, one round trip.  The
    // loads cover every chunk slot, used or not, so they need not wait for
    // the position (nchunk); stale slots are never read back.
    constexpr int kRegChunks = 12, kRegRows = 3;
    const int nmax = a.n_chunks_max;
    const bool rows_fit = H <= kRegRows * kNT;
    const bool fast = nchunk <= kRegChunks && rows_fit;
    float cv[kRegRows][kRegChunks];
    if (rows_fit) {
#pragma unroll
        for (int k = 0; k < kRegRows; ++k) {
            const int o = tid + kNT * k;
            const int hq = o < H ? o / a.hd : 0, d = o < H ? o - hq * a.hd : 0;
            const float* ph = a.part + (size_t)hq * nmax * stride + 2 + d;
#pragma unroll
            for (int c = 0; c < kRegChunks; ++c)
                cv[k][c] = (o < H && c < nmax) ? __ldcg(ph + (size_t)c * stride) : 0.0f;
        }
    }
    for (int e = tid; e < a.heads * nmax; e += kNT) {
        const float* pc = a.part + (size_t)e * stride;
        mls[2 * e] = __ldcg(pc);
        mls[2 * e + 1] = __ldcg(pc + 1);
    }
    __syncthreads();
    for (int hq = warp; hq < a.heads; hq += kNT / 32) {
        float M = -INFINITY;
        for (int c = lane; c < nchunk; c += 32) M = fmaxf(M, mls[2 * (hq * nmax + c)]);
        M = warp_max(M);
        float L = 0.0f;
        for (int c = lane; c < nchunk; c += 32) {
            const int e = hq * nmax + c;
            const float f = expf(__fsub_rn(mls[2 * e], M));
            L = __fadd_rn(L, __fmul_rn(mls[2 * e + 1], f));
            mls[2 * e] = f;
        }
        L = warp_sum(L);
        if (lane == 0) invl[hq] = L > 0.0f ? __fdiv_rn(1.0f, L) : 0.0f;
    }
    __syncthreads();
    if (fast) {
#pragma unroll
        for (int k = 0; k < kRegRows; ++k) {
            const int o = tid + kNT * k;
            if (o < H) {
                const int hq = o / a.hd;
                float acc = 0.0f;
#pragma unroll
                for (int c = 0; c < kRegChunks; ++c)
                    if (c < nchunk) acc = __fadd_rn(acc, __fmul_rn(cv[k][c], mls[2 * (hq * nmax + c)]));
                xs[o] = __fmul_rn(acc, invl[hq]);
            }
        }
        __syncthreads();
        return;
    }
    for (int o = tid; o < H; o += kNT) {
        const int hq = o / a.hd, d = o - hq * a.hd;
        const float* ph = a.part + (size_t)hq * a.n_chunks_max * stride + 2 + d;
        float acc = 0.0f;
        for (int c0 = 0; c0 < nchunk; c0 += 8) {
            float cv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) cv[u] = c0 + u < nchunk ? __ldcg(ph + (size_t)(c0 + u) * stride) : 0.0f;
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (c0 + u < nchunk) acc = __fadd_rn(acc, __fmul_rn(cv[u], mls[2 * (hq * nmax + c0 + u)]));
        }
        xs[o] = __fmul_rn(acc, invl[hq]);
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------
// One QuantizedLinear on a single activation row, with the operations around
// it fused:
//   prologue  optional RMSNorm / LayerNorm of x (norm 284-319), then the
//             per-row activation quantizer (quantization.cpp:202-212); every
//             block computes it redundantly from x (K <= a few thousand), so
//             no separate launch and no grid-wide sync are needed.
//   body      warp-per-column int8 dot (dp4a) over the weight panel.
//   epilogue  float(acc) * s_row * s_col + bias, then store / GELU / residual
//             add (y = y + out, the reference's math::add(input, attended)).
// `skip_prefill`: the lm_head skips positions whose logits nobody reads.
// ---------------------------------------------------------------------------
template <int kType, int kPro, int kEpi>
__global__ void __launch_bounds__(kThreads) linear_kernel(const float* __restrict__ x, int K, int Kp,
                                                          const float* __restrict__ nw, const float* __restrict__ nb,
                                                          float eps, const uint8_t* __restrict__ panel,
                                                          const float* __restrict__ scales, int N,
                                                          const float* __restrict__ bias, float* y,
                                                          const State* __restrict__ st, int skip_prefill,
                                                          const MergeArgs merge, const ArgmaxArgs am) {
    extern __shared__ __align__(16) float lsm[];
    float* xs = lsm;                                          // [Kp] fp32 (normalised) activations
    int8_t* qs = reinterpret_cast<int8_t*>(lsm + Kp);         // [Kp] codes
    __shared__ float red[96];
    __shared__ unsigned long long blk_key;
    __shared__ int blk_nan;
    constexpr int kPre = 8;  // 16-byte weight chunks per lane fetched before the dependency wait (K <= 4096 INT8)
    const int lane = threadIdx.x & 31;
    const int warps_total = gridDim.x * (kThreads / 32);
    const size_t cb = kType == kInt8 ? (size_t)Kp : (size_t)(Kp >> 1);
    const int chunks = (int)(cb >> 4);
    const int first_col = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);

    // Weights do not depend on earlier kernels: start fetching this warp's
    // first column, then let the next kernel launch, then wait for the
    // producer of x (programmatic dependent launch).
    uint4 pre[kPre];
#pragma unroll
    for (int u = 0; u < kPre; ++u) {
        const int c = lane + 32 * u;
        pre[u] = (first_col < N && c < chunks) ? ld_stream_u4(panel + (size_t)first_col * cb + (size_t)c * 16)
                                               : make_uint4(0, 0, 0, 0);
    }
    const bool lead = lane == 0 && first_col < N;  // lane 0 finishes the warp's columns
    const float pre_scale = lead ? scales[first_col] : 0.0f;
    const float pre_bias = (lead && bias) ? bias[first_col] : 0.0f;
    // this thread's norm weights (and LayerNorm biases), also independent of
    // earlier kernels
    float nwr[kNormRegs], nbr[kNormRegs];
#pragma unroll
    for (int k = 0; k < kNormRegs; ++k) {
        const int i = threadIdx.x + kThreads * k;
        nwr[k] = ((kPro == kProRms || kPro == kProLayer) && i < K) ? nw[i] : 0.0f;
        nbr[k] = (kPro == kProLayer && i < K) ? nb[i] : 0.0f;
    }
    pdl_launch_dependents();
    pdl_wait_primary();
    if (skip_prefill && __ldcg(&st->pos) + 1 < __ldcg(&st->prompt_len)) return;
    // The residual is final once the kernel before this one completed (its
    // own wait covered every kernel before it): load it with the row.
    const float pre_res = (kEpi == kEpiResidual && lead) ? __ldcg(y + first_col) : 0.0f;

    if (kPro == kProMerge) {
        // context row from the attention chunks (shared memory after xs, qs)
        float* mls = lsm + Kp + Kp / 4;
        const int nchunk = (__ldcg(&st->pos) + kAttnChunk) / kAttnChunk;
        merge_rows<kThreads>(merge, nchunk, xs, mls, mls + 2 * merge.heads * merge.n_chunks_max);
        for (int i = K + threadIdx.x; i < Kp; i += kThreads) xs[i] = 0.0f;
    } else {
        load_row<kThreads>(x, K, Kp, xs);
    }
    __syncthreads();
    if (kEpi == kEpiLogits && threadIdx.x == 0) blk_key = 0ull, blk_nan = 0;
    const float s = quantize_row<kThreads>(xs, qs, K, Kp, kType, kPro, nw, nb, nwr, nbr, eps, red);
    unsigned long long best = 0ull;
    int nan = 0;

    for (int col = first_col; col < N; col += warps_total) {
        const uint8_t* wc = panel + (size_t)col * cb;
        const bool have_pre = col == first_col;
        int acc[1] = {0};
#pragma unroll
        for (int u = 0; u < kPre; ++u) {
            const int c = lane + 32 * u;
            if (c < chunks) {
                const uint4 w = have_pre ? pre[u] : ld_stream_u4(wc + (size_t)c * 16);
                if (kType == kInt8)
                    dot16_int8<1>(w, qs, Kp, c * 16, acc);
                else
                    dot16_int4<1>(w, qs, Kp, c * 32, acc);
            }
        }
        for (int c = lane + 32 * kPre; c < chunks; c += 32) {
            const uint4 w = ld_stream_u4(wc + (size_t)c * 16);
            if (kType == kInt8)
                dot16_int8<1>(w, qs, Kp, c * 16, acc);
            else
                dot16_int4<1>(w, qs, Kp, c * 32, acc);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], o);
        if (lane == 0) {
            float v = zq_epilogue(acc[0], s, have_pre ? pre_scale : scales[col]);
            if (bias) v = x86_add(v, have_pre ? pre_bias : bias[col]);
            if (kEpi == kEpiStore || kEpi == kEpiLogits) y[col] = v;
            else if (kEpi == kEpiGelu) y[col] = gelu_ref(v);
            else y[col] = x86_add(have_pre ? pre_res : __ldcg(y + col), v);
            if (kEpi == kEpiLogits) {
                if (isnan(v)) {
                    nan = 1;
                } else {
                    const unsigned long long k = argmax_key(v, col);
                    if (k > best) best = k;
                }
            }
        }
    }
    if (kEpi == kEpiLogits) {
        if (lane == 0) {
            if (best) atomicMax(&blk_key, best);
            if (nan) blk_nan = 1;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            am.slots[blockIdx.x] = blk_key;
            if (blk_nan) atomicExch(am.nan, 1);
        }
    }
}

// ---------------------------------------------------------------------------
// Greedy choice (sample_next with top_k = 1, 82-174): the highest logit,
// lowest id on ties, folded into one key by the lm_head kernel.  The
// reference returns token 0 when its softmax denominator is not finite (any
// NaN logit, or a maximum of +-inf).  During prefill the step only advances
// the position.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) next_token_kernel(ArgmaxArgs am, int nslots, int V, int32_t* tokens,
                                                         State* st) {
    __shared__ unsigned long long wbest[8];
    pdl_launch_dependents();
    pdl_wait_primary();
    const int pos = __ldcg(&st->pos);
    const bool choose = pos + 1 >= __ldcg(&st->prompt_len);
    if (choose) {
        unsigned long long best = 0ull;
        for (int i = threadIdx.x; i < nslots; i += 256) {
            const unsigned long long k = __ldcg(am.slots + i);
            if (k > best) best = k;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            if (other > best) best = other;
        }
        if ((threadIdx.x & 31) == 0) wbest[threadIdx.x >> 5] = best;
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    if (choose) {
        unsigned long long best = wbest[0];
        for (int w = 1; w < 8; ++w)
            if (wbest[w] > best) best = wbest[w];
        tokens[pos + 1] = token_from_key(best, __ldcg(am.nan), V);
        *am.nan = 0;  // ready for the next step's lm_head
    }
    st->pos = pos + 1;
}

// Repetition penalty and n-gram block of a greedy step, read by the captured
// step from device memory so that one graph serves every setting.
struct PenaltyCfg {
    float rep;  // repetition_penalty (1 = off)
    int ngram;  // no_repeat_ngram_size (0 = off)
};

constexpr int kPenaltyThreads = 1024;

// Block-wide maximum of 64-bit keys; every thread gets the result.
__device__ unsigned long long block_max_key(unsigned long long v, unsigned long long* sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, v, o);
        if (other > v) v = other;
    }
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    unsigned long long best = sh[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
        if (sh[w] > best) best = sh[w];
    return best;
}

// Greedy choice with the repetition penalty and the n-gram block of
// sample_next (82-174, with top_k = 1) over the full logits row and the token
// history tokens[0, pos] (the prompt and the tokens generated so far):
//   value = logit, divided by the penalty (value >= 0) or multiplied by it
//   (value < 0) for tokens of the history; -inf for tokens that followed an
//   earlier occurrence of the last n - 1 tokens; if no value is finite and a
//   block applied, the raw logits instead (120-128).  The token is the
//   largest value (lowest id on ties), or 0 when the reference's softmax
//   denominator is not finite: a NaN value, or a maximum of +-inf.
// One block; `bits` holds 2 * ceil(V / 32) words of dynamic shared memory.
__global__ void __launch_bounds__(kPenaltyThreads) next_token_penalized_kernel(const float* logits, int V,
                                                                               int32_t* tokens, State* st,
                                                                               const PenaltyCfg* pc, int* nan_flag) {
    extern __shared__ uint32_t bits[];
    __shared__ unsigned long long red[kPenaltyThreads / 32];
    __shared__ int flags;  // bit 0: a block applies; 1: NaN value; 2: finite value; 3: NaN logit
    pdl_launch_dependents();
    pdl_wait_primary();
    const int tid = threadIdx.x;
    const int pos = __ldcg(&st->pos);
    if (pos + 1 < __ldcg(&st->prompt_len)) {  // prefill: no choice
        if (tid == 0) st->pos = pos + 1;
        return;
    }
    const int words = (V + 31) >> 5;
    uint32_t* seen = bits;
    uint32_t* blocked = bits + words;
    for (int i = tid; i < 2 * words; i += kPenaltyThreads) bits[i] = 0u;
    if (tid == 0) flags = 0;
    __syncthreads();
    const float rep = pc->rep;
    const int n = pc->ngram;
    const int len = pos + 1;
    if (rep != 1.0f)
        for (int i = tid; i < len; i += kPenaltyThreads) {
            const int t = __ldcg(tokens + i);
            if (t >= 0 && t < V) atomicOr(&seen[t >> 5], 1u << (t & 31));
        }
    if (n > 0 && len >= n) {
        const int pl = n - 1;
        for (int start = tid; start + n <= len; start += kPenaltyThreads) {
            bool match = true;
            for (int k = 0; k < pl && match; ++k) match = __ldcg(tokens + start + k) == __ldcg(tokens + len - pl + k);
            if (!match) continue;
            const int t = __ldcg(tokens + start + pl);
            atomicOr(&flags, 1);
            if (t >= 0 && t < V) atomicOr(&blocked[t >> 5], 1u << (t & 31));
        }
    }
    __syncthreads();
    const bool have_block = flags & 1;
    unsigned long long best = 0ull, best_raw = 0ull;
    int f = 0;
    for (int id = tid; id < V; id += kPenaltyThreads) {
        const float raw = __ldcg(logits + id);
        float v = raw;
        if (rep != 1.0f && ((seen[id >> 5] >> (id & 31)) & 1u)) v = v >= 0.0f ? __fdiv_rn(v, rep) : __fmul_rn(v, rep);
        if (have_block && ((blocked[id >> 5] >> (id & 31)) & 1u)) v = -INFINITY;
        if (isnan(v)) {
            f |= 2;
        } else {
            const unsigned long long k = argmax_key(v, id);
            if (k > best) best = k;
            if (isfinite(v)) f |= 4;
        }
        if (isnan(raw)) {
            f |= 8;
        } else {
            const unsigned long long k = argmax_key(raw, id);
            if (k > best_raw) best_raw = k;
        }
    }
    if (f) atomicOr(&flags, f);
    best = block_max_key(best, red);
    best_raw = block_max_key(best_raw, red);
    if (tid != 0) return;
    const int fl = flags;
    const bool use_raw = !(fl & 4) && (fl & 1);
    tokens[pos + 1] = use_raw ? token_from_key(best_raw, fl & 8, V) : token_from_key(best, fl & 2, V);
    *nan_flag = 0;  // the lm_head raised it on a NaN logit; unused here
    st->pos = pos + 1;
}

// ===========================================================================
// Persistent decode: the whole greedy generation in one cooperative launch.
//
// The multi-kernel step above pays a launch and a dependency hand-over for
// each of its ~5 kernels per layer, and every one of them is latency-bound
// (a few MB of weights per kernel).  Here one CTA per SM runs every step; the
// phases of a step are separated by a grid barrier, and before arriving at a
// barrier each warp already loads everything of the next phase that does not
// depend on it: its weight columns, their scales and biases, the residual
// values it will add, and each thread its norm weights.  After the barrier
// only the activation row, its norm and quantization, the dots and the
// stores remain.  Per step and layer:
//   A  (layer 0: embedding lookup) norm1 -> quantize -> q|k|v columns
//   B  attention items (KV group, 64-position chunk): RoPE, KV append by the
//      first chunk, scores, chunk softmax, partial context (m, l, c)
//   C  merge the chunks' (m, l, c) into the context row -> out_proj columns,
//      residual add into h
//   D  norm2 -> ff_up columns, GELU
//   E  ff_down columns, residual add into h
// then, when the step's logits are needed, the final norm and lm_head
// columns; the greedy argmax is folded into that phase (per-CTA maximum of
// an order-preserving key, one 64-bit atomicMax per CTA) and every CTA reads
// the chosen token after the next barrier.
//
// Each thread owns the row elements tid, tid + 512, ... in every phase, so a
// row needs no barrier between its load and its reductions; a block
// reduction costs one __syncthreads.  Every barrier wait is bounded: on
// timeout the kernel records an error and all CTAs leave at their next
// barrier.  Data written by other CTAs is read through L2 (ld.global.cg).
// ===========================================================================
constexpr int kStepThreads = 512;
constexpr int kStepWarps = kStepThreads / 32;
constexpr int kPreSlots = 8;          // 16-byte weight chunks per lane loaded before a barrier
constexpr int kMaxColsPerWarp = 8;    // columns one warp reduces at once
constexpr int kHeadBatch = 4;         // query heads of a KV group handled together
constexpr int kAttnPosPerWarp = kAttnChunk / kStepWarps;  // 4
constexpr int kRowRegs = 4;           // norm weights per thread held in registers (K <= 2048)
constexpr int kMergeChunks = 12;      // attention chunks merged from registers (contexts <= 768)

struct LinDesc {
    const uint8_t* panel;
    const float* scales;
    const float* bias;
    int K, Kp, N;
};

struct LayerDesc {
    LinDesc qkv, out, up, down;
    const float *n1w, *n1b, *n2w, *n2b;
    int rms1, rms2;
};

struct StepParams {
    const LayerDesc* layers;
    int n_layers;
    LinDesc head;
    const float* final_w;
    const uint8_t* emb_panel;
    const float* emb_scales;
    int emb_Kp;
    const float* pe;
    const float* rcos;
    const float* rsin;
    float* h;
    float* qkv;
    float* ff;
    float* part;  // [heads][n_chunks_max][kMaxHeadDim + 2]
    float* kc;
    float* vc;
    int32_t* tokens;
    State* state;
    unsigned long long* keys;  // [2] argmax keys, by step parity
    int* nan_flags;            // [2]
    unsigned int* bar;         // grid barrier arrivals (zero at launch)
    float* step_logits;        // [new tokens][V] or null
    uint32_t* err;
    int H, F, V, heads, kvh, hd, max_seq, n_chunks_max, xmax;
    float eps, scale;
    int prompt_len, n_steps;
};

__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid-wide barrier of a cooperative launch (all CTAs resident): the k-th
// barrier of the launch waits for the arrival counter to reach k * gridDim.
// Returns false when this or another CTA gave up on a wait.
__device__ bool grid_barrier(unsigned int* ctr, unsigned int target, uint32_t* err, int* flag_sh) {
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = *(volatile uint32_t*)err == kDevErrNone;
        if (ok) {
            // release: this CTA's writes (ordered before by __syncthreads)
            // are visible to whoever observes the arrival
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
            if (ld_acquire_u32(ctr) < target) {
                const uint64_t t0 = global_timer_ns();
                uint32_t spins = 0;
                while (ld_acquire_u32(ctr) < target) {
                    if ((++spins & 255u) == 0u) {
                        if (*(volatile uint32_t*)err != kDevErrNone) {
                            ok = 0;
                            break;
                        }
                        if (global_timer_ns() - t0 > 4000000000ull) {
                            atomicCAS(err, kDevErrNone, kDevErrTimeoutPeer);
                            ok = 0;
                            break;
                        }
                    }
                }
            }
        }
        *flag_sh = ok;
    }
    __syncthreads();
    return *flag_sh != 0;
}

// Block reductions with one __syncthreads: the r-th reduction of a row
// prologue writes its warp partials to buffer r of three 32-float buffers
// (a row needs at most three; the prologue ends with a barrier before the
// next one starts), and every thread adds the partials in the same order.
__device__ __forceinline__ float block_sum1(float v, float* red, int& rsel) {
    v = warp_sum(v);
    float* b = red + 32 * rsel;
    ++rsel;
    if ((threadIdx.x & 31) == 0) b[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < kStepWarps; ++w) t = __fadd_rn(t, b[w]);
    return t;
}
__device__ __forceinline__ float block_max1(float v, float* red, int& rsel) {
    v = warp_max(v);
    float* b = red + 32 * rsel;
    ++rsel;
    if ((threadIdx.x & 31) == 0) b[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = b[0];
#pragma unroll
    for (int w = 1; w < kStepWarps; ++w) t = fmaxf(t, b[w]);
    return t;
}

struct NormPre {
    float w[kRowRegs], b[kRowRegs];
};

__device__ __forceinline__ void prefetch_norm(const float* nw, const float* nb, int K, NormPre& np) {
#pragma unroll
    for (int k = 0; k < kRowRegs; ++k) {
        const int i = threadIdx.x + kStepThreads * k;
        np.w[k] = (nw && i < K) ? nw[i] : 0.0f;
        np.b[k] = (nb && i < K) ? nb[i] : 0.0f;
    }
}

// The row prologue of the step kernel: the same arithmetic as quantize_row
// (norm 284-319, then quantization.cpp:202-212) on the elements this thread
// owns, xs[tid + 512 k] for k >= 0 (already written by this thread, [K, Kp)
// zero).  Returns the row scale; qs is complete when it returns.
__device__ float quantize_row_step(float* xs, int8_t* qs, int K, int Kp, int type, int pro,
                                   const float* __restrict__ nw, const float* __restrict__ nb, const NormPre& np,
                                   float eps, float* red) {
    const int tid = threadIdx.x;
    int rsel = 0;
    if (pro == kProRms) {
        float ss = 0.0f;
        for (int i = tid; i < K; i += kStepThreads) ss = __fadd_rn(ss, __fmul_rn(xs[i], xs[i]));
        ss = block_sum1(ss, red, rsel);
        const float var = __fdiv_rn(ss, (float)K);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
        for (int k = 0; k < kRowRegs; ++k) {
            const int i = tid + kStepThreads * k;
            if (i < K) xs[i] = __fmul_rn(__fmul_rn(xs[i], inv), np.w[k]);
        }
        for (int i = tid + kStepThreads * kRowRegs; i < K; i += kStepThreads)
            xs[i] = __fmul_rn(__fmul_rn(xs[i], inv), nw[i]);
    } else if (pro == kProLayer) {
        float sm = 0.0f;
        for (int i = tid; i < K; i += kStepThreads) sm = __fadd_rn(sm, xs[i]);
        sm = block_sum1(sm, red, rsel);
        const float mean = __fdiv_rn(sm, (float)K);
        float ss = 0.0f;
        for (int i = tid; i < K; i += kStepThreads) {
            const float c = __fsub_rn(xs[i], mean);
            ss = __fadd_rn(ss, __fmul_rn(c, c));
        }
        ss = block_sum1(ss, red, rsel);
        const float var = __fdiv_rn(ss, (float)K);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
        for (int k = 0; k < kRowRegs; ++k) {
            const int i = tid + kStepThreads * k;
            if (i < K) xs[i] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xs[i], mean), inv), np.w[k]), np.b[k]);
        }
        for (int i = tid + kStepThreads * kRowRegs; i < K; i += kStepThreads)
            xs[i] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xs[i], mean), inv), nw[i]), nb[i]);
    }
    float m = 0.0f;
    for (int i = tid; i < K; i += kStepThreads) m = fmaxf(m, fabsf(xs[i]));
    m = block_max1(m, red, rsel);
    const float s = zq_scale_from_absmax(m, 127.0f);
    const float rcp = zq_quant_rcp(s);
    for (int i = tid; i < Kp; i += kStepThreads) {
        const int8_t code = i < K ? (int8_t)zq_quantize_value_rcp(xs[i], s, rcp, 127) : (int8_t)0;
        qs[i] = code;
    }
    __syncthreads();
    return s;
}

struct Pre {
    uint4 w[kPreSlots];
    float sc, bi, res;  // lane j < columns: scale, bias and residual of the warp's column j
};

// This warp's columns of L are gw, gw + W, ... (at most kMaxColsPerWarp at a
// time); its lanes take the columns' 16-byte chunks in order, so slot u of
// lane l holds flat chunk l + 32u.  Lane j also loads column j's scale and
// bias and, when `res` is given, the residual value res[col].
template <int kType>
__device__ __forceinline__ void prefetch_cols(const LinDesc& L, int gw, int W, int lane, const float* res, Pre& pre) {
    const int cb = kType == kInt8 ? L.Kp : (L.Kp >> 1);
    const int chunks = cb >> 4;
    int ncols = gw < L.N ? (L.N - gw + W - 1) / W : 0;
    if (ncols > kMaxColsPerWarp) ncols = kMaxColsPerWarp;
    const int total = ncols * chunks;
    if (ncols <= 1) {
        const uint8_t* base = L.panel + (size_t)gw * cb;
#pragma unroll
        for (int u = 0; u < kPreSlots; ++u) {
            const int f = lane + 32 * u;
            pre.w[u] = f < total ? ld_stream_u4(base + (size_t)f * 16) : make_uint4(0u, 0u, 0u, 0u);
        }
    } else {
        int ci = 0, c = lane;  // flat chunk lane + 32u = column ci, chunk c
        while (c >= chunks) c -= chunks, ++ci;
#pragma unroll
        for (int u = 0; u < kPreSlots; ++u) {
            pre.w[u] = ci < ncols ? ld_stream_u4(L.panel + (size_t)(gw + ci * W) * cb + (size_t)c * 16)
                                  : make_uint4(0u, 0u, 0u, 0u);
            c += 32;
            while (c >= chunks) c -= chunks, ++ci;
        }
    }
    const int col = gw + lane * W;
    const bool mine = lane < ncols;
    pre.sc = mine ? L.scales[col] : 0.0f;
    pre.bi = (mine && L.bias) ? L.bias[col] : 0.0f;
    pre.res = (mine && res) ? __ldcg(res + col) : 0.0f;
}

// Dots of this warp's columns against the codes in shared memory; for every
// column epi(col, acc, scale, bias, residual) runs on lane 0.  The first
// round uses what prefetch_cols loaded; later rounds reload `pre` in place.
template <int kType, class Epi>
__device__ __forceinline__ void run_cols(const LinDesc& L, int gw, int W, int lane, Pre& pre, const float* res,
                                         const int8_t* qs, Epi&& epi) {
    const int cb = kType == kInt8 ? L.Kp : (L.Kp >> 1);
    const int chunks = cb >> 4;
    for (int first = gw, group = 0; first < L.N; first += kMaxColsPerWarp * W, ++group) {
        int ncols = (L.N - first + W - 1) / W;
        if (ncols > kMaxColsPerWarp) ncols = kMaxColsPerWarp;
        const int total = ncols * chunks;
        int acc[kMaxColsPerWarp];
#pragma unroll
        for (int j = 0; j < kMaxColsPerWarp; ++j) acc[j] = 0;
        if (ncols == 1) {
            // one column: flat chunk f is chunk f of column `first`
            const uint8_t* base = L.panel + (size_t)first * cb;
            for (int f0 = 0; f0 < total; f0 += 32 * kPreSlots) {
                if (group != 0 || f0 != 0) {
#pragma unroll
                    for (int u = 0; u < kPreSlots; ++u) {
                        const int f = f0 + lane + 32 * u;
                        if (f < total) pre.w[u] = ld_stream_u4(base + (size_t)f * 16);
                    }
                }
                int d[1] = {0};
#pragma unroll
                for (int u = 0; u < kPreSlots; ++u) {
                    const int f = f0 + lane + 32 * u;
                    if (f < total) {
                        if (kType == kInt8)
                            dot16_int8<1>(pre.w[u], qs, L.Kp, f * 16, d);
                        else
                            dot16_int4<1>(pre.w[u], qs, L.Kp, f * 32, d);
                    }
                }
                acc[0] += d[0];
            }
        } else
        for (int f0 = 0; f0 < total; f0 += 32 * kPreSlots) {
            if (group != 0 || f0 != 0) {
#pragma unroll
                for (int u = 0; u < kPreSlots; ++u) {
                    const int f = f0 + lane + 32 * u;
                    if (f < total) {
                        const int ci = f / chunks, c = f - ci * chunks;
                        pre.w[u] = ld_stream_u4(L.panel + (size_t)(first + ci * W) * cb + (size_t)c * 16);
                    }
                }
            }
            int ci = 0, c = f0 + lane;  // flat chunk f0 + lane + 32u = column ci, chunk c
            while (c >= chunks) c -= chunks, ++ci;
#pragma unroll
            for (int u = 0; u < kPreSlots; ++u) {
                if (ci < ncols) {
                    int d[1] = {0};
                    if (kType == kInt8)
                        dot16_int8<1>(pre.w[u], qs, L.Kp, c * 16, d);
                    else
                        dot16_int4<1>(pre.w[u], qs, L.Kp, c * 32, d);
#pragma unroll
                    for (int j = 0; j < kMaxColsPerWarp; ++j)
                        if (j == ci) acc[j] += d[0];
                }
                c += 32;
                while (c >= chunks) c -= chunks, ++ci;
            }
        }
#pragma unroll
        for (int j = 0; j < kMaxColsPerWarp; ++j) {
            if (j < ncols) {
                int v = acc[j];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                float sc = __shfl_sync(0xffffffffu, pre.sc, j);
                float bi = __shfl_sync(0xffffffffu, pre.bi, j);
                float rs = __shfl_sync(0xffffffffu, pre.res, j);
                const int col = first + j * W;
                if (lane == 0) {
                    if (group != 0) {
                        sc = L.scales[col];
                        bi = L.bias ? L.bias[col] : 0.0f;
                        rs = res ? __ldcg(res + col) : 0.0f;
                    }
                    epi(col, v, sc, bi, rs);
                }
            }
        }
    }
}

// Query rows of heads h0 .. h0+nh-1 into q_s (row stride kMaxHeadDim), with
// RoPE at `pos` (apply_rope 347-384) when the model uses it.
__device__ __forceinline__ void load_queries(const StepParams& p, float* q_s, int h0, int nh, int pos, int tid) {
    const int hd = p.hd, half = hd >> 1;
    if (p.rcos) {
        for (int e = tid; e < nh * half; e += kStepThreads) {
            const int i = e / half, t = e - i * half;
            const float* qsrc = p.qkv + (size_t)(h0 + i) * hd;
            const float qe = __ldcg(qsrc + 2 * t), qo = __ldcg(qsrc + 2 * t + 1);
            const float c = p.rcos[(size_t)pos * half + t], sn = p.rsin[(size_t)pos * half + t];
            q_s[i * kMaxHeadDim + 2 * t] = __fsub_rn(__fmul_rn(qe, c), __fmul_rn(qo, sn));
            q_s[i * kMaxHeadDim + 2 * t + 1] = __fadd_rn(__fmul_rn(qe, sn), __fmul_rn(qo, c));
        }
    } else {
        for (int e = tid; e < nh * hd; e += kStepThreads) {
            const int i = e / hd, d = e - i * hd;
            q_s[i * kMaxHeadDim + d] = __ldcg(p.qkv + (size_t)(h0 + i) * hd + d);
        }
    }
}

// One attention item: query heads of KV group `grp` against positions
// [chunk*64, chunk*64 + 64) <= pos; writes each head's (m, l, c) partial.
__device__ __noinline__ void attention_item(const StepParams& p, int grp, int chunk, int pos, int li, float* q_s, float* kn,
                               float* vn, float* sc, float* mh, float* wpart) {
    constexpr int kPerLane = kMaxHeadDim / 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hd = p.hd, half = hd >> 1;
    const int rep = p.heads / p.kvh;
    const size_t cache_layer = (size_t)p.kvh * p.max_seq * hd;
    float* kc_l = p.kc + (size_t)li * cache_layer;
    float* vc_l = p.vc + (size_t)li * cache_layer;
    const float* ksrc = p.qkv + (size_t)p.heads * hd + (size_t)grp * hd;
    const float* vsrc = p.qkv + (size_t)(p.heads + p.kvh) * hd + (size_t)grp * hd;
    // Every load is issued before the first wait: the cached keys and values
    // of this warp's positions, the new key and value, the first queries.
    // The cache rows are loaded whatever the position (every row below
    // max_seq exists), so these loads need not wait for `pos`; rows past it
    // are zeroed once it is known.
    float kr[kAttnPosPerWarp][kPerLane], vr[kAttnPosPerWarp][kPerLane];
#pragma unroll
    for (int i = 0; i < kAttnPosPerWarp; ++i) {
        const int j = chunk * kAttnChunk + warp * kAttnPosPerWarp + i;
        const float* kj = kc_l + ((size_t)grp * p.max_seq + j) * hd;
        const float* vj = vc_l + ((size_t)grp * p.max_seq + j) * hd;
#pragma unroll
        for (int r = 0; r < kPerLane; ++r) {
            const int d = lane + 32 * r;
            const bool row = d < hd && j < p.max_seq;
            kr[i][r] = row ? __ldcg(kj + d) : 0.0f;
            vr[i][r] = row ? __ldcg(vj + d) : 0.0f;
        }
    }
    if (chunk * kAttnChunk > pos) return;  // a chunk past the position (the whole block leaves)
    if (p.rcos) {
        if (tid < half) {
            const float c = p.rcos[(size_t)pos * half + tid], sn = p.rsin[(size_t)pos * half + tid];
            const float ke = __ldcg(ksrc + 2 * tid), ko = __ldcg(ksrc + 2 * tid + 1);
            kn[2 * tid] = __fsub_rn(__fmul_rn(ke, c), __fmul_rn(ko, sn));
            kn[2 * tid + 1] = __fadd_rn(__fmul_rn(ke, sn), __fmul_rn(ko, c));
        }
    } else if (tid < hd) {
        kn[tid] = __ldcg(ksrc + tid);
    }
    if (tid < hd) vn[tid] = __ldcg(vsrc + tid);
    load_queries(p, q_s, grp * rep, rep < kHeadBatch ? rep : kHeadBatch, pos, tid);
    __syncthreads();
    if (chunk == 0 && tid < hd) {
        kc_l[((size_t)grp * p.max_seq + pos) * hd + tid] = kn[tid];
        vc_l[((size_t)grp * p.max_seq + pos) * hd + tid] = vn[tid];
    }
#pragma unroll
    for (int i = 0; i < kAttnPosPerWarp; ++i) {
        const int j = chunk * kAttnChunk + warp * kAttnPosPerWarp + i;
        if (j == pos) {
#pragma unroll
            for (int r = 0; r < kPerLane; ++r) {
                const int d = lane + 32 * r;
                if (d < hd) kr[i][r] = kn[d], vr[i][r] = vn[d];
            }
        } else if (j > pos) {
#pragma unroll
            for (int r = 0; r < kPerLane; ++r) kr[i][r] = vr[i][r] = 0.0f;
        }
    }
    for (int hb = 0; hb < rep; hb += kHeadBatch) {
        const int nh = rep - hb < kHeadBatch ? rep - hb : kHeadBatch;
        if (hb > 0) {  // the previous batch ended with a barrier: q_s is free
            load_queries(p, q_s, grp * rep + hb, nh, pos, tid);
            __syncthreads();
        }
        // scores (forward_block 424-451 for the newest row)
        for (int i2 = 0; i2 < nh; ++i2) {
#pragma unroll
            for (int i = 0; i < kAttnPosPerWarp; ++i) {
                float part = 0.0f;
#pragma unroll
                for (int r = 0; r < kPerLane; ++r) {
                    const int d = lane + 32 * r;
                    if (d < hd) part = __fadd_rn(part, __fmul_rn(q_s[i2 * kMaxHeadDim + d], kr[i][r]));
                }
                part = warp_sum(part);
                const int t = warp * kAttnPosPerWarp + i;
                const int j = chunk * kAttnChunk + t;
                if (lane == 0) sc[i2 * kAttnChunk + t] = j <= pos ? __fmul_rn(part, p.scale) : -INFINITY;
            }
        }
        __syncthreads();
        // chunk softmax: warp i2 takes head i2
        if (warp < nh) {
            const float a0 = sc[warp * kAttnChunk + lane], a1 = sc[warp * kAttnChunk + lane + 32];
            const float m = warp_max(fmaxf(a0, a1));
            const float e0 = a0 == -INFINITY ? 0.0f : expf(__fsub_rn(a0, m));
            const float e1 = a1 == -INFINITY ? 0.0f : expf(__fsub_rn(a1, m));
            const float l = warp_sum(__fadd_rn(e0, e1));
            sc[warp * kAttnChunk + lane] = e0;
            sc[warp * kAttnChunk + lane + 32] = e1;
            if (lane == 0) mh[warp] = m, mh[kHeadBatch + warp] = l;
        }
        __syncthreads();
        // partial context of this warp's positions
        for (int i2 = 0; i2 < nh; ++i2) {
#pragma unroll
            for (int r = 0; r < kPerLane; ++r) {
                float a = 0.0f;
#pragma unroll
                for (int i = 0; i < kAttnPosPerWarp; ++i)
                    a = __fadd_rn(a, __fmul_rn(sc[i2 * kAttnChunk + warp * kAttnPosPerWarp + i], vr[i][r]));
                const int d = lane + 32 * r;
                if (d < hd) wpart[(warp * kHeadBatch + i2) * kMaxHeadDim + d] = a;
            }
        }
        __syncthreads();
        for (int e = tid; e < nh * hd; e += kStepThreads) {
            const int i2 = e / hd, d = e - i2 * hd;
            float c = 0.0f;
#pragma unroll
            for (int w = 0; w < kStepWarps; ++w) c = __fadd_rn(c, wpart[(w * kHeadBatch + i2) * kMaxHeadDim + d]);
            float* dst = p.part + ((size_t)(grp * rep + hb + i2) * p.n_chunks_max + chunk) * (kMaxHeadDim + 2);
            dst[2 + d] = c;
            if (d == 0) dst[0] = mh[i2], dst[1] = mh[kHeadBatch + i2];
        }
        __syncthreads();
    }
}

// Attention of the kernel chain: one block of 512 threads per (KV group,
// 64-position chunk) runs attention_item; blocks of chunks past the current
// position return at once, so one launch shape serves every position.  The
// out_proj kernel that follows merges the chunks (kProMerge).
constexpr int kAttnSmemFloats = kHeadBatch * kMaxHeadDim + 2 * kMaxHeadDim + kHeadBatch * kAttnChunk +
                                2 * kHeadBatch + kStepWarps * kHeadBatch * kMaxHeadDim;
__global__ void __launch_bounds__(kStepThreads) attn_chunk_kernel(const __grid_constant__ StepParams p, int li) {
    extern __shared__ __align__(16) float asm_[];
    float* q_s = asm_;
    float* kn = q_s + kHeadBatch * kMaxHeadDim;
    float* vn = kn + kMaxHeadDim;
    float* sc = vn + kMaxHeadDim;
    float* mh = sc + kHeadBatch * kAttnChunk;
    float* wpart = mh + 2 * kHeadBatch;
    pdl_launch_dependents();
    pdl_wait_primary();
    const int pos = __ldcg(&p.state->pos);
    const int grp = blockIdx.x / p.n_chunks_max, chunk = blockIdx.x - grp * p.n_chunks_max;
    attention_item(p, grp, chunk, pos, li, q_s, kn, vn, sc, mh, wpart);  // returns at once past pos
}

// Context row of the attention: merges the chunks' (m, l, c) partials into
// xs[o], o = heads * hd, for the elements this thread owns:
// M = max m, L = sum l e^(m - M), ctx = (sum c e^(m - M)) / L.
__device__ __noinline__ void merge_context(const StepParams& p, int nchunk, float* xs, float* mls, float* invl) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int H = p.H, hd = p.hd;
    const size_t stride = kMaxHeadDim + 2;
    const bool fast = nchunk <= kMergeChunks && H <= 2 * kStepThreads;
    float cv[2][kMergeChunks];
    if (fast) {  // this thread's partial contexts, loaded with the (m, l) pairs
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int o = tid + kStepThreads * k;
            const int hq = o / hd, d = o - hq * hd;
            const float* ph = p.part + (size_t)hq * p.n_chunks_max * stride + 2 + d;
#pragma unroll
            for (int c = 0; c < kMergeChunks; ++c)
                cv[k][c] = (o < H && c < nchunk) ? __ldcg(ph + (size_t)c * stride) : 0.0f;
        }
    }
    for (int e = tid; e < p.heads * nchunk; e += kStepThreads) {
        const int hq = e / nchunk, c = e - hq * nchunk;
        const float* pc = p.part + ((size_t)hq * p.n_chunks_max + c) * stride;
        mls[2 * e] = __ldcg(pc);
        mls[2 * e + 1] = __ldcg(pc + 1);
    }
    __syncthreads();
    for (int hq = warp; hq < p.heads; hq += kStepWarps) {
        float M = -INFINITY;
        for (int c = lane; c < nchunk; c += 32) M = fmaxf(M, mls[2 * (hq * nchunk + c)]);
        M = warp_max(M);
        float L = 0.0f;
        for (int c = lane; c < nchunk; c += 32) {
            const int e = hq * nchunk + c;
            const float f = expf(__fsub_rn(mls[2 * e], M));
            L = __fadd_rn(L, __fmul_rn(mls[2 * e + 1], f));
            mls[2 * e] = f;
        }
        L = warp_sum(L);
        if (lane == 0) invl[hq] = L > 0.0f ? __fdiv_rn(1.0f, L) : 0.0f;
    }
    __syncthreads();
    if (fast) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int o = tid + kStepThreads * k;
            if (o < H) {
                const int hq = o / hd;
                float acc = 0.0f;
#pragma unroll
                for (int c = 0; c < kMergeChunks; ++c)
                    if (c < nchunk) acc = __fadd_rn(acc, __fmul_rn(cv[k][c], mls[2 * (hq * nchunk + c)]));
                xs[o] = __fmul_rn(acc, invl[hq]);
            }
        }
    } else {
        for (int o = tid; o < H; o += kStepThreads) {
            const int hq = o / hd, d = o - hq * hd;
            const float* ph = p.part + (size_t)hq * p.n_chunks_max * stride + 2 + d;
            float acc = 0.0f;
            for (int c = 0; c < nchunk; ++c)
                acc = __fadd_rn(acc, __fmul_rn(__ldcg(ph + (size_t)c * stride), mls[2 * (hq * nchunk + c)]));
            xs[o] = __fmul_rn(acc, invl[hq]);
        }
    }
}

// Per-CTA control block at the start of the step kernel's shared memory.
struct StepCtl {
    float red[96];
    unsigned long long cta_key;
    int cta_nan;
    int flag;
};
constexpr int kStepCtlFloats = (int)((sizeof(StepCtl) + 15) / 16 * 4);

struct StepSmem {
    StepCtl* ctl;
    float* xs;
    int8_t* qs;
    float *q_s, *kn, *vn, *sc, *mh, *wpart, *mls, *invl;
    LayerDesc* lds;
};

__device__ __forceinline__ StepSmem step_smem(const StepParams& p) {
    extern __shared__ __align__(16) float ssm[];
    StepSmem m;
    m.ctl = reinterpret_cast<StepCtl*>(ssm);
    m.xs = ssm + kStepCtlFloats;                                       // [xmax]
    m.qs = reinterpret_cast<int8_t*>(m.xs + p.xmax);                   // [xmax]
    m.q_s = m.xs + p.xmax + p.xmax / 4;                                // [kHeadBatch][kMaxHeadDim]
    m.kn = m.q_s + kHeadBatch * kMaxHeadDim;                           // [kMaxHeadDim]
    m.vn = m.kn + kMaxHeadDim;                                         // [kMaxHeadDim]
    m.sc = m.vn + kMaxHeadDim;                                         // [kHeadBatch][kAttnChunk]
    m.mh = m.sc + kHeadBatch * kAttnChunk;                             // [2][kHeadBatch]
    m.wpart = m.mh + 2 * kHeadBatch;                                   // [kStepWarps][kHeadBatch][kMaxHeadDim]
    m.mls = m.wpart + kStepWarps * kHeadBatch * kMaxHeadDim;           // [heads][n_chunks_max][2]
    m.invl = m.mls + 2 * p.heads * p.n_chunks_max;                     // [heads]
    m.lds = reinterpret_cast<LayerDesc*>(m.invl + p.heads + (p.heads & 1));  // [n_layers]
    return m;
}

enum RowSrc { kRowEmbed = 0, kRowGlobal = 1, kRowMerge = 2 };
enum EpiKind { kEpStore = 0, kEpGelu = 1, kEpResidual = 2, kEpLogits = 3 };

struct PhaseArgs {
    LinDesc L;
    const float* nw;
    const float* nb;
    int pro;
    int row_src;      // RowSrc
    const float* row; // kRowGlobal: the activation row in global memory
    int K;            // row length
    int epi;          // EpiKind
    float* out;       // destination of the columns (kEpLogits: per-step logits or null)
    const float* res; // kEpResidual: residual source (out itself)
};

// One decode linear as a phase of the step kernel: load this warp's weight
// columns (and scales, biases, residuals) and this thread's norm weights,
// wait at the grid barrier (when `barrier_target` is not 0), build and
// quantize the activation row, then the dots and the epilogue.  Kept out of
// line so that every phase runs the same, warm, instructions.
template <int kType>
__device__ __noinline__ bool linear_phase(const StepParams& p, const PhaseArgs& a, unsigned int barrier_target, int tok,
                                          int pos, int nchunk) {
    const StepSmem m = step_smem(p);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int W = gridDim.x * kStepWarps;
    const int gw = blockIdx.x * kStepWarps + warp;
    Pre pre;
    NormPre np;
    prefetch_cols<kType>(a.L, gw, W, lane, a.epi == kEpResidual ? a.res : nullptr, pre);
    if (a.pro != kProNone) prefetch_norm(a.nw, a.nb, a.K, np);
    if (barrier_target && !grid_barrier(p.bar, barrier_target, p.err, &m.ctl->flag)) return false;
    float* xs = m.xs;
    if (a.row_src == kRowEmbed) {
        // token_lookup (271-282) [+ sinusoidal PE]
        for (int j = tid; j < a.K; j += kStepThreads) {
            int code;
            if (kType == kInt8) {
                code = (int8_t)p.emb_panel[(size_t)j * p.emb_Kp + tok];
            } else {
                const uint8_t b = p.emb_panel[(size_t)j * (p.emb_Kp >> 1) + panel_int4_byte(tok)];
                const int nib = (b >> panel_int4_shift(tok)) & 0x0F;
                code = nib < 8 ? nib : nib - 16;
            }
            float v = x86_mul((float)code, p.emb_scales[j]);
            if (p.pe) v = x86_add(v, p.pe[(size_t)pos * a.K + j]);
            xs[j] = v;
            if (blockIdx.x == 0) p.h[j] = v;  // residual stream, read after the next barriers
        }
    } else if (a.row_src == kRowGlobal) {
        load_row<kStepThreads>(a.row, a.K, a.K, xs);
    } else {
        merge_context(p, nchunk, xs, m.mls, m.invl);
    }
    for (int j = a.K + tid; j < a.L.Kp; j += kStepThreads) xs[j] = 0.0f;
    if (a.epi == kEpLogits && tid == 0) m.ctl->cta_key = 0ull, m.ctl->cta_nan = 0;
    const float srow = quantize_row_step(xs, m.qs, a.K, a.L.Kp, kType, a.pro, a.nw, a.nb, np, p.eps, m.ctl->red);
    unsigned long long best = 0ull;
    int nan = 0;
    run_cols<kType>(a.L, gw, W, lane, pre, a.epi == kEpResidual ? a.res : nullptr, m.qs,
                    [&](int col, int acc, float s_col, float b, float r) {
                        float v = zq_epilogue(acc, srow, s_col);
                        if (a.L.bias) v = x86_add(v, b);
                        switch (a.epi) {
                            case kEpStore: a.out[col] = v; break;
                            case kEpGelu: a.out[col] = gelu_ref(v); break;
                            case kEpResidual: a.out[col] = x86_add(r, v); break;
                            default:
                                if (a.out) a.out[col] = v;
                                if (isnan(v)) {
                                    nan = 1;
                                } else {
                                    const unsigned long long k = argmax_key(v, col);
                                    if (k > best) best = k;
                                }
                        }
                    });
    if (a.epi == kEpLogits) {
        if (lane == 0) {
            if (best) atomicMax(&m.ctl->cta_key, best);
            if (nan) m.ctl->cta_nan = 1;
        }
        __syncthreads();
    }
    return true;
}

template <int kType>
__global__ void __launch_bounds__(kStepThreads, 1) step_kernel(const __grid_constant__ StepParams p) {
    const StepSmem m = step_smem(p);
    const int tid = threadIdx.x;
    const unsigned int G = gridDim.x;
    const int H = p.H;

    // layer descriptors into shared memory (read by every phase)
    {
        const int words = p.n_layers * (int)(sizeof(LayerDesc) / sizeof(int));
        const int* src = reinterpret_cast<const int*>(p.layers);
        int* dst = reinterpret_cast<int*>(m.lds);
        for (int i = tid; i < words; i += kStepThreads) dst[i] = src[i];
    }
    __syncthreads();

    int pos = __ldcg(&p.state->pos);
    int tok = __ldcg(p.tokens + pos);
    bool ok = true;
    bool need_barrier = false;  // h was written since the last barrier
    unsigned int nbar = 0;      // barriers passed in this launch
    for (int step = 0; step < p.n_steps && ok; ++step, ++pos) {
        const bool want_logits = pos + 1 >= p.prompt_len;
        const int nchunk = (pos + kAttnChunk) / kAttnChunk;
        for (int li = 0; li < p.n_layers && ok; ++li) {
            const LayerDesc& Ld = m.lds[li];
            PhaseArgs a;
            // ---- A: (layer 0: embedding) norm1 -> q|k|v ----------------
            a.L = Ld.qkv;
            a.nw = Ld.n1w;
            a.nb = Ld.n1b;
            a.pro = Ld.rms1 ? kProRms : kProLayer;
            a.row_src = li == 0 ? kRowEmbed : kRowGlobal;
            a.row = p.h;
            a.K = H;
            a.epi = kEpStore;
            a.out = p.qkv;
            a.res = nullptr;
            const bool bar_a = li > 0 || need_barrier;
            if (bar_a) ++nbar;
            ok = linear_phase<kType>(p, a, bar_a ? nbar * G : 0u, tok, pos, nchunk);
            if (!ok) break;
            // ---- B: attention items ------------------------------------
            ++nbar;
            ok = grid_barrier(p.bar, nbar * G, p.err, &m.ctl->flag);
            if (!ok) break;
            if (li == 0 && blockIdx.x == 0 && tid == 0) {
                // every CTA has read the previous step's argmax key by now
                p.keys[(step + 1) & 1] = 0ull;
                p.nan_flags[(step + 1) & 1] = 0;
            }
            for (int item = blockIdx.x; item < p.kvh * nchunk; item += G)
                attention_item(p, item / nchunk, item % nchunk, pos, li, m.q_s, m.kn, m.vn, m.sc, m.mh, m.wpart);
            // ---- C: context merge -> out_proj, residual -----------------
            a.L = Ld.out;
            a.nw = a.nb = nullptr;
            a.pro = kProNone;
            a.row_src = kRowMerge;
            a.epi = kEpResidual;
            a.out = p.h;
            a.res = p.h;
            ok = linear_phase<kType>(p, a, ++nbar * G, tok, pos, nchunk);
            if (!ok) break;
            // ---- D: norm2 -> ff_up, GELU --------------------------------
            a.L = Ld.up;
            a.nw = Ld.n2w;
            a.nb = Ld.n2b;
            a.pro = Ld.rms2 ? kProRms : kProLayer;
            a.row_src = kRowGlobal;
            a.row = p.h;
            a.epi = kEpGelu;
            a.out = p.ff;
            a.res = nullptr;
            ok = linear_phase<kType>(p, a, ++nbar * G, tok, pos, nchunk);
            if (!ok) break;
            // ---- E: ff_down, residual -----------------------------------
            a.L = Ld.down;
            a.nw = a.nb = nullptr;
            a.pro = kProNone;
            a.row = p.ff;
            a.K = p.F;
            a.epi = kEpResidual;
            a.out = p.h;
            a.res = p.h;
            ok = linear_phase<kType>(p, a, ++nbar * G, tok, pos, nchunk);
        }
        if (!ok) break;
        need_barrier = true;
        if (want_logits) {
            // ---- final RMS norm (forward 492) -> lm_head -> argmax key --
            PhaseArgs a;
            a.L = p.head;
            a.nw = p.final_w;
            a.nb = nullptr;
            a.pro = kProRms;
            a.row_src = kRowGlobal;
            a.row = p.h;
            a.K = H;
            a.epi = kEpLogits;
            a.out = p.step_logits ? p.step_logits + (size_t)(pos + 1 - p.prompt_len) * p.V : nullptr;
            a.res = nullptr;
            ok = linear_phase<kType>(p, a, ++nbar * G, tok, pos, nchunk);
            if (!ok) break;
            if (tid == 0) {
                if (m.ctl->cta_key) atomicMax(p.keys + (step & 1), m.ctl->cta_key);
                if (m.ctl->cta_nan) atomicExch(p.nan_flags + (step & 1), 1);
            }
            ok = grid_barrier(p.bar, ++nbar * G, p.err, &m.ctl->flag);
            if (!ok) break;
            tok = token_from_key(__ldcg(p.keys + (step & 1)), __ldcg(p.nan_flags + (step & 1)), p.V);
            if (blockIdx.x == 0 && tid == 0) p.tokens[pos + 1] = tok;
            need_barrier = false;  // the argmax barrier ordered every read of h
        } else {
            tok = __ldcg(p.tokens + pos + 1);  // the prompt's next token
        }
    }
    if (blockIdx.x == 0 && tid == 0 && ok) p.state->pos = pos;
}

}  // namespace lm
}  // namespace zq

// ===========================================================================
// Host side
// ===========================================================================

namespace {

using zq::lm::State;

constexpr uint32_t kModelMagic = 0x4d4c5a51u;  // "QZLM" (quantized_language_model.cpp:557)
constexpr uint32_t kModelVersion = 1;          // 558

struct HostTensor {
    std::vector<size_t> dims;
    std::vector<float> data;  // empty tensor: no dims, no data
    size_t size() const { return data.size(); }
};

struct HostLinear {
    zq::ZyqRecord w;
    HostTensor bias;
};

struct HostBlock {
    bool rms1 = true, rms2 = true;
    HostTensor n1w, n1b, n2w, n2b;
    HostLinear q, k, v, o, up, down;
};

struct LmStatus {
    zq_status s = ZQ_OK;
    std::string msg;
};

class Reader {
public:
    Reader(const uint8_t* p, size_t n) : p_(p), n_(n) {}
    bool read(void* dst, size_t k) {
        if (!p_ || off_ > n_ || n_ - off_ < k) return false;
        std::memcpy(dst, p_ + off_, k);
        off_ += k;
        return true;
    }
    const uint8_t* here() const { return p_ + off_; }
    size_t left() const { return n_ - off_; }
    void skip(size_t k) { off_ += k; }

private:
    const uint8_t* p_;
    size_t n_, off_ = 0;
};

const char* kCorrupted = "ZYRON quantized model: corrupted file";

struct ParseError {
    zq_status s;
    std::string msg;
};

uint32_t rd_u32(Reader& r) {
    uint32_t v;
    if (!r.read(&v, 4)) throw ParseError{ZQ_ERR_RUNTIME, kCorrupted};
    return v;
}
uint64_t rd_u64(Reader& r) {
    uint64_t v;
    if (!r.read(&v, 8)) throw ParseError{ZQ_ERR_RUNTIME, kCorrupted};
    return v;
}
float rd_f32(Reader& r) {
    float v;
    if (!r.read(&v, 4)) throw ParseError{ZQ_ERR_RUNTIME, kCorrupted};
    return v;
}

// qread_tensor (quantized_language_model.cpp:605-612 region): rank, dims,
// size, data; rank 0 with size 0 is the empty tensor.
HostTensor rd_tensor(Reader& r) {
    HostTensor t;
    const uint64_t rank = rd_u64(r);
    if (rank > 16) throw ParseError{ZQ_ERR_RUNTIME, "ZYRON quantized model: invalid tensor rank"};
    size_t expect = 1;
    for (uint64_t i = 0; i < rank; ++i) {
        const uint64_t d = rd_u64(r);
        if (d == 0) throw ParseError{ZQ_ERR_INVALID_ARGUMENT, "ZYRON Shape: dimensions must be > 0"};
        if (expect > std::numeric_limits<size_t>::max() / d)
            throw ParseError{ZQ_ERR_OVERFLOW, "ZYRON Shape: element count overflow"};
        expect *= (size_t)d;
        t.dims.push_back((size_t)d);
    }
    const uint64_t size = rd_u64(r);
    if (rank == 0 && size == 0) return HostTensor{};
    if (size != expect) throw ParseError{ZQ_ERR_RUNTIME, "ZYRON quantized model: tensor size mismatch"};
    if (size > r.left() / sizeof(float)) throw ParseError{ZQ_ERR_RUNTIME, kCorrupted};
    t.data.resize((size_t)size);
    r.read(t.data.data(), (size_t)size * sizeof(float));
    return t;
}

HostLinear rd_linear(Reader& r) {
    HostLinear l;
    zq_status s = zq::parse_zyq(r.here(), r.left(), &l.w);
    if (s != ZQ_OK) throw ParseError{s, zq_last_error()};
    r.skip(l.w.consumed);
    l.bias = rd_tensor(r);
    // QuantizedLinear(QuantizedMatrix, Tensor) checks (quantized_linear.cpp:8-14)
    if (l.bias.size() != 0 && (l.bias.dims.size() != 1 || l.bias.size() != l.w.cols))
        throw ParseError{ZQ_ERR_INVALID_ARGUMENT, "ZYRON QuantizedLinear: bias shape mismatch"};
    return l;
}

// transformer::Config::validate (include/zyron/transformer/config.hpp:32-68).
void validate_config(const zq_lm_info& c, size_t qat_bits, float dropout) {
    const size_t kvh = c.num_kv_heads == 0 ? c.num_heads : c.num_kv_heads;
    if (c.vocab_size == 0 || c.hidden_size == 0 || c.num_layers == 0 || c.num_heads == 0 ||
        c.intermediate_size == 0 || c.max_sequence_length == 0)
        throw ParseError{ZQ_ERR_INVALID_ARGUMENT, "ZYRON Transformer: dimensions must be > 0"};
    if (c.hidden_size % c.num_heads != 0)
        throw ParseError{ZQ_ERR_INVALID_ARGUMENT, "ZYRON Transformer: hidden_size must be divisible by num_heads"};
    if (kvh == 0 || kvh > c.num_heads || c.num_heads % kvh != 0)
        throw ParseError{ZQ_ERR_INVALID_ARGUMENT,
                         "ZYRON Transformer: num_kv_heads must divide num_heads and be <= num_heads"};
    if (c.use_rope && ((c.hidden_size / c.num_heads) % 2 != 0))
        throw ParseError{ZQ_ERR_INVALID_ARGUMENT, "ZYRON Transformer: RoPE requires an even attention head dimension"};
    if (!(c.norm_eps > 0.0f)) throw ParseError{ZQ_ERR_INVALID_ARGUMENT, "ZYRON Transformer: norm_eps must be > 0"};
    if (!(c.rope_theta > 0.0f) || !std::isfinite(c.rope_theta))
        throw ParseError{ZQ_ERR_INVALID_ARGUMENT, "ZYRON Transformer: rope_theta must be finite and > 0"};
    if (!(dropout >= 0.0f) || dropout >= 1.0f || !std::isfinite(dropout))
        throw ParseError{ZQ_ERR_INVALID_ARGUMENT, "ZYRON Transformer: dropout must be finite and in [0, 1)"};
    if (qat_bits != 4 && qat_bits != 8)
        throw ParseError{ZQ_ERR_INVALID_ARGUMENT, "ZYRON Transformer: qat_bits must be 4 or 8"};
}

size_t tensor_bytes(const HostTensor& t) { return t.size() * sizeof(float); }
size_t zyq_bytes(const zq::ZyqRecord& w) { return w.payload_bytes + w.cols * sizeof(float); }

struct DevLayer {
    bool rms1 = true, rms2 = true;
    float *n1w = nullptr, *n1b = nullptr, *n2w = nullptr, *n2b = nullptr;
    zq_weight *qkv = nullptr, *out = nullptr, *up = nullptr, *down = nullptr;
    float *b_qkv = nullptr, *b_out = nullptr, *b_up = nullptr, *b_down = nullptr;
};

}  // namespace

struct zq_lm {
    zq_lm_info info{};
    int device = 0;
    zq_weight* emb = nullptr;
    float* pe = nullptr;
    float* final_w = nullptr;
    std::vector<DevLayer> layers;
    zq_weight* head = nullptr;
    float* b_head = nullptr;
    // runtime buffers
    float *h = nullptr, *qkv = nullptr, *ff = nullptr, *logits = nullptr;
    float *kc = nullptr, *vc = nullptr;
    float *rcos = nullptr, *rsin = nullptr;
    float* attn_part = nullptr;          // [heads][splits][128 + 2] chunk partials
    int attn_splits = 1;
    int32_t* tokens = nullptr;
    State* state = nullptr;
    std::vector<void*> allocations;
    cudaGraphExec_t graph_one = nullptr;
    cudaGraphExec_t graph_chunk = nullptr;
    // the same step ending in the penalised greedy choice
    cudaGraphExec_t graph_one_pen = nullptr;
    cudaGraphExec_t graph_chunk_pen = nullptr;
    zq::lm::PenaltyCfg* penalty = nullptr;  // read by next_token_penalized_kernel
    size_t penalty_smem = 0;                // its bitmaps
    // persistent decode (step_kernel): layer descriptors, barrier, argmax keys
    zq::lm::LayerDesc* layer_desc = nullptr;
    unsigned int* bar = nullptr;
    unsigned long long* keys = nullptr;
    int* nan_flags = nullptr;
    unsigned long long* head_slots = nullptr;  // the lm_head blocks' argmax keys (kernel chain)
    int head_blocks = 0;                       // lm_head grid: one resident wave
    int step_grid = 0;  // 0: cooperative launch unavailable, use the kernel chain
    size_t step_smem = 0;
    int xmax = 0;
    int chunk = 16;
    int persistent = 0;  // ZQ_LM_OPT_PERSISTENT
    // Used when the caller passes no stream: graph capture needs a stream
    // that is not a default stream.
    cudaStream_t own_stream = nullptr;
    ~zq_lm();
};

zq_lm::~zq_lm() {
    int cur = 0;
    cudaGetDevice(&cur);
    if (cur != device) cudaSetDevice(device);
    if (graph_one) cudaGraphExecDestroy(graph_one);
    if (graph_chunk) cudaGraphExecDestroy(graph_chunk);
    if (graph_one_pen) cudaGraphExecDestroy(graph_one_pen);
    if (graph_chunk_pen) cudaGraphExecDestroy(graph_chunk_pen);
    if (own_stream) cudaStreamDestroy(own_stream);
    zq_weight_destroy(emb);
    zq_weight_destroy(head);
    for (auto& l : layers) {
        zq_weight_destroy(l.qkv);
        zq_weight_destroy(l.out);
        zq_weight_destroy(l.up);
        zq_weight_destroy(l.down);
    }
    for (void* p : allocations) cudaFree(p);
    if (cur != device) cudaSetDevice(cur);
}

namespace {

template <class T>
cudaError_t dev_alloc(zq_lm* lm, T** p, size_t count) {
    void* q = nullptr;
    cudaError_t e = cudaMalloc(&q, count * sizeof(T) > 0 ? count * sizeof(T) : 16);
    if (e == cudaSuccess) {
        lm->allocations.push_back(q);
        *p = static_cast<T*>(q);
    }
    return e;
}

cudaError_t upload_tensor(zq_lm* lm, const HostTensor& t, float** out, cudaStream_t st) {
    *out = nullptr;
    if (t.size() == 0) return cudaSuccess;
    cudaError_t e = dev_alloc(lm, out, t.size());
    if (e == cudaSuccess) e = cudaMemcpyAsync(*out, t.data.data(), t.size() * sizeof(float), cudaMemcpyHostToDevice, st);
    return e;
}

zq_status make_weight(const zq::ZyqRecord& r, void* stream, zq_weight** out) {
    return zq_weight_create(r.type, r.rows, r.cols, r.scales.data(), r.payload, r.payload_bytes, stream, out);
}

#define LM_CUDA(call)                                             \
    do {                                                          \
        cudaError_t _e = (call);                                  \
        if (_e != cudaSuccess) return zq::cuda_error(_e, #call);  \
    } while (0)

#define LM_OK(call)                      \
    do {                                 \
        zq_status _s = (call);           \
        if (_s != ZQ_OK) return _s;      \
    } while (0)

size_t linear_smem(int Kp) { return (size_t)Kp * sizeof(float) + (size_t)Kp; }

// One column per warp (8 per block): every column's weights are loaded
// before the dependency wait; blocks beyond the resident ones run as a
// second wave.
int linear_blocks(const zq_weight* w) { return (int)((w->N + 7) / 8); }

// Every decode-step kernel is launched with programmatic dependent launch:
// it may start (and prefetch constant weights) while its predecessor runs,
// and waits in griddepcontrol.wait before reading anything the predecessor
// writes.
template <class... Params, class... Args>
cudaError_t launch_pdl(void (*kern)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<Params>(args)...);
}



constexpr size_t kMaxLinearSmem = 200 * 1024;

template <int kType, int kPro, int kEpi>
cudaError_t prepare_linear_t() {
    return cudaFuncSetAttribute(zq::lm::linear_kernel<kType, kPro, kEpi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)kMaxLinearSmem);
}

template <int kType>
cudaError_t prepare_type() {
    using namespace zq::lm;
    cudaError_t e = prepare_linear_t<kType, kProNone, kEpiStore>();
    if (e == cudaSuccess) e = prepare_linear_t<kType, kProNone, kEpiGelu>();
    if (e == cudaSuccess) e = prepare_linear_t<kType, kProNone, kEpiResidual>();
    if (e == cudaSuccess) e = prepare_linear_t<kType, kProRms, kEpiStore>();
    if (e == cudaSuccess) e = prepare_linear_t<kType, kProRms, kEpiGelu>();
    if (e == cudaSuccess) e = prepare_linear_t<kType, kProRms, kEpiResidual>();
    if (e == cudaSuccess) e = prepare_linear_t<kType, kProLayer, kEpiStore>();
    if (e == cudaSuccess) e = prepare_linear_t<kType, kProLayer, kEpiGelu>();
    if (e == cudaSuccess) e = prepare_linear_t<kType, kProLayer, kEpiResidual>();
    if (e == cudaSuccess) e = prepare_linear_t<kType, kProMerge, kEpiResidual>();
    if (e == cudaSuccess) e = prepare_linear_t<kType, kProRms, kEpiLogits>();
    return e;
}

// Kernel attributes are set once at load, outside any stream capture.
cudaError_t prepare_kernels() {
    cudaError_t e = prepare_type<ZQ_TYPE_INT8>();
    if (e == cudaSuccess) e = prepare_type<ZQ_TYPE_INT4>();
    return e;
}

template <int kType, int kPro, int kEpi>
cudaError_t launch_linear_t(const float* x, const float* nw, const float* nb, float eps, const zq_weight* w,
                            const float* bias, float* y, const State* st, int skip_prefill, cudaStream_t s,
                            zq::lm::MergeArgs merge, zq::lm::ArgmaxArgs am, int max_blocks) {
    auto kern = zq::lm::linear_kernel<kType, kPro, kEpi>;
    size_t smem = linear_smem(w->Kp);
    if (kPro == zq::lm::kProMerge) smem += (2 * (size_t)merge.heads * merge.n_chunks_max + merge.heads) * sizeof(float);
    const int blocks = max_blocks > 0 ? std::min(max_blocks, linear_blocks(w)) : linear_blocks(w);
    return launch_pdl(kern, dim3(blocks), dim3(zq::lm::kThreads), smem, s, x, (int)w->K, w->Kp, nw, nb, eps,
                      (const uint8_t*)w->panel, (const float*)w->scales, (int)w->N, bias, y, st, skip_prefill, merge,
                      am);
}

template <int kPro, int kEpi>
cudaError_t launch_linear(const float* x, const float* nw, const float* nb, float eps, const zq_weight* w,
                          const float* bias, float* y, const State* st, int skip_prefill, cudaStream_t s,
                          zq::lm::MergeArgs merge = {}, zq::lm::ArgmaxArgs am = {}, int max_blocks = 0) {
    return w->type == ZQ_TYPE_INT8 ? launch_linear_t<ZQ_TYPE_INT8, kPro, kEpi>(x, nw, nb, eps, w, bias, y, st,
                                                                             skip_prefill, s, merge, am, max_blocks)
                                   : launch_linear_t<ZQ_TYPE_INT4, kPro, kEpi>(x, nw, nb, eps, w, bias, y, st,
                                                                             skip_prefill, s, merge, am, max_blocks);
}

// The lm_head's grid: at most one resident wave.  Its warps stride over the
// columns, so the wave covers them all; (N + 7) / 8 blocks of one column per
// warp would run in several waves that each repeat the row's norm and
// quantization (vocab 16384: 2048 blocks, 4 resident per SM).
int head_blocks_for(const zq_weight* head) {
    using namespace zq::lm;
    const int full = linear_blocks(head);
    int dev = 0, sms = 0, per_sm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return full;
    const size_t smem = linear_smem(head->Kp);
    const cudaError_t e =
        head->type == ZQ_TYPE_INT8
            ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, linear_kernel<ZQ_TYPE_INT8, kProRms, kEpiLogits>,
                                                            kThreads, smem)
            : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, linear_kernel<ZQ_TYPE_INT4, kProRms, kEpiLogits>,
                                                            kThreads, smem);
    if (e != cudaSuccess || per_sm < 1 || sms < 1) return full;
    return std::min(full, sms * per_sm);
}

template <int kEpi>
cudaError_t launch_normed(bool rms, const float* x, const float* nw, const float* nb, float eps, const zq_weight* w,
                          const float* bias, float* y, const State* st, int skip, cudaStream_t s) {
    return rms ? launch_linear<zq::lm::kProRms, kEpi>(x, nw, nb, eps, w, bias, y, st, skip, s)
               : launch_linear<zq::lm::kProLayer, kEpi>(x, nw, nb, eps, w, bias, y, st, skip, s);
}

// Enqueue one decode step (all kernels) on `s`; `penalized` ends it with the
// greedy choice under the repetition penalty and n-gram block.
cudaError_t enqueue_step(zq_lm* lm, cudaStream_t s, bool penalized = false) {
    const zq_lm_info& c = lm->info;
    const int hd = (int)(c.hidden_size / c.num_heads);
    const int kvh = (int)(c.num_kv_heads == 0 ? c.num_heads : c.num_kv_heads);
    const float eps = c.norm_eps;
    const int hidden = (int)c.hidden_size;
    cudaError_t e = launch_pdl(zq::lm::embed_kernel, dim3((hidden + 255) / 256), dim3(256), 0, s,
                               (const uint8_t*)lm->emb->panel, lm->emb->type, lm->emb->Kp,
                               (const float*)lm->emb->scales, hidden, (const int32_t*)lm->tokens,
                               (const State*)lm->state, (const float*)lm->pe, lm->h);
    // attention chunks (attn_chunk_kernel) and their merge (kProMerge)
    zq::lm::StepParams ap{};
    ap.qkv = lm->qkv;
    ap.part = lm->attn_part;
    ap.kc = lm->kc;
    ap.vc = lm->vc;
    ap.state = lm->state;
    ap.rcos = c.use_rope ? lm->rcos : nullptr;
    ap.rsin = c.use_rope ? lm->rsin : nullptr;
    ap.H = hidden;
    ap.heads = (int)c.num_heads;
    ap.kvh = kvh;
    ap.hd = hd;
    ap.max_seq = (int)c.max_sequence_length;
    ap.n_chunks_max = lm->attn_splits;
    ap.scale = 1.0f / std::sqrt(static_cast<float>(hd));
    const zq::lm::MergeArgs merge{lm->attn_part, (int)c.num_heads, hd, lm->attn_splits};
    for (size_t li = 0; li < lm->layers.size() && e == cudaSuccess; ++li) {
        const DevLayer& L = lm->layers[li];
        e = launch_normed<zq::lm::kEpiStore>(L.rms1, lm->h, L.n1w, L.n1b, eps, L.qkv, L.b_qkv, lm->qkv, lm->state, 0, s);
        if (e != cudaSuccess) break;
        e = launch_pdl(zq::lm::attn_chunk_kernel, dim3((unsigned)(kvh * lm->attn_splits)), dim3(zq::lm::kStepThreads),
                       zq::lm::kAttnSmemFloats * sizeof(float), s, ap, (int)li);
        if (e != cudaSuccess) break;
        e = launch_linear<zq::lm::kProMerge, zq::lm::kEpiResidual>(nullptr, nullptr, nullptr, eps, L.out, L.b_out, lm->h,
                                                                   lm->state, 0, s, merge);
        if (e != cudaSuccess) break;
        e = launch_normed<zq::lm::kEpiGelu>(L.rms2, lm->h, L.n2w, L.n2b, eps, L.up, L.b_up, lm->ff, lm->state, 0, s);
        if (e != cudaSuccess) break;
        e = launch_linear<zq::lm::kProNone, zq::lm::kEpiResidual>(lm->ff, nullptr, nullptr, eps, L.down, L.b_down,
                                                                  lm->h, lm->state, 0, s);
    }
    if (e != cudaSuccess) return e;
    // final norm is always RMS without bias (forward 492); the lm_head folds
    // the greedy choice into lm->keys[0] / lm->nan_flags[0]
    const zq::lm::ArgmaxArgs am{lm->head_slots, lm->nan_flags};
    e = launch_linear<zq::lm::kProRms, zq::lm::kEpiLogits>(lm->h, lm->final_w, nullptr, eps, lm->head, lm->b_head,
                                                           lm->logits, lm->state, 1, s, {}, am, lm->head_blocks);
    if (e != cudaSuccess) return e;
    if (penalized)
        return launch_pdl(zq::lm::next_token_penalized_kernel, dim3(1), dim3(zq::lm::kPenaltyThreads),
                          lm->penalty_smem, s, (const float*)lm->logits, (int)c.vocab_size, lm->tokens, lm->state,
                          (const zq::lm::PenaltyCfg*)lm->penalty, lm->nan_flags);
    return launch_pdl(zq::lm::next_token_kernel, dim3(1), dim3(256), 0, s, am, lm->head_blocks, (int)c.vocab_size,
                      lm->tokens, lm->state);
}

zq::lm::LinDesc lin_desc(const zq_weight* w, const float* bias) {
    return zq::lm::LinDesc{w->panel, w->scales, bias, (int)w->K, w->Kp, (int)w->N};
}

// Descriptors, barrier and grid of the persistent decode kernel.  A model
// that cannot run it (no cooperative launch, or no room for one CTA per SM)
// keeps step_grid = 0 and decodes with the kernel chain.
cudaError_t prepare_persistent(zq_lm* lm, cudaStream_t st) {
    const zq_lm_info& c = lm->info;
    std::vector<zq::lm::LayerDesc> h(lm->layers.size());
    int kmax = lm->head->Kp;
    for (size_t i = 0; i < lm->layers.size(); ++i) {
        const DevLayer& L = lm->layers[i];
        h[i].qkv = lin_desc(L.qkv, L.b_qkv);
        h[i].out = lin_desc(L.out, L.b_out);
        h[i].up = lin_desc(L.up, L.b_up);
        h[i].down = lin_desc(L.down, L.b_down);
        h[i].n1w = L.n1w;
        h[i].n1b = L.n1b;
        h[i].n2w = L.n2w;
        h[i].n2b = L.n2b;
        h[i].rms1 = L.rms1;
        h[i].rms2 = L.rms2;
        kmax = std::max({kmax, L.qkv->Kp, L.out->Kp, L.up->Kp, L.down->Kp});
    }
    cudaError_t e = dev_alloc(lm, &lm->layer_desc, h.size());
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(lm->layer_desc, h.data(), h.size() * sizeof(h[0]), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = dev_alloc(lm, &lm->bar, 1);
    if (e == cudaSuccess) e = dev_alloc(lm, &lm->keys, 2);
    if (e == cudaSuccess) e = dev_alloc(lm, &lm->nan_flags, 2);
    lm->head_blocks = head_blocks_for(lm->head);
    if (e == cudaSuccess) e = dev_alloc(lm, &lm->head_slots, (size_t)lm->head_blocks);
    if (e != cudaSuccess) return e;
    lm->xmax = (kmax + 31) / 32 * 32;
    using namespace zq::lm;
    const size_t att = (size_t)kHeadBatch * kMaxHeadDim + 2 * kMaxHeadDim + (size_t)kHeadBatch * kAttnChunk +
                       2 * kHeadBatch + (size_t)kStepWarps * kHeadBatch * kMaxHeadDim +
                       2 * c.num_heads * (size_t)lm->attn_splits + c.num_heads + (c.num_heads & 1);
    lm->step_smem = ((size_t)kStepCtlFloats + lm->xmax + lm->xmax / 4 + att) * sizeof(float) +
                    h.size() * sizeof(zq::lm::LayerDesc);
    int coop = 0, sms = 0, per_sm = 0;
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, lm->device);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, lm->device);
    const void* kern = c.type == ZQ_TYPE_INT8 ? (const void*)step_kernel<zq::kInt8> : (const void*)step_kernel<zq::kInt4>;
    lm->step_grid = 0;
    if (!coop || lm->step_smem > kMaxLinearSmem) return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lm->step_smem);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kStepThreads, lm->step_smem);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return cudaSuccess;
    }
    if (per_sm >= 1) lm->step_grid = sms;
    return cudaSuccess;
}

// All `steps` decode steps as one cooperative launch of step_kernel.
cudaError_t launch_persistent(zq_lm* lm, int steps, int prompt_len, float* step_logits_dev, uint32_t* err,
                              cudaStream_t st) {
    const zq_lm_info& c = lm->info;
    zq::lm::StepParams p{};
    p.layers = lm->layer_desc;
    p.n_layers = (int)lm->layers.size();
    p.head = lin_desc(lm->head, lm->b_head);
    p.final_w = lm->final_w;
    p.emb_panel = lm->emb->panel;
    p.emb_scales = lm->emb->scales;
    p.emb_Kp = lm->emb->Kp;
    p.pe = lm->pe;
    p.rcos = c.use_rope ? lm->rcos : nullptr;
    p.rsin = c.use_rope ? lm->rsin : nullptr;
    p.h = lm->h;
    p.qkv = lm->qkv;
    p.ff = lm->ff;
    p.part = lm->attn_part;
    p.kc = lm->kc;
    p.vc = lm->vc;
    p.tokens = lm->tokens;
    p.state = lm->state;
    p.keys = lm->keys;
    p.nan_flags = lm->nan_flags;
    p.bar = lm->bar;
    p.step_logits = step_logits_dev;
    p.err = err;
    p.H = (int)c.hidden_size;
    p.F = (int)c.intermediate_size;
    p.V = (int)c.vocab_size;
    p.heads = (int)c.num_heads;
    p.kvh = (int)(c.num_kv_heads == 0 ? c.num_heads : c.num_kv_heads);
    p.hd = (int)(c.hidden_size / c.num_heads);
    p.max_seq = (int)c.max_sequence_length;
    p.n_chunks_max = lm->attn_splits;
    p.xmax = lm->xmax;
    p.eps = c.norm_eps;
    p.scale = 1.0f / std::sqrt(static_cast<float>(p.hd));
    p.prompt_len = prompt_len;
    p.n_steps = steps;
    cudaError_t e = cudaMemsetAsync(lm->bar, 0, sizeof(unsigned int), st);
    if (e == cudaSuccess) e = cudaMemsetAsync(lm->keys, 0, 2 * sizeof(unsigned long long), st);
    if (e == cudaSuccess) e = cudaMemsetAsync(lm->nan_flags, 0, 2 * sizeof(int), st);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)lm->step_grid);
    cfg.blockDim = dim3(zq::lm::kStepThreads);
    cfg.dynamicSmemBytes = lm->step_smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return c.type == ZQ_TYPE_INT8 ? cudaLaunchKernelEx(&cfg, zq::lm::step_kernel<zq::kInt8>, p)
                                  : cudaLaunchKernelEx(&cfg, zq::lm::step_kernel<zq::kInt4>, p);
}

cudaError_t build_graph(zq_lm* lm, int steps, cudaGraphExec_t* out, cudaStream_t s, bool penalized = false) {
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return e;
    for (int i = 0; i < steps && e == cudaSuccess; ++i) e = enqueue_step(lm, s, penalized);
    cudaError_t e2 = cudaStreamEndCapture(s, &g);
    if (e == cudaSuccess) e = e2;
    if (e == cudaSuccess) e = cudaGraphInstantiate(out, g, 0);
    if (g) cudaGraphDestroy(g);
    return e;
}

zq_status fail_lm(zq_status s, const std::string& msg) { return zq::set_error(s, msg.c_str()); }

}  // namespace

extern "C" {

zq_status zq_lm_load(const void* bytes, size_t len, void* stream, zq_lm** out) {
    if (!out) return fail_lm(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null output handle");
    *out = nullptr;
    Reader r(static_cast<const uint8_t*>(bytes), len);
    zq_lm_info c{};
    int type = 0;
    std::vector<HostBlock> blocks;
    zq::ZyqRecord emb;
    HostTensor pe, final_w;
    HostLinear head;
    try {
        // QuantizedLanguageModel::load (quantized_language_model.cpp:627-642)
        if (rd_u32(r) != kModelMagic || rd_u32(r) != kModelVersion)
            throw ParseError{ZQ_ERR_RUNTIME, "ZYRON quantized model: unsupported format"};
        type = (int)rd_u32(r);
        if (type != 1 && type != 2) throw ParseError{ZQ_ERR_RUNTIME, "ZYRON quantized model: invalid type"};
        // q_read_config (581-587)
        c.vocab_size = rd_u64(r);
        c.hidden_size = rd_u64(r);
        c.num_layers = rd_u64(r);
        c.num_heads = rd_u64(r);
        c.num_kv_heads = rd_u64(r);
        c.intermediate_size = rd_u64(r);
        c.max_sequence_length = rd_u64(r);
        c.norm_eps = rd_f32(r);
        c.use_rms_norm = rd_u32(r) != 0;
        c.causal = rd_u32(r) != 0;
        c.use_rope = rd_u32(r) != 0;
        c.tie_word_embeddings = rd_u32(r) != 0;
        c.rope_theta = rd_f32(r);
        const float dropout = rd_f32(r);
        (void)rd_u32(r);  // use_qat
        const uint64_t qat_bits = rd_u64(r);
        validate_config(c, (size_t)qat_bits, dropout);
        zq_status s = zq::parse_zyq(r.here(), r.left(), &emb);
        if (s != ZQ_OK) throw ParseError{s, zq_last_error()};
        r.skip(emb.consumed);
        pe = rd_tensor(r);
        final_w = rd_tensor(r);
        const uint64_t nblocks = rd_u64(r);
        if (nblocks != c.num_layers) throw ParseError{ZQ_ERR_RUNTIME, "ZYRON quantized model: layer count mismatch"};
        for (uint64_t i = 0; i < nblocks; ++i) {
            HostBlock b;
            b.rms1 = rd_u32(r) != 0;
            b.n1w = rd_tensor(r);
            b.n1b = rd_tensor(r);
            b.rms2 = rd_u32(r) != 0;
            b.n2w = rd_tensor(r);
            b.n2b = rd_tensor(r);
            b.q = rd_linear(r);
            b.k = rd_linear(r);
            b.v = rd_linear(r);
            b.o = rd_linear(r);
            b.up = rd_linear(r);
            b.down = rd_linear(r);
            blocks.push_back(std::move(b));
        }
        head = rd_linear(r);
    } catch (const ParseError& pe_) {
        return fail_lm(pe_.s, pe_.msg);
    }
    c.type = type;

    // Shape consistency the device kernels rely on (the reference would fail
    // later, inside forward()).
    const size_t H = c.hidden_size, V = c.vocab_size, F = c.intermediate_size;
    const size_t kvh = c.num_kv_heads == 0 ? c.num_heads : c.num_kv_heads;
    const size_t hd = H / c.num_heads;
    auto bad = [](const char* what) { return fail_lm(ZQ_ERR_INVALID_ARGUMENT, std::string("zyron_b200: ") + what); };
    if (hd > (size_t)zq::lm::kMaxHeadDim) return bad("head dimension above 128 is not supported on the device");
    if (linear_smem(zq::padded_k(type, (int)std::max(H, F))) > kMaxLinearSmem)
        return bad("hidden or intermediate size too large for the device decode kernels");
    if (emb.rows != V || emb.cols != H) return bad("token embedding shape does not match the config");
    if (head.w.rows != H || head.w.cols != V) return bad("lm_head shape does not match the config");
    if (final_w.size() != H) return bad("final norm weight size does not match the config");
    if (!c.use_rope && pe.size() != c.max_sequence_length * H) return bad("positional encoding shape mismatch");
    for (const auto& b : blocks) {
        if (b.q.w.rows != H || b.q.w.cols != H || b.k.w.rows != H || b.k.w.cols != kvh * hd || b.v.w.rows != H ||
            b.v.w.cols != kvh * hd || b.o.w.rows != H || b.o.w.cols != H || b.up.w.rows != H || b.up.w.cols != F ||
            b.down.w.rows != F || b.down.w.cols != H)
            return bad("block projection shapes do not match the config");
        if (b.n1w.size() != H || b.n2w.size() != H || (!b.rms1 && b.n1b.size() != H) || (!b.rms2 && b.n2b.size() != H))
            return bad("block norm shapes do not match the config");
        if (b.q.w.type != type || b.k.w.type != type || b.v.w.type != type)
            return bad("q/k/v projections must share one quantization type");
    }

    // quantized_bytes / float_reference_bytes as load() computes them (636-641, 644-664)
    size_t qb = zyq_bytes(emb) + tensor_bytes(pe) + tensor_bytes(final_w) + zyq_bytes(head.w) + tensor_bytes(head.bias);
    size_t fb = emb.rows * emb.cols * 4 + tensor_bytes(pe) + tensor_bytes(final_w) + head.w.rows * head.w.cols * 4 +
                tensor_bytes(head.bias);
    for (const auto& b : blocks) {
        qb += tensor_bytes(b.n1w) + tensor_bytes(b.n1b) + tensor_bytes(b.n2w) + tensor_bytes(b.n2b);
        fb += tensor_bytes(b.n1w) + tensor_bytes(b.n1b) + tensor_bytes(b.n2w) + tensor_bytes(b.n2b);
        for (const HostLinear* l : {&b.q, &b.k, &b.v, &b.o, &b.up, &b.down}) {
            qb += zyq_bytes(l->w);
            fb += l->w.rows * l->w.cols * 4 + tensor_bytes(l->bias);
        }
    }
    c.quantized_bytes = qb;
    c.float_reference_bytes = fb;

    // ---- upload ---------------------------------------------------------
    auto* lm = new (std::nothrow) zq_lm;
    if (!lm) return fail_lm(ZQ_ERR_RUNTIME, "zyron_b200: out of host memory");
    lm->info = c;
    cudaGetDevice(&lm->device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : cudaStreamPerThread;
    auto cleanup = [&](zq_status s) {
        delete lm;
        return s;
    };
    cudaError_t e0 = prepare_kernels();
    if (e0 != cudaSuccess) return cleanup(zq::cuda_error(e0, "kernel attributes"));
    zq_status s = make_weight(emb, stream, &lm->emb);
    if (s != ZQ_OK) return cleanup(s);
    s = make_weight(head.w, stream, &lm->head);
    if (s != ZQ_OK) return cleanup(s);
    cudaError_t e = upload_tensor(lm, head.bias, &lm->b_head, st);
    if (e == cudaSuccess) e = upload_tensor(lm, final_w, &lm->final_w, st);
    if (e == cudaSuccess && !c.use_rope) e = upload_tensor(lm, pe, &lm->pe, st);
    for (const auto& b : blocks) {
        if (e != cudaSuccess) break;
        DevLayer d;
        d.rms1 = b.rms1;
        d.rms2 = b.rms2;
        zq_weight *wq = nullptr, *wk = nullptr, *wv = nullptr;
        s = make_weight(b.q.w, stream, &wq);
        if (s == ZQ_OK) s = make_weight(b.k.w, stream, &wk);
        if (s == ZQ_OK) s = make_weight(b.v.w, stream, &wv);
        if (s == ZQ_OK) {
            zq_weight* parts[3] = {wq, wk, wv};
            s = zq::concat_cols(parts, 3, stream, &d.qkv);
        }
        zq_weight_destroy(wq);
        zq_weight_destroy(wk);
        zq_weight_destroy(wv);
        if (s == ZQ_OK) s = make_weight(b.o.w, stream, &d.out);
        if (s == ZQ_OK) s = make_weight(b.up.w, stream, &d.up);
        if (s == ZQ_OK) s = make_weight(b.down.w, stream, &d.down);
        lm->layers.push_back(d);  // owned weights are released by ~zq_lm
        if (s != ZQ_OK) return cleanup(s);
        DevLayer& L = lm->layers.back();
        e = upload_tensor(lm, b.n1w, &L.n1w, st);
        if (e == cudaSuccess) e = upload_tensor(lm, b.n1b, &L.n1b, st);
        if (e == cudaSuccess) e = upload_tensor(lm, b.n2w, &L.n2w, st);
        if (e == cudaSuccess) e = upload_tensor(lm, b.n2b, &L.n2b, st);
        // concatenated q|k|v bias; a missing bias adds zeros
        if (e == cudaSuccess && (b.q.bias.size() || b.k.bias.size() || b.v.bias.size())) {
            HostTensor cat;
            const size_t nq = b.q.w.cols, nk = b.k.w.cols, nv = b.v.w.cols;
            cat.dims = {nq + nk + nv};
            cat.data.assign(nq + nk + nv, 0.0f);
            if (b.q.bias.size()) std::memcpy(cat.data.data(), b.q.bias.data.data(), nq * 4);
            if (b.k.bias.size()) std::memcpy(cat.data.data() + nq, b.k.bias.data.data(), nk * 4);
            if (b.v.bias.size()) std::memcpy(cat.data.data() + nq + nk, b.v.bias.data.data(), nv * 4);
            e = upload_tensor(lm, cat, &L.b_qkv, st);
        }
        if (e == cudaSuccess) e = upload_tensor(lm, b.o.bias, &L.b_out, st);
        if (e == cudaSuccess) e = upload_tensor(lm, b.up.bias, &L.b_up, st);
        if (e == cudaSuccess) e = upload_tensor(lm, b.down.bias, &L.b_down, st);
    }
    // runtime buffers
    const size_t T = c.max_sequence_length;
    if (e == cudaSuccess) e = dev_alloc(lm, &lm->h, H);
    if (e == cudaSuccess) e = dev_alloc(lm, &lm->qkv, H + 2 * kvh * hd);
    if (e == cudaSuccess) e = dev_alloc(lm, &lm->ff, F);
    if (e == cudaSuccess) e = dev_alloc(lm, &lm->logits, V);
    if (e == cudaSuccess) e = dev_alloc(lm, &lm->kc, c.num_layers * kvh * T * hd);
    if (e == cudaSuccess) e = dev_alloc(lm, &lm->vc, c.num_layers * kvh * T * hd);
    lm->attn_splits = (int)((T + zq::lm::kAttnChunk - 1) / zq::lm::kAttnChunk);
    if (e == cudaSuccess)
        e = dev_alloc(lm, &lm->attn_part, c.num_heads * (size_t)lm->attn_splits * (zq::lm::kMaxHeadDim + 2));
    if (e == cudaSuccess) e = dev_alloc(lm, &lm->tokens, T + 2);
    if (e == cudaSuccess) e = dev_alloc(lm, &lm->state, 1);
    if (e == cudaSuccess) e = dev_alloc(lm, &lm->penalty, 1);
    lm->penalty_smem = 2 * ((V + 31) / 32) * sizeof(uint32_t);
    if (e == cudaSuccess && lm->penalty_smem > 48 * 1024) {
        if (lm->penalty_smem <= kMaxLinearSmem)
            e = cudaFuncSetAttribute(zq::lm::next_token_penalized_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)lm->penalty_smem);
        else
            lm->penalty_smem = 0;  // vocabulary too large for the device bitmaps: penalties are applied on the host
    }
    if (e == cudaSuccess && c.use_rope) {
        // apply_rope factors (quantized_language_model.cpp:367-374), computed
        // with the same float formula: angle = pos / pow(theta, 2p / hd).
        const size_t half = hd / 2;
        std::vector<float> cs(T * half), sn(T * half);
        for (size_t p = 0; p < T; ++p) {
            const float absolute = static_cast<float>(p);
            for (size_t pair = 0; pair < half; ++pair) {
                const float exponent = (2.0f * static_cast<float>(pair)) / static_cast<float>(hd);
                const float angle = absolute / std::pow(c.rope_theta, exponent);
                cs[p * half + pair] = std::cos(angle);
                sn[p * half + pair] = std::sin(angle);
            }
        }
        e = dev_alloc(lm, &lm->rcos, T * half);
        if (e == cudaSuccess) e = dev_alloc(lm, &lm->rsin, T * half);
        if (e == cudaSuccess) e = cudaMemcpyAsync(lm->rcos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(lm->rsin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    }
    if (e == cudaSuccess) e = prepare_persistent(lm, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&lm->own_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return cleanup(zq::cuda_error(e, "language model upload"));
    *out = lm;
    return ZQ_OK;
}

zq_status zq_lm_set_option(zq_lm* lm, int option, int value, int* previous) {
    if (!lm) return fail_lm(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null model");
    if (option != ZQ_LM_OPT_PERSISTENT) return fail_lm(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: unknown model option");
    if (value != 0 && value != 1) return fail_lm(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: option value must be 0 or 1");
    if (previous) *previous = lm->persistent;
    lm->persistent = value;
    return ZQ_OK;
}

zq_status zq_lm_get_info(const zq_lm* lm, zq_lm_info* info) {
    if (!lm || !info) return fail_lm(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null argument");
    *info = lm->info;
    return ZQ_OK;
}

zq_status zq_lm_generate(zq_lm* lm, const int64_t* prompt, size_t prompt_len, const zq_generation_config* config,
                         int64_t* out_tokens, size_t out_cap, size_t* out_len, float* step_logits, void* stream) {
    if (!lm) return fail_lm(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null model");
    const zq_lm_info& c = lm->info;
    // generate_batch checks, in its order (quantized_language_model.cpp:503-517)
    zq_status vs = zq::check_generation_config(config);
    if (vs != ZQ_OK) return vs;
    const zq_generation_config& cfg = *config;
    if (prompt_len == 0 || !prompt) return fail_lm(ZQ_ERR_INVALID_ARGUMENT, "ZYRON QuantizedLanguageModel: empty prompt");
    if (prompt_len > c.max_sequence_length)
        return fail_lm(ZQ_ERR_INVALID_ARGUMENT, "ZYRON QuantizedLanguageModel: prompt exceeds context");
    if (cfg.top_k > c.vocab_size)
        return fail_lm(ZQ_ERR_INVALID_ARGUMENT, "ZYRON QuantizedLanguageModel: top_k exceeds vocabulary");
    // tokens stop growing once they reach max_sequence_length (539-545)
    size_t n_new = 0;
    if (cfg.max_new_tokens > 0) {
        const size_t room = c.max_sequence_length > prompt_len ? c.max_sequence_length - prompt_len : 1;
        n_new = cfg.max_new_tokens < room ? cfg.max_new_tokens : room;
    }
    const size_t total = prompt_len + n_new;
    if (out_len) *out_len = total;
    if (!out_tokens || out_cap < total)
        return fail_lm(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: output token buffer too small");
    if (n_new == 0) {  // the reference's loop never runs, so nothing reads the ids
        for (size_t i = 0; i < prompt_len; ++i) out_tokens[i] = prompt[i];
        return ZQ_OK;
    }
    // token_lookup (271-282), which the first forward runs
    for (size_t i = 0; i < prompt_len; ++i)
        if (prompt[i] < 0 || (uint64_t)prompt[i] >= c.vocab_size)
            return fail_lm(ZQ_ERR_OUT_OF_RANGE, "ZYRON QuantizedLanguageModel: token id out of range");
    for (size_t i = 0; i < prompt_len; ++i) out_tokens[i] = prompt[i];

    int cur = 0;
    LM_CUDA(cudaGetDevice(&cur));
    if (cur != lm->device) return fail_lm(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: model lives on another device");
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : lm->own_stream;
    std::vector<int32_t> tok(c.max_sequence_length + 2, 0);
    for (size_t i = 0; i < prompt_len; ++i) tok[i] = (int32_t)prompt[i];
    State s0{0, (int)prompt_len, {0, 0}};
    LM_CUDA(cudaMemcpyAsync(lm->tokens, tok.data(), tok.size() * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    LM_CUDA(cudaMemcpyAsync(lm->state, &s0, sizeof s0, cudaMemcpyHostToDevice, st));
    // the lm_head's argmax key starts cleared
    LM_CUDA(cudaMemsetAsync(lm->keys, 0, 2 * sizeof(unsigned long long), st));
    LM_CUDA(cudaMemsetAsync(lm->nan_flags, 0, 2 * sizeof(int), st));

    const size_t steps = prompt_len - 1 + n_new;  // last step produces the last new token
    const bool penalties = cfg.repetition_penalty != 1.0f || cfg.no_repeat_ngram_size > 0;
    const bool greedy = cfg.top_k == 1 && (!penalties || lm->penalty_smem > 0);

    if (!greedy) {
        // Sampling: every step's logits go to the host, where the reference's
        // sample_next (82-174) picks the token from std::mt19937(seed)
        // (520), which is then written into the device token history.  The
        // prompt's positions need no choice and run as graph replays.
        std::mt19937 rng(cfg.seed);
        std::vector<float> row(c.vocab_size);
        if (!lm->graph_one) LM_CUDA(build_graph(lm, 1, &lm->graph_one, st));
        for (size_t i = 0; i + 1 < prompt_len; ++i) LM_CUDA(cudaGraphLaunch(lm->graph_one, st));
        for (size_t g = 0; g < n_new; ++g) {
            LM_CUDA(cudaGraphLaunch(lm->graph_one, st));
            LM_CUDA(cudaMemcpyAsync(row.data(), lm->logits, c.vocab_size * sizeof(float), cudaMemcpyDeviceToHost, st));
            LM_CUDA(cudaStreamSynchronize(st));
            if (step_logits) std::memcpy(step_logits + g * c.vocab_size, row.data(), c.vocab_size * sizeof(float));
            const size_t t = zq::sample_row(rng, row.data(), c.vocab_size, out_tokens, prompt_len + g, cfg);
            out_tokens[prompt_len + g] = (int64_t)t;
            tok[prompt_len + g] = (int32_t)t;
            // the step's own greedy choice sits in the same slot; overwrite it
            if (g + 1 < n_new)
                LM_CUDA(cudaMemcpyAsync(lm->tokens + prompt_len + g, &tok[prompt_len + g], sizeof(int32_t),
                                        cudaMemcpyHostToDevice, st));
        }
        LM_CUDA(cudaStreamSynchronize(st));
        return ZQ_OK;
    }

    if (penalties) {
        const zq::lm::PenaltyCfg pc{cfg.repetition_penalty, (int)std::min<size_t>(cfg.no_repeat_ngram_size, 1u << 30)};
        LM_CUDA(cudaMemcpyAsync(lm->penalty, &pc, sizeof pc, cudaMemcpyHostToDevice, st));
    }
    // ZQ_LM_OPT_PERSISTENT: every step in one cooperative launch of
    // step_kernel (when the device allows it); otherwise the kernel chain
    // replayed from CUDA graphs.
    if (!penalties && lm->step_grid > 0 && lm->persistent) {
        // persistent decode: every step in one cooperative launch
        uint32_t* err = nullptr;
        zq_status es = zq::device_error_word(&err);
        if (es != ZQ_OK) return es;
        float* dlog = nullptr;
        if (step_logits) LM_CUDA(cudaMallocAsync(&dlog, n_new * c.vocab_size * sizeof(float), st));
        cudaError_t le = launch_persistent(lm, (int)steps, (int)prompt_len, dlog, err, st);
        if (le == cudaSuccess && dlog)
            le = cudaMemcpyAsync(step_logits, dlog, n_new * c.vocab_size * sizeof(float), cudaMemcpyDeviceToHost, st);
        if (dlog) cudaFreeAsync(dlog, st);
        LM_CUDA(le);
    } else if (step_logits) {
        // parity mode: per step, copy the logits that chose each new token
        for (size_t i = 0; i < steps; ++i) {
            LM_CUDA(enqueue_step(lm, st, penalties));
            if (i + 1 >= prompt_len) {
                const size_t g = i + 1 - prompt_len;
                LM_CUDA(cudaMemcpyAsync(step_logits + g * c.vocab_size, lm->logits, c.vocab_size * sizeof(float),
                                        cudaMemcpyDeviceToHost, st));
            }
        }
    } else {
        cudaGraphExec_t& one = penalties ? lm->graph_one_pen : lm->graph_one;
        cudaGraphExec_t& chunk = penalties ? lm->graph_chunk_pen : lm->graph_chunk;
        if (!one) LM_CUDA(build_graph(lm, 1, &one, st, penalties));
        if (!chunk && steps >= (size_t)lm->chunk) LM_CUDA(build_graph(lm, lm->chunk, &chunk, st, penalties));
        size_t done = 0;
        while (steps - done >= (size_t)lm->chunk && chunk) {
            LM_CUDA(cudaGraphLaunch(chunk, st));
            done += lm->chunk;
        }
        while (done < steps) {
            LM_CUDA(cudaGraphLaunch(one, st));
            ++done;
        }
    }
    LM_CUDA(cudaMemcpyAsync(tok.data(), lm->tokens, total * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    LM_CUDA(cudaStreamSynchronize(st));
    for (size_t i = prompt_len; i < total; ++i) out_tokens[i] = tok[i];
    return ZQ_OK;
}

zq_status zq_lm_generate_greedy(zq_lm* lm, const int64_t* prompt, size_t prompt_len, size_t max_new_tokens,
                                int64_t* out_tokens, size_t out_cap, size_t* out_len, float* step_logits,
                                void* stream) {
    zq_generation_config cfg{};
    cfg.max_new_tokens = max_new_tokens;
    cfg.temperature = 1.0f;
    cfg.top_k = 1;
    cfg.top_p = 1.0f;
    cfg.repetition_penalty = 1.0f;
    cfg.no_repeat_ngram_size = 0;
    cfg.seed = 0;
    return zq_lm_generate(lm, prompt, prompt_len, &cfg, out_tokens, out_cap, out_len, step_logits, stream);
}

zq_status zq_lm_destroy(zq_lm* lm) {
    delete lm;
    return ZQ_OK;
}

}  // extern "C"
