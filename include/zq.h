/*
 * zq.h -- C ABI of the B200 quantized matmul library (libzyron_b200.so).
 *
 * This is the boundary under ZYRON's `zyron::quantization` API.  The C++20
 * drop-in (zyron_b200/cpp: QuantizedMatrix, quantize, matmul, QuantizedLinear)
 * and the Python bindings (zyron_b200/_lib.py) both call only these entry
 * points.  Plain pointers and sizes; no C++ or torch types.
 *
 * Conventions
 *   - Weights are the reference's logical [rows = K][cols = N] matrix.
 *     Host payloads use the reference storage: column-major (element (r, c)
 *     at linear index c*K + r), INT4 two codes per byte with the low nibble
 *     holding the even linear index (reference: src/quantization/
 *     quantization.cpp:52-67, 155).
 *   - Activations x are fp32 row-major [m][K], outputs y fp32 row-major
 *     [m][N].  Pointers named *_dev / x / y / out are device pointers on the
 *     weight's device; *_host pointers are host memory (pinned or pageable).
 *   - `stream` is a cudaStream_t; NULL selects the calling thread's
 *     per-thread default stream.  Compute calls are asynchronous on it unless
 *     stated otherwise.
 *   - Every call validates its arguments on the host before any launch and
 *     returns a zq_status.  zq_last_error() gives the calling thread's last
 *     message; messages of errors the reference also raises are identical to
 *     the reference's (e.g. "ZYRON quantization: weights are empty").
 *   - There is no CPU fallback: without a usable sm_100 device every compute
 *     call fails with ZQ_ERR_CUDA.
 */
#ifndef ZQ_H
#define ZQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum zq_status {
    ZQ_OK = 0,
    ZQ_ERR_INVALID_ARGUMENT = 1, /* reference: std::invalid_argument */
    ZQ_ERR_OUT_OF_RANGE = 2,     /* reference: std::out_of_range */
    ZQ_ERR_OVERFLOW = 3,         /* reference: std::overflow_error */
    ZQ_ERR_RUNTIME = 4,          /* reference: std::runtime_error (format, I/O) */
    ZQ_ERR_CUDA = 5,             /* a CUDA runtime call failed */
    ZQ_ERR_DEVICE_TIMEOUT = 6    /* a bounded device-side wait gave up */
} zq_status;

/* zyron::quantization::Type values (include/zyron/quantization/quantization.hpp:13-16). */
#define ZQ_TYPE_INT8 1
#define ZQ_TYPE_INT4 2

/* A quantized weight resident in device memory (replaces the storage of
 * zyron::quantization::QuantizedMatrix, quantization.hpp:18-52). */
typedef struct zq_weight zq_weight;

/* Last error message of the calling thread ("" if none). */
const char* zq_last_error(void);

/* ABI version of this header (bumped on incompatible changes). */
int zq_abi_version(void);
#define ZQ_ABI_VERSION 1

/* ---- weights ------------------------------------------------------------ */

/* Upload a quantized matrix given in the reference's host storage: `scales`
 * has `cols` floats, `payload` has rows*cols bytes (INT8) or
 * ceil(rows*cols/2) bytes (INT4).  The device copy is made on the current
 * device.  Replaces the storage fill of quantize() / QuantizedMatrix::load
 * (quantization.cpp:121-162, 269-311) with a device upload. */
zq_status zq_weight_create(int type, size_t rows, size_t cols, const float* scales_host,
                           const void* payload_host, size_t payload_bytes, void* stream,
                           zq_weight** out);

/* quantize() on the device: w_dev is fp32 row-major [rows][cols] on the
 * current device.  Bit-identical to the reference's quantize()
 * (quantization.cpp:121-162). */
zq_status zq_weight_quantize(const float* w_dev, size_t rows, size_t cols, int type, void* stream,
                             zq_weight** out);

/* quantize() from host memory: w_host is fp32 row-major [rows][cols]; it is
 * copied to the current device and quantized there.  Synchronous. */
zq_status zq_weight_quantize_host(const float* w_host, size_t rows, size_t cols, int type, void* stream,
                                  zq_weight** out);

/* Parse one .zyq record from memory and upload it (QuantizedMatrix::load(istream),
 * quantization.cpp:269-311: same checks, same order, same messages).  On
 * success *consumed is the number of bytes of the record. */
zq_status zq_weight_load_zyq(const void* bytes, size_t len, size_t* consumed, void* stream,
                             zq_weight** out);

/* Serialise to the .zyq format (QuantizedMatrix::save(ostream),
 * quantization.cpp:247-261).  Call with buf == NULL to get the size in *len.
 * Synchronous. */
zq_status zq_weight_save_zyq(const zq_weight* w, void* buf, size_t cap, size_t* len, void* stream);

/* Shape / type / payload size in the reference's storage / device ordinal. */
zq_status zq_weight_info(const zq_weight* w, int* type, size_t* rows, size_t* cols,
                         size_t* payload_bytes, int* device);

/* Copy scales and the reference-layout payload back to the host.  Synchronous. */
zq_status zq_weight_download(const zq_weight* w, float* scales_host, void* payload_host, void* stream);

/* A new weight holding columns [col_begin, col_end) of `w` (device to device,
 * current device).  Used for column-parallel sharding: a column's codes and
 * scale are independent of every other column. */
zq_status zq_weight_slice_cols(const zq_weight* w, size_t col_begin, size_t col_end, void* stream,
                               zq_weight** out);

zq_status zq_weight_destroy(zq_weight* w);

/* ---- compute ------------------------------------------------------------ */

/* zq_matmul whose output goes to n_dst (1..8) buffers at once: element
 * (r, c) of the [m][cols] result is stored at dsts[i][r*ldy + col_offset + c]
 * for every i.  The buffers may be other GPUs' memory mapped into this process
 * (CUDA IPC or peer access): each output tile is then written over NVLink as
 * soon as the tensor cores finish it, so the all-gather of column-sharded
 * outputs (rank g passes col_offset = g*cols and every rank's full [m][ldy]
 * output) runs inside the matmul instead of after it.  Stores are complete
 * when the kernel completes; synchronise with the peers (e.g. a collective
 * barrier) before reading their columns.  m must exceed 8 (the tensor-core
 * path).  Same workspace rule as zq_matmul.  No counterpart in the reference
 * (which runs on one host). */
zq_status zq_matmul_multi(const zq_weight* w, const float* x, size_t m, const float* bias, float* const* dsts,
                          int n_dst, size_t ldy, size_t col_offset, void* workspace, size_t workspace_bytes,
                          void* stream);

/* Device scratch needed by zq_matmul for `m` activation rows. */
size_t zq_matmul_workspace_bytes(const zq_weight* w, size_t m);

/* The per-row dynamic activation quantizer on its own (quantization.cpp:
 * 202-212): q is int8 [m][ldq] with ldq >= k (codes in [0, k), zeros in
 * [k, ldq)), row_scale fp32 [m], all device. */
zq_status zq_quantize_rows(const float* x, size_t m, size_t k, int8_t* q, size_t ldq, float* row_scale,
                           void* stream);

/* Row length of the activation codes zq_matmul_codes expects for `w`
 * (K rounded up to a multiple of 128 codes). */
size_t zq_weight_padded_k(const zq_weight* w);

/* quantization::matmul (quantization.cpp:177-238) followed, when bias is not
 * NULL, by QuantizedLinear::forward's bias add (quantized_linear.cpp:33-50).
 * x [m][rows], bias [cols] or NULL, y [m][cols]; all device pointers.
 * m <= 8 runs the HBM-bound GEMV, larger m the tcgen05 GEMM.  `workspace`
 * must hold zq_matmul_workspace_bytes(w, m) bytes and must not be shared by
 * calls that may overlap on the GPU.  Results are bit-identical to the
 * reference. */
zq_status zq_matmul(const zq_weight* w, const float* x, size_t m, const float* bias, float* y,
                    void* workspace, size_t workspace_bytes, void* stream);

/* zq_matmul with the activation quantizer already applied: q is int8
 * [m][zq_weight_padded_k(w)] (as written by zq_quantize_rows with that ldq),
 * row_scale fp32 [m].  Lets a producer kernel emit codes directly and lets
 * the matmul kernel be timed on its own.  Same workspace rule as zq_matmul. */
zq_status zq_matmul_codes(const zq_weight* w, const int8_t* q, const float* row_scale, size_t m,
                          const float* bias, float* y, void* workspace, size_t workspace_bytes, void* stream);

/* zq_matmul for callers that cannot allocate device memory or pass a
 * workspace (plugin hosts that hand over only input and output buffers,
 * pool allocators that forbid raw cudaMalloc, loops that must not
 * synchronise on an allocation).  No counterpart in the reference: its
 * matmul runs on the host.  Scratch comes from a fixed array compiled into
 * the library (ZQ_NOALLOC_SCRATCH_BYTES per device, held until exit); calls
 * needing more (zq_matmul_workspace_bytes(w, m) larger than that) fail with
 * ZQ_ERR_INVALID_ARGUMENT.  Allocates nothing.  The first call on each device
 * resolves the array's device address and should precede any stream capture;
 * the address is kept for the life of the process, so a cudaDeviceReset()
 * invalidates it and the entry point must not be used on that device after
 * one.
 * All calls on a device share the array: calls that may overlap on the GPU
 * race and must be serialised.  Same results as zq_matmul. */
#define ZQ_NOALLOC_SCRATCH_BYTES (8u << 20)
zq_status zq_matmul_noalloc(const zq_weight* w, const float* x, size_t m, const float* bias, float* y,
                            void* stream);

/* The same computation from host buffers to host buffers: copies x (and
 * bias) to the device, runs zq_matmul, copies y back and synchronises the
 * stream.  Device buffers are cached per thread and grow as needed. */
zq_status zq_matmul_host(const zq_weight* w, const float* x_host, size_t m, const float* bias_host,
                         float* y_host, void* stream);

/* QuantizedMatrix::dequantize() (quantization.cpp:164-175): out is fp32
 * row-major [rows][cols] on the device. */
zq_status zq_dequantize(const zq_weight* w, float* out, void* stream);

/* dequantize() into host memory: out_host is fp32 row-major [rows][cols].
 * Synchronous. */
zq_status zq_dequantize_host(const zq_weight* w, float* out_host, void* stream);

/* ---- column-sharded matmul over NCCL ------------------------------------ */

/* Columns [*begin, *end) of rank `rank` when n_cols columns are split over
 * `world` ranks: contiguous, the first n_cols % world ranks one column wider.
 * zq_matmul_sharded expects each rank's shard to be exactly this range (e.g.
 * zq_weight_slice_cols(w, begin, end, ...)). */
zq_status zq_shard_range(size_t n_cols, int world, int rank, size_t* begin, size_t* end);

/* NCCL communicator helpers for hosts without their own NCCL binding.  NCCL
 * is loaded at run time (libnccl.so.2; a process that already loaded it, e.g.
 * through PyTorch, shares that copy).  The unique id is ZQ_NCCL_UNIQUE_ID_BYTES
 * opaque bytes that rank 0 creates and every rank passes to
 * zq_nccl_comm_init, with its own device current.  *comm is an ncclComm_t. */
#define ZQ_NCCL_UNIQUE_ID_BYTES 128
zq_status zq_nccl_get_unique_id(void* id_out);
zq_status zq_nccl_comm_init(int nranks, const void* id, int rank, void** comm);
zq_status zq_nccl_comm_destroy(void* comm);

/* Workspace zq_matmul_sharded needs for m rows of an n_cols-column weight
 * split over `world` ranks (0 for invalid arguments). */
size_t zq_matmul_sharded_workspace_bytes(const zq_weight* shard, size_t m, size_t n_cols, int world);

/* The sharded path of quantization::matmul (the reference runs it on one
 * host; the column split follows from quantization.cpp:141-159, one scale
 * per column).  y [m][n_cols] (full output, on every rank) = matmul(x, W)
 * with W's columns sharded over the ranks of `nccl_comm` (an ncclComm_t on
 * the current device): this rank holds `shard`, its zq_shard_range columns,
 * and bias_shard (or NULL) for them.  Every rank computes its block with
 * zq_matmul (same activation codes everywhere, no exchange), then one
 * ncclAllGather on `stream` joins the blocks.  Bit-identical to zq_matmul on
 * the whole weight.  Every rank must make the same call (same m and n_cols)
 * in the same order; a rank that fails validation issues no collective, so
 * the others' gather waits until the communicator is aborted or times out. */
zq_status zq_matmul_sharded(const zq_weight* shard, const float* x, size_t m, const float* bias_shard, float* y,
                            size_t n_cols, void* nccl_comm, void* workspace, size_t workspace_bytes, void* stream);

/* ---- peer buffers (for zq_matmul_multi across processes) ---------------- */

/* A device allocation exported from one process for another (CUDA IPC). */
typedef struct zq_ipc_handle {
    unsigned char handle[64];
    uint64_t offset; /* of the exported pointer inside its allocation */
    int device;
    int pad;
} zq_ipc_handle;

/* Export the allocation that contains `dev_ptr` (memory from cudaMalloc or a
 * pool built on it) for use by other processes. */
zq_status zq_ipc_export(const void* dev_ptr, zq_ipc_handle* out);

/* Map an exported allocation into this process so that kernels on the
 * CURRENT device can read and write it (peer access over NVLink is enabled
 * for the current device).  *dev_ptr is the exported pointer's address here. */
zq_status zq_ipc_import(const zq_ipc_handle* h, void** dev_ptr);

/* Unmap what zq_ipc_import mapped (pass the pointer it returned). */
zq_status zq_ipc_close(void* dev_ptr);

/* Options of one weight's matmuls (every call with that weight, on any
 * thread; results never depend on them).  *previous (may be NULL) receives
 * the old value.
 *   ZQ_OPT_DECODE_KERNEL: the kernel for plain matmuls with few activation
 *     rows --
 *       ZQ_DECODE_TENSOR_CORE: the tcgen05 decode kernel for m <= 16 (weights
 *         streamed by TMA, work split evenly over the SMs);
 *       ZQ_DECODE_CUDA_CORE: the dp4a warp-per-column GEMV for m <= 8;
 *       ZQ_DECODE_AUTO (default): the GEMV for m <= 4, the tcgen05 kernel for
 *         5 <= m <= 16.
 *     Larger m always runs the tcgen05 GEMM.
 *   ZQ_OPT_RESERVED_SMS: streaming multiprocessors kept out of the matmul
 *     kernels' grids (default 0), so work running concurrently on other
 *     streams -- e.g. a collective of the previous output block -- finds free
 *     SMs.
 *   ZQ_OPT_GEMM_GROUP_M: M-tiles per group of the GEMM's tile order (default
 *     32; 0 = all), which bounds the L2 working set of large GEMMs.
 * No counterpart in the reference (its matmul has no kernel choices). */
#define ZQ_OPT_DECODE_KERNEL 1
#define ZQ_OPT_RESERVED_SMS 2
#define ZQ_OPT_GEMM_GROUP_M 3
#define ZQ_DECODE_AUTO 0
#define ZQ_DECODE_TENSOR_CORE 1
#define ZQ_DECODE_CUDA_CORE 2
zq_status zq_weight_set_option(zq_weight* w, int option, int value, int* previous);

/* Synchronise `stream`, then read and clear the current device's error word
 * (0 = none; otherwise which bounded wait gave up).  Returns
 * ZQ_ERR_DEVICE_TIMEOUT when the word was set. */
zq_status zq_device_error(void* stream, uint32_t* code);

/* Failure-path test of the bounded device waits (no counterpart in the
 * reference; not for production use).  Runs zq_matmul_codes on the tcgen05
 * decode kernel (1 <= m <= 16) with the finisher of every column block that
 * several CTAs share waiting for one more partial sum than exists, so that
 * wait gives up after limit_ns (1e5 to 1e9 ns): the kernel records the
 * timeout in the error word, skips those blocks' outputs, releases its
 * resources and returns.  The call succeeds; zq_device_error() then returns
 * ZQ_ERR_DEVICE_TIMEOUT with code 5 and clears the word, and later calls run
 * normally.  Nothing faults and nothing waits without a limit. */
zq_status zq_test_decode_wait_timeout(const zq_weight* w, const int8_t* q, const float* row_scale, size_t m,
                                      float* y, void* workspace, size_t workspace_bytes, uint64_t limit_ns,
                                      void* stream);

/* ---- quantized language model (device-resident decode) ----------------- */

/* A QuantizedLanguageModel with weights, KV cache and activations resident on
 * one device (replaces the host model of
 * include/zyron/model/quantized_language_model.hpp:17-89). */
typedef struct zq_lm zq_lm;

/* transformer::Config of the loaded model (include/zyron/transformer/
 * config.hpp:10-25) plus the type and the byte counts of
 * QuantizedLanguageModel::quantized_bytes / float_reference_bytes. */
typedef struct zq_lm_info {
    size_t vocab_size, hidden_size, num_layers, num_heads, num_kv_heads, intermediate_size, max_sequence_length;
    float norm_eps;
    int use_rms_norm, causal, use_rope, tie_word_embeddings;
    float rope_theta;
    int type;
    size_t quantized_bytes, float_reference_bytes;
} zq_lm_info;

/* Parse a .zyqmodel image (QuantizedLanguageModel::save/load format,
 * src/model/quantized_language_model.cpp:615-642: same checks and messages)
 * and upload it to the current device. */
zq_status zq_lm_load(const void* bytes, size_t len, void* stream, zq_lm** out);

zq_status zq_lm_get_info(const zq_lm* lm, zq_lm_info* info);

/* Options of one model's decode loop.  *previous (may be NULL) receives the
 * old value.
 *   ZQ_LM_OPT_PERSISTENT: 1 runs every greedy step without penalties in one
 *     cooperative launch of a persistent kernel (when the device allows it),
 *     0 (default) replays the chain of per-phase kernels from CUDA graphs.
 *     Both give the same tokens. */
#define ZQ_LM_OPT_PERSISTENT 1
zq_status zq_lm_set_option(zq_lm* lm, int option, int value, int* previous);

/* QuantizedLanguageModel::generate with GenerationConfig{top_k = 1} (greedy;
 * quantized_language_model.cpp:496-547).  Writes prompt + new tokens to
 * out_tokens (capacity out_cap) and their count to *out_len; generation stops
 * after max_new_tokens or when the sequence reaches max_sequence_length, as in
 * the reference.  Ties between equal logits go to the lowest id.  When
 * step_logits is not NULL it receives, for every new token, the vocab_size
 * logits it was chosen from (parity testing; runs without CUDA graphs).
 * Synchronous.  Runs on `stream` (which must not be a default stream, since
 * the decode steps are captured as a CUDA graph), or on the model's own
 * stream when `stream` is NULL. */
zq_status zq_lm_generate_greedy(zq_lm* lm, const int64_t* prompt, size_t prompt_len, size_t max_new_tokens,
                                int64_t* out_tokens, size_t out_cap, size_t* out_len, float* step_logits,
                                void* stream);

/* GenerationConfig (include/zyron/model/generation.hpp:13-21).  The
 * reference's quantized sampler validates `temperature` but does not use it
 * (quantized_language_model.cpp:71-80, 82-174); neither does this library. */
typedef struct zq_generation_config {
    size_t max_new_tokens;
    float temperature;
    size_t top_k;          /* 0: no top-k cut; 1: greedy */
    float top_p;           /* in (0, 1] */
    float repetition_penalty;   /* >= 1; 1 = off */
    size_t no_repeat_ngram_size; /* 0 = off */
    uint32_t seed;         /* std::mt19937 seed of the draws */
} zq_generation_config;

/* QuantizedLanguageModel::generate (quantized_language_model.cpp:496-547) for
 * any GenerationConfig: same validation order and messages, and, given the
 * same logits, the same tokens as the reference's sample_next (82-174).
 *   - top_k == 1 without penalties: greedy on the device (as
 *     zq_lm_generate_greedy);
 *   - top_k == 1 with repetition_penalty != 1 or no_repeat_ngram_size > 0:
 *     the penalty and the n-gram block are applied on the device, over the
 *     device token history, before the greedy choice (lowest id on ties);
 *   - any other top_k: each step's logits are copied to the host and sampled
 *     there with the reference's softmax, std::sort, top-k/top-p cuts and one
 *     std::mt19937(seed) draw per token (zq_sample_next).
 * Output, step_logits and stream are as for zq_lm_generate_greedy. */
zq_status zq_lm_generate(zq_lm* lm, const int64_t* prompt, size_t prompt_len, const zq_generation_config* config,
                         int64_t* out_tokens, size_t out_cap, size_t* out_len, float* step_logits, void* stream);

zq_status zq_lm_destroy(zq_lm* lm);

/* ---- checkpoint conversion --------------------------------------------- */

/* zyron_quantize (tools/zyron_quantize.cpp:33-48): a .zyron training
 * checkpoint (src/model/checkpoint.cpp:145-232; versions 1-4) in memory to a
 * .zyqmodel image (QuantizedLanguageModel(model, type) then save,
 * quantized_language_model.cpp:178-269, 615-625), byte-identical to the
 * reference tool's output.  The checkpoint is validated with the reference's
 * checks, order and messages (format, config, optimizer and scheduler
 * hyper-parameters, parameter and moment shapes, tokenizer data); every
 * weight matrix is quantized on the current device.  *out receives a buffer
 * of *out_len bytes to release with zq_free_buffer; *compression_ratio (may
 * be NULL) QuantizedLanguageModel::compression_ratio() of the result.
 * Synchronous. */
zq_status zq_quantize_checkpoint(const void* checkpoint, size_t len, int type, void* stream, void** out,
                                 size_t* out_len, double* compression_ratio);

/* transformer::Config (include/zyron/transformer/config.hpp:10-26). */
typedef struct zq_lm_config {
    size_t vocab_size, hidden_size, num_layers, num_heads, num_kv_heads, intermediate_size, max_sequence_length;
    float norm_eps;
    int use_rms_norm, causal, use_rope, tie_word_embeddings;
    float rope_theta, dropout;
    int use_qat;
    size_t qat_bits;
} zq_lm_config;

/* QuantizedLanguageModel(LanguageModel(config, seed), type).save(): the
 * .zyqmodel image of a freshly initialised model (language_model.cpp:52-75;
 * quantized_language_model.cpp:178-269, 615-625).  The parameters are drawn
 * as the reference's constructors draw them -- std::mt19937 and
 * std::uniform_real_distribution<float> per tensor, with the same seeds,
 * ranges and order -- so on the same standard library the image is
 * byte-identical to the reference's.  The config is validated as
 * Config::validate does; weights are quantized on the current device.
 * Output as for zq_quantize_checkpoint.  Synchronous. */
zq_status zq_lm_init_image(const zq_lm_config* config, uint32_t seed, int type, void* stream, void** out,
                           size_t* out_len, double* compression_ratio);
void zq_free_buffer(void* p);

/* ---- token sampling (host) --------------------------------------------- */

/* The state of sample_next's random draws: std::mt19937(seed), as created
 * once per generate call (quantized_language_model.cpp:520). */
typedef struct zq_sampler zq_sampler;
zq_status zq_sampler_create(uint32_t seed, zq_sampler** out);
zq_status zq_sampler_destroy(zq_sampler* s);

/* sample_next (quantized_language_model.cpp:82-174) over one row of `vocab`
 * host logits: repetition penalty over `history` (the prompt and the tokens
 * generated so far), n-gram block, softmax, sort by probability, top-k, top-p
 * and one draw from `s`.  Host only; no device work.  Validates `config` as
 * validate_generation_config does (71-80), and top_k <= vocab. */
zq_status zq_sample_next(zq_sampler* s, const float* logits, size_t vocab, const int64_t* history,
                         size_t history_len, const zq_generation_config* config, int64_t* token);

#ifdef __cplusplus
}
#endif

#endif /* ZQ_H */
