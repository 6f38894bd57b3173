// zq_checkpoint.cpp -- zyron_quantize: a .zyron training checkpoint to a
// .zyqmodel quantized model, with every weight quantized on the device.
//
// The reference tool (tools/zyron_quantize.cpp:33-48) loads the checkpoint
// (src/model/checkpoint.cpp:145-179), restores it into a LanguageModel, an
// AdamW optimizer, a warmup-cosine scheduler and a BPE tokenizer (181-232),
// builds QuantizedLanguageModel(model, type) (quantized_language_model.cpp:
// 178-269) and saves it (615-625).  Here the same file is parsed with the
// same checks, in the same order and with the same messages; the model's
// parameters are taken in LanguageModel::parameters() order
// (src/model/language_model.cpp:192-206); each weight matrix is quantized
// with the library's device quantize() (bit-identical to the reference's);
// and the .zyqmodel bytes are written in the reference's layout.  The
// sinusoidal position table is computed on the host with the reference's
// float expression, so the output is byte-identical to the reference tool's.
#include "zq.h"

#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <new>
#include <random>
#include <string>
#include <vector>

namespace zq {
zq_status set_error(zq_status s, const char* msg);
}

namespace {

struct Fail {
    zq_status status;
    std::string msg;
};

[[noreturn]] void fail(zq_status s, const std::string& m) { throw Fail{s, m}; }

// Bounded little-endian reader; a short read is the reference's
// "ZYRON checkpoint: corrupted file" (read_exact, checkpoint.cpp:23-26).
struct Reader {
    const uint8_t* p;
    size_t len, off = 0;
    void read(void* dst, size_t n) {
        if (off > len || len - off < n) fail(ZQ_ERR_RUNTIME, "ZYRON checkpoint: corrupted file");
        std::memcpy(dst, p + off, n);
        off += n;
    }
    uint64_t u64() {
        uint64_t v;
        read(&v, 8);
        return v;
    }
    uint32_t u32() {
        uint32_t v;
        read(&v, 4);
        return v;
    }
    float f32() {
        float v;
        read(&v, 4);
        return v;
    }
};

// transformer::Config with the reference's defaults
// (include/zyron/transformer/config.hpp:10-26).
struct Config {
    uint64_t vocab = 260, hidden = 128, layers = 2, heads = 4, kv_heads = 0, ffn = 512, max_seq = 128;
    float eps = 1e-5f;
    bool rms = true, causal = true, rope = true, tie = true;
    float theta = 10000.0f, dropout = 0.0f;
    bool qat = false;
    uint64_t qat_bits = 8;
    uint64_t kvh() const { return kv_heads == 0 ? heads : kv_heads; }
};

// Config::validate (config.hpp:32-66).
void validate(const Config& c) {
    if (c.vocab == 0 || c.hidden == 0 || c.layers == 0 || c.heads == 0 || c.ffn == 0 || c.max_seq == 0)
        fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON Transformer: dimensions must be > 0");
    if (c.hidden % c.heads != 0)
        fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON Transformer: hidden_size must be divisible by num_heads");
    if (c.kvh() == 0 || c.kvh() > c.heads || c.heads % c.kvh() != 0)
        fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON Transformer: num_kv_heads must divide num_heads and be <= num_heads");
    if (c.rope && ((c.hidden / c.heads) % 2 != 0))
        fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON Transformer: RoPE requires an even attention head dimension");
    if (!(c.eps > 0.0f)) fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON Transformer: norm_eps must be > 0");
    if (!(c.theta > 0.0f) || !std::isfinite(c.theta))
        fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON Transformer: rope_theta must be finite and > 0");
    if (!(c.dropout >= 0.0f) || c.dropout >= 1.0f || !std::isfinite(c.dropout))
        fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON Transformer: dropout must be finite and in [0, 1)");
    if (c.qat_bits != 4 && c.qat_bits != 8) fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON Transformer: qat_bits must be 4 or 8");
}

// read_config (checkpoint.cpp:43-71): versions 1-4 carry more fields.
Config read_config(Reader& r, uint32_t version) {
    Config c;
    c.vocab = r.u64();
    c.hidden = r.u64();
    c.layers = r.u64();
    c.heads = r.u64();
    c.ffn = r.u64();
    c.max_seq = r.u64();
    c.eps = r.f32();
    c.rms = r.u32() != 0;
    c.causal = r.u32() != 0;
    if (version >= 2) {
        c.kv_heads = r.u64();
        c.rope = r.u32() != 0;
        c.tie = r.u32() != 0;
        c.theta = r.f32();
        if (version >= 3) {
            c.dropout = r.f32();
            if (version >= 4) {
                c.qat = r.u32() != 0;
                c.qat_bits = r.u64();
            }
        }
    } else {
        c.kv_heads = c.heads;
        c.rope = false;
        c.tie = false;
    }
    validate(c);
    return c;
}

struct Tensor {
    std::vector<uint64_t> dims;
    const float* data = nullptr;  // into the checkpoint bytes (may be unaligned: copy before use)
    uint64_t count = 0;
};

// Shape(dims) validation and size (include/zyron/core/shape.hpp).
uint64_t shape_size(const std::vector<uint64_t>& dims) {
    uint64_t result = 1;
    for (uint64_t d : dims) {
        if (d == 0) fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON Shape: dimensions must be > 0");
        if (result > std::numeric_limits<uint64_t>::max() / d)
            fail(ZQ_ERR_OVERFLOW, "ZYRON Shape: element count overflow");
        result *= d;
    }
    return result;
}

// read_tensor (checkpoint.cpp:80-93).
Tensor read_tensor(Reader& r) {
    const uint64_t rank = r.u64();
    if (rank > 64) fail(ZQ_ERR_RUNTIME, "ZYRON checkpoint: invalid tensor rank");
    Tensor t;
    for (uint64_t i = 0; i < rank; ++i) t.dims.push_back(r.u64());
    const uint64_t size = shape_size(t.dims);
    t.count = r.u64();
    if (t.count != size) fail(ZQ_ERR_RUNTIME, "ZYRON checkpoint: tensor size mismatch");
    if (t.count > (r.len - r.off) / sizeof(float)) fail(ZQ_ERR_RUNTIME, "ZYRON checkpoint: corrupted file");
    t.data = reinterpret_cast<const float*>(r.p + r.off);
    r.off += t.count * sizeof(float);
    return t;
}

// read_tensor_vector (checkpoint.cpp:98-104).
std::vector<Tensor> read_tensors(Reader& r) {
    const uint64_t n = r.u64();
    if (n > 1000000) fail(ZQ_ERR_RUNTIME, "ZYRON checkpoint: too many tensors");
    std::vector<Tensor> out;
    out.reserve((size_t)n);
    for (uint64_t i = 0; i < n; ++i) out.push_back(read_tensor(r));
    return out;
}

// validate_hyperparameters (src/training/adamw.cpp:10-16).
void check_adamw(float lr, float b1, float b2, float eps, float wd) {
    if (!(lr >= 0.0f) || !std::isfinite(lr)) fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON AdamW: invalid learning rate");
    if (!(b1 >= 0.0f && b1 < 1.0f) || !std::isfinite(b1)) fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON AdamW: invalid beta1");
    if (!(b2 >= 0.0f && b2 < 1.0f) || !std::isfinite(b2)) fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON AdamW: invalid beta2");
    if (!(eps > 0.0f) || !std::isfinite(eps)) fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON AdamW: invalid epsilon");
    if (!(wd >= 0.0f) || !std::isfinite(wd)) fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON AdamW: invalid weight decay");
}

// WarmupCosineScheduler's constructor checks (src/training/scheduler.cpp:19-26).
void check_scheduler(float base, uint64_t warmup, uint64_t total, float min_lr) {
    if (!(base >= 0.0f) || !std::isfinite(base))
        fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON Scheduler: invalid base learning rate");
    if (total == 0) fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON Scheduler: total_steps must be > 0");
    if (warmup > total) fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON Scheduler: warmup_steps > total_steps");
    if (!(min_lr >= 0.0f) || !std::isfinite(min_lr) || min_lr > base)
        fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON Scheduler: invalid minimum learning rate");
}

// BPE::load(istream)'s structure checks (src/tokenizer/bpe.cpp:490-529): the
// tokenizer is restored but not part of the quantized model.
void check_tokenizer(const uint8_t* p, size_t len) {
    size_t off = 0;
    auto u32 = [&]() -> uint32_t {
        if (len - off < 4) fail(ZQ_ERR_RUNTIME, "ZYRON BPE: corrupted tokenizer file");
        uint32_t v;
        std::memcpy(&v, p + off, 4);
        off += 4;
        return v;
    };
    auto str = [&]() -> uint32_t {
        const uint32_t n = u32();
        if (n != 0) {
            if (len - off < n) fail(ZQ_ERR_RUNTIME, "ZYRON BPE: corrupted tokenizer string");
            off += n;
        }
        return n;
    };
    if (u32() != 0x4e42595au || u32() != 1u) fail(ZQ_ERR_RUNTIME, "ZYRON BPE: unsupported tokenizer format");
    const uint32_t vocab = u32();
    const uint32_t merges = u32();
    if (vocab < 260) fail(ZQ_ERR_RUNTIME, "ZYRON BPE: invalid vocabulary size");
    bool empty_special = false;
    for (int i = 0; i < 4; ++i) empty_special = (str() == 0) || empty_special;
    if (empty_special) fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON BPE: special tokens must not be empty");  // reset (39-45)
    for (uint32_t i = 0; i < vocab; ++i) str();
    for (uint32_t i = 0; i < merges; ++i) {
        u32();
        u32();
        u32();
    }
}

// The model's parameter shapes in LanguageModel::parameters() order
// (language_model.cpp:192-206; transformer_block.cpp:60-70; attention.cpp:
// 368-377; feed_forward.cpp:32-37; linear.cpp:142-146; normalization.cpp).
// With tied embeddings the lm_head contributes only its bias: its weight is
// the embedding's, already listed.
std::vector<std::vector<uint64_t>> parameter_shapes(const Config& c) {
    const uint64_t H = c.hidden, V = c.vocab, F = c.ffn, kvd = c.kvh() * (c.hidden / c.heads);
    std::vector<std::vector<uint64_t>> s;
    s.push_back({V, H});
    for (uint64_t l = 0; l < c.layers; ++l) {
        s.push_back({H});
        if (!c.rms) s.push_back({H});
        s.push_back({H, H});
        s.push_back({H});
        s.push_back({H, kvd});
        s.push_back({kvd});
        s.push_back({H, kvd});
        s.push_back({kvd});
        s.push_back({H, H});
        s.push_back({H});
        s.push_back({H});
        if (!c.rms) s.push_back({H});
        s.push_back({H, F});
        s.push_back({F});
        s.push_back({F, H});
        s.push_back({H});
    }
    s.push_back({H});
    if (!c.tie) s.push_back({H, V});
    s.push_back({V});
    return s;
}

// Output buffer in the reference's little-endian save format
// (quantized_language_model.cpp:575-625).
struct Writer {
    std::vector<uint8_t> b;
    void put(const void* p, size_t n) {
        const uint8_t* q = static_cast<const uint8_t*>(p);
        b.insert(b.end(), q, q + n);
    }
    void u32(uint32_t v) { put(&v, 4); }
    void u64(uint64_t v) { put(&v, 8); }
    void f32(float v) { put(&v, 4); }
    // qwrite_tensor (582-590): an empty tensor is rank 0, size 0.
    void tensor(const std::vector<uint64_t>& dims, const float* data, uint64_t count) {
        if (count == 0) {
            u64(0);
            u64(0);
            return;
        }
        u64(dims.size());
        for (uint64_t d : dims) u64(d);
        u64(count);
        put(data, count * sizeof(float));
    }
    void tensor(const Tensor& t) { tensor(t.dims, t.data, t.count); }
};

std::vector<float> copy_floats(const Tensor& t) {
    std::vector<float> v((size_t)t.count);
    if (t.count) std::memcpy(v.data(), t.data, t.count * sizeof(float));
    return v;
}

// quantize(w [rows][cols]) on the device, appended as a .zyq record
// (QuantizedMatrix::save).  Returns the record's payload + scale bytes
// (QuantizedMatrix::bytes, quantization.cpp:104-109).
uint64_t put_quantized(Writer& w, const float* data, uint64_t rows, uint64_t cols, int type, void* stream) {
    zq_weight* q = nullptr;
    zq_status s = zq_weight_quantize_host(data, rows, cols, type, stream, &q);
    if (s != ZQ_OK) fail(s, zq_last_error());
    size_t n = 0;
    s = zq_weight_save_zyq(q, nullptr, 0, &n, stream);
    if (s == ZQ_OK) {
        const size_t at = w.b.size();
        w.b.resize(at + n);
        s = zq_weight_save_zyq(q, w.b.data() + at, n, &n, stream);
    }
    size_t payload = 0;
    if (s == ZQ_OK) s = zq_weight_info(q, nullptr, nullptr, nullptr, &payload, nullptr);
    const std::string msg = s == ZQ_OK ? "" : zq_last_error();
    zq_weight_destroy(q);
    if (s != ZQ_OK) fail(s, msg);
    return payload + cols * sizeof(float);
}

struct Result {
    std::vector<uint8_t> bytes;
    uint64_t quantized_bytes = 0, float_bytes = 0;
};

Result build_image(const Config& c, const std::vector<Tensor>& params, int type, void* stream);

Result convert(const uint8_t* data, size_t len, int type, void* stream) {
    Reader r{data, len};
    // Checkpoint::load (145-179)
    if (r.u32() != 0x4e52595au) fail(ZQ_ERR_RUNTIME, "ZYRON checkpoint: unsupported format");
    const uint32_t version = r.u32();
    if (version < 1 || version > 4) fail(ZQ_ERR_RUNTIME, "ZYRON checkpoint: unsupported format");
    const Config c = read_config(r, version);
    r.u64();  // training step
    r.u64();  // optimizer step
    const float lr = r.f32(), b1 = r.f32(), b2 = r.f32(), eps = r.f32(), wd = r.f32();
    r.u64();  // scheduler step
    const float base_lr = r.f32();
    const uint64_t warmup = r.u64(), total = r.u64();
    const float min_lr = r.f32();
    const std::vector<Tensor> params = read_tensors(r);
    const std::vector<Tensor> m1 = read_tensors(r);
    const std::vector<Tensor> m2 = read_tensors(r);
    const uint64_t tok_size = r.u64();
    if (tok_size > r.len - r.off) fail(ZQ_ERR_RUNTIME, "ZYRON checkpoint: corrupted file");
    const uint8_t* tok = r.p + r.off;

    // zyron_quantize: LanguageModel(config, 42), AdamW and the scheduler
    // from the checkpoint's hyper-parameters, then Checkpoint::restore.
    check_adamw(lr, b1, b2, eps, wd);
    check_scheduler(base_lr, warmup, total, min_lr);
    const auto shapes = parameter_shapes(c);
    if (shapes.size() != params.size()) fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON checkpoint: parameter count mismatch");
    for (size_t i = 0; i < shapes.size(); ++i)
        if (shapes[i] != params[i].dims) fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON checkpoint: parameter shape mismatch");
    if (m1.size() != params.size() || m2.size() != params.size())
        fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON AdamW: checkpoint state parameter count mismatch");
    for (size_t i = 0; i < params.size(); ++i)
        if (m1[i].dims != params[i].dims || m2[i].dims != params[i].dims)
            fail(ZQ_ERR_INVALID_ARGUMENT, "ZYRON AdamW: checkpoint moment shape mismatch");
    if (tok_size == 0) fail(ZQ_ERR_RUNTIME, "ZYRON checkpoint: tokenizer data missing");
    check_tokenizer(tok, (size_t)tok_size);
    return build_image(c, params, type, stream);
}

// QuantizedLanguageModel(model, type) and save (quantized_language_model.cpp:
// 178-269, 615-625) of a model whose parameters, in parameters() order and
// with the shapes of parameter_shapes(c), are `params`.
Result build_image(const Config& c, const std::vector<Tensor>& params, int type, void* stream) {
    const uint64_t H = c.hidden, V = c.vocab, F = c.ffn, kvd = c.kvh() * (c.hidden / c.heads);
    Result res;
    Writer w;
    w.u32(0x4d4c5a51u);
    w.u32(1u);
    w.u32((uint32_t)type);
    w.u64(c.vocab);
    w.u64(c.hidden);
    w.u64(c.layers);
    w.u64(c.heads);
    w.u64(c.kv_heads);
    w.u64(c.ffn);
    w.u64(c.max_seq);
    w.f32(c.eps);
    w.u32(c.rms);
    w.u32(c.causal);
    w.u32(c.rope);
    w.u32(c.tie);
    w.f32(c.theta);
    w.f32(c.dropout);
    w.u32(c.qat);
    w.u64(c.qat_bits);
    size_t pi = 0;
    const std::vector<float> emb = copy_floats(params[pi++]);
    uint64_t qb = put_quantized(w, emb.data(), V, H, type, stream);
    uint64_t fb = V * H * 4;
    // sinusoidal table for models without RoPE (199-208), same float formula
    if (!c.rope) {
        std::vector<float> pe((size_t)(c.max_seq * H), 0.0f);
        constexpr float base = 10000.0f;
        const float hidden = static_cast<float>(H);
        for (uint64_t pos = 0; pos < c.max_seq; ++pos)
            for (uint64_t i = 0; i < H; i += 2) {
                const float exponent = static_cast<float>(i) / hidden;
                const float angle = static_cast<float>(pos) / std::pow(base, exponent);
                pe[pos * H + i] = std::sin(angle);
                if (i + 1 < H) pe[pos * H + i + 1] = std::cos(angle);
            }
        w.tensor({c.max_seq, H}, pe.data(), pe.size());
        qb += pe.size() * 4;
        fb += pe.size() * 4;
    } else {
        w.tensor({}, nullptr, 0);
    }
    // final norm weight, then the blocks
    const Tensor* final_norm = &params[params.size() - (c.tie ? 2 : 3)];
    w.tensor(*final_norm);
    qb += final_norm->count * 4;
    fb += final_norm->count * 4;
    w.u64(c.layers);
    for (uint64_t l = 0; l < c.layers; ++l) {
        const Tensor& n1w = params[pi++];
        const Tensor* n1b = c.rms ? nullptr : &params[pi++];
        const Tensor* lin[6][2];
        for (int k = 0; k < 4; ++k) {
            lin[k][0] = &params[pi++];
            lin[k][1] = &params[pi++];
        }
        const Tensor& n2w = params[pi++];
        const Tensor* n2b = c.rms ? nullptr : &params[pi++];
        for (int k = 4; k < 6; ++k) {
            lin[k][0] = &params[pi++];
            lin[k][1] = &params[pi++];
        }
        w.u32(c.rms);
        w.tensor(n1w);
        if (n1b) w.tensor(*n1b); else w.tensor({}, nullptr, 0);
        w.u32(c.rms);
        w.tensor(n2w);
        if (n2b) w.tensor(*n2b); else w.tensor({}, nullptr, 0);
        const uint64_t norms = (n1w.count + (n1b ? n1b->count : 0) + n2w.count + (n2b ? n2b->count : 0)) * 4;
        qb += norms;
        fb += norms;
        const uint64_t in_f[6] = {H, H, H, H, H, F}, out_f[6] = {H, kvd, kvd, H, F, H};
        for (int k = 0; k < 6; ++k) {
            const std::vector<float> wk = copy_floats(*lin[k][0]);
            qb += put_quantized(w, wk.data(), in_f[k], out_f[k], type, stream);
            w.tensor(*lin[k][1]);
            fb += in_f[k] * out_f[k] * 4 + lin[k][1]->count * 4;
        }
    }
    // lm_head: effective_weight() -- the transposed embedding when tied
    // (linear.cpp:148-152) -- and its bias
    pi++;  // final norm, written above
    std::vector<float> head;
    if (c.tie) {
        head.resize((size_t)(H * V));
        for (uint64_t v = 0; v < V; ++v)
            for (uint64_t h = 0; h < H; ++h) head[h * V + v] = emb[v * H + h];
    } else {
        head = copy_floats(params[pi++]);
    }
    const Tensor& head_bias = params[pi++];
    qb += put_quantized(w, head.data(), H, V, type, stream);
    w.tensor(head_bias);
    qb += head_bias.count * 4;
    fb += H * V * 4 + head_bias.count * 4;
    res.bytes = std::move(w.b);
    res.quantized_bytes = qb;
    res.float_bytes = fb;
    return res;
}

// The parameters of LanguageModel(config, seed) (language_model.cpp:52-75),
// in parameters() order.  Every random tensor is Tensor::random(shape, -lim,
// lim, s) (src/core/tensor.cpp:165-172): a fresh std::mt19937(s) and one
// std::uniform_real_distribution<float>(-lim, lim) draw per element in
// row-major order, so the values equal the reference's bit for bit on the
// same standard library.  The seeds follow the constructors: the embedding
// (range 0.02, embedding.hpp:17) takes seed + 1; the transformer seed + 100,
// its block l that + 100 l (transformer.cpp:44-47); a block's attention + 10
// and its feed-forward + 20 (transformer_block.cpp:13-14); q, k, v and out
// projections + 1..4 (attention.cpp:102-105); up and down + 1, + 2
// (feed_forward.cpp:8-9); an untied lm_head seed + 200.  Linear weights use
// the Xavier limit sqrt(6 / (in + out)) in float (linear.cpp:13-26); norm
// weights are ones, norm and linear biases zeros.
std::vector<std::vector<float>> init_parameters(const Config& c, uint32_t seed) {
    const auto shapes = parameter_shapes(c);
    std::vector<std::vector<float>> out;
    out.reserve(shapes.size());
    auto random = [&](uint64_t rows, uint64_t cols, float lim, uint32_t s) {
        std::vector<float> v((size_t)(rows * cols));
        std::mt19937 rng(s);
        std::uniform_real_distribution<float> dist(-lim, lim);
        for (float& x : v) x = dist(rng);
        out.push_back(std::move(v));
    };
    auto fill = [&](uint64_t n, float value) { out.push_back(std::vector<float>((size_t)n, value)); };
    auto linear = [&](uint64_t in, uint64_t o, uint32_t s) {
        random(in, o, std::sqrt(6.0f / static_cast<float>(in + o)), s);
        fill(o, 0.0f);
    };
    const uint64_t H = c.hidden, V = c.vocab, F = c.ffn, kvd = c.kvh() * (c.hidden / c.heads);
    random(V, H, 0.02f, seed + 1u);
    const uint32_t transformer_seed = seed + 100u;
    for (uint64_t l = 0; l < c.layers; ++l) {
        const uint32_t block = transformer_seed + static_cast<uint32_t>(l * 100);
        const uint32_t attn = block + 10u, ffn = block + 20u;
        fill(H, 1.0f);
        if (!c.rms) fill(H, 0.0f);
        linear(H, H, attn + 1u);
        linear(H, kvd, attn + 2u);
        linear(H, kvd, attn + 3u);
        linear(H, H, attn + 4u);
        fill(H, 1.0f);
        if (!c.rms) fill(H, 0.0f);
        linear(H, F, ffn + 1u);
        linear(F, H, ffn + 2u);
    }
    fill(H, 1.0f);
    if (!c.tie) random(H, V, std::sqrt(6.0f / static_cast<float>(H + V)), seed + 200u);
    fill(V, 0.0f);
    if (out.size() != shapes.size()) fail(ZQ_ERR_RUNTIME, "zyron_b200: parameter list mismatch");
    for (size_t i = 0; i < out.size(); ++i)
        if (out[i].size() != shape_size(shapes[i])) fail(ZQ_ERR_RUNTIME, "zyron_b200: parameter size mismatch");
    return out;
}

}  // namespace

extern "C" {

zq_status zq_quantize_checkpoint(const void* checkpoint, size_t len, int type, void* stream, void** out,
                                 size_t* out_len, double* compression_ratio) {
    if (!out || !out_len) return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null output");
    *out = nullptr;
    *out_len = 0;
    if (type != ZQ_TYPE_INT8 && type != ZQ_TYPE_INT4)
        return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "--bits must be 4 or 8");
    try {
        Result r = convert(static_cast<const uint8_t*>(checkpoint), checkpoint ? len : 0, type, stream);
        void* buf = std::malloc(r.bytes.size());
        if (!buf) return zq::set_error(ZQ_ERR_RUNTIME, "zyron_b200: out of host memory");
        std::memcpy(buf, r.bytes.data(), r.bytes.size());
        *out = buf;
        *out_len = r.bytes.size();
        if (compression_ratio)
            *compression_ratio = r.quantized_bytes == 0 ? 0.0 : (double)r.float_bytes / (double)r.quantized_bytes;
        return ZQ_OK;
    } catch (const Fail& f) {
        return zq::set_error(f.status, f.msg.c_str());
    } catch (const std::bad_alloc&) {
        return zq::set_error(ZQ_ERR_RUNTIME, "zyron_b200: out of host memory");
    }
}

zq_status zq_lm_init_image(const zq_lm_config* config, uint32_t seed, int type, void* stream, void** out,
                           size_t* out_len, double* compression_ratio) {
    if (!out || !out_len || !config) return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null argument");
    *out = nullptr;
    *out_len = 0;
    if (type != ZQ_TYPE_INT8 && type != ZQ_TYPE_INT4)
        return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: type must be INT8 or INT4");
    try {
        Config c;
        c.vocab = config->vocab_size;
        c.hidden = config->hidden_size;
        c.layers = config->num_layers;
        c.heads = config->num_heads;
        c.kv_heads = config->num_kv_heads;
        c.ffn = config->intermediate_size;
        c.max_seq = config->max_sequence_length;
        c.eps = config->norm_eps;
        c.rms = config->use_rms_norm != 0;
        c.causal = config->causal != 0;
        c.rope = config->use_rope != 0;
        c.tie = config->tie_word_embeddings != 0;
        c.theta = config->rope_theta;
        c.dropout = config->dropout;
        c.qat = config->use_qat != 0;
        c.qat_bits = config->qat_bits;
        validate(c);
        const std::vector<std::vector<float>> store = init_parameters(c, seed);
        const auto shapes = parameter_shapes(c);
        std::vector<Tensor> params(store.size());
        for (size_t i = 0; i < store.size(); ++i) {
            params[i].dims = shapes[i];
            params[i].data = store[i].data();
            params[i].count = store[i].size();
        }
        Result r = build_image(c, params, type, stream);
        void* buf = std::malloc(r.bytes.size());
        if (!buf) return zq::set_error(ZQ_ERR_RUNTIME, "zyron_b200: out of host memory");
        std::memcpy(buf, r.bytes.data(), r.bytes.size());
        *out = buf;
        *out_len = r.bytes.size();
        if (compression_ratio)
            *compression_ratio = r.quantized_bytes == 0 ? 0.0 : (double)r.float_bytes / (double)r.quantized_bytes;
        return ZQ_OK;
    } catch (const Fail& f) {
        return zq::set_error(f.status, f.msg.c_str());
    } catch (const std::bad_alloc&) {
        return zq::set_error(ZQ_ERR_RUNTIME, "zyron_b200: out of host memory");
    }
}

void zq_free_buffer(void* p) { std::free(p); }

}  // extern "C"
