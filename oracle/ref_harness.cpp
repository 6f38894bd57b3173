// ref_harness.cpp -- C entry points over the compiled ZYRON reference.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together
// with the reference's own unmodified sources (src/**/*.cpp of ZYRON) into
// oracle/_ref/libzyron_ref.so.  Tests use it to pin the C restatement
// (oracle/zq_oracle.c) against the real reference, to generate golden
// vectors, and bench.py's reference arm uses it as the timed CPU baseline.
// The product library never links it.
//
// Every function forwards to the reference's public API:
//   zyron::quantization::quantize / matmul / QuantizedMatrix::{dequantize,
//   save, load}            (include/zyron/quantization/quantization.hpp:18-58)
//   QuantizedLinear::forward (include/zyron/quantization/quantized_linear.hpp:10-31)
//   QuantizedLanguageModel   (include/zyron/model/quantized_language_model.hpp)
//   runtime::set_num_threads / num_threads (include/zyron/core/runtime.hpp:16-17)
#include "zyron/core/runtime.hpp"
#include "zyron/model/checkpoint.hpp"
#include "zyron/tokenizer/bpe.hpp"
#include "zyron/training/adamw.hpp"
#include "zyron/training/scheduler.hpp"
#include "zyron/core/tensor.hpp"
#include "zyron/model/language_model.hpp"
#include "zyron/model/quantized_language_model.hpp"
#include "zyron/quantization/quantization.hpp"
#include "zyron/quantization/quantized_linear.hpp"
#include "zyron/transformer/config.hpp"

#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <random>
#include <sstream>
#include <string>
#include <vector>

namespace zq = zyron::quantization;

namespace {
thread_local std::string g_err;

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::invalid_argument& e) {
        g_err = e.what();
        return 1;
    } catch (const std::out_of_range& e) {
        g_err = e.what();
        return 2;
    } catch (const std::overflow_error& e) {
        g_err = e.what();
        return 3;
    } catch (const std::exception& e) {
        g_err = e.what();
        return 4;
    }
}

zyron::Tensor tensor_from(const float* data, std::vector<std::size_t> dims) {
    zyron::Tensor t{zyron::Shape(std::move(dims))};
    std::memcpy(t.data(), data, t.size() * sizeof(float));
    return t;
}
}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

void ref_set_threads(std::size_t n) { zyron::runtime::set_num_threads(n); }
std::size_t ref_num_threads() { return zyron::runtime::num_threads(); }

// quantize(): w row-major [K][N]; returns an owned QuantizedMatrix handle.
int ref_quantize(const float* w, std::size_t K, std::size_t N, int type, void** out) {
    return guarded([&] {
        auto t = tensor_from(w, {K, N});
        *out = new zq::QuantizedMatrix(zq::quantize(t, static_cast<zq::Type>(type)));
    });
}

void ref_free(void* h) { delete static_cast<zq::QuantizedMatrix*>(h); }

// Serialise to the .zyq byte format (QuantizedMatrix::save(ostream)).
// Call once with buf == nullptr to learn the size.
int ref_save_zyq(const void* h, void* buf, std::size_t cap, std::size_t* len) {
    return guarded([&] {
        std::ostringstream os(std::ios::binary);
        static_cast<const zq::QuantizedMatrix*>(h)->save(os);
        const std::string s = os.str();
        *len = s.size();
        if (buf) {
            if (cap < s.size()) throw std::runtime_error("ref_save_zyq: buffer too small");
            std::memcpy(buf, s.data(), s.size());
        }
    });
}

// Parse .zyq bytes (QuantizedMatrix::load(istream)).
int ref_load_zyq(const void* buf, std::size_t len, void** out) {
    return guarded([&] {
        std::string s(static_cast<const char*>(buf), len);
        std::istringstream is(s, std::ios::binary);
        *out = new zq::QuantizedMatrix(zq::QuantizedMatrix::load(is));
    });
}

// Scales and the raw column-major payload, read through value() so the
// harness relies only on the public API.
int ref_scales(const void* h, float* scales) {
    return guarded([&] {
        const auto& q = *static_cast<const zq::QuantizedMatrix*>(h);
        std::memcpy(scales, q.scales().data(), q.cols() * sizeof(float));
    });
}

int ref_codes(const void* h, std::int8_t* codes) {
    return guarded([&] {
        const auto& q = *static_cast<const zq::QuantizedMatrix*>(h);
        for (std::size_t c = 0; c < q.cols(); ++c)
            for (std::size_t r = 0; r < q.rows(); ++r) codes[c * q.rows() + r] = q.value(c, r);
    });
}

std::size_t ref_bytes(const void* h) { return static_cast<const zq::QuantizedMatrix*>(h)->bytes(); }

// quantization::matmul(): x row-major [M][K] -> y row-major [M][N].
int ref_matmul(const void* h, const float* x, std::size_t M, std::size_t K, float* y) {
    return guarded([&] {
        const auto& q = *static_cast<const zq::QuantizedMatrix*>(h);
        auto t = tensor_from(x, {M, K});
        auto out = zq::matmul(t, q);
        std::memcpy(y, out.data(), out.size() * sizeof(float));
    });
}

// QuantizedLinear(QuantizedMatrix, bias).forward(x).  bias may be null.
int ref_linear_forward(const void* h, const float* bias, const float* x, std::size_t M,
                       std::size_t K, float* y) {
    return guarded([&] {
        const auto& q = *static_cast<const zq::QuantizedMatrix*>(h);
        zyron::Tensor b;
        if (bias) b = tensor_from(bias, {q.cols()});
        zq::QuantizedLinear lin(q, b);
        auto out = lin.forward(tensor_from(x, {M, K}));
        std::memcpy(y, out.data(), out.size() * sizeof(float));
    });
}

int ref_dequantize(const void* h, float* out) {
    return guarded([&] {
        auto t = static_cast<const zq::QuantizedMatrix*>(h)->dequantize();
        std::memcpy(out, t.data(), t.size() * sizeof(float));
    });
}

// ---------------------------------------------------------------------------
// Quantized language model (include/zyron/model/quantized_language_model.hpp)
// ---------------------------------------------------------------------------

struct RefQlm {
    std::unique_ptr<zyron::model::QuantizedLanguageModel> m;
};

// Build LanguageModel(config, seed) and quantize it; the config fields mirror
// transformer::Config (include/zyron/transformer/config.hpp).
int ref_qlm_create(std::size_t vocab, std::size_t hidden, std::size_t layers, std::size_t heads,
                   std::size_t kv_heads, std::size_t ffn, std::size_t max_seq, int use_rope,
                   int use_rms_norm, int tie, std::uint32_t seed, int type, void** out) {
    return guarded([&] {
        auto cfg = zyron::transformer::tiny(vocab);
        cfg.vocab_size = vocab;
        cfg.hidden_size = hidden;
        cfg.num_layers = layers;
        cfg.num_heads = heads;
        cfg.num_kv_heads = kv_heads;
        cfg.intermediate_size = ffn;
        cfg.max_sequence_length = max_seq;
        cfg.use_rope = use_rope != 0;
        cfg.use_rms_norm = use_rms_norm != 0;
        cfg.tie_word_embeddings = tie != 0;
        cfg.dropout = 0.0f;
        cfg.validate();
        zyron::model::LanguageModel lm(cfg, seed);
        auto* r = new RefQlm;
        r->m = std::make_unique<zyron::model::QuantizedLanguageModel>(lm, static_cast<zq::Type>(type));
        *out = r;
    });
}

void ref_qlm_free(void* h) { delete static_cast<RefQlm*>(h); }

int ref_qlm_save(const void* h, const char* path) {
    return guarded([&] { static_cast<const RefQlm*>(h)->m->save(path); });
}

int ref_qlm_load(const char* path, void** out) {
    return guarded([&] {
        auto* r = new RefQlm;
        r->m = std::make_unique<zyron::model::QuantizedLanguageModel>(
            zyron::model::QuantizedLanguageModel::load(path));
        *out = r;
    });
}

// forward(ids) -> logits [T][vocab] (batch 1).
int ref_qlm_forward(const void* h, const std::size_t* ids, std::size_t T, float* logits) {
    return guarded([&] {
        std::vector<std::size_t> v(ids, ids + T);
        auto out = static_cast<const RefQlm*>(h)->m->forward(v);
        std::memcpy(logits, out.data(), out.size() * sizeof(float));
    });
}

// Greedy generate (top_k = 1).  out receives prompt + new tokens; *out_len
// its length.
int ref_qlm_generate_greedy(const void* h, const std::size_t* ids, std::size_t T,
                            std::size_t max_new, std::size_t* out, std::size_t* out_len) {
    return guarded([&] {
        std::vector<std::size_t> v(ids, ids + T);
        zyron::model::GenerationConfig gc;
        gc.max_new_tokens = max_new;
        gc.top_k = 1;
        gc.top_p = 1.0f;
        gc.temperature = 1.0f;
        gc.repetition_penalty = 1.0f;
        gc.no_repeat_ngram_size = 0;
        gc.seed = 0;
        auto res = static_cast<const RefQlm*>(h)->m->generate(v, gc);
        std::memcpy(out, res.data(), res.size() * sizeof(std::size_t));
        *out_len = res.size();
    });
}

// generate() with a full GenerationConfig (include/zyron/model/generation.hpp:
// 13-21).  out receives prompt + new tokens; *out_len its length.
int ref_qlm_generate(const void* h, const std::size_t* ids, std::size_t T, std::size_t max_new, float temperature,
                     std::size_t top_k, float top_p, float repetition_penalty, std::size_t no_repeat_ngram_size,
                     std::uint32_t seed, std::size_t* out, std::size_t* out_len) {
    return guarded([&] {
        std::vector<std::size_t> v(ids, ids + T);
        zyron::model::GenerationConfig gc;
        gc.max_new_tokens = max_new;
        gc.temperature = temperature;
        gc.top_k = top_k;
        gc.top_p = top_p;
        gc.repetition_penalty = repetition_penalty;
        gc.no_repeat_ngram_size = no_repeat_ngram_size;
        gc.seed = seed;
        auto res = static_cast<const RefQlm*>(h)->m->generate(v, gc);
        std::memcpy(out, res.data(), res.size() * sizeof(std::size_t));
        *out_len = res.size();
    });
}

// Checkpoint::save (src/model/checkpoint.cpp:106-143) of LanguageModel(config,
// seed) whose parameters and optimizer moments are overwritten with
// uniform(-0.5, 0.5) draws (std::mt19937(seed + 1000 + i) for tensor i, so
// no two tensors are alike), an AdamW(lr 3e-4) and a warmup-cosine scheduler
// (3e-4, 10, 100, 1e-5), and a BPE tokenizer trained to 270 tokens on a
// fixed text.  Written as version 4, the format the reference saves.
int ref_checkpoint_save(const char* path, std::size_t vocab, std::size_t hidden, std::size_t layers,
                        std::size_t heads, std::size_t kv_heads, std::size_t ffn, std::size_t max_seq, int use_rope,
                        int use_rms_norm, int tie, std::uint32_t seed) {
    return guarded([&] {
        auto cfg = zyron::transformer::tiny(vocab);
        cfg.vocab_size = vocab;
        cfg.hidden_size = hidden;
        cfg.num_layers = layers;
        cfg.num_heads = heads;
        cfg.num_kv_heads = kv_heads;
        cfg.intermediate_size = ffn;
        cfg.max_sequence_length = max_seq;
        cfg.use_rope = use_rope != 0;
        cfg.use_rms_norm = use_rms_norm != 0;
        cfg.tie_word_embeddings = tie != 0;
        cfg.dropout = 0.0f;
        cfg.validate();
        zyron::model::LanguageModel lm(cfg, seed);
        auto params = lm.parameters();
        for (std::size_t i = 0; i < params.size(); ++i) {
            std::mt19937 rng(seed + 1000u + static_cast<std::uint32_t>(i));
            std::uniform_real_distribution<float> d(-0.5f, 0.5f);
            auto& t = params[i]->value();
            for (std::size_t k = 0; k < t.size(); ++k) t[k] = d(rng);
        }
        zyron::training::AdamW opt(params, 3e-4f, 0.9f, 0.95f, 1e-8f, 0.1f);
        zyron::training::WarmupCosineScheduler sched(3e-4f, 10, 100, 1e-5f);
        zyron::tokenizer::BPE tok;
        tok.train_text("the quick brown fox jumps over the lazy dog; the lazy dog sleeps. "
                       "quantized models run fast on tensor cores, the quick fox said.",
                       270);
        zyron::model::Checkpoint::save(path, lm, opt, sched, tok, 7);
    });
}

}  // extern "C"
