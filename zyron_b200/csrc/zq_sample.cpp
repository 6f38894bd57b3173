// zq_sample.cpp -- token sampling of ZYRON's QuantizedLanguageModel on the
// host, over one row of logits the device computed.
//
// The reference's sample_next (src/model/quantized_language_model.cpp:82-174)
// draws from an std::mt19937 with std::uniform_real_distribution<float> after
// an std::sort of the whole vocabulary by probability.  The order std::sort
// leaves equal probabilities in, and the draws, are those of the C++ standard
// library, so the sampler is host code built with the same compiler and
// library as the reference: given the same logits it returns the same token.
// The steps are restated here in the reference's order with the same float
// operations (penalty, n-gram block, max, sequential exp sum, probabilities,
// sort, top-k, top-p, draw); only the bookkeeping differs (bitmaps instead of
// std::find over the history and a std::map of n-gram prefixes, which give
// the same membership answers).
#include "zq.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <limits>
#include <new>
#include <random>
#include <vector>

namespace zq {
zq_status set_error(zq_status s, const char* msg);
}

struct zq_sampler {
    std::mt19937 rng;
};

namespace {

struct Candidate {
    std::size_t id;
    float probability;
};

// Whether `id` is a member of the bitmap.
inline bool has(const std::vector<uint32_t>& bits, std::size_t id) { return (bits[id >> 5] >> (id & 31)) & 1u; }
inline void put(std::vector<uint32_t>& bits, std::size_t id) { bits[id >> 5] |= 1u << (id & 31); }

}  // namespace

namespace zq {

// validate_generation_config (quantized_language_model.cpp:71-80): same
// checks, order and messages.
zq_status check_generation_config(const zq_generation_config* c) {
    if (!c) return set_error(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null generation config");
    if (!(c->temperature > 0.0f) || !std::isfinite(c->temperature))
        return set_error(ZQ_ERR_INVALID_ARGUMENT, "ZYRON QuantizedLanguageModel: invalid temperature");
    if (!(c->top_p > 0.0f) || c->top_p > 1.0f || !std::isfinite(c->top_p))
        return set_error(ZQ_ERR_INVALID_ARGUMENT, "ZYRON QuantizedLanguageModel: invalid top_p");
    if (!(c->repetition_penalty >= 1.0f) || !std::isfinite(c->repetition_penalty))
        return set_error(ZQ_ERR_INVALID_ARGUMENT, "ZYRON QuantizedLanguageModel: invalid repetition_penalty");
    return ZQ_OK;
}

// sample_next (82-174) for one row of `vocab` logits; history holds the
// prompt and the tokens generated so far.
std::size_t sample_row(std::mt19937& rng, const float* logits, std::size_t vocab, const int64_t* history,
                       std::size_t len, const zq_generation_config& cfg) {
    // Tokens of the history (repetition penalty, 116-121).
    std::vector<uint32_t> seen((vocab + 31) / 32, 0u);
    if (cfg.repetition_penalty != 1.0f)
        for (std::size_t i = 0; i < len; ++i)
            if (history[i] >= 0 && (uint64_t)history[i] < vocab) put(seen, (std::size_t)history[i]);

    // n-gram block (96-108): the tokens that followed an earlier occurrence
    // of the last n - 1 tokens.  The reference keeps a map from every
    // (n - 1)-gram prefix of the history to its followers and looks up the
    // current prefix; scanning the history for that prefix gives the same
    // set.  `blocked_found` is the reference's `blocked != seen_ngrams.end()`.
    std::vector<uint32_t> blocked((vocab + 31) / 32, 0u);
    bool blocked_found = false;
    const std::size_t n = cfg.no_repeat_ngram_size;
    if (n > 0 && len >= n) {
        const std::size_t pl = n - 1;
        const int64_t* prefix = history + (len - pl);
        for (std::size_t start = 0; start + n <= len; ++start) {
            if (!std::equal(history + start, history + start + pl, prefix)) continue;
            blocked_found = true;
            const int64_t t = history[start + pl];
            if (t >= 0 && (uint64_t)t < vocab) put(blocked, (std::size_t)t);
        }
    }

    // Penalised and blocked values and their maximum (110-128).
    float max_logit = -std::numeric_limits<float>::infinity();
    std::vector<float> values(vocab);
    for (std::size_t id = 0; id < vocab; ++id) {
        float value = logits[id];
        if (cfg.repetition_penalty != 1.0f && has(seen, id))
            value = value >= 0.0f ? value / cfg.repetition_penalty : value * cfg.repetition_penalty;
        if (blocked_found && has(blocked, id)) value = -std::numeric_limits<float>::infinity();
        values[id] = value;
        max_logit = std::max(max_logit, value);
    }
    bool any_finite = false;
    for (float value : values) any_finite = any_finite || std::isfinite(value);
    if (!any_finite && blocked_found) {
        for (std::size_t id = 0; id < vocab; ++id) values[id] = logits[id];
        max_logit = *std::max_element(values.begin(), values.end());
    }

    // Softmax with a sequential denominator (130-136).
    float denominator = 0.0f;
    for (float value : values) denominator += std::exp(value - max_logit);
    if (!(denominator > 0.0f) || !std::isfinite(denominator)) return 0;
    std::vector<Candidate> candidates;
    candidates.reserve(vocab);
    for (std::size_t id = 0; id < vocab; ++id)
        candidates.push_back({id, std::exp(values[id] - max_logit) / denominator});

    // Sort by probability, then the top-k and top-p cuts (138-160).
    std::sort(candidates.begin(), candidates.end(),
              [](const Candidate& a, const Candidate& b) { return a.probability > b.probability; });
    if (cfg.top_k != 0 && cfg.top_k < candidates.size()) candidates.resize(cfg.top_k);
    if (cfg.top_p < 1.0f) {
        float cumulative = 0.0f;
        std::size_t keep = 0;
        for (const Candidate& c : candidates) {
            cumulative += c.probability;
            ++keep;
            if (cumulative >= cfg.top_p) break;
        }
        candidates.resize(std::max<std::size_t>(1, keep));
    }

    // One draw over the kept mass (162-173).
    float probability_sum = 0.0f;
    for (const Candidate& c : candidates) probability_sum += c.probability;
    if (!(probability_sum > 0.0f)) return candidates.front().id;
    std::uniform_real_distribution<float> distribution(0.0f, probability_sum);
    const float draw = distribution(rng);
    float cumulative = 0.0f;
    for (const Candidate& c : candidates) {
        cumulative += c.probability;
        if (draw <= cumulative) return c.id;
    }
    return candidates.back().id;
}

}  // namespace zq

extern "C" {

zq_status zq_sampler_create(uint32_t seed, zq_sampler** out) {
    if (!out) return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null output handle");
    *out = new (std::nothrow) zq_sampler{std::mt19937(seed)};
    if (!*out) return zq::set_error(ZQ_ERR_RUNTIME, "zyron_b200: out of host memory");
    return ZQ_OK;
}

zq_status zq_sampler_destroy(zq_sampler* s) {
    delete s;
    return ZQ_OK;
}

zq_status zq_sample_next(zq_sampler* s, const float* logits, size_t vocab, const int64_t* history, size_t history_len,
                         const zq_generation_config* config, int64_t* token) {
    if (!s || !token) return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null argument");
    zq_status st = zq::check_generation_config(config);
    if (st != ZQ_OK) return st;
    if (vocab == 0 || !logits) return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: empty logits");
    if (config->top_k > vocab)
        return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "ZYRON QuantizedLanguageModel: top_k exceeds vocabulary");
    if (history_len > 0 && !history) return zq::set_error(ZQ_ERR_INVALID_ARGUMENT, "zyron_b200: null history");
    try {
        *token = (int64_t)zq::sample_row(s->rng, logits, vocab, history, history_len, *config);
    } catch (const std::bad_alloc&) {
        return zq::set_error(ZQ_ERR_RUNTIME, "zyron_b200: out of host memory");
    }
    return ZQ_OK;
}

}  // extern "C"
