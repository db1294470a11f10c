// Test infrastructure only (the checker, never the product): a C ABI over the reference's own CPU
// sampler, compiled unmodified from its sources by oracle/Makefile. Python tests, the golden-fixture
// generator and bench.py's reference arm load the resulting oracle/_ref/libref_sampler.so with ctypes.
//
// Wrapped reference symbols:
//   sample(logits, SamplingParams, history, banned, u)   src/families/qwen3-tts/sampler.cpp:103-111
//   candidates(logits, SamplingParams, history, banned)  src/families/qwen3-tts/sampler.cpp:69-101
//   pick(weights, u)                                     src/common/sampling.cpp:9-19
//   uniform(std::mt19937_64&)                            src/common/sampling.cpp:5-7
//   haru::candidates(logits, haru::Sampling)             src/families/haru/sampler.cpp:18-61
//   drama3::candidates(logits, drama3::Sampling)         src/families/drama3/sampler.cpp:30-60
//   haru::Dry::update / penalties, shape_logits          src/families/haru/sampler.cpp:82-124
//
// Status codes (identical to the product's per-row codes, include/speech_sampler_b200.h):
//   0 ok; 1 Error(OutOfRange, "repetition_penalty"); 2 Error(OutOfRange, "temperature");
//   3 std::runtime_error "no token has a finite logit"; 4 Error(Device) (Haru's NaN refusal);
//   5 any other exception (message copied out).
#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <exception>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "error.h"
#include "drama3/sampler.h"
#include "haru/sampler.h"
#include "qwen3-tts/sampler.h"
#include "sampling.h"

namespace {

/** Same field order and sizes as ssb_params in include/speech_sampler_b200.h. */
struct RefParams {
    int32_t greedy;
    float temperature;
    int32_t top_k;
    float top_p;
    float repetition_penalty;
    float presence_penalty;   // not a reference parameter: ignored here (see ref_time_rows)
    float frequency_penalty;  // not a reference parameter: ignored here (see ref_time_rows)
    int32_t flavor;           // not a reference parameter: ignored here
};

SamplingParams to_params(const RefParams * p) {
    SamplingParams s;
    s.greedy = p->greedy != 0;
    s.temperature = p->temperature;
    s.top_k = p->top_k;
    s.top_p = p->top_p;
    s.repetition_penalty = p->repetition_penalty;
    return s;
}

thread_local std::string g_message;

int classify(const std::exception & e) {
    g_message = e.what();
    if (const Error * err = dynamic_cast<const Error *>(&e)) {
        if (err->fault() == Fault::OutOfRange && err->input() == "repetition_penalty") return 1;
        if (err->fault() == Fault::OutOfRange && err->input() == "temperature") return 2;
        if (err->fault() == Fault::Device) return 4;
        return 5;
    }
    if (g_message == "no token has a finite logit to pick from") return 3;
    return 5;
}

std::vector<bool> banned_of(const uint8_t * banned, int32_t banned_len) {
    std::vector<bool> b;
    if (banned) b.assign(banned, banned + banned_len);
    return b;
}

}  // namespace

extern "C" {

const char * ref_last_message() { return g_message.c_str(); }

/** sample(logits, p, history, banned, u); banned is one byte per token (nullable = none). */
int ref_sample(const float * logits, int32_t n, const RefParams * p, const int32_t * history, int32_t hlen,
               const uint8_t * banned, int32_t banned_len, double u, int32_t * id) {
    try {
        const std::vector<float> row(logits, logits + n);
        const std::vector<int32_t> h(history, history + (history ? hlen : 0));
        *id = sample(row, to_params(p), h, banned_of(banned, banned_len), u);
        return 0;
    } catch (const std::exception & e) {
        *id = -1;
        return classify(e);
    }
}

/** candidates(logits, p, history, banned): writes up to `cap` tokens and weights and the full count. */
int ref_candidates(const float * logits, int32_t n, const RefParams * p, const int32_t * history, int32_t hlen,
                   const uint8_t * banned, int32_t banned_len, int32_t * tokens, double * weights, int32_t cap,
                   int32_t * count) {
    try {
        const std::vector<float> row(logits, logits + n);
        const std::vector<int32_t> h(history, history + (history ? hlen : 0));
        const Candidates c = candidates(row, to_params(p), h, banned_of(banned, banned_len));
        *count = (int32_t) c.tokens.size();
        for (int32_t i = 0; i < *count && i < cap; i++) {
            tokens[i] = c.tokens[(size_t) i];
            weights[i] = c.weights[(size_t) i];
        }
        return 0;
    } catch (const std::exception & e) {
        *count = 0;
        return classify(e);
    }
}

int32_t ref_pick(const double * weights, int32_t n, double u) {
    return (int32_t) pick(std::vector<double>(weights, weights + n), u);
}

/** n draws of uniform() from std::mt19937_64(seed). */
void ref_uniform(uint64_t seed, int64_t n, double * out) {
    std::mt19937_64 rng(seed);
    for (int64_t i = 0; i < n; i++) out[i] = uniform(rng);
}

/** haru::candidates(logits, {temperature, top_k, top_p}). */
int ref_haru_candidates(const float * logits, int32_t n, float temperature, int32_t top_k, float top_p,
                        int32_t * tokens, double * weights, int32_t cap, int32_t * count) {
    try {
        haru::Sampling s;
        s.temperature = temperature;
        s.top_k = top_k;
        s.top_p = top_p;
        const Candidates c = haru::candidates(std::vector<float>(logits, logits + n), s);
        *count = (int32_t) c.tokens.size();
        for (int32_t i = 0; i < *count && i < cap; i++) {
            tokens[i] = c.tokens[(size_t) i];
            weights[i] = c.weights[(size_t) i];
        }
        return 0;
    } catch (const std::exception & e) {
        *count = 0;
        return classify(e);
    }
}

/** drama3::candidates(logits, {temperature, top_k, top_p}). */
int ref_drama3_candidates(const float * logits, int32_t n, float temperature, int32_t top_k, float top_p,
                          int32_t * tokens, double * weights, int32_t cap, int32_t * count) {
    try {
        drama3::Sampling s;
        s.temperature = temperature;
        s.top_k = top_k;
        s.top_p = top_p;
        const Candidates c = drama3::candidates(std::vector<float>(logits, logits + n), s);
        *count = (int32_t) c.tokens.size();
        for (int32_t i = 0; i < *count && i < cap; i++) {
            tokens[i] = c.tokens[(size_t) i];
            weights[i] = c.weights[(size_t) i];
        }
        return 0;
    } catch (const std::exception & e) {
        *count = 0;
        return classify(e);
    }
}

/** Same layout as ssb_dry_config. */
struct RefDryConfig {
    double multiplier, base, max_penalty;
    int32_t allowed_length, lookback, max_match_length, reserved;
};

static haru::Dry make_dry(const RefDryConfig * c, const int32_t * exempt, int32_t n_exempt) {
    haru::DryConfig d;
    d.multiplier = c->multiplier;
    d.base = c->base;
    d.max_penalty = c->max_penalty;
    d.allowed_length = c->allowed_length;
    d.lookback = c->lookback;
    d.max_match_length = c->max_match_length;
    return haru::Dry(d, std::vector<int32_t>(exempt, exempt + n_exempt));
}

/** haru::Dry::update over `tokens`, the penalties() after each: [n_tokens, cap] and counts [n_tokens]. */
void ref_dry_run(const RefDryConfig * c, const int32_t * exempt, int32_t n_exempt, const int32_t * tokens,
                 int64_t n_tokens, int32_t * pen_tokens, double * pen_values, int32_t cap, int32_t * counts) {
    haru::Dry dry = make_dry(c, exempt, n_exempt);
    for (int64_t s = 0; s < n_tokens; s++) {
        dry.update(tokens[s]);
        const auto & p = dry.penalties();
        counts[s] = (int32_t) p.size();
        for (size_t i = 0; i < p.size() && (int32_t) i < cap; i++) {
            pen_tokens[s * cap + (int64_t) i] = p[i].first;
            pen_values[s * cap + (int64_t) i] = p[i].second;
        }
    }
}

/** shape_logits(logits, dry after `tokens`, silent, {pad, eop, eos}, eop_bias, must_speak) in place. */
void ref_haru_shape(float * logits, int32_t n, const RefDryConfig * c, const int32_t * exempt, int32_t n_exempt,
                    const int32_t * tokens, int64_t n_tokens, const float * silent, int32_t pad, int32_t eop,
                    int32_t eos, float eop_bias, int32_t must_speak) {
    haru::Dry dry = make_dry(c, exempt, n_exempt);
    for (int64_t s = 0; s < n_tokens; s++) dry.update(tokens[s]);
    std::vector<float> l(logits, logits + n);
    haru::TextIds ids;
    ids.pad = pad;
    ids.eop = eop;
    ids.eos = eos;
    haru::shape_logits(l, dry, silent, ids, eop_bias, must_speak != 0);
    std::copy(l.begin(), l.end(), logits);
}

/**
 * The CPU baseline: sample() over `rows` rows split statically over `threads` std::thread workers, one
 * row per call as the reference's decode loops call it. Row vectors, histories and ban lists are built
 * before the clock starts (the call sites hold them already); the timed region is the sample() calls.
 *
 * The reference has no presence/frequency penalty. Where p asks for one (and the repetition penalty is
 * 1, so the order of processors is unaffected), it is applied to the row copy inside the timed region
 * before sample(), in fp32 as the engine defines it: l -= frequency*count; l -= presence.
 *
 * banned: one byte per token; banned_ld = 0 shares one list across rows. hlens nullable (= hld for all,
 * with negative ids skipped by the reference itself). Returns seconds, or -1 on a bad argument.
 */
double ref_time_rows(const float * logits, int64_t rows, int32_t n, int64_t ld, const RefParams * p,
                     const int32_t * history, int64_t hld, const int32_t * hlens, const uint8_t * banned,
                     int64_t banned_ld, const double * u, int32_t threads, int32_t * ids, int32_t * status) {
    if (rows <= 0 || n <= 0 || threads <= 0) return -1;
    const bool ext = p->presence_penalty != 0.0f || p->frequency_penalty != 0.0f;
    if (ext && p->repetition_penalty != 1.0f) return -1;
    const SamplingParams sp = to_params(p);
    std::vector<std::vector<float>> lv((size_t) rows);
    std::vector<std::vector<int32_t>> hv((size_t) rows);
    std::vector<std::vector<bool>> bv(banned ? (banned_ld ? (size_t) rows : 1) : 0);
    for (int64_t r = 0; r < rows; r++) {
        lv[(size_t) r].assign(logits + r * ld, logits + r * ld + n);
        if (history) {
            const int64_t len = hlens ? hlens[r] : hld;
            hv[(size_t) r].assign(history + r * hld, history + r * hld + len);
        }
    }
    for (size_t b = 0; b < bv.size(); b++) bv[b].assign(banned + (int64_t) b * banned_ld, banned + (int64_t) b * banned_ld + n);
    const std::vector<bool> none;

    auto work = [&](int64_t r0, int64_t r1) {
        std::vector<float> row;
        std::vector<int32_t> sorted;
        for (int64_t r = r0; r < r1; r++) {
            const std::vector<float> * src = &lv[(size_t) r];
            if (ext) {
                row = lv[(size_t) r];
                sorted = hv[(size_t) r];
                std::sort(sorted.begin(), sorted.end());
                for (size_t i = 0; i < sorted.size();) {
                    size_t j = i;
                    while (j < sorted.size() && sorted[j] == sorted[i]) j++;
                    const int32_t t = sorted[i];
                    if (t >= 0 && t < n) {
                        float l = row[(size_t) t];
                        l = l - p->frequency_penalty * (float) (j - i);
                        l = l - p->presence_penalty;
                        row[(size_t) t] = l;
                    }
                    i = j;
                }
                src = &row;
            }
            const std::vector<bool> & b = bv.empty() ? none : bv[banned_ld ? (size_t) r : 0];
            try {
                ids[r] = sample(*src, sp, hv[(size_t) r], b, sp.greedy ? 0.0 : u[r]);
                status[r] = 0;
            } catch (const std::exception & e) {
                ids[r] = -1;
                status[r] = classify(e);
            }
        }
    };

    const auto t0 = std::chrono::steady_clock::now();
    if (threads == 1) {
        work(0, rows);
    } else {
        std::vector<std::thread> pool;
        const int64_t per = (rows + threads - 1) / threads;
        for (int32_t t = 0; t < threads; t++) {
            const int64_t r0 = std::min<int64_t>(rows, (int64_t) t * per), r1 = std::min<int64_t>(rows, r0 + per);
            if (r0 < r1) pool.emplace_back(work, r0, r1);
        }
        for (auto & th : pool) th.join();
    }
    const auto t1 = std::chrono::steady_clock::now();
    return std::chrono::duration<double>(t1 - t0).count();
}

int32_t ref_hardware_concurrency() { return (int32_t) std::thread::hardware_concurrency(); }

}  // extern "C"
