// Test infrastructure only: checks the C++ call-site wrapper (include/speech_sampler_b200.hpp) against
// the reference it stands in for. Compiled by oracle/Makefile against the reference's own headers and
// sampler sources (unmodified, where they lie under $(REF)) and linked with the engine
// (speech.cpp_b200/libspeech_sampler_b200.so); Python tests load it with ctypes. Each entry point runs
// the same call through the reference and through the wrapper and reports both outcomes:
//   adapter_sample       sample(logits, SamplingParams, history, banned, u)   qwen3-tts/sampler.cpp:103-111
//   adapter_haru         haru::candidates + pick                               haru/sampler.cpp:18-61
//   adapter_drama3       drama3::candidates + pick                             drama3/sampler.cpp:30-60
//   adapter_talker_loop  the talker's decode loop (qwen3-tts/synthesizer.cpp:120-131): sample(..., rng)
//                        with Generation::banned per frame and the code predictor's draws between
//                        frames, for `steps` frames; ids of both sides and whether both generators
//                        end in the same state
#include <cstdint>
#include <cstring>
#include <exception>
#include <random>
#include <string>
#include <vector>

#include "drama3/sampler.h"
#include "error.h"
#include "haru/sampler.h"
#include "json.h"
#include "qwen3-tts/sampler.h"
#include "sampling.h"

#define SSB_SPEECH_CPP 1
#define SSB_SPEECH_CPP_HARU 1
#define SSB_SPEECH_CPP_DRAMA3 1
#include "speech_sampler_b200.hpp"

namespace {

/** Same field order and sizes as ssb_params (include/speech_sampler_b200.h). */
struct CheckParams {
    int32_t greedy;
    float temperature;
    int32_t top_k;
    float top_p;
    float repetition_penalty;
    float presence_penalty;
    float frequency_penalty;
    int32_t flavor;
};

/** How a call ended: kind 0 returned `id`; 1 threw Error (fault, input); 2 threw std::runtime_error;
 * 3 threw anything else. The message is what() (truncated to fit). */
struct Outcome {
    int32_t id;
    int32_t kind;
    int32_t fault;
    char input[64];
    char message[448];
};

SamplingParams qwen_params(const CheckParams * p) {
    SamplingParams s;
    s.greedy = p->greedy != 0;
    s.temperature = p->temperature;
    s.top_k = p->top_k;
    s.top_p = p->top_p;
    s.repetition_penalty = p->repetition_penalty;
    return s;
}

void copy_text(char * dst, size_t cap, const std::string & s) {
    const size_t n = s.size() < cap - 1 ? s.size() : cap - 1;
    std::memcpy(dst, s.data(), n);
    dst[n] = 0;
}

template <typename Body>
void record(Outcome * o, Body && body) {
    std::memset(o, 0, sizeof(*o));
    o->id = -1;
    try {
        o->id = body();
        o->kind = 0;
    } catch (const Error & e) {
        o->kind = 1;
        o->fault = (int32_t) e.fault();
        copy_text(o->input, sizeof(o->input), e.input());
        copy_text(o->message, sizeof(o->message), e.what());
    } catch (const std::runtime_error & e) {
        o->kind = 2;
        copy_text(o->message, sizeof(o->message), e.what());
    } catch (const std::exception & e) {
        o->kind = 3;
        copy_text(o->message, sizeof(o->message), e.what());
    }
}

thread_local std::string g_message;

std::vector<bool> banned_of(const uint8_t * banned, int32_t n) {
    std::vector<bool> b;
    if (banned) b.assign(banned, banned + n);
    return b;
}

}  // namespace

extern "C" {

/** sample(logits, p, history, banned, u): the reference's into *ref, the wrapper's into *adapter. */
void adapter_sample(const float * logits, int32_t n, const CheckParams * p, const int32_t * history, int32_t hlen,
                    const uint8_t * banned, int32_t banned_len, double u, Outcome * adapter, Outcome * ref) {
    const std::vector<float> row(logits, logits + n);
    const std::vector<int32_t> h(history, history + (history ? hlen : 0));
    const std::vector<bool> b = banned_of(banned, banned_len);
    const SamplingParams s = qwen_params(p);
    record(ref, [&] { return sample(row, s, h, b, u); });
    record(adapter, [&] { return ssb::speechcpp::sample(row, s, h, b, u); });
}

/** tokens[pick(weights, u)] of haru::candidates, by the reference and by the wrapper. */
void adapter_haru(const float * logits, int32_t n, float temperature, int32_t top_k, float top_p, double u,
                  Outcome * adapter, Outcome * ref) {
    const std::vector<float> row(logits, logits + n);
    haru::Sampling s;
    s.temperature = temperature;
    s.top_k = top_k;
    s.top_p = top_p;
    record(ref, [&] {
        const Candidates c = haru::candidates(row, s);
        return c.tokens[(size_t) pick(c.weights, u)];
    });
    record(adapter, [&] { return ssb::speechcpp::haru_sample(ssb::thread_context(), row, s, u); });
}

/** tokens[pick(weights, u)] of drama3::candidates, by the reference and by the wrapper. */
void adapter_drama3(const float * logits, int32_t n, float temperature, int32_t top_k, float top_p, double u,
                    Outcome * adapter, Outcome * ref) {
    const std::vector<float> row(logits, logits + n);
    drama3::Sampling s;
    s.temperature = temperature;
    s.top_k = top_k;
    s.top_p = top_p;
    record(ref, [&] {
        const Candidates c = drama3::candidates(row, s);
        return c.tokens[(size_t) pick(c.weights, u)];
    });
    record(adapter, [&] { return ssb::speechcpp::drama3_sample(ssb::thread_context(), row, s, u); });
}

/**
 * The talker's loop over `steps` frames of `logits` [steps, vocab]: each frame samples with the talker's
 * settings, the history of the frames before and Generation::banned(vocab, eos, frame) (the reference's
 * own Generation, built from a stub model file holding these settings), then draws `cp_draws` uniforms
 * as the code predictor does when it samples. The reference runs sample(..., rng); the wrapper runs
 * mode 0: ssb::speechcpp::sample(..., std::vector<bool> banned, rng), mode 1: the same with the cached
 * TalkerBanMask. Both generators start from `seed`. Returns 0, or -1 when a side threw (the message:
 * adapter_last_message()). *rng_equal = both generators end in the same state.
 */
int64_t adapter_talker_loop(const float * logits, int64_t steps, int32_t vocab, const CheckParams * p, int32_t eos,
                            int32_t suppressed, int32_t min_frames, int32_t cp_draws, uint64_t seed, int32_t mode,
                            int32_t * ids_adapter, int32_t * ids_ref, int32_t * rng_equal) {
    try {
        ModelFile m;
        const std::string t = "qwen3-tts.generation.talker.", c = "qwen3-tts.generation.code_predictor.";
        m.set(t + "do_sample", p->greedy ? 0.0 : 1.0);
        m.set(t + "temperature", p->temperature);
        m.set(t + "top_k", p->top_k);
        m.set(t + "top_p", p->top_p);
        m.set(t + "repetition_penalty", p->repetition_penalty);
        m.set(c + "do_sample", 1.0);
        m.set(c + "temperature", 0.9);
        m.set(c + "top_k", 50);
        m.set(c + "top_p", 1.0);
        m.set(c + "repetition_penalty", 1.0);
        m.set("qwen3-tts.generation.min_frames", min_frames);
        m.set("qwen3-tts.generation.max_frames", (double) steps);
        m.set("qwen3-tts.talker.suppressed_tokens", suppressed);
        const Generation g(m);
        ssb::TalkerBanMask cached(vocab, eos, g.suppressed_tokens, g.min_frames);
        std::mt19937_64 rng_ref(seed), rng_ad(seed);
        std::vector<int32_t> hist_ref, hist_ad;
        for (int64_t s = 0; s < steps; s++) {
            const std::vector<float> row(logits + s * vocab, logits + (s + 1) * vocab);
            const int frames = (int) s;
            ids_ref[s] = sample(row, g.talker, hist_ref, g.banned(vocab, eos, frames), rng_ref);
            hist_ref.push_back(ids_ref[s]);
            if (mode == 0)
                ids_adapter[s] = ssb::speechcpp::sample(row, g.talker, hist_ad, g.banned(vocab, eos, frames), rng_ad);
            else
                ids_adapter[s] = ssb::speechcpp::sample(ssb::thread_context(), row, g.talker, hist_ad, cached, frames, rng_ad);
            hist_ad.push_back(ids_adapter[s]);
            for (int d = 0; d < cp_draws; d++) {
                uniform(rng_ref);
                uniform(rng_ad);
            }
        }
        *rng_equal = rng_ref == rng_ad ? 1 : 0;
        return 0;
    } catch (const std::exception & e) {
        g_message = e.what();
        *rng_equal = 0;
        return -1;
    }
}

const char * adapter_last_message() { return g_message.c_str(); }

}  // extern "C"
