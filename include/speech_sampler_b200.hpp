/*
 * C++ host wrapper of the B200 sampler's C ABI (speech_sampler_b200.h) for speech.cpp's call sites.
 * Header-only, C++17.
 *
 * Part 1, always available: an RAII context, the engine's mask layout, the talker's suppress mask built
 * once per min_frames state (Generation::banned, src/families/qwen3-tts/sampler.cpp:62-67), and one-row
 * host calls returning the id and the row status.
 *
 * Part 2, where the reference's headers are included before this one and the including file defines
 * SSB_SPEECH_CPP (qwen3-tts/sampler.h, json.h), SSB_SPEECH_CPP_HARU (haru/sampler.h) or
 * SSB_SPEECH_CPP_DRAMA3 (drama3/sampler.h): the reference's own call signatures in namespace
 * ssb::speechcpp, each sampling on the device and throwing the exception the reference throws for the
 * same row:
 *   sample(logits, SamplingParams, history, banned, double u)           qwen3-tts/sampler.cpp:103-111
 *   sample(logits, SamplingParams, history, banned, std::mt19937_64 &)  qwen3-tts/sampler.cpp:113-116
 *   haru_sample(logits, haru::Sampling, u)    = candidates() then pick()  haru/sampler.cpp:18-61
 *   drama3_sample(logits, drama3::Sampling, u) = candidates() then pick()  drama3/sampler.cpp:30-60
 * The rng overload draws uniform() only where the row draws (not greedy), as the reference does, so a
 * seeded decode loop consumes the same numbers. A call-level failure of the engine (a CUDA error, a size
 * beyond its limits) becomes an Error of the matching Fault.
 */
#pragma once

#include <cstdint>
#include <random>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "speech_sampler_b200.h"

namespace ssb {

/* A failed call of the C ABI (not a row status): the ssb_status and ssb_last_error()'s message. */
class EngineError : public std::runtime_error {
public:
    EngineError(ssb_status status, const std::string & message) : std::runtime_error(message), status_(status) {}
    ssb_status status() const { return status_; }

private:
    ssb_status status_;
};

inline void check(ssb_status s) {
    if (s != SSB_OK) throw EngineError(s, ssb_last_error());
}

/* One sampling context (scratch, staging, cached masks) on one device. Movable, not copyable. */
class Context {
public:
    explicit Context(int device = 0) { check(ssb_context_create(device, &ctx_)); }
    ~Context() {
        if (ctx_) ssb_context_destroy(ctx_);
    }
    Context(const Context &) = delete;
    Context & operator=(const Context &) = delete;
    Context(Context && o) noexcept : ctx_(std::exchange(o.ctx_, nullptr)) {}
    Context & operator=(Context && o) noexcept {
        if (this != &o) {
            if (ctx_) ssb_context_destroy(ctx_);
            ctx_ = std::exchange(o.ctx_, nullptr);
        }
        return *this;
    }

    ssb_context * get() const { return ctx_; }
    void reserve(int32_t rows, int32_t vocab) { check(ssb_context_reserve(ctx_, rows, vocab)); }
    /* Device pointers in `r`; asynchronous on `stream` (a cudaStream_t, or null). */
    void sample_rows(const ssb_rows & r, void * stream = nullptr) { check(ssb_sample_rows(ctx_, &r, stream)); }
    /* Host pointers in `r`; returns when ids and status are written. */
    void sample_host(const ssb_rows & r, void * stream = nullptr) { check(ssb_sample_host(ctx_, &r, stream)); }
    /* A device copy of `words` owned by the context (ssb_context_mask). */
    const uint32_t * upload_mask(const std::vector<uint32_t> & words) {
        const uint32_t * d = nullptr;
        check(ssb_context_mask(ctx_, words.data(), (int64_t) words.size(), &d));
        return d;
    }

private:
    ssb_context * ctx_ = nullptr;
};

/* The calling thread's context on `device` (created on first use): the context the reference-signature
 * calls of part 2 use when given none. */
inline Context & thread_context(int device = 0) {
    thread_local Context ctx(device);
    return ctx;
}

/* The engine's mask layout: bit (t & 31) of word t >> 5 is token t. Entries of `banned` past `vocab`
 * are ignored and a shorter `banned` leaves the rest allowed (restricted(), qwen3-tts/sampler.cpp:40-42). */
inline std::vector<uint32_t> pack_mask(const std::vector<bool> & banned, int vocab) {
    std::vector<uint32_t> words((size_t) (vocab + 31) / 32, 0u);
    const size_t n = banned.size() < (size_t) vocab ? banned.size() : (size_t) vocab;
    for (size_t i = 0; i < n; i++)
        if (banned[i]) words[i >> 5] |= 1u << (i & 31);
    return words;
}

/*
 * Generation::banned(vocab, end_of_speech, frames) (qwen3-tts/sampler.cpp:62-67) packed once per
 * min_frames state: the last `suppressed_tokens` ids but the end of speech, and the end of speech while
 * frames < min_frames. host(frames) serves ssb_sample_host, device(ctx, frames) ssb_sample_rows (copied
 * to the context on first use).
 */
class TalkerBanMask {
public:
    TalkerBanMask(int vocab, int32_t end_of_speech, int suppressed_tokens, int min_frames)
        : vocab_(vocab), min_frames_(min_frames) {
        late_.assign((size_t) (vocab + 31) / 32, 0u);
        const int first = suppressed_tokens < vocab ? vocab - suppressed_tokens : 0;
        for (int i = first; i < vocab; i++)
            if (i != end_of_speech) late_[(size_t) i >> 5] |= 1u << (i & 31);
        early_ = late_;
        if (end_of_speech >= 0 && end_of_speech < vocab) early_[(size_t) end_of_speech >> 5] |= 1u << (end_of_speech & 31);
    }
    int vocab() const { return vocab_; }
    const std::vector<uint32_t> & host(int frames) const { return frames < min_frames_ ? early_ : late_; }
    const uint32_t * device(Context & ctx, int frames) {
        const bool early = frames < min_frames_;
        for (const Cached & c : device_)
            if (c.ctx == ctx.get() && c.early == early) return c.words;
        device_.push_back(Cached{ctx.get(), early, ctx.upload_mask(host(frames))});
        return device_.back().words;
    }

private:
    struct Cached {
        ssb_context * ctx;
        bool early;
        const uint32_t * words;
    };
    int vocab_ = 0, min_frames_ = 0;
    std::vector<uint32_t> early_, late_;
    std::vector<Cached> device_;
};

/* The id and row status (ssb_row_status) of one sampled row. */
struct RowResult {
    int32_t id = -1;
    int32_t status = SSB_ROW_OK;
};

/* One f32 row from host memory, as the reference's sample() receives it: `mask` (host words, or null)
 * bans its set bits; `history` of `history_len` ids (or null). */
inline RowResult sample_host_row(Context & ctx, const float * logits, int32_t vocab, const ssb_params & p,
                                 const int32_t * history, int64_t history_len, const uint32_t * mask, double u) {
    RowResult out;
    ssb_rows r{};
    r.logits = logits;
    r.ld = vocab;
    r.dtype = SSB_F32;
    r.rows = 1;
    r.vocab = vocab;
    r.params = p;
    r.history = history_len > 0 ? history : nullptr;
    r.history_ld = history_len > 0 ? history_len : 0;
    r.mask = mask;
    r.mask_kind = mask ? SSB_MASK_BAN : SSB_MASK_NONE;
    r.u = &u;
    r.ids = &out.id;
    r.status = &out.status;
    ctx.sample_host(r);
    return out;
}

}  // namespace ssb

#if defined(SSB_SPEECH_CPP) || defined(SSB_SPEECH_CPP_HARU) || defined(SSB_SPEECH_CPP_DRAMA3)
namespace ssb {
namespace speechcpp {

/* The reference's Fault of a call-level failure of the engine (src/common/error.h:8-21). */
inline Fault fault_of(ssb_status s) {
    switch (s) {
        case SSB_INVALID_ARGUMENT: return Fault::InvalidArgument;
        case SSB_OUT_OF_RANGE: return Fault::OutOfRange;
        case SSB_OUT_OF_MEMORY: return Fault::OutOfMemory;
        default: return Fault::Device;
    }
}

/* One host row through the engine, an engine failure rethrown as the reference's Error. */
inline RowResult host_row(Context & ctx, const std::vector<float> & logits, const ssb_params & p,
                          const std::vector<int32_t> & history, const uint32_t * mask, double u) {
    try {
        return sample_host_row(ctx, logits.data(), (int32_t) logits.size(), p, history.data(),
                               (int64_t) history.size(), mask, u);
    } catch (const EngineError & e) {
        throw Error(fault_of(e.status()), e.what());
    }
}

/* A row status the reference has no exception for: a fault of the device. */
[[noreturn]] inline void device_fault(int32_t status) {
    throw Error(Fault::Device, "the sampler could not sample a row on the device (row status " + std::to_string(status) + ")");
}

}  // namespace speechcpp
}  // namespace ssb
#endif

#ifdef SSB_SPEECH_CPP
namespace ssb {
namespace speechcpp {

inline ssb_params to_params(const SamplingParams & p) {
    return ssb_params{p.greedy ? 1 : 0, p.temperature, p.top_k, p.top_p, p.repetition_penalty, 0.0f, 0.0f,
                      SSB_FLAVOR_QWEN3_TTS};
}

/* The exception the reference's sample() throws for a row that ended with `status`: the penalty's
 * Error (qwen3-tts/sampler.cpp:43-48), temperature_overflow() (sampler.cpp:82-83, sampling.cpp:21-25),
 * the runtime_error of a row without a finite logit (sampler.cpp:49). */
[[noreturn]] inline void rethrow(int32_t status, const SamplingParams & p) {
    switch (status) {
        case SSB_ROW_PENALTY_OVERFLOW:
            throw Error(Fault::OutOfRange,
                        "the repetition penalty " + json_number(p.repetition_penalty) +
                            " pushes a logit beyond the range of a float; give a penalty nearer 1",
                        "repetition_penalty");
        case SSB_ROW_TEMPERATURE_OVERFLOW: throw temperature_overflow(p.temperature);
        case SSB_ROW_NO_FINITE_LOGIT: throw std::runtime_error("no token has a finite logit to pick from");
        default: device_fault(status);
    }
}

/* sample(logits, p, history, banned, u) (qwen3-tts/sampler.cpp:103-111) on the device. */
inline int32_t sample(Context & ctx, const std::vector<float> & logits, const SamplingParams & p,
                      const std::vector<int32_t> & history, const std::vector<bool> & banned, double u) {
    const std::vector<uint32_t> mask = banned.empty() ? std::vector<uint32_t>() : pack_mask(banned, (int) logits.size());
    const RowResult r = host_row(ctx, logits, to_params(p), history, mask.empty() ? nullptr : mask.data(), u);
    if (r.status != SSB_ROW_OK) rethrow(r.status, p);
    return r.id;
}

/* sample(logits, p, history, banned, rng) (qwen3-tts/sampler.cpp:113-116): the next uniform() of `rng`
 * where p draws, none where p is greedy. */
inline int32_t sample(Context & ctx, const std::vector<float> & logits, const SamplingParams & p,
                      const std::vector<int32_t> & history, const std::vector<bool> & banned, std::mt19937_64 & rng) {
    return sample(ctx, logits, p, history, banned, p.greedy ? 0.0 : uniform(rng));
}

/* The talker's step with its ban mask cached: banned = Generation::banned(vocab, end_of_speech, frames). */
inline int32_t sample(Context & ctx, const std::vector<float> & logits, const SamplingParams & p,
                      const std::vector<int32_t> & history, const TalkerBanMask & banned, int frames,
                      std::mt19937_64 & rng) {
    const double u = p.greedy ? 0.0 : uniform(rng);
    const RowResult r = host_row(ctx, logits, to_params(p), history, banned.host(frames).data(), u);
    if (r.status != SSB_ROW_OK) rethrow(r.status, p);
    return r.id;
}

/* The same calls on the calling thread's context. */
inline int32_t sample(const std::vector<float> & logits, const SamplingParams & p, const std::vector<int32_t> & history,
                      const std::vector<bool> & banned, double u) {
    return sample(thread_context(), logits, p, history, banned, u);
}
inline int32_t sample(const std::vector<float> & logits, const SamplingParams & p, const std::vector<int32_t> & history,
                      const std::vector<bool> & banned, std::mt19937_64 & rng) {
    return sample(thread_context(), logits, p, history, banned, rng);
}

}  // namespace speechcpp
}  // namespace ssb
#endif

#ifdef SSB_SPEECH_CPP_HARU
namespace ssb {
namespace speechcpp {

/* tokens[pick(weights, u)] of haru::candidates(logits, s) (haru/sampler.cpp:18-61) on the device, with
 * its exceptions: a NaN or +inf logit is the device's Error (:21-23), an overflowing temperature
 * temperature_overflow() (:34). A temperature of 0 or less takes the first maximum whatever u is. */
inline int32_t haru_sample(Context & ctx, const std::vector<float> & logits, const haru::Sampling & s, double u) {
    const ssb_params p{0, s.temperature, s.top_k, s.top_p, 1.0f, 0.0f, 0.0f, SSB_FLAVOR_HARU};
    const RowResult r = host_row(ctx, logits, p, {}, nullptr, u);
    switch (r.status) {
        case SSB_ROW_OK: return r.id;
        case SSB_ROW_NON_FINITE_INPUT:
            throw Error(Fault::Device, "the model computed a logit that is not a number; run it on another device");
        case SSB_ROW_TEMPERATURE_OVERFLOW: throw temperature_overflow(s.temperature);
        default: device_fault(r.status);
    }
}

}  // namespace speechcpp
}  // namespace ssb
#endif

#ifdef SSB_SPEECH_CPP_DRAMA3
namespace ssb {
namespace speechcpp {

/* tokens[pick(weights, u)] of drama3::candidates(logits, s) (drama3/sampler.cpp:30-60) on the device,
 * with its exceptions: a non-finite logit is the device's Error (:35-37), a temperature that takes the
 * largest logit beyond a float temperature_overflow() (:47). */
inline int32_t drama3_sample(Context & ctx, const std::vector<float> & logits, const drama3::Sampling & s, double u) {
    const ssb_params p{0, s.temperature, s.top_k, s.top_p, 1.0f, 0.0f, 0.0f, SSB_FLAVOR_DRAMA3};
    const RowResult r = host_row(ctx, logits, p, {}, nullptr, u);
    switch (r.status) {
        case SSB_ROW_OK: return r.id;
        case SSB_ROW_NON_FINITE_INPUT:
            throw Error(Fault::Device,
                        "the device computed logits that are not finite numbers; run the model on another device or "
                        "with another weight type");
        case SSB_ROW_TEMPERATURE_OVERFLOW: throw temperature_overflow(s.temperature);
        default: device_fault(r.status);
    }
}

}  // namespace speechcpp
}  // namespace ssb
#endif
