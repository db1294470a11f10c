/*
 * speech_sampler_b200 — the C ABI of the B200 token-sampling and logit-processing engine.
 *
 * This is the boundary a speech.cpp build links against in place of its CPU sampler. Every call takes
 * plain device pointers and sizes (no C++ or torch types), never throws, never falls back to the CPU,
 * and reports failures as an ssb_status plus a thread-local message (ssb_last_error()). Per-row
 * numerical refusals (the reference's exceptions) come back as ssb_row_status codes in `status[]`.
 *
 * Reference interfaces replaced (paths in the speech.cpp source tree):
 *   sample(logits, SamplingParams, history, banned, u)  src/families/qwen3-tts/sampler.h:61-62, .cpp:103-111
 *   sample(..., std::mt19937_64&)                       src/families/qwen3-tts/sampler.h:65-66, .cpp:113-116
 *   candidates(logits, SamplingParams, history, banned) src/families/qwen3-tts/sampler.h:52-53, .cpp:69-101
 *   GraphSampler::pick/draw/read (device picks)         src/families/qwen3-tts/graph-sampler.h:30-45
 *   Qwen3Readback::Pick (device argmax, ASR greedy)     src/common/qwen3-decoder.h:80-92, .cpp:422-437
 *   Qwen3Decoder verify() argmax over [n, vocab]        src/common/qwen3-decoder.cpp:492-510
 *   host greedy max_element (ASR)                       src/families/qwen3-asr/decoder.cpp:108-113
 *   haru::candidates, drama3::candidates (+ pick)       src/families/haru/sampler.cpp:18-61, drama3/sampler.cpp:30-60
 *   haru::Dry::update / penalties, shape_logits         src/families/haru/sampler.cpp:82-124
 *   Error(Fault, message, input) refusals               src/common/error.h:8-38
 */
#ifndef SPEECH_SAMPLER_B200_H
#define SPEECH_SAMPLER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define SSB_API __attribute__((visibility("default")))
#else
#define SSB_API
#endif

/* Call status. Mirrors the reference's Fault kinds (src/common/error.h:8-21) that this path can raise. */
typedef enum ssb_status {
    SSB_OK = 0,
    SSB_INVALID_ARGUMENT = 1, /* Fault::InvalidArgument: a null pointer, a negative size, a bad enum */
    SSB_OUT_OF_RANGE = 2,     /* Fault::OutOfRange: a size beyond an engine limit (message names it) */
    SSB_DEVICE = 3,           /* Fault::Device: a CUDA error */
    SSB_OUT_OF_MEMORY = 4     /* Fault::OutOfMemory: device scratch could not be allocated */
} ssb_status;

/*
 * Per-row outcome, written to status[row]. The C++ host wrapper (speech_sampler_b200.hpp) turns each
 * into the reference's exception:
 *   PENALTY_OVERFLOW     -> Error(OutOfRange, ..., "repetition_penalty")   qwen3-tts/sampler.cpp:43-47
 *   TEMPERATURE_OVERFLOW -> temperature_overflow(T), input "temperature"   sampling.cpp:21-25, sampler.cpp:82-83
 *   NO_FINITE_LOGIT      -> std::runtime_error("no token has a finite logit to pick from")  sampler.cpp:49
 *   NON_FINITE_INPUT     -> Error(Device, ...)  a NaN among the restricted logits (haru/sampler.cpp:21-23)
 *   INVALID_ROW          -> a row whose own parameters exceed the launch's bounds (ssb_rows.max_top_k)
 *   DEVICE_TIMEOUT       -> Error(Device, ...): the row's logits did not arrive in shared memory within
 *                           the kernel's bounded wait (a device fault; never expected)
 */
typedef enum ssb_row_status {
    SSB_ROW_OK = 0,
    SSB_ROW_PENALTY_OVERFLOW = 1,
    SSB_ROW_TEMPERATURE_OVERFLOW = 2,
    SSB_ROW_NO_FINITE_LOGIT = 3,
    SSB_ROW_NON_FINITE_INPUT = 4,
    SSB_ROW_INVALID_ROW = 5,
    SSB_ROW_DEVICE_TIMEOUT = 6
} ssb_row_status;

typedef enum ssb_dtype { SSB_F32 = 0, SSB_BF16 = 1 } ssb_dtype;

/* BAN: a set bit removes the token (the reference's `banned`, qwen3-tts/sampler.cpp:40-42).
 * ALLOW: a clear bit removes the token (extension: the complement of `banned`). */
typedef enum ssb_mask_kind { SSB_MASK_NONE = 0, SSB_MASK_BAN = 1, SSB_MASK_ALLOW = 2 } ssb_mask_kind;

/*
 * The family whose candidate rule a row follows. Every family takes the restricted logits (penalties,
 * then the mask) and draws with pick() (src/common/sampling.cpp:9-19).
 *   QWEN3_TTS  candidates()/sample(), src/families/qwen3-tts/sampler.cpp:69-111 (the default)
 *   HARU       haru::candidates(), src/families/haru/sampler.cpp:18-61: float32 softmax, a temperature of
 *              0 or less (or greedy) draws the first maximum, top_k 0 or >= vocab keeps every token,
 *              top-p gives 0 weight to the tokens past it; NaN or +inf -> SSB_ROW_NON_FINITE_INPUT
 *   DRAMA3     drama3::candidates(), src/families/drama3/sampler.cpp:30-60: temperature at least 1e-5,
 *              top_k at least 1, the softmax over every token, the token that passes top_p dropped; any
 *              non-finite stored logit -> SSB_ROW_NON_FINITE_INPUT; tokens the mask bans are no
 *              candidates (SSB_ROW_NO_FINITE_LOGIT when none is left)
 * HARU and DRAMA3 keep at most 8192 candidates: a larger effective top-k is refused (SSB_OUT_OF_RANGE;
 * SSB_ROW_INVALID_ROW for a row of row_params beyond max_top_k), every row of a call must have the
 * call's family (SSB_ROW_INVALID_ROW otherwise), and ssb_sample_rows_noalloc takes QWEN3_TTS only.
 */
typedef enum ssb_flavor { SSB_FLAVOR_QWEN3_TTS = 0, SSB_FLAVOR_HARU = 1, SSB_FLAVOR_DRAMA3 = 2 } ssb_flavor;

/*
 * Sampling settings of one row. The first five fields are the reference's SamplingParams
 * (src/families/qwen3-tts/sampler.h:12-24) with the same meaning and defaults
 * {greedy 0, temperature 1, top_k 0 (= every token), top_p 1, repetition_penalty 1}. The penalties
 * after them are extensions (0 = off): for each distinct in-range history id with c occurrences,
 * after the repetition penalty, l = l - frequency_penalty * c; l = l - presence_penalty (fp32).
 * Haru's and Drama 3's Sampling {temperature, top_k, top_p} (haru/sampler.h:13-19,
 * drama3/sampler.h:12-17) map onto the same fields with `flavor` set.
 */
typedef struct ssb_params {
    int32_t greedy;
    float temperature;
    int32_t top_k;
    float top_p;
    float repetition_penalty;
    float presence_penalty;
    float frequency_penalty;
    int32_t flavor; /* ssb_flavor (0: Qwen3-TTS) */
} ssb_params;

/*
 * One batch of independent rows; every pointer is DEVICE memory unless it says otherwise.
 * Row r's logits are logits + r*ld (dtype elements, ld >= vocab). Row r's mask words are
 * mask + r*mask_ld (bit (t & 31) of word t >> 5 is token t; mask_ld 0 shares one mask by all rows).
 * Row r's history is history + r*history_ld, of history_len[r] ids (or history_ld ids where
 * history_len is NULL); ids outside [0, vocab) are skipped, as the reference skips them
 * (qwen3-tts/sampler.cpp:35), so -1 padding is allowed.
 * u[r] is the number uniform() drew for row r (sampling.cpp:5-7); greedy rows never read it.
 * row_params (nullable) gives each row its own settings; the launch then needs max_top_k, the
 * largest effective top-k of any drawing row (0 = some row keeps every token); a row beyond it gets
 * SSB_ROW_INVALID_ROW. Without row_params, `params` applies to all rows and max_top_k is ignored.
 */
typedef struct ssb_rows {
    const void *logits;
    int64_t ld;
    int32_t dtype; /* ssb_dtype */
    int32_t rows;
    int32_t vocab;
    int32_t max_top_k;
    ssb_params params;
    const ssb_params *row_params;
    const int32_t *history;
    int64_t history_ld;
    const int32_t *history_len;
    const uint32_t *mask;
    int64_t mask_ld;
    int32_t mask_kind; /* ssb_mask_kind */
    int32_t reserved;  /* must be 0 */
    const double *u;
    int32_t *ids;    /* out: the sampled token, -1 where status != OK */
    int32_t *status; /* out: ssb_row_status */
} ssb_rows;

typedef struct ssb_context ssb_context;

/* Engine limits (also reported in messages). */
#define SSB_MAX_VOCAB 16777216      /* 2^24 tokens per row */
#define SSB_MAX_STREAM_HISTORY 8192 /* history_ld limit for rows of more than SSB_SMALL_VOCAB tokens */
#define SSB_SMALL_VOCAB 8192        /* rows up to this size are sampled whole from shared memory */

/* Library version, "major.minor.patch". */
SSB_API const char *ssb_version(void);

/* The message of the last failing call on this thread ("" after a success). */
SSB_API const char *ssb_last_error(void);

/* A context on CUDA device `device`: owns the split-row scratch and the host-call staging buffers.
 * One context per device and stream; calls on one context must not overlap in time. */
SSB_API ssb_status ssb_context_create(int32_t device, ssb_context **out);
SSB_API ssb_status ssb_context_destroy(ssb_context *ctx);

/* Allocates scratch for batches up to max_rows rows of max_vocab tokens, so that later calls of that
 * size allocate nothing (required before capturing them into a CUDA graph). */
SSB_API ssb_status ssb_context_reserve(ssb_context *ctx, int32_t max_rows, int32_t max_vocab);

/*
 * Samples every row of `rows` on `stream` (a cudaStream_t; NULL = the legacy default stream):
 * penalties -> mask -> temperature -> top-k -> softmax (double) -> top-p -> pick, or the first
 * maximum for greedy rows, exactly as the reference's sample() (qwen3-tts/sampler.cpp:103-111) with
 * ties broken by lowest token index. Asynchronous: ids/status are valid once the stream reaches them.
 */
SSB_API ssb_status ssb_sample_rows(ssb_context *ctx, const ssb_rows *rows, void *stream);

/*
 * The parity / debug export of candidates() (qwen3-tts/sampler.cpp:69-101): for each row, up to `cap`
 * kept tokens in candidate order with their weights (normalized by the sum over the top-k, before
 * the top-p cut, as the reference returns them) into tokens[row*cap ..], weights[row*cap ..], and
 * the full kept count into count[row]. `processed` (nullable, f32 [rows, vocab]) receives the
 * restricted logits: penalties and mask applied, before the temperature. Also writes ids/status.
 */
SSB_API ssb_status ssb_candidates_rows(ssb_context *ctx, const ssb_rows *rows, int32_t cap, int32_t *tokens,
                                       double *weights, int32_t *count, float *processed, void *stream);

/*
 * A device copy of a mask that many calls share (the talker's suppress mask of Generation::banned,
 * src/families/qwen3-tts/sampler.cpp:62-67, built once per min_frames state instead of per step):
 * copies `words` uint32 words (the ssb_rows.mask layout) from host memory, synchronously, into memory
 * the context owns, and returns its device address in *device_words, valid until the context is
 * destroyed. No counterpart in the reference, which builds a std::vector<bool> per call.
 */
SSB_API ssb_status ssb_context_mask(ssb_context *ctx, const uint32_t *host_words, int64_t words,
                                    const uint32_t **device_words);

/*
 * The restricted logits alone, the reference's restricted() (qwen3-tts/sampler.cpp:29-51) for a batch:
 * the repetition penalty (and the presence/frequency extension) over each row's distinct history ids,
 * then the mask (-inf where banned / not allowed), before the temperature, into out (f32, row r at
 * out + r * out_ld, out_ld >= vocab). Reads logits, ld, rows, vocab, dtype, params / row_params,
 * history* and mask*; ids, status and u are not used (may be null). History ids outside [0, vocab)
 * are ignored. history_ld is at most SSB_MAX_STREAM_HISTORY. Asynchronous on `stream`.
 */
SSB_API ssb_status ssb_restrict_rows(ssb_context *ctx, const ssb_rows *rows, float *out, int64_t out_ld, void *stream);

/*
 * sample() for HOST buffers, as the reference's call sites hold them (a logits readback, a history
 * vector, a ban list): copies the inputs to context-owned device buffers, samples, copies ids and
 * status back and waits for the stream. Pointers in `rows` are HOST pointers here.
 */
SSB_API ssb_status ssb_sample_host(ssb_context *ctx, const ssb_rows *rows, void *stream);

/*
 * ssb_sample_rows without a context and without any device allocation, for callers that cannot call
 * cudaMalloc (a runtime that owns all device memory through its own pool, or a process that must not
 * grow its footprint or synchronize the device on its decode path). No counterpart in the reference.
 * Pointers in `rows` are device pointers, as for ssb_sample_rows. The split-row scratch is a fixed
 * array of about 2.03 MiB inside the library, held by every GPU that loads it; the first call on each
 * device looks up its address, clears its per-row arrival counters once and waits for the device (make
 * it before any stream capture); every launch leaves the counters at 0 again. Takes QWEN3_TTS rows of
 * more than SSB_SMALL_VOCAB tokens, 16-byte aligned, with a top-k of at most 128 or greedy; anything
 * else is SSB_OUT_OF_RANGE. Calls share the array: calls that overlap on the GPU race and must not be
 * made.
 */
SSB_API ssb_status ssb_sample_rows_noalloc(const ssb_rows *rows, void *stream);

/* ---------------------------------------------------------------- device-resident chains */

/*
 * The embedding rows of the drawn ids (ggml_get_rows of the next step's table, as the code predictor's
 * chain feeds each pick to the next codebook: src/families/qwen3-tts/talker.cpp:58-64): after the rows
 * are sampled, out[r, 0:dim] = table[ids[r], 0:dim]; a row whose status is not SSB_ROW_OK (or whose id
 * is outside [0, table_rows)) gets zeros. Everything stays on the device and in stream order, so a
 * chain of steps can be captured into one CUDA graph with no readback between picks.
 */
typedef struct ssb_embed {
    const void *table;  /* [table_rows, ld] device */
    int64_t ld;         /* elements between table rows (>= dim) */
    int32_t table_rows;
    int32_t dtype;      /* ssb_dtype of table and out */
    int32_t dim;        /* elements per embedding row */
    int32_t reserved;   /* must be 0 */
    void *out;          /* [rows, out_ld] device */
    int64_t out_ld;     /* elements between out rows (>= dim) */
} ssb_embed;

/* ssb_sample_rows, then the embedding rows of the drawn ids (ids and status are written as usual). */
SSB_API ssb_status ssb_sample_embed_rows(ssb_context *ctx, const ssb_rows *rows, const ssb_embed *embed,
                                         void *stream);

/*
 * The LM head fused with the greedy pick (Qwen3Readback::Pick, src/common/qwen3-decoder.cpp:422-437, and
 * verify()'s argmax over [n, vocab], :492-510): ids[r] = the first maximum over tokens v of
 * hidden[r] . weight[v], with bf16 inputs and fp32 accumulation on the tensor cores; the logits are never
 * written. rows 1..256, dim a multiple of 64, hidden_ld and weight_ld multiples of 8 elements, both base
 * pointers 16-byte aligned. max_logit (the winning logit) and status are optional. Calls on one context
 * must not overlap on the GPU (they share the context's per-row maxima).
 */
typedef struct ssb_lm_head {
    const void *hidden;  /* [rows, hidden_ld] bf16 device */
    int64_t hidden_ld;
    int32_t rows;
    int32_t dim;
    const void *weight;  /* [vocab, weight_ld] bf16 device: one row per token */
    int64_t weight_ld;
    int32_t vocab;
    int32_t dtype;       /* SSB_BF16 */
    int32_t *ids;        /* [rows] */
    float *max_logit;    /* [rows] or null */
    int32_t *status;     /* [rows] or null: SSB_ROW_OK, or SSB_ROW_DEVICE_TIMEOUT */
} ssb_lm_head;

SSB_API ssb_status ssb_lm_head_argmax(ssb_context *ctx, const ssb_lm_head *head, void *stream);

/* ---------------------------------------------------------------- vocabulary-sharded rows */

/*
 * A row whose columns are split over several GPUs (a tensor-parallel LM head) is sampled from each
 * rank's best candidates instead of the whole row: step 1 on every rank (ssb_shard_select), one
 * all-gather of the records (ssb_shard_sample does it over NCCL, speech_sampler_b200_nccl.h), step 2 on
 * every rank (ssb_shard_merge), which writes the same ids and statuses on every rank as ssb_sample_rows
 * on the whole rows. A record holds k_cap composites per row plus one word (k_cap a power of two in
 * [1, 1024], at least every drawing row's effective top-k; greedy rows need 1); rows that keep more
 * (top_k 0 over a large vocabulary) come back SSB_ROW_INVALID_ROW.
 */
/* words (uint64) of one rank's records: rows * (k_cap + 1) */
SSB_API int64_t ssb_shard_record_words(int32_t rows, int32_t k_cap);

/* Step 1: `slice` holds columns [col_offset, col_offset + slice->vocab) of rows of vocab_total tokens
 * (col_offset a multiple of 32); its history holds the rows' GLOBAL token ids and its mask (if any) the
 * whole rows' mask words. Writes rows * (k_cap + 1) words to `records` (device). */
SSB_API ssb_status ssb_shard_select(ssb_context *ctx, const ssb_rows *slice, int32_t col_offset, int32_t vocab_total,
                                    int32_t k_cap, uint64_t *records, void *stream);

/* Step 2: `records` = the world ranks' records one after another ([world][rows][k_cap + 1], device);
 * rows' params / row_params, u, ids and status are used (its logits, history and mask are not). */
SSB_API ssb_status ssb_shard_merge(ssb_context *ctx, const ssb_rows *rows, int32_t vocab_total, int32_t world,
                                   int32_t k_cap, const uint64_t *records, void *stream);

/* The restricted logits (ssb_restrict_rows) of a slice [col_offset, col_offset + slice->vocab) of rows of
 * vocab_total tokens, taking the rows' GLOBAL history ids and whole-row mask words as ssb_shard_select does:
 * the first step of the restricted-slice exchange (every row of any top-k, top-k 0 included). */
SSB_API ssb_status ssb_restrict_slice(ssb_context *ctx, const ssb_rows *slice, int32_t col_offset, int32_t vocab_total,
                                      float *out, int64_t out_ld, void *stream);

/* ---------------------------------------------------------------- Haru's logit shaping and DRY */

/* DryConfig (haru/sampler.h:37-40, read by file_dry, haru/sampler.cpp:63-73). */
typedef struct ssb_dry_config {
    double multiplier;
    double base;
    double max_penalty;
    int32_t allowed_length;
    int32_t lookback;
    int32_t max_match_length;
    int32_t reserved; /* must be 0 */
} ssb_dry_config;

/* The DRY state of `streams` text streams on the device (haru::Dry, haru/sampler.h:49-69): each stream's
 * last lookback + max_match_length + 1 drawn tokens but the exempt ones, and its penalties. */
typedef struct ssb_dry ssb_dry;

#define SSB_DRY_MAX_WINDOW 8192 /* lookback + max_match_length + 1 limit */
#define SSB_DRY_MAX_EXEMPT 64

/* Creates the state of `streams` empty streams on the context's device; `exempt` (host, n_exempt ids)
 * are the tokens Dry(config, exempt) leaves out (haru/dialogue.cpp:128 passes PAD, EOP and EOS). */
SSB_API ssb_status ssb_dry_create(ssb_context *ctx, const ssb_dry_config *config, int32_t streams,
                                  const int32_t *exempt, int32_t n_exempt, ssb_dry **out);
SSB_API ssb_status ssb_dry_destroy(ssb_dry *dry);

/* Dry::update(token) (haru/sampler.cpp:86-110) for every stream: tokens[s] (device, [streams]) is
 * stream s's drawn token; a negative token leaves the stream as it is. Asynchronous on `stream`: the
 * tokens may be the ids an ssb_sample_rows call wrote just before on the same stream. */
SSB_API ssb_status ssb_dry_update(ssb_dry *dry, const int32_t *tokens, void *stream);

/* Dry::penalties() of stream `s` (by rising token), copied to host memory after the work queued on
 * `stream`: up to `cap` entries and the full count. */
SSB_API ssb_status ssb_dry_penalties(const ssb_dry *dry, int32_t s, int32_t *tokens, double *penalties, int32_t cap,
                                     int32_t *count, void *stream);

/* shape_logits() (haru/sampler.cpp:116-124) for rows of f32 logits on the device, in place: row r is
 * stream r of `dry` (or no DRY penalty when dry is null); each DRY penalty rounded to float is
 * subtracted from its token's logit, PAD's and EOP's logits are replaced by silent[r * silent_ld + 0]
 * and [+ 1] (plus eop_bias where it is not 0), and where must_speak[r] is nonzero PAD, EOP and EOS are
 * set to -inf. Rows then go to ssb_sample_rows with params.flavor = SSB_FLAVOR_HARU. */
typedef struct ssb_haru_shape {
    float *logits;             /* [rows, ld] f32, device, modified in place */
    int64_t ld;
    int32_t rows;              /* at most the DRY state's streams when dry is given */
    int32_t vocab;
    const float *silent;       /* [rows, silent_ld] device: PAD's and EOP's logits of the silent head */
    int64_t silent_ld;         /* >= 2 */
    int32_t pad, eop, eos;     /* haru::TextIds (haru/sampler.h:43-45), each in [0, vocab) */
    float eop_bias;
    const int32_t *must_speak; /* [rows] device, or null (no row must speak) */
} ssb_haru_shape;

SSB_API ssb_status ssb_haru_shape_rows(ssb_context *ctx, const ssb_haru_shape *shape, const ssb_dry *dry,
                                       void *stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* SPEECH_SAMPLER_B200_H */
