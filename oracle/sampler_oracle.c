/*
 * TEST INFRASTRUCTURE ONLY — the checker, never the product. Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / reference legs may load this library (oracle/liboracle.so).
 *
 * A plain-C restatement of the reference's token sampler, with the extensions the B200 engine adds.
 * Each step cites the reference line it restates (paths relative to the speech.cpp source tree):
 *
 *   uniform(rng)        src/common/sampling.cpp:5-7          rng() * 2^-64 over std::mt19937_64
 *   pick(w, u)          src/common/sampling.cpp:9-19         cumulative share in double, "> u", else last
 *   restricted()        src/families/qwen3-tts/sampler.cpp:29-51
 *   candidates()        src/families/qwen3-tts/sampler.cpp:69-101
 *   sample(..., u)      src/families/qwen3-tts/sampler.cpp:103-111
 *   haru::candidates()  src/families/haru/sampler.cpp:18-61
 *
 * Where it departs from the reference (each one "parity unpinned by the reference"):
 *   - ties: the reference's candidates() sorts with logits[a] > logits[b] and no index tie-break
 *     (qwen3-tts/sampler.cpp:78-79, std::partial_sort is unstable); here equal scaled logits are
 *     ordered by lowest token index, the comparator of haru/sampler.cpp:39. Greedy is the first
 *     maximum, as std::max_element gives (qwen3-tts/sampler.cpp:107).
 *   - presence/frequency penalties (not in the reference): applied after the repetition penalty to
 *     each distinct in-range history id with c occurrences, in fp32 without contraction:
 *         l = l - frequency * (float)c;   l = l - presence;
 *     only when presence != 0 or frequency != 0 (either way the arithmetic is a no-op otherwise).
 *   - allow-mask (not in the reference): the complement of the ban list.
 *   - bf16 rows (not in the reference): widened exactly to fp32 before any arithmetic.
 *   - NaN: a NaN among the restricted logits (after penalties and mask) gives status 4
 *     (NON_FINITE_INPUT), as haru::candidates refuses NaN (haru/sampler.cpp:21-23); the reference's
 *     max_element / partial_sort give order-dependent results there. A NaN among the logits scaled
 *     by the temperature (only a degenerate temperature of 0, +-inf or NaN can make one) gives
 *     status 2 (TEMPERATURE_OVERFLOW).
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off; no fast-math).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { ORC_OK = 0, ORC_PENALTY_OVERFLOW = 1, ORC_TEMPERATURE_OVERFLOW = 2, ORC_NO_FINITE_LOGIT = 3,
       ORC_NON_FINITE_INPUT = 4, ORC_INVALID = 6 };
enum { ORC_F32 = 0, ORC_BF16 = 1 };
enum { ORC_MASK_NONE = 0, ORC_MASK_BAN = 1, ORC_MASK_ALLOW = 2 };

/* Same layout as ssb_params in include/speech_sampler_b200.h; the first five fields are the
 * reference's SamplingParams (src/families/qwen3-tts/sampler.h:12-24). */
typedef struct {
    int32_t greedy;
    float temperature;
    int32_t top_k;
    float top_p;
    float repetition_penalty;
    float presence_penalty;
    float frequency_penalty;
    int32_t reserved;
} oracle_params;

/* ---- MT19937-64 (Matsumoto & Nishimura, 2000), the engine behind std::mt19937_64 ---- */
typedef struct {
    uint64_t mt[312];
    int mti;
} oracle_mt64;

void oracle_mt64_seed(oracle_mt64 * g, uint64_t seed) {
    g->mt[0] = seed;
    for (int i = 1; i < 312; i++) g->mt[i] = 6364136223846793005ULL * (g->mt[i - 1] ^ (g->mt[i - 1] >> 62)) + (uint64_t) i;
    g->mti = 312;
}

uint64_t oracle_mt64_next(oracle_mt64 * g) {
    const uint64_t upper = 0xFFFFFFFF80000000ULL, lower = 0x7FFFFFFFULL, matrix = 0xB5026F5AA96619E9ULL;
    if (g->mti >= 312) {
        for (int i = 0; i < 312; i++) {
            const uint64_t x = (g->mt[i] & upper) | (g->mt[(i + 1) % 312] & lower);
            g->mt[i] = g->mt[(i + 156) % 312] ^ (x >> 1) ^ ((x & 1ULL) ? matrix : 0ULL);
        }
        g->mti = 0;
    }
    uint64_t x = g->mt[g->mti++];
    x ^= (x >> 29) & 0x5555555555555555ULL;
    x ^= (x << 17) & 0x71D67FFFEDA60000ULL;
    x ^= (x << 37) & 0xFFF7EEE000000000ULL;
    x ^= x >> 43;
    return x;
}

/* uniform(): sampling.cpp:5-7 — the 64-bit draw converted to double (round to nearest) times 2^-64. */
double oracle_uniform_next(oracle_mt64 * g) { return (double) oracle_mt64_next(g) * 0x1.0p-64; }

void oracle_uniform(uint64_t seed, int64_t n, double * out) {
    oracle_mt64 g;
    oracle_mt64_seed(&g, seed);
    for (int64_t i = 0; i < n; i++) out[i] = oracle_uniform_next(&g);
}

/* pick(): sampling.cpp:9-19. */
int32_t oracle_pick(const double * w, int32_t n, double u) {
    double sum = 0;
    for (int32_t i = 0; i < n; i++) sum += w[i];
    const int32_t last = n - 1;
    double cumulative = 0;
    for (int32_t i = 0; i < last; i++) {
        cumulative += w[i] / sum;
        if (cumulative > u) return i;
    }
    return last;
}

/* ---- ordering: (value desc, index asc) ---- */
typedef struct {
    float v;
    int32_t i;
} orc_entry;

/* 1 when a comes before b in the candidate order. */
static int orc_before(const orc_entry * a, const orc_entry * b) {
    return a->v > b->v || (a->v == b->v && a->i < b->i);
}

static int orc_cmp(const void * pa, const void * pb) {
    const orc_entry * a = (const orc_entry *) pa, * b = (const orc_entry *) pb;
    if (orc_before(a, b)) return -1;
    if (orc_before(b, a)) return 1;
    return 0;
}

/* min-heap on the candidate order (root = the entry that comes last) */
static void heap_down(orc_entry * h, int32_t n, int32_t i) {
    for (;;) {
        int32_t l = 2 * i + 1, r = l + 1, m = i;
        if (l < n && orc_before(&h[m], &h[l])) m = l;
        if (r < n && orc_before(&h[m], &h[r])) m = r;
        if (m == i) return;
        orc_entry t = h[i];
        h[i] = h[m];
        h[m] = t;
        i = m;
    }
}

/* The first k of v[0..n) in candidate order, written sorted to out[0..k). */
static void top_k_sorted(const float * v, int32_t n, int32_t k, orc_entry * out) {
    if (k >= n / 4) {
        for (int32_t i = 0; i < n; i++) out[i].v = v[i], out[i].i = i;
        qsort(out, (size_t) n, sizeof(orc_entry), orc_cmp);
        return;
    }
    for (int32_t i = 0; i < k; i++) out[i].v = v[i], out[i].i = i;
    for (int32_t i = k / 2 - 1; i >= 0; i--) heap_down(out, k, i);
    for (int32_t i = k; i < n; i++) {
        orc_entry e = {v[i], i};
        if (orc_before(&e, &out[0])) {
            out[0] = e;
            heap_down(out, k, 0);
        }
    }
    qsort(out, (size_t) k, sizeof(orc_entry), orc_cmp);
}

static float widen(const void * logits, int dtype, int64_t i) {
    if (dtype == ORC_BF16) {
        const uint32_t bits = (uint32_t) ((const uint16_t *) logits)[i] << 16;
        float f;
        memcpy(&f, &bits, 4);
        return f;
    }
    return ((const float *) logits)[i];
}

static int cmp_i32(const void * a, const void * b) {
    const int32_t x = *(const int32_t *) a, y = *(const int32_t *) b;
    return (x > y) - (x < y);
}

/*
 * restricted(): qwen3-tts/sampler.cpp:29-51, plus the extensions. Writes the restricted logits to r[n]
 * and returns a status; *top gets their maximum.
 */
static int restrict_row(const void * logits, int dtype, int32_t n, const oracle_params * p, const int32_t * history,
                        int32_t hlen, const uint32_t * mask, int mask_kind, float * r, float * top) {
    for (int32_t i = 0; i < n; i++) r[i] = widen(logits, dtype, i);
    const int ext = p->presence_penalty != 0.0f || p->frequency_penalty != 0.0f;
    if ((p->repetition_penalty != 1.0f || ext) && hlen > 0) {
        /* distinct in-range ids with their counts: sort a copy (the reference's `seen` bitmap, :33-39) */
        int32_t * h = (int32_t *) malloc(sizeof(int32_t) * (size_t) hlen);
        memcpy(h, history, sizeof(int32_t) * (size_t) hlen);
        qsort(h, (size_t) hlen, sizeof(int32_t), cmp_i32);
        for (int32_t a = 0; a < hlen;) {
            int32_t b = a;
            while (b < hlen && h[b] == h[a]) b++;
            const int32_t t = h[a];
            if (t >= 0 && t < n) {
                float l = r[t];
                if (p->repetition_penalty != 1.0f) l = l < 0 ? l * p->repetition_penalty : l / p->repetition_penalty;
                if (ext) {
                    l = l - p->frequency_penalty * (float) (b - a);
                    l = l - p->presence_penalty;
                }
                r[t] = l;
            }
            a = b;
        }
        free(h);
    }
    if (mask && mask_kind != ORC_MASK_NONE) {
        for (int32_t i = 0; i < n; i++) {
            const int bit = (int) ((mask[i >> 5] >> (i & 31)) & 1u);
            if ((mask_kind == ORC_MASK_BAN && bit) || (mask_kind == ORC_MASK_ALLOW && !bit)) r[i] = -INFINITY;
        }
    }
    for (int32_t i = 0; i < n; i++)
        if (isnan(r[i])) return ORC_NON_FINITE_INPUT;
    float m = r[0];
    for (int32_t i = 1; i < n; i++)
        if (m < r[i]) m = r[i]; /* std::max_element: the first of the largest */
    *top = m;
    if (m == INFINITY && p->repetition_penalty != 1.0f) return ORC_PENALTY_OVERFLOW;
    if (!isfinite(m)) return ORC_NO_FINITE_LOGIT;
    return ORC_OK;
}

/*
 * One row of sample() / candidates(). Outputs (each nullable):
 *   id         the token sample() returns (-1 on a status other than 0)
 *   processed  [n] the restricted logits (penalties and mask applied, before the temperature)
 *   tokens / weights / count: candidates() — up to `cap` entries, *count = the full number kept;
 *              for a greedy row: the single argmax with weight 1.
 *   keep_mass  the cumulative normalized weight at the top-p cut (1 without top-p), for tests that
 *              measure the distance of u from the nearest decision boundary.
 */
int oracle_sample_row(const void * logits, int dtype, int32_t n, const oracle_params * p, const int32_t * history,
                      int32_t hlen, const uint32_t * mask, int mask_kind, double u, int32_t * id, float * processed,
                      int32_t * tokens, double * weights, int32_t cap, int32_t * count) {
    if (id) *id = -1;
    if (count) *count = 0;
    if (n <= 0 || !p) return ORC_INVALID;
    float * r = (float *) malloc(sizeof(float) * (size_t) n);
    float top = 0;
    int st = restrict_row(logits, dtype, n, p, history, hlen, mask, mask_kind, r, &top);
    if (processed) memcpy(processed, r, sizeof(float) * (size_t) n);
    if (st != ORC_OK) {
        free(r);
        return st;
    }
    if (p->greedy) {
        int32_t best = 0;
        for (int32_t i = 1; i < n; i++)
            if (r[best] < r[i]) best = i;
        if (id) *id = best;
        if (count) *count = 1;
        if (tokens && cap > 0) tokens[0] = best;
        if (weights && cap > 0) weights[0] = 1.0;
        free(r);
        return ORC_OK;
    }
    /* candidates(): qwen3-tts/sampler.cpp:72-99 */
    for (int32_t i = 0; i < n; i++) {
        r[i] = r[i] / p->temperature;
        if (isnan(r[i])) {
            free(r);
            return ORC_TEMPERATURE_OVERFLOW;
        }
    }
    const int32_t k = p->top_k > 0 ? (p->top_k < n ? p->top_k : n) : n;
    orc_entry * e = (orc_entry *) malloc(sizeof(orc_entry) * (size_t) (k >= n / 4 ? n : k));
    top_k_sorted(r, n, k, e);
    const float max_logit = e[0].v;
    if (!isfinite(max_logit)) {
        free(e);
        free(r);
        return ORC_TEMPERATURE_OVERFLOW;
    }
    double * w = (double *) malloc(sizeof(double) * (size_t) k);
    double sum = 0;
    for (int32_t i = 0; i < k; i++) sum += w[i] = exp((double) e[i].v - max_logit);
    for (int32_t i = 0; i < k; i++) w[i] /= sum;
    int32_t keep = k;
    if (p->top_p < 1.0f) {
        double cumulative = 0;
        keep = 0;
        while (keep < k) {
            cumulative += w[keep++];
            if (cumulative >= p->top_p) break;
        }
    }
    if (count) *count = keep;
    for (int32_t i = 0; i < keep && i < cap; i++) {
        if (tokens) tokens[i] = e[i].i;
        if (weights) weights[i] = w[i];
    }
    if (id) *id = e[oracle_pick(w, keep, u)].i;
    free(w);
    free(e);
    free(r);
    return ORC_OK;
}

/* Many rows (row-major, leading dimensions in elements / words; mask_ld 0 shares one mask). */
void oracle_sample_rows(const void * logits, int dtype, int64_t rows, int32_t n, int64_t ld, const oracle_params * p,
                        int32_t params_per_row, const int32_t * history, int64_t hld, const int32_t * hlens,
                        const uint32_t * mask, int64_t mask_ld, int mask_kind, const double * u, int32_t * ids,
                        int32_t * status, float * processed) {
    const size_t es = dtype == ORC_BF16 ? 2 : 4;
    for (int64_t r = 0; r < rows; r++) {
        const oracle_params * pr = params_per_row ? p + r : p;
        const int32_t hl = history ? (hlens ? hlens[r] : (int32_t) hld) : 0;
        status[r] = oracle_sample_row((const char *) logits + (size_t) (r * ld) * es, dtype, n, pr,
                                      history ? history + r * hld : NULL, hl, mask ? mask + r * mask_ld : NULL,
                                      mask_kind, u ? u[r] : 0.0, &ids[r], processed ? processed + r * (int64_t) n : NULL,
                                      NULL, NULL, 0, NULL);
    }
}

/*
 * haru::candidates(): haru/sampler.cpp:18-61 — float32 softmax, lowest-index ties, top-p zeroing the
 * weights of tokens whose preceding cumulative share reaches top_p. Returns a status (4 for NaN/+inf,
 * 2 for a temperature overflow); writes up to cap entries and *count = k.
 */
int oracle_haru_candidates(const float * logits, int32_t n, float temperature, int32_t top_k, float top_p,
                           int32_t * tokens, double * weights, int32_t cap, int32_t * count) {
    *count = 0;
    for (int32_t i = 0; i < n; i++)
        if (isnan(logits[i]) || logits[i] == INFINITY) return ORC_NON_FINITE_INPUT;
    if (temperature <= 0.0f) {
        int32_t best = 0;
        for (int32_t i = 1; i < n; i++)
            if (logits[best] < logits[i]) best = i;
        *count = 1;
        if (cap > 0) tokens[0] = best, weights[0] = 1.0;
        return ORC_OK;
    }
    float * s = (float *) malloc(sizeof(float) * (size_t) n);
    for (int32_t i = 0; i < n; i++) {
        s[i] = logits[i] / temperature;
        if (isfinite(logits[i]) && !isfinite(s[i])) {
            free(s);
            return ORC_TEMPERATURE_OVERFLOW;
        }
    }
    const int32_t k = top_k > 0 && top_k < n ? top_k : n;
    orc_entry * e = (orc_entry *) malloc(sizeof(orc_entry) * (size_t) (k >= n / 4 ? n : k));
    top_k_sorted(s, n, k, e);
    float * q = (float *) malloc(sizeof(float) * (size_t) k);
    float sum = 0.0f;
    for (int32_t i = 0; i < k; i++) {
        q[i] = expf(e[i].v - e[0].v);
        sum += q[i];
    }
    for (int32_t i = 0; i < k; i++) q[i] /= sum;
    *count = k;
    float cumulative = 0.0f;
    for (int32_t i = 0; i < k; i++) {
        double wi = q[i];
        if (top_p > 0.0f && top_p < 1.0f) {
            cumulative += q[i];
            if (!(cumulative - q[i] < top_p)) wi = 0.0;
        }
        if (i < cap) tokens[i] = e[i].i, weights[i] = wi;
    }
    free(q);
    free(e);
    free(s);
    return ORC_OK;
}

/*
 * drama3::candidates(): drama3/sampler.cpp:30-60 — the logits divided by max(T, 1e-5) (:31-39, any
 * non-finite logit is the device's error), k = min(max(top_k, 1), n), the k best by falling scaled
 * logit with lowest-index ties (:40-45), the largest not finite -> temperature overflow (:46-47), the
 * double sum of exp(s - top) over every token in index order (:48-49), then the tokens in order while
 * the running share stays at most top_p, the first always (:50-58), each with weight exp(s - top).
 * Returns a status (4 non-finite input, 2 temperature overflow); writes up to cap entries and *count.
 */
int oracle_drama3_candidates(const float * logits, int32_t n, float temperature, int32_t top_k, float top_p,
                             int32_t * tokens, double * weights, int32_t cap, int32_t * count) {
    *count = 0;
    const float t = temperature > 1e-5f ? temperature : 1e-5f;
    float * s = (float *) malloc(sizeof(float) * (size_t) n);
    for (int32_t i = 0; i < n; i++) {
        if (!isfinite(logits[i])) {
            free(s);
            return ORC_NON_FINITE_INPUT;
        }
        s[i] = logits[i] / t;
    }
    const int32_t k = top_k < 1 ? 1 : (top_k < n ? top_k : n);
    orc_entry * e = (orc_entry *) malloc(sizeof(orc_entry) * (size_t) (k >= n / 4 ? n : k));
    top_k_sorted(s, n, k, e);
    const float top = e[0].v;
    if (!isfinite(top)) {
        free(e);
        free(s);
        return ORC_TEMPERATURE_OVERFLOW;
    }
    double sum = 0.0;
    for (int32_t i = 0; i < n; i++) sum += exp((double) s[i] - top);
    double cumulative = 0.0;
    int32_t kept = 0;
    for (int32_t r = 0; r < k; r++) {
        const double p = exp((double) e[r].v - top);
        cumulative += p / sum;
        if (r > 0 && cumulative > top_p) break;
        if (r < cap) tokens[r] = e[r].i, weights[r] = p;
        kept++;
    }
    *count = kept;
    free(e);
    free(s);
    return ORC_OK;
}

/*
 * haru::Dry (haru/sampler.cpp:82-114). The settings have ssb_dry_config's layout. oracle_dry_run feeds
 * `tokens` to Dry::update one after another and writes the penalties after each (by rising token, up to
 * cap per step: pen_tokens/pen_values [n_tokens, cap], counts [n_tokens]). An exempt token leaves the
 * state, penalties included, as it was (:87).
 */
typedef struct {
    double multiplier, base, max_penalty;
    int32_t allowed_length, lookback, max_match_length, reserved;
} orc_dry_config;

typedef struct {
    int32_t token, length;
} orc_match;

static int orc_match_cmp(const void * a, const void * b) {
    const orc_match * x = (const orc_match *) a, * y = (const orc_match *) b;
    if (x->token != y->token) return x->token < y->token ? -1 : 1;
    return (x->length > y->length) - (x->length < y->length);
}

static int orc_in(const int32_t * ids, int32_t n, int32_t t) {
    for (int32_t i = 0; i < n; i++)
        if (ids[i] == t) return 1;
    return 0;
}

void oracle_dry_run(const orc_dry_config * c, const int32_t * exempt, int32_t n_exempt, const int32_t * tokens,
                    int64_t n_tokens, int32_t * pen_tokens, double * pen_values, int32_t cap, int32_t * counts) {
    const int64_t size = (int64_t) c->lookback + c->max_match_length + 1;
    int32_t * h = (int32_t *) malloc(sizeof(int32_t) * (size_t) (size + 1));
    orc_match * m = (orc_match *) malloc(sizeof(orc_match) * (size_t) (size + 1));
    int32_t * pt = (int32_t *) malloc(sizeof(int32_t) * (size_t) (size + 1));
    double * pv = (double *) malloc(sizeof(double) * (size_t) (size + 1));
    int64_t hn = 0;
    int32_t np = 0;
    for (int64_t s = 0; s < n_tokens; s++) {
        const int32_t token = tokens[s];
        if (!orc_in(exempt, n_exempt, token)) {
            h[hn++] = token;
            if (hn > size) {
                memmove(h, h + (hn - size), sizeof(int32_t) * (size_t) size);
                hn = size;
            }
            np = 0;
            const int32_t need = c->allowed_length > 1 ? c->allowed_length : 1;
            if (hn >= need) {
                int32_t nm = 0;
                const int32_t last = h[hn - 1];
                const int64_t jlo = hn - 1 - c->lookback > 0 ? hn - 1 - c->lookback : 0;
                for (int64_t j = hn - 2; j >= jlo; j--) {
                    if (h[j] != last) continue;
                    int32_t length = 1;
                    while (length < c->max_match_length && j - length >= 0 && h[j - length] == h[hn - 1 - length]) length++;
                    if (length >= c->allowed_length) m[nm].token = h[j + 1], m[nm].length = length, nm++;
                }
                qsort(m, (size_t) nm, sizeof(orc_match), orc_match_cmp);
                for (int32_t i = 0; i < nm; i++) {
                    if (i + 1 < nm && m[i + 1].token == m[i].token) continue;  /* the longest is last */
                    if (orc_in(exempt, n_exempt, m[i].token)) continue;
                    const double pen = c->multiplier * pow(c->base, (double) (m[i].length - c->allowed_length));
                    pt[np] = m[i].token;
                    pv[np] = pen < c->max_penalty ? pen : c->max_penalty;  /* std::min(max_penalty, pen) */
                    np++;
                }
            }
        }
        counts[s] = np;
        for (int32_t i = 0; i < np && i < cap; i++) {
            pen_tokens[s * cap + i] = pt[i];
            pen_values[s * cap + i] = pv[i];
        }
    }
    free(pv);
    free(pt);
    free(m);
    free(h);
}

/*
 * shape_logits() (haru/sampler.cpp:116-124) on one f32 row in place: each penalty rounded to float
 * subtracted from its token's logit, PAD's and EOP's logits replaced by silent[0] and silent[1], the EOP
 * bias added where it is not 0, and PAD, EOP and EOS to -inf where the row must speak.
 */
void oracle_haru_shape(float * logits, const int32_t * pen_tokens, const double * pen_values, int32_t n_pen,
                       const float * silent, int32_t pad, int32_t eop, int32_t eos, float eop_bias, int32_t must_speak) {
    for (int32_t i = 0; i < n_pen; i++) logits[pen_tokens[i]] -= (float) pen_values[i];
    logits[pad] = silent[0];
    logits[eop] = silent[1];
    if (eop_bias != 0.0f) logits[eop] += eop_bias;
    if (must_speak) logits[pad] = logits[eop] = logits[eos] = -INFINITY;
}
