// Large-vocabulary rows (vocab > SSB_SMALL_VOCAB, e.g. Qwen3's 151936): the logits row is streamed
// once from HBM and reduced on the fly. This is the HBM-bound hot path.
//
// Work decomposition: `splits` CTAs per row, each owning `chunk` consecutive columns; with one split
// a CTA finishes its row alone, otherwise the last CTA to arrive (per-row counter) merges the partial
// results the others left in global scratch. No CTA ever waits on another.
//
// Staging: thread 0 streams the CTA's columns through a ring of kStages shared-memory stages of
// kStageBytes with TMA bulk copies (cp.async.bulk, completion counted on an mbarrier per stage); the
// block barrier that ends a stage frees its slot for the copy kStages ahead. Rows whose base or pitch
// is not 16-byte aligned take a plain-load path (one element per thread per iteration).
//
// Each stage is reduced in two phases per thread:
//   fast  — per 16-byte group: a NaN-propagating max (bf16x2 packed for bf16) folded into the row's
//           restricted maximum (qwen3-tts/sampler.cpp:43-49), and one compare against the running
//           threshold. Groups that pass, or that hold a masked or history token, are flagged.
//   slow  — only the flagged groups: widen, substitute -inf for masked tokens and the penalized value
//           for history tokens, then
//           mode 0 (all rows greedy): the first maximum, qwen3-tts/sampler.cpp:105-108;
//           mode 1 (top-k draws; greedy rows as the top-1 of unscaled logits): each element that can
//           reach the threshold is divided by the temperature exactly as the reference does
//           (qwen3-tts/sampler.cpp:73), keyed as a composite (value, then lowest index) and, when it
//           is not below the threshold composite, appended to a shared candidate buffer.
// The threshold starts as the k-th largest of the first stage's group maxima (k elements are at least
// that large, so no element below it can be among the k best) and rises whenever the buffer passes
// half full: two 8-bit digits of a radix select give the bucket that holds the k-th candidate, and
// everything below it leaves the buffer. Candidates that find the buffer full stay pending in their
// thread and are tested again, from the still-resident stage, after the raise. Comparison on
// composites is exact whatever the order in which elements arrive. At the end the candidates are cut
// to exactly the k best and sorted, and draw_row replays the reference's double-precision
// softmax, top-p cut and pick.
#include <climits>
#include <cuda_bf16.h>

#include "ssb_device.cuh"
#include "ssb_kernels.h"

namespace ssb {

namespace {

constexpr int kStageBytes = 16384;
constexpr int kStages = 3;
constexpr int kGroupsPerThread = kStageBytes / 16 / kStreamThreads;  // 16-byte groups per thread per stage
constexpr int kSeeds = kGroupsPerThread * kStreamThreads;            // group maxima of the first stage
constexpr uint32_t kWaitLimit = 1u << 22;                            // bounded mbarrier polls
constexpr int kWarpSortMax = 256;                                    // the final cut sorts this many in one warp

static_assert(kGroupsPerThread * kStreamThreads * 16 == kStageBytes, "stage must split evenly");

__device__ __forceinline__ uint32_t smem_addr(const void * p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// One arrival that also expects `bytes` of transaction (the bulk copy's completion).
__device__ __forceinline__ void mbar_expect(uint64_t * bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t * bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for phase `parity` of `bar`, giving up after kWaitLimit polls (returns false).
__device__ __forceinline__ bool mbar_wait(uint64_t * bar, uint32_t parity) {
    for (uint32_t n = 0; n < kWaitLimit; n++)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// Bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) from global to this CTA's
// shared memory, completing on `bar`. No multicast.
__device__ __forceinline__ void bulk_load(void * dst, const void * src, uint32_t bytes, uint64_t * bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

// NaN-propagating max of the elements of a 16-byte group.
template <typename TIn> __device__ __forceinline__ float group_max(const uint4 & r);
template <> __device__ __forceinline__ float group_max<uint16_t>(const uint4 & r) {
    const __nv_bfloat162 a = __hmax2_nan(*reinterpret_cast<const __nv_bfloat162 *>(&r.x),
                                         *reinterpret_cast<const __nv_bfloat162 *>(&r.y));
    const __nv_bfloat162 b = __hmax2_nan(*reinterpret_cast<const __nv_bfloat162 *>(&r.z),
                                         *reinterpret_cast<const __nv_bfloat162 *>(&r.w));
    const __nv_bfloat162 m = __hmax2_nan(a, b);
    const uint32_t w = *reinterpret_cast<const uint32_t *>(&m);
    return max_nan(bf16_lo(w), bf16_hi(w));
}
template <> __device__ __forceinline__ float group_max<float>(const uint4 & r) {
    return max_nan(max_nan(__uint_as_float(r.x), __uint_as_float(r.y)), max_nan(__uint_as_float(r.z), __uint_as_float(r.w)));
}

// Multiplicative hash of a token id into `bits` bits (Knuth's multiplicative method).
__device__ __forceinline__ uint32_t hash_token(int32_t t, int bits) { return ((uint32_t) t * 0x9E3779B1u) >> (32 - bits); }

// Per-CTA constants of the stream.
struct Ctx {
    int c0;
    int mask_kind;
    const uint32_t * mrow;
    bool penal;
    const uint32_t * hbits;
    const int32_t * hkey;
    const float * hval;
    int hbits_n;  // log2 of the hash table size
    float tscale;
    bool fast;
    bool scale;
    float * processed;
    uint64_t * buf;
    int * count;
    int cap;
    int high;
};

// Per-thread running state.
struct Run {
    float acc;        // restricted maximum, NaN-propagating
    int nan_scaled;   // a scaled logit was NaN
    uint64_t best;    // mode 0: composite of the first maximum
    float best_v;     // mode 0: its value
    uint64_t theta;   // mode 1: a candidate enters iff its composite >= theta
    float theta_lo;   // mode 1: raw logits below this cannot reach theta
    int over;         // mode 1: the buffer passed half full
};

__device__ __forceinline__ float history_value(const Ctx & c, int32_t t) {
    const uint32_t mask = (1u << c.hbits_n) - 1u;
    uint32_t h = hash_token(t, c.hbits_n);
    for (uint32_t n = 0; n <= mask && c.hkey[h] != t; n++) h = (h + 1) & mask;
    return c.hval[h];
}

// Mask and history bits of a group of G columns at col0 (col0 % G == 0).
template <int G>
__device__ __forceinline__ void special_bits(const Ctx & c, int col0, uint32_t vmask, uint32_t & mb, uint32_t & hb) {
    mb = 0, hb = 0;
    if (c.mrow) {
        const uint32_t w = __ldg(c.mrow + (col0 >> 5)) >> (col0 & 31);
        mb = (c.mask_kind == SSB_MASK_BAN ? w : ~w) & vmask;
    }
    if (c.penal) hb = (c.hbits[(col0 - c.c0) >> 5] >> ((col0 - c.c0) & 31)) & vmask;
}

// Appends composite `cv` to the candidate buffer; false when the buffer is full (the caller keeps it
// pending). Per-thread atomics: after the first stage only a few elements per stage get here.
__device__ __forceinline__ bool append(const Ctx & c, Run & r, uint64_t cv) {
    const int slot = atomicAdd(c.count, 1);
    if (slot + 1 > c.high) r.over = 1;
    if (slot < c.cap) {
        c.buf[slot] = cv;
        return true;
    }
    return false;
}

// The slow phase of one group: widen, substitute, and the per-element work of the mode. `only`
// restricts it to the elements of a retry (bits), with the row statistics already taken.
template <typename TIn, int G, int kMode, bool kDebug>
__device__ __forceinline__ uint32_t slow_group(const Ctx & c, Run & r, const uint4 & raw, int col0, uint32_t vmask,
                                               uint32_t only, bool first_pass) {
    float v[G];
    if (G == 1) {
        v[0] = __uint_as_float(raw.x);
    } else {
        Elem<TIn>::unpack(raw, v);
    }
    uint32_t mb, hb;
    special_bits<G>(c, col0, vmask, mb, hb);
    if (mb | hb) {
#pragma unroll
        for (int e = 0; e < G; e++) {
            if ((mb >> e) & 1u) v[e] = -kInf;
            else if ((hb >> e) & 1u) v[e] = history_value(c, col0 + e);
        }
    }
    if (first_pass) {
#pragma unroll
        for (int e = 0; e < G; e++) {
            if ((vmask >> e) & 1u) {
                r.acc = max_nan(r.acc, v[e]);
                if (kDebug && c.processed) c.processed[col0 + e] = v[e];
            }
        }
    }
    uint32_t dropped = 0;
#pragma unroll
    for (int e = 0; e < G; e++) {
        if (!((vmask >> e) & 1u) || !((only >> e) & 1u)) continue;
        if (kMode == 0) {
            const uint64_t cv = composite(v[e], (uint32_t) (col0 + e));
            if (v[e] == v[e] && cv > r.best) r.best = cv, r.best_v = v[e];
        } else if (v[e] >= r.theta_lo) {
            const float sc = c.scale ? __fdiv_rn(v[e], c.tscale) : v[e];
            r.nan_scaled |= sc != sc;
            const uint64_t cv = composite(sc, (uint32_t) (col0 + e));
            if (cv >= r.theta && !append(c, r, cv)) dropped |= 1u << e;
        }
    }
    return dropped;
}

// Shared state of the candidate buffer.
struct BufShared {
    int count;
    int nsel;
    uint64_t theta;
    float theta_lo;
};

// Keeps the buffer entries selected by st (key >= st.prefix) and returns how many; block-wide.
__device__ int keep_selected(uint64_t * buf, uint64_t * tmp, int n, const SelectState & st, BufShared & bs) {
    if (threadIdx.x == 0) bs.nsel = 0;
    __syncthreads();
    for (int base = 0; base < n; base += blockDim.x) {
        const int i = base + (int) threadIdx.x;
        const uint64_t cv = i < n ? buf[i] : 0;
        const bool take = i < n && selected(cv, st);
        const unsigned m = __ballot_sync(0xffffffffu, take);
        if (m) {
            const int leader = __ffs(m) - 1;
            int slot = 0;
            if (lane_id() == leader) slot = atomicAdd(&bs.nsel, __popc(m));
            slot = __shfl_sync(0xffffffffu, slot, leader);
            if (take) tmp[slot + __popc(m & ((1u << lane_id()) - 1u))] = cv;
        }
    }
    __syncthreads();
    const int kept = bs.nsel;
    for (int i = threadIdx.x; i < kept; i += blockDim.x) buf[i] = tmp[i];
    __syncthreads();
    return kept;
}

// Raises the threshold to the bucket (top 16 bits) of the k-th best buffered candidate and drops
// everything below it; if ties still leave the buffer over half full, cuts it to exactly the k best.
// Block-wide. Returns the number of candidates kept (>= min(k, n)).
__device__ int raise_threshold(uint64_t * buf, uint64_t * tmp, int k, int cap, int high, float tscale, bool fast,
                               BufShared & bs, SelectState & st) {
    const int n = bs.count < cap ? bs.count : cap;
    int kept = n;
    if (n > k) {
        radix_select(n, k, [&](int i) { return buf[i]; }, st, 2);
        kept = keep_selected(buf, tmp, n, st, bs);
        if (kept > high) {
            radix_select(kept, k, [&](int i) { return buf[i]; }, st, 8);
            kept = keep_selected(buf, tmp, kept, st, bs);
        }
        if (threadIdx.x == 0 && st.prefix > bs.theta) {
            bs.theta = st.prefix;
            bs.theta_lo = raw_bound(composite_value(st.prefix), tscale, fast);
        }
    }
    if (threadIdx.x == 0) bs.count = kept;
    __syncthreads();
    return kept;
}

// Cuts the buffer to exactly its min(k, n) best, sorted descending into sel; block-wide.
__device__ int final_cut(uint64_t * buf, uint64_t * tmp, uint64_t * sel, int k, int cap, float tscale, bool fast,
                         BufShared & bs, SelectState & st) {
    int n = bs.count < cap ? bs.count : cap;
    if (n > kWarpSortMax && n > k) {
        radix_select(n, k, [&](int i) { return buf[i]; }, st, 8);
        n = keep_selected(buf, tmp, n, st, bs);
    }
    const int kk = n < k ? n : k;
    if (n <= kWarpSortMax) {
        if (threadIdx.x < 32) {
            uint64_t x[kWarpSortMax / 32];
#pragma unroll
            for (int r = 0; r < kWarpSortMax / 32; r++) {
                const int i = r * 32 + (int) threadIdx.x;
                x[r] = i < n ? buf[i] : 0ull;
            }
            warp_sort_desc<kWarpSortMax / 32>(x);
#pragma unroll
            for (int r = 0; r < kWarpSortMax / 32; r++) {
                const int i = r * 32 + (int) threadIdx.x;
                if (i < kk) sel[i] = x[r];
            }
        }
        __syncthreads();
    } else {
        const int np2 = next_pow2(kk);
        for (int i = threadIdx.x; i < np2; i += blockDim.x) sel[i] = i < kk ? buf[i] : 0ull;
        __syncthreads();
        bitonic_sort_desc(sel, np2);
    }
    (void) tscale;
    (void) fast;
    return kk;
}

template <typename TIn, int kMode, bool kVec, bool kDebug>
__global__ void __launch_bounds__(kStreamThreads, 2) stream_rows_kernel(const StreamArgs sa) {
    const RowsArgs & a = sa.r;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ SelectState sel;
    __shared__ BufShared bs;
    __shared__ float s_redf[32];
    __shared__ uint64_t s_red64[32];
    __shared__ int s_redi[32];
    __shared__ int s_last, s_abort;
    __shared__ __align__(8) uint64_t s_full[kStages];

    const int splits = sa.splits;
    const int row = blockIdx.x / splits;
    const int split = blockIdx.x - row * splits;
    const int vocab = a.vocab;
    const ssb_params pp = a.row_params ? a.row_params[row] : a.params;
    const RowParams p = resolve_params(pp, vocab);
    const bool greedy_row = kMode == 0 || p.greedy;
    const int k = greedy_row ? 1 : p.k;
    if (kMode == 1 && a.row_params && !p.greedy && p.k > a.k_bound) {
        if (split == 0 && threadIdx.x == 0) {
            a.ids[row] = -1, a.status[row] = SSB_ROW_INVALID_ROW;
            if (kDebug && a.dbg_count) a.dbg_count[row] = 0;
        }
        return;
    }
    const int c0 = split * sa.chunk;
    const int c1 = min(vocab, c0 + sa.chunk);
    const int len = c1 - c0;

    // ---- shared memory: [ring] [history bitmap] [hash keys] [hash values] [buffer] [tmp] [selected]
    unsigned char * ring = smem;
    unsigned char * after_ring = smem + (kVec ? kStages * kStageBytes : 0);
    const int hw_alloc = (((sa.chunk + 31) >> 5) + 3) & ~3;  // bitmap words, padded to 16 bytes
    uint32_t * s_hbits = reinterpret_cast<uint32_t *>(after_ring);
    int32_t * s_hkey = reinterpret_cast<int32_t *>(s_hbits + hw_alloc);
    float * s_hval = reinterpret_cast<float *>(s_hkey + sa.hist_slots);
    uint64_t * s_buf = reinterpret_cast<uint64_t *>(s_hval + sa.hist_slots);  // hist_slots is even
    uint64_t * s_tmp = s_buf + sa.cap;
    uint64_t * s_sel = s_tmp + sa.cap;

    const TIn * src = reinterpret_cast<const TIn *>(a.logits) + (int64_t) row * a.ld;
    constexpr int G = kVec ? Elem<TIn>::kVec : 1;
    constexpr int kStageElems = kStageBytes / (int) sizeof(TIn);
    const int nvec = kVec ? len / G : 0;  // 16-byte groups of the chunk
    const int nstages = kVec ? (nvec * 16 + kStageBytes - 1) / kStageBytes : 0;
    const char * gsrc = reinterpret_cast<const char *>(src + c0);

    // ---- start the first stages' copies before anything else
    if (threadIdx.x == 0) {
        s_abort = 0;
        if (kVec) {
            for (int q = 0; q < kStages; q++) mbar_init(&s_full[q], 1);
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            for (int q = 0; q < kStages && q < nstages; q++) {
                const uint32_t bytes = (uint32_t) min(kStageBytes, nvec * 16 - q * kStageBytes);
                mbar_expect(&s_full[q], bytes);
                bulk_load(ring + q * kStageBytes, gsrc + (size_t) q * kStageBytes, bytes, &s_full[q]);
            }
        }
    }

    // ---- history: a hash table of the distinct in-range ids, their counts then penalized values
    const int32_t * hist = a.history ? a.history + (int64_t) row * a.history_ld : nullptr;
    int hlen = 0;
    if (hist) {
        hlen = a.history_len ? a.history_len[row] : (int) a.history_ld;
        hlen = hlen < 0 ? 0 : (hlen > (int) a.history_ld ? (int) a.history_ld : hlen);
    }
    const bool penal = p.history_applies && hlen > 0;
    const int hbits_n = sa.hist_slots > 1 ? 31 - __clz(sa.hist_slots) : 1;
    if (penal) {
        const int nw = (sa.chunk + 31) >> 5;
        for (int i = threadIdx.x; i < nw; i += blockDim.x) s_hbits[i] = 0;
        for (int i = threadIdx.x; i < sa.hist_slots; i += blockDim.x) s_hkey[i] = -1, s_hval[i] = 0.0f;
        __syncthreads();
        const uint32_t hmask = (uint32_t) sa.hist_slots - 1u;
        for (int i = threadIdx.x; i < hlen; i += blockDim.x) {
            const int32_t t = hist[i];
            if (t < c0 || t >= c1) continue;
            uint32_t h = hash_token(t, hbits_n);
            for (uint32_t n = 0; n <= hmask; n++) {
                const int32_t old = atomicCAS(&s_hkey[h], -1, t);
                if (old == -1 || old == t) {
                    atomicAdd(&s_hval[h], 1.0f);  // the count, exact in fp32 below 2^24
                    break;
                }
                h = (h + 1) & hmask;
            }
        }
        __syncthreads();
        for (int i = threadIdx.x; i < sa.hist_slots; i += blockDim.x) {
            const int32_t t = s_hkey[i];
            if (t >= 0) {
                s_hval[i] = penalize(Elem<TIn>::load1(src, t), (int) s_hval[i], p);
                atomicOr(&s_hbits[(t - c0) >> 5], 1u << ((t - c0) & 31));
            }
        }
    }
    if (kMode == 1 && threadIdx.x == 0) {
        bs.count = 0;
        bs.theta = 0;
        bs.theta_lo = -kInf;
    }
    __syncthreads();

    Ctx c;
    c.c0 = c0;
    c.mask_kind = a.mask_kind;
    c.mrow = (a.mask && a.mask_kind != SSB_MASK_NONE) ? a.mask + (int64_t) row * a.mask_ld : nullptr;
    c.penal = penal;
    c.hbits = s_hbits;
    c.hkey = s_hkey;
    c.hval = s_hval;
    c.hbits_n = hbits_n;
    c.scale = !greedy_row;
    c.tscale = greedy_row ? 1.0f : p.temperature;
    c.fast = greedy_row ? true : p.fast_scale;
    c.processed = (kDebug && a.dbg_processed) ? a.dbg_processed + (int64_t) row * vocab : nullptr;
    c.buf = s_buf;
    c.count = &bs.count;
    c.cap = sa.cap;
    c.high = sa.cap / 2;
    Run r;
    r.acc = -kInf;
    r.nan_scaled = 0;
    r.best = 0;
    r.best_v = -kInf;
    r.theta = 0;
    r.theta_lo = -kInf;
    r.over = 0;
    const bool special = c.mrow != nullptr || penal;

    // raises the threshold while a candidate is pending or the buffer passed half full; block-wide
    auto settle = [&](uint32_t & pending, auto && retry) {
        if (kMode != 1) return;
        while (__syncthreads_or(r.over || pending)) {
            raise_threshold(s_buf, s_tmp, k, c.cap, c.high, c.tscale, c.fast, bs, sel);
            r.over = 0;
            r.theta = bs.theta;
            r.theta_lo = bs.theta_lo;
            pending = retry(pending);
        }
    };

    if (kVec) {
        for (int st = 0; st < nstages; st++) {
            const int slot = st % kStages;
            const uint4 * stage = reinterpret_cast<const uint4 *>(ring + slot * kStageBytes);
            if (!mbar_wait(&s_full[slot], (uint32_t) (st / kStages) & 1u)) s_abort = 1;
            const int sbase = c0 + st * kStageElems;
            const int sgroups = min(kStageBytes, nvec * 16 - st * kStageBytes) / 16;
            // fast phase
            uint32_t flagged = 0;
            float gmax[kGroupsPerThread];
#pragma unroll
            for (int j = 0; j < kGroupsPerThread; j++) {
                const int g = j * kStreamThreads + (int) threadIdx.x;
                gmax[j] = -kInf;
                if (g >= sgroups) continue;
                bool flag = kDebug;
                if (special) {
                    uint32_t mb, hb;
                    special_bits<G>(c, sbase + g * G, (uint32_t) ((1ull << G) - 1), mb, hb);
                    flag |= (mb | hb) != 0;
                }
                if (!flag) {
                    const float gm = group_max<TIn>(stage[g]);
                    gmax[j] = gm;
                    r.acc = max_nan(r.acc, gm);
                    flag = kMode == 0 ? gm > r.best_v : gm >= r.theta_lo;
                }
                flagged |= (uint32_t) flag << j;
            }
            // first stage of a top-k row: the k-th largest group maximum is a lower bound of the k-th
            // largest element, so the threshold starts there (for a positive temperature, which keeps
            // the order of the logits)
            if (kMode == 1 && st == 0 && k <= kSeeds && c.fast) {  // x -> x/T must be increasing
                uint64_t * seeds = s_tmp;  // kSeeds <= cap entries
#pragma unroll
                for (int j = 0; j < kGroupsPerThread; j++) {
                    const float gm = gmax[j];
                    seeds[j * kStreamThreads + threadIdx.x] = (uint64_t) order_key(gm == gm ? gm : -kInf) << 32;
                }
                __syncthreads();
                radix_select(kSeeds, k, [&](int i) { return seeds[i]; }, sel, 2);
                const float s0raw = composite_value(sel.prefix);
                if (s0raw > -kInf) {
                    const float s0 = c.scale ? __fdiv_rn(s0raw, c.tscale) : s0raw;
                    r.theta = (uint64_t) order_key(s0) << 32;
                    r.theta_lo = raw_bound(s0, c.tscale, c.fast);
                    // groups flagged against the open threshold are re-tested against the seed
                    flagged = 0;
#pragma unroll
                    for (int j = 0; j < kGroupsPerThread; j++) {
                        const int g = j * kStreamThreads + (int) threadIdx.x;
                        if (g < sgroups) flagged |= (uint32_t) (kDebug || gmax[j] >= r.theta_lo || gmax[j] != gmax[j] ||
                                                                (special && gmax[j] == -kInf)) << j;
                    }
                }
                if (threadIdx.x == 0) {
                    bs.theta = r.theta;
                    bs.theta_lo = r.theta_lo;
                }
                __syncthreads();
            }
            // slow phase: only flagged groups
            uint32_t pending = 0;
            while (flagged) {
                const int j = __ffs(flagged) - 1;
                flagged &= flagged - 1;
                const int g = j * kStreamThreads + (int) threadIdx.x;
                pending |= slow_group<TIn, G, kMode, kDebug>(c, r, stage[g], sbase + g * G, (uint32_t) ((1ull << G) - 1),
                                                             ~0u, true) << (j * G);
            }
            settle(pending, [&](uint32_t pend) {
                uint32_t still = 0;
                while (pend) {
                    const int j = (__ffs(pend) - 1) / G;
                    const uint32_t pj = (pend >> (j * G)) & (uint32_t) ((1ull << G) - 1);
                    pend &= ~((uint32_t) ((1ull << G) - 1) << (j * G));
                    const int g = j * kStreamThreads + (int) threadIdx.x;
                    still |= slow_group<TIn, G, kMode, kDebug>(c, r, stage[g], sbase + g * G,
                                                               (uint32_t) ((1ull << G) - 1), pj, false) << (j * G);
                }
                return still;
            });
            __syncthreads();  // every thread is done with this stage: its slot may be refilled
            if (threadIdx.x == 0 && st + kStages < nstages) {
                const int nx = st + kStages;
                const uint32_t bytes = (uint32_t) min(kStageBytes, nvec * 16 - nx * kStageBytes);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_expect(&s_full[slot], bytes);
                bulk_load(ring + slot * kStageBytes, gsrc + (size_t) nx * kStageBytes, bytes, &s_full[slot]);
            }
        }
    }
    // columns past the last whole 16-byte group (all columns on the unaligned path): one per thread
    {
        const int cstart = c0 + nvec * G;
        const int iters = (c1 - cstart + kStreamThreads - 1) / kStreamThreads;
        for (int it = 0; it < iters; it++) {
            const int col = cstart + it * kStreamThreads + (int) threadIdx.x;
            const bool ok = col < c1;
            uint4 raw = make_uint4(ok ? __float_as_uint(Elem<TIn>::load1(src, col)) : 0u, 0u, 0u, 0u);
            uint32_t pending = ok ? slow_group<TIn, 1, kMode, kDebug>(c, r, raw, col, 1u, ~0u, true) : 0u;
            settle(pending, [&](uint32_t pend) {
                return pend ? slow_group<TIn, 1, kMode, kDebug>(c, r, raw, col, 1u, pend, false) : 0u;
            });
        }
    }

    // ---- this CTA's result
    __syncthreads();
    int kk = 1;
    if (kMode == 1) kk = final_cut(s_buf, s_tmp, s_sel, k, c.cap, c.tscale, c.fast, bs, sel);
    const float rmax = block_max_nan(r.acc, s_redf);
    const int nanf = block_or(r.nan_scaled, s_redi) | (s_abort ? 2 : 0);
    uint64_t best = 0;
    if (kMode == 0) best = block_max_u64(r.best, s_red64);

    float row_max = rmax;
    int row_flags = nanf;
    if (splits > 1) {
        const int64_t slot = (int64_t) row * splits + split;
        if (kMode == 0) {
            if (threadIdx.x == 0) sa.part_cand[slot * sa.r.k_bound] = best;
        } else {
            for (int i = threadIdx.x; i < kk; i += blockDim.x) sa.part_cand[slot * sa.r.k_bound + i] = s_sel[i];
        }
        if (threadIdx.x == 0) {
            sa.part_n[slot] = kk;
            sa.part_max[slot] = rmax;
            sa.part_flags[slot] = nanf;
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) s_last = atomicAdd(&sa.counters[row], 1u) == (unsigned) (splits - 1);
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        if (threadIdx.x == 0) sa.counters[row] = 0;  // ready for the next launch
        // ---- the last CTA of the row merges every split's result
        float m = -kInf;
        int f = 0;
        for (int q = threadIdx.x; q < splits; q += blockDim.x) {
            m = max_nan(m, __ldcg(sa.part_max + (int64_t) row * splits + q));
            f |= __ldcg(sa.part_flags + (int64_t) row * splits + q);
        }
        row_max = block_max_nan(m, s_redf);
        f = __reduce_or_sync(0xffffffffu, f);
        __syncthreads();
        if (lane_id() == 0) s_redi[warp_id()] = f;
        __syncthreads();
        row_flags = 0;
        for (int q = 0; q < (int) (blockDim.x >> 5); q++) row_flags |= s_redi[q];
        if (kMode == 0) {
            uint64_t b = 0;
            for (int q = threadIdx.x; q < splits; q += blockDim.x) {
                const uint64_t cv = __ldcg(reinterpret_cast<const unsigned long long *>(sa.part_cand) +
                                           ((int64_t) row * splits + q) * sa.r.k_bound);
                b = cv > b ? cv : b;
            }
            best = block_max_u64(b, s_red64);
        } else {
            // gather every split's candidates into the buffer, raising the threshold whenever it could overflow
            const int total_slots = splits * sa.r.k_bound;
            const int room = sa.cap - k;
            if (threadIdx.x == 0) bs.count = 0, bs.theta = 0, bs.theta_lo = -kInf;
            __syncthreads();
            for (int b0 = 0; b0 < total_slots; b0 += room) {
                const int nb = min(room, total_slots - b0);
                for (int i0 = 0; i0 < nb; i0 += blockDim.x) {  // warp-uniform trip count
                    const int ii = i0 + (int) threadIdx.x;
                    bool take = false;
                    uint64_t cv = 0;
                    if (ii < nb) {
                        const int i = b0 + ii;
                        const int q = i / sa.r.k_bound, j = i - q * sa.r.k_bound;
                        const int64_t sl = (int64_t) row * splits + q;
                        if (j < __ldcg(sa.part_n + sl)) {
                            take = true;
                            cv = __ldcg(reinterpret_cast<const unsigned long long *>(sa.part_cand) + sl * sa.r.k_bound + j);
                        }
                    }
                    const unsigned mm = __ballot_sync(0xffffffffu, take);
                    if (mm) {
                        const int leader = __ffs(mm) - 1;
                        int sl2 = 0;
                        if (lane_id() == leader) sl2 = atomicAdd(&bs.count, __popc(mm));
                        sl2 = __shfl_sync(0xffffffffu, sl2, leader);
                        const int at = sl2 + __popc(mm & ((1u << lane_id()) - 1u));
                        if (take && at < sa.cap) s_buf[at] = cv;
                    }
                }
                __syncthreads();
                if (b0 + nb < total_slots) {
                    // cut to exactly k so that `room` entries fit
                    const int n = bs.count < sa.cap ? bs.count : sa.cap;
                    if (n > k) {
                        radix_select(n, k, [&](int i) { return s_buf[i]; }, sel, 8);
                        const int kept = keep_selected(s_buf, s_tmp, n, sel, bs);
                        if (threadIdx.x == 0) bs.count = kept;
                        __syncthreads();
                    }
                }
            }
            kk = final_cut(s_buf, s_tmp, s_sel, k, sa.cap, c.tscale, c.fast, bs, sel);
        }
    }

    // ---- finalize the row (one CTA)
    int32_t * id_out = a.ids + row;
    int32_t * st_out = a.status + row;
    RowOut out{id_out, st_out, nullptr, nullptr, nullptr, 0};
    if (kDebug) {
        out.tokens = a.dbg_tokens ? a.dbg_tokens + (int64_t) row * a.dbg_cap : nullptr;
        out.weights = a.dbg_weights ? a.dbg_weights + (int64_t) row * a.dbg_cap : nullptr;
        out.count = a.dbg_count ? a.dbg_count + row : nullptr;
        out.cap = a.dbg_cap;
    }
    int stt = (row_flags & 2) ? SSB_ROW_DEVICE_TIMEOUT : restricted_status(row_max, p.rep);
    if (stt == SSB_ROW_OK && !greedy_row && (row_flags & 1)) stt = SSB_ROW_TEMPERATURE_OVERFLOW;
    if (stt != SSB_ROW_OK) {
        if (threadIdx.x == 0) {
            *id_out = -1, *st_out = stt;
            if (out.count) *out.count = 0;
        }
        return;
    }
    if (kMode == 0 || greedy_row) {
        if (kMode == 1) best = kk > 0 ? s_sel[0] : 0;  // sorted: the first is the best
        if (threadIdx.x == 0) {
            *id_out = (int32_t) composite_index(best), *st_out = SSB_ROW_OK;
            if (out.count) *out.count = 1;
            if (out.tokens && out.cap > 0) out.tokens[0] = *id_out, out.weights[0] = 1.0;
        }
        return;
    }
    const double u = a.u ? a.u[row] : 0.0;
    if (warp_id() == 0) draw_row(s_sel, kk, p, u, reinterpret_cast<double *>(s_buf), out);
}

template <typename TIn, int kMode, bool kVec, bool kDebug>
void * kernel_ptr() {
    return reinterpret_cast<void *>(stream_rows_kernel<TIn, kMode, kVec, kDebug>);
}

void * select_kernel(int mode, bool bf16, bool vec, bool debug) {
#define SSB_PICK(T, M)                                                                                  \
    return vec ? (debug ? kernel_ptr<T, M, true, true>() : kernel_ptr<T, M, true, false>())            \
               : (debug ? kernel_ptr<T, M, false, true>() : kernel_ptr<T, M, false, false>())
    if (bf16) {
        if (mode == 0) SSB_PICK(uint16_t, 0);
        SSB_PICK(uint16_t, 1);
    }
    if (mode == 0) SSB_PICK(float, 0);
    SSB_PICK(float, 1);
#undef SSB_PICK
}

}  // namespace

size_t stream_smem_bytes(int mode, bool vec, int chunk, int hist_slots, int cap, int sel_slots) {
    const size_t hwords = (size_t) ((((chunk + 31) >> 5) + 3) & ~3);
    size_t bytes = (vec ? (size_t) kStages * kStageBytes : 0) + hwords * 4 + (size_t) hist_slots * 8;
    if (mode == 1) bytes += (size_t) cap * 16 + (size_t) sel_slots * 8;
    return bytes;
}

int stream_blocks_per_sm(int mode, bool bf16, bool vec, size_t smem) {
    void * kern = select_kernel(mode, bf16, vec, false);
    if (ssb::set_max_dynamic_smem((const void *) kern, smem) != cudaSuccess) return 0;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kStreamThreads, smem) != cudaSuccess) return 0;
    return n;
}

cudaError_t launch_stream(const StreamArgs & a, int mode, bool bf16, bool vec, bool debug, cudaStream_t stream) {
    const size_t smem = stream_smem_bytes(mode, vec, a.chunk, a.hist_slots, a.cap, a.sel_slots);
    void * kern = select_kernel(mode, bf16, vec, debug);
    cudaError_t e = ssb::set_max_dynamic_smem((const void *) kern, smem);
    if (e != cudaSuccess) return e;
    void * args[] = {const_cast<StreamArgs *>(&a)};
    return cudaLaunchKernel(kern, dim3((unsigned) (a.r.rows * a.splits)), dim3(kStreamThreads), args, smem, stream);
}

}  // namespace ssb
