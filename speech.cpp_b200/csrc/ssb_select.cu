// Large-vocabulary rows with top-k <= 128 (every drawing configuration of the Qwen3 text decoders and
// the talker) and all-greedy batches: the HBM-bound hot path.
//
// One CTA streams `chunk` consecutive columns of one row (several CTAs per row when the batch is small;
// the last to finish merges their results, as in ssb_stream.cu). Warp-specialized:
//   producer warp  streams the chunk through a ring of kStages shared-memory stages with TMA bulk
//                  copies (cp.async.bulk + mbarrier complete_tx), refilling a slot as soon as all
//                  consumer warps have released it (an "empty" mbarrier per slot);
//   8 consumers    reduce each stage with no block-wide synchronization:
//     fast path, per 16-byte group: a NaN-propagating max (bf16x2 packed for bf16) folded into the
//       restricted maximum (qwen3-tts/sampler.cpp:43-49) and one compare against the CTA's threshold.
//       Groups holding a masked or history token, or reaching the threshold, are flagged.
//     slow path: the flagged groups of a warp form a work list that its lanes take one each: widen,
//       substitute -inf for masked tokens and the penalized value for history tokens, divide by the
//       temperature exactly as the reference does (qwen3-tts/sampler.cpp:73), and key each element as a
//       composite (value, then lowest index: the order of qwen3-tts/sampler.cpp:78-79 with
//       haru/sampler.cpp:39's tie-break).
//   greedy (KW = 0): the first maximum (qwen3-tts/sampler.cpp:105-108), kept as the CTA's largest
//     composite by a shared 64-bit atomic max; a group is flagged when its maximum reaches its value.
//   top-k (KW > 0): candidates (composites at or above the threshold) collect in a per-warp shared
//     buffer; a full buffer is sorted by a bitonic network in registers and merged, under a lock with a
//     bounded wait, into the CTA's shared queue of its best 32*KW composites. The threshold is the
//     queue's k-th entry (plus one): every composite below it has k better ones already, so filtering
//     on it is exact. The first stage seeds it with the k-th largest group maximum of each warp (k
//     elements are at least that large; for a positive temperature, which keeps the logits' order).
// Candidates are pre-tested on raw logits against raw_bound() so that the division runs only near the
// top. The queue is the CTA's exact top-k, and finalize_draw replays the reference's double-precision
// softmax, top-p cut and pick.
#include <climits>
#include <cuda_bf16.h>

#include "ssb_device.cuh"
#include "ssb_kernels.h"

namespace ssb {

namespace {

constexpr int kStageBytes = 16384;
constexpr int kStages = 3;
constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + the producer warp
constexpr int kGroupsPerThread = kStageBytes / 16 / kConsumers;
constexpr int kWarpBuf = 128;              // candidate buffer entries per consumer warp
constexpr int kDefer = 64;                 // deferred flagged groups per consumer warp
constexpr uint32_t kWaitLimit = 1u << 22;  // bounded mbarrier polls
constexpr uint32_t kLockLimit = 1u << 22;  // bounded lock attempts

static_assert(kGroupsPerThread * kConsumers * 16 == kStageBytes, "stage must split evenly");
static_assert(kGroupsPerThread == 4, "the work list enumerates four groups per lane");

__device__ __forceinline__ uint32_t smem_addr(const void * p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect(uint64_t * bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t * bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
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

__device__ __forceinline__ void bulk_load(void * dst, const void * src, uint32_t bytes, uint64_t * bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

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

// Element i (= r * 32 + lane) of a warp-distributed array, for a warp-uniform i.
template <int R>
__device__ __forceinline__ uint64_t warp_get(const uint64_t (&x)[R], int i) {
    uint64_t v = 0;
#pragma unroll
    for (int r = 0; r < R; r++)
        if (r == (i >> 5)) v = x[r];
    return __shfl_sync(0xffffffffu, v, i & 31);
}

// Merges the sorted (descending) 32*KW elements of `q` with the sorted 32*KW elements of `t`, keeping
// the best 32*KW sorted in q: max against t reversed gives a bitonic sequence holding the best half,
// which a bitonic clean-up sorts.
template <int KW>
__device__ __forceinline__ void warp_merge_sorted(uint64_t (&q)[KW], const uint64_t (&t)[KW]) {
    const int lane = lane_id();
#pragma unroll
    for (int r = 0; r < KW; r++) {
        const uint64_t o = __shfl_sync(0xffffffffu, t[KW - 1 - r], 31 - lane);
        q[r] = q[r] > o ? q[r] : o;
    }
#pragma unroll
    for (int j = 16 * KW; j > 0; j >>= 1) {
#pragma unroll
        for (int r = 0; r < KW; r++) {
            if (j >= 32) {
                const int rp = r ^ (j >> 5);
                if (rp > r) {
                    const uint64_t a = q[r], b = q[rp];
                    if (a < b) q[r] = b, q[rp] = a;
                }
            } else {
                const uint64_t o = shfl_xor(q[r], j);
                const bool keep_max = (lane & j) == 0;
                q[r] = keep_max ? (q[r] > o ? q[r] : o) : (q[r] < o ? q[r] : o);
            }
        }
    }
}

// Shared state of the CTA's selection.
struct Shared {
    uint64_t theta;     // a candidate enters iff its composite >= theta (top-k)
    uint64_t best;      // greedy: the largest composite seen
    uint32_t seed_key;  // greedy: order key of the largest group maximum seen in a warp's first stage
    int lock;
    int abort;
};

// Sorts a warp's candidate buffer and merges its best into the CTA queue `gq` under the lock; raises
// the threshold to the queue's k-th entry. Warp-wide; not inlined, so one copy of the networks exists.
template <int QN, int R>
__device__ __noinline__ void publish(const uint64_t * wbuf, int wn, uint64_t * gq, int k, Shared * sh) {
    const int lane = lane_id();
    uint64_t x[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
        const int i = r * 32 + lane;
        x[r] = i < wn ? wbuf[i] : 0ull;
    }
    warp_sort_desc<R>(x);
    uint64_t t[QN];
#pragma unroll
    for (int r = 0; r < QN; r++) t[r] = r < R ? x[r < R ? r : 0] : 0ull;
    int got = 0;
    if (lane == 0) {
        for (uint32_t n = 0; n < kLockLimit; n++) {
            if (atomicCAS(&sh->lock, 0, 1) == 0) {
                got = 1;
                break;
            }
        }
    }
    got = __shfl_sync(0xffffffffu, got, 0);
    if (!got) {
        if (lane == 0) sh->abort = 1;
        return;
    }
    __threadfence_block();
    uint64_t q[QN];
#pragma unroll
    for (int r = 0; r < QN; r++) q[r] = reinterpret_cast<volatile uint64_t *>(gq)[r * 32 + lane];
    warp_merge_sorted<QN>(q, t);
#pragma unroll
    for (int r = 0; r < QN; r++) reinterpret_cast<volatile uint64_t *>(gq)[r * 32 + lane] = q[r];
    const uint64_t kth = warp_get<QN>(q, k - 1);
    __threadfence_block();
    __syncwarp();
    if (lane == 0) {
        if (kth) atomicMax(reinterpret_cast<unsigned long long *>(&sh->theta), (unsigned long long) (kth + 1));
        atomicExch(&sh->lock, 0);
    }
    __syncwarp();
}

struct Ctx {
    int c0;
    int mask_kind;
    const uint32_t * mrow;
    bool penal;
    const uint32_t * hbits;
    const int32_t * hkey;
    const float * hval;
    int hbits_n;
    float tscale;
    bool fast;
    bool scale;
    float * processed;
};

__device__ __forceinline__ float history_value(const Ctx & c, int32_t t) {
    const uint32_t mask = (1u << c.hbits_n) - 1u;
    uint32_t h = hash_token(t, c.hbits_n);
    for (uint32_t n = 0; n <= mask && c.hkey[h] != t; n++) h = (h + 1) & mask;
    return c.hval[h];
}

template <int G>
__device__ __forceinline__ uint32_t special_bits(const Ctx & c, int col0) {
    uint32_t mb = 0, hb = 0;
    constexpr uint32_t full = (uint32_t) ((1ull << G) - 1);
    if (c.mrow) {
        const uint32_t w = __ldg(c.mrow + (col0 >> 5)) >> (col0 & 31);
        mb = (c.mask_kind == SSB_MASK_BAN ? w : ~w) & full;
    }
    if (c.penal) hb = (c.hbits[(col0 - c.c0) >> 5] >> ((col0 - c.c0) & 31)) & full;
    return mb | (hb << 16);
}

// The restricted logit of column `col` whose raw value is x.
__device__ __forceinline__ float restrict1(const Ctx & c, float x, int col, uint32_t sb, int e) {
    if ((sb >> e) & 1u) return -kInf;
    if ((sb >> (16 + e)) & 1u) return history_value(c, col);
    return x;
}

template <typename TIn, int KW, bool kDebug>
__global__ void __launch_bounds__(kThreads, 2) select_rows_kernel(const StreamArgs sa) {
    const RowsArgs & a = sa.r;
    constexpr int G = Elem<TIn>::kVec;
    constexpr int kStageElems = kStageBytes / (int) sizeof(TIn);
    constexpr int QN = KW > 0 ? KW : 1;  // registers per lane of the CTA queue
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t s_full[kStages];
    __shared__ __align__(8) uint64_t s_empty[kStages];
    __shared__ Shared sh;
    __shared__ float s_redf[32];
    __shared__ uint64_t s_red64[32];
    __shared__ int s_redi[32];
    __shared__ int s_last;

    const int warp = warp_id(), lane = lane_id();
    const bool producer = warp == kConsumerWarps;
    const int splits = sa.splits;
    const int row = blockIdx.x / splits;
    const int split = blockIdx.x - row * splits;
    const int vocab = a.vocab;
    const ssb_params pp = a.row_params ? a.row_params[row] : a.params;
    const RowParams p = resolve_params(pp, vocab);
    const bool greedy_row = KW == 0 || p.greedy;
    const int k = greedy_row ? 1 : p.k;
    if (KW > 0 && a.row_params && !p.greedy && p.k > a.k_bound) {
        if (split == 0 && threadIdx.x == 0) {
            a.ids[row] = -1, a.status[row] = SSB_ROW_INVALID_ROW;
            if (kDebug && a.dbg_count) a.dbg_count[row] = 0;
        }
        return;
    }
    const int c0 = split * sa.chunk;
    const int c1 = min(vocab, c0 + sa.chunk);
    const int len = c1 - c0;
    const int nvec = len / G;
    const int nstages = (nvec * 16 + kStageBytes - 1) / kStageBytes;

    // ---- shared memory: [ring] [history bitmap] [hash keys] [hash values] [warp buffers] [queue] [selected]
    unsigned char * ring = smem;
    const int hw_alloc = (((sa.chunk + 31) >> 5) + 3) & ~3;
    uint32_t * s_hbits = reinterpret_cast<uint32_t *>(smem + kStages * kStageBytes);
    int32_t * s_hkey = reinterpret_cast<int32_t *>(s_hbits + hw_alloc);
    float * s_hval = reinterpret_cast<float *>(s_hkey + sa.hist_slots);
    uint64_t * s_wbuf = reinterpret_cast<uint64_t *>(s_hval + sa.hist_slots);  // [kConsumerWarps][kWarpBuf]
    uint64_t * s_queue = s_wbuf + kConsumerWarps * kWarpBuf;                    // [32*QN]
    uint64_t * s_sel = s_queue + 32 * QN;                                      // [max(sel_slots, 32*QN)]
    uint4 * s_draw = reinterpret_cast<uint4 *>(s_sel + (sa.sel_slots > 32 * QN ? sa.sel_slots : 32 * QN));  // [8][kDefer]
    int * s_dcol = reinterpret_cast<int *>(s_draw + kConsumerWarps * kDefer);                               // [8][kDefer]

    const TIn * src = reinterpret_cast<const TIn *>(a.logits) + (int64_t) row * a.ld;
    const char * gsrc = reinterpret_cast<const char *>(src + c0);

    if (threadIdx.x == 0) {
        sh.theta = 0;
        sh.best = 0;
        sh.seed_key = 0;
        sh.lock = 0;
        sh.abort = 0;
        for (int q = 0; q < kStages; q++) mbar_init(&s_full[q], 1), mbar_init(&s_empty[q], kConsumerWarps);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int q = 0; q < kStages && q < nstages; q++) {
            const uint32_t bytes = (uint32_t) min(kStageBytes, nvec * 16 - q * kStageBytes);
            mbar_expect(&s_full[q], bytes);
            bulk_load(ring + q * kStageBytes, gsrc + (size_t) q * kStageBytes, bytes, &s_full[q]);
        }
    }
    if (KW > 0)
        for (int i = threadIdx.x; i < 32 * QN; i += blockDim.x) s_queue[i] = 0;

    // ---- history: hash table of the distinct in-range ids (duplicates combined per warp first)
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
        for (int base = 0; base < hlen; base += blockDim.x) {  // warp-uniform trip count
            const int i = base + (int) threadIdx.x;
            const int32_t t = i < hlen ? hist[i] : -1;
            const bool in = t >= c0 && t < c1;
            const unsigned m = __ballot_sync(0xffffffffu, in);
            if (in) {
                const unsigned peers = __match_any_sync(m, t);
                if (lane == __ffs(peers) - 1) {
                    uint32_t h = hash_token(t, hbits_n);
                    for (uint32_t n = 0; n <= hmask; n++) {
                        const int32_t old = atomicCAS(&s_hkey[h], -1, t);
                        if (old == -1 || old == t) {
                            atomicAdd(&s_hval[h], (float) __popc(peers));  // counts, exact below 2^24
                            break;
                        }
                        h = (h + 1) & hmask;
                    }
                }
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
    const bool special = c.mrow != nullptr || penal;

    float acc = -kInf;
    int nan_scaled = 0;
    uint64_t theta = 0;   // top-k: composites below it cannot be among the k best; greedy: the best so far
    float thr = -kInf;    // raw logits below thr cannot reach theta
    uint64_t * wbuf = s_wbuf + warp * kWarpBuf;
    int wn = 0;           // warp-uniform count of wbuf

    // refreshes theta/thr from the shared state
    auto refresh = [&]() {
        const uint64_t t = *reinterpret_cast<volatile uint64_t *>(KW > 0 ? &sh.theta : &sh.best);
        if (t > theta) {
            theta = t;
            const float b = KW > 0 ? raw_bound(composite_value(theta), c.tscale, c.fast) : composite_value(theta);
            thr = b > thr ? b : thr;
        }
        if (KW == 0) {
            const uint32_t sk = *reinterpret_cast<volatile uint32_t *>(&sh.seed_key);
            if (sk) {
                const float b = key_value(sk);
                thr = b > thr ? b : thr;
            }
        }
    };
    // merges the warp's buffered candidates into the CTA queue (sorting only as many as it holds)
    auto flush = [&]() {
        __syncwarp();
        if (wn <= 32) publish<QN, 1>(wbuf, wn, s_queue, k, &sh);
        else if (wn <= 64) publish<QN, 2>(wbuf, wn, s_queue, k, &sh);
        else publish<QN, 4>(wbuf, wn, s_queue, k, &sh);
        wn = 0;
        refresh();
    };
    // appends each lane's candidate `cv` (where `has`) to the warp buffer; flushes when it could overflow
    auto append = [&](bool has, uint64_t cv) {
        const unsigned m = __ballot_sync(0xffffffffu, has);
        if (!m) return;
        if (has) wbuf[wn + __popc(m & ((1u << lane) - 1u))] = cv;
        wn += __popc(m);
        if (wn > kWarpBuf - 32) flush();
    };
    // top-k: the per-element test of a candidate (restricted value v at column col), warp-uniform
    auto element = [&](bool valid, float v, int col) {
        bool has = false;
        uint64_t cv = 0;
        if (valid && v >= thr) {
            const float sc = c.scale ? __fdiv_rn(v, c.tscale) : v;
            nan_scaled |= sc != sc;
            cv = composite(sc, (uint32_t) col);
            has = cv >= theta;
        }
        append(has, cv);
    };
    // one flagged group per lane (has): widen, restrict, fold into the statistics, test its elements
    auto process_item = [&](bool has, const uint4 & raw, int col0) {
        float v[G];
        uint32_t sb = 0;
        if (has) {
            Elem<TIn>::unpack(raw, v);
            sb = special ? special_bits<G>(c, col0) : 0u;
        } else {
#pragma unroll
            for (int e = 0; e < G; e++) v[e] = -kInf;
        }
        uint64_t lbest = 0;
#pragma unroll
        for (int e = 0; e < G; e++) {
            if (has) {
                v[e] = restrict1(c, v[e], col0 + e, sb, e);
                acc = max_nan(acc, v[e]);
                if (kDebug && c.processed) c.processed[col0 + e] = v[e];
            }
            if (KW == 0) {
                if (has && v[e] == v[e] && v[e] >= thr) {
                    const uint64_t cv = composite(v[e], (uint32_t) (col0 + e));
                    lbest = cv > lbest ? cv : lbest;
                }
            } else {
                element(has, v[e], col0 + e);
            }
        }
        return lbest;
    };
    // greedy: folds each lane's best composite of an item into the CTA's best, once per warp
    auto greedy_fold = [&](uint64_t lbest) {
        const uint64_t m = warp_max_u64(lbest);
        if (m > theta) {
            if (lane == 0) atomicMax(reinterpret_cast<unsigned long long *>(&sh.best), (unsigned long long) m);
            theta = m;
            const float b = composite_value(m);
            thr = b > thr ? b : thr;
        }
    };

    // the deferred flagged groups of this warp, 32 per pass; then the candidates reach the CTA queue
    int dn = 0;  // warp-uniform count of deferred groups
    auto process_deferred = [&]() {
        __syncwarp();
        for (int base = 0; base < dn; base += 32) {  // warp-uniform
            const int item = base + lane;
            const bool has = item < dn;
            const uint4 raw = has ? s_draw[warp * kDefer + item] : make_uint4(0, 0, 0, 0);
            const int col0 = has ? s_dcol[warp * kDefer + item] : c0;
            process_item(has, raw, col0);
        }
        dn = 0;
        if (wn >= 32) flush();
        __syncwarp();
    };
    auto consumer_sync = [&]() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory"); };

    if (producer) {
        if (lane == 0) {
            for (int st = kStages; st < nstages; st++) {
                const int slot = st % kStages;
                if (!mbar_wait(&s_empty[slot], (uint32_t) ((st / kStages) - 1) & 1u)) sh.abort = 1;
                const uint32_t bytes = (uint32_t) min(kStageBytes, nvec * 16 - st * kStageBytes);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_expect(&s_full[slot], bytes);
                bulk_load(ring + slot * kStageBytes, gsrc + (size_t) st * kStageBytes, bytes, &s_full[slot]);
            }
        }
    } else {
        const int tid = (int) threadIdx.x;  // 0 .. kConsumers-1
        for (int st = 0; st < nstages; st++) {
            const int slot = st % kStages;
            const uint4 * stage = reinterpret_cast<const uint4 *>(ring + slot * kStageBytes);
            if (!mbar_wait(&s_full[slot], (uint32_t) (st / kStages) & 1u)) sh.abort = 1;
            refresh();
            const int sbase = c0 + st * kStageElems;
            const int sgroups = min(kStageBytes, nvec * 16 - st * kStageBytes) / 16;
            // fast path
            uint32_t flagged = 0;
            float gmax[kGroupsPerThread];
#pragma unroll
            for (int j = 0; j < kGroupsPerThread; j++) {
                const int g = j * kConsumers + tid;
                gmax[j] = -kInf;
                if (g >= sgroups) continue;
                bool flag = kDebug || (special && special_bits<G>(c, sbase + g * G) != 0);
                if (!flag) {
                    const float gm = group_max<TIn>(stage[g]);
                    gmax[j] = gm;
                    acc = max_nan(acc, gm);
                    flag = gm >= thr;
                }
                flagged |= (uint32_t) flag << j;
            }
            // greedy: the warp's largest group maximum of the first stage is a value the maximum reaches
            if (KW == 0 && st == 0) {
                float wm = -kInf;
#pragma unroll
                for (int j = 0; j < kGroupsPerThread; j++)
                    if (gmax[j] == gmax[j] && gmax[j] > wm) wm = gmax[j];
#pragma unroll
                for (int o = 16; o; o >>= 1) wm = fmaxf(wm, __shfl_xor_sync(0xffffffffu, wm, o));
                if (wm > thr) {
                    if (lane == 0) atomicMax(&sh.seed_key, order_key(wm));
                    thr = wm;
                    flagged = 0;
#pragma unroll
                    for (int j = 0; j < kGroupsPerThread; j++) {
                        const int g = j * kConsumers + tid;
                        if (g < sgroups)
                            flagged |= (uint32_t) (kDebug || gmax[j] >= thr || gmax[j] != gmax[j] ||
                                                   (special && special_bits<G>(c, sbase + g * G) != 0))
                                       << j;
                    }
                }
            }
            // top-k: the first stage seeds the CTA's threshold with the k-th largest of its group maxima
            // (k elements are at least that large; a positive temperature keeps the logits' order)
            if (KW > 0 && st == 0 && c.fast) {
                uint64_t seeds[kGroupsPerThread];
#pragma unroll
                for (int j = 0; j < kGroupsPerThread; j++)
                    seeds[j] = (uint64_t) order_key(gmax[j] == gmax[j] ? gmax[j] : -kInf) << 32;
                warp_sort_desc<kGroupsPerThread>(seeds);
#pragma unroll
                for (int r = 0; r < QN; r++) s_wbuf[warp * kWarpBuf + r * 32 + lane] = seeds[r];
                consumer_sync();
                if (warp == 0) {
                    uint64_t q[QN];
#pragma unroll
                    for (int r = 0; r < QN; r++) q[r] = s_wbuf[r * 32 + lane];
                    for (int w = 1; w < kConsumerWarps; w++) {
                        uint64_t t[QN];
#pragma unroll
                        for (int r = 0; r < QN; r++) t[r] = s_wbuf[w * kWarpBuf + r * 32 + lane];
                        warp_merge_sorted<QN>(q, t);
                    }
                    const float s0raw = composite_value(warp_get<QN>(q, k - 1));
                    if (lane == 0 && s0raw > -kInf) {
                        const float s0 = c.scale ? __fdiv_rn(s0raw, c.tscale) : s0raw;
                        atomicMax(reinterpret_cast<unsigned long long *>(&sh.theta), (unsigned long long) order_key(s0) << 32);
                    }
                }
                consumer_sync();
                refresh();
                flagged = 0;
#pragma unroll
                for (int j = 0; j < kGroupsPerThread; j++) {
                    const int g = j * kConsumers + tid;
                    if (g < sgroups)
                        flagged |= (uint32_t) (kDebug || gmax[j] >= thr || gmax[j] != gmax[j] ||
                                               (special && special_bits<G>(c, sbase + g * G) != 0))
                                   << j;
                }
            }
            // the warp's flagged groups
            unsigned bl[kGroupsPerThread];
            int total = 0;
#pragma unroll
            for (int j = 0; j < kGroupsPerThread; j++) bl[j] = __ballot_sync(0xffffffffu, (flagged >> j) & 1u), total += __popc(bl[j]);
            if (KW > 0 && total > 0 && dn + total > kDefer) process_deferred();
            if (KW > 0 && total > 0 && total <= kDefer) {
                // top-k: defer them (raw bytes and column) and take them 32 at a time
                int off = 0;
#pragma unroll
                for (int j = 0; j < kGroupsPerThread; j++) {
                    if ((flagged >> j) & 1u) {
                        const int pos = dn + off + __popc(bl[j] & ((1u << lane) - 1u));
                        const int g = j * kConsumers + tid;
                        s_draw[warp * kDefer + pos] = stage[g];
                        s_dcol[warp * kDefer + pos] = sbase + g * G;
                    }
                    off += __popc(bl[j]);
                }
                dn += total;
                if (dn >= 32) process_deferred();
            } else {
                // greedy, or a flood larger than the deferred list: the groups straight from the stage
                for (int base = 0; base < total; base += 32) {  // warp-uniform
                    const int item = base + lane;
                    const bool has = item < total;
                    int jj = 0, r = item;
                    const int n0 = __popc(bl[0]), n1 = __popc(bl[1]), n2 = __popc(bl[2]);
                    if (r >= n0) { r -= n0; jj = 1; if (r >= n1) { r -= n1; jj = 2; if (r >= n2) { r -= n2; jj = 3; } } }
                    const unsigned bj = jj == 0 ? bl[0] : (jj == 1 ? bl[1] : (jj == 2 ? bl[2] : bl[3]));
                    const int srcl = has ? (int) __fns(bj, 0, r + 1) : 0;
                    const int g = jj * kConsumers + warp * 32 + srcl;
                    const uint64_t lbest = process_item(has, has ? stage[g] : make_uint4(0, 0, 0, 0), sbase + g * G);
                    if (KW == 0) greedy_fold(lbest);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_empty[slot]);
        }
        if (KW > 0 && dn > 0) process_deferred();
        // columns past the last whole 16-byte group: one per lane
        for (int base = c0 + nvec * G; base < c1; base += kConsumers) {  // warp-uniform trip count
            const int col = base + tid;
            const bool ok = col < c1;
            float v = -kInf;
            if (ok) {
                v = Elem<TIn>::load1(src, col);
                if (special) v = restrict1(c, v, col, special_bits<1>(c, col), 0);
                acc = max_nan(acc, v);
                if (kDebug && c.processed) c.processed[col] = v;
            }
            refresh();
            if (KW == 0) greedy_fold(ok && v == v && v >= thr ? composite(v, (uint32_t) col) : 0ull);
            else element(ok, v, col);
        }
        if (KW > 0 && wn > 0) flush();
        if (KW == 0 && lane == 0)
            atomicMax(reinterpret_cast<unsigned long long *>(&sh.best), (unsigned long long) theta);
    }

    // ---- this CTA's result
    __syncthreads();
    const float rmax = block_max_nan(acc, s_redf);
    const int nanf = block_or(nan_scaled, s_redi) | (sh.abort ? 2 : 0);
    uint64_t best = sh.best;
    int kk = 1;
    if (KW > 0) {
        for (int i = threadIdx.x; i < 32 * QN; i += blockDim.x) s_sel[i] = s_queue[i];
        __syncthreads();
        int nz = 0;
        for (int i = 0; i < 32 * QN && s_sel[i] != 0; i++) nz++;
        kk = nz < k ? nz : k;
    }

    float row_max = rmax;
    int row_flags = nanf;
    if (splits > 1) {
        const int64_t slot = (int64_t) row * splits + split;
        if (KW == 0) {
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
        float m = -kInf;
        int f = 0;
        for (int q = threadIdx.x; q < splits; q += blockDim.x) {
            m = max_nan(m, __ldcg(sa.part_max + (int64_t) row * splits + q));
            f |= __ldcg(sa.part_flags + (int64_t) row * splits + q);
        }
        row_max = block_max_nan(m, s_redf);
        row_flags = block_or(f & 1, s_redi) | (block_or(f & 2, s_redi) ? 2 : 0);
        if (KW == 0) {
            uint64_t b = 0;
            for (int q = threadIdx.x; q < splits; q += blockDim.x) {
                const uint64_t cv = __ldcg(reinterpret_cast<const unsigned long long *>(sa.part_cand) +
                                           ((int64_t) row * splits + q) * sa.r.k_bound);
                b = cv > b ? cv : b;
            }
            best = block_max_u64(b, s_red64);
        } else {
            // each consumer warp merges the lists of splits w, w+8, ...; warp 0 merges the warps' results
            if (warp < kConsumerWarps) {
                uint64_t q[QN];
#pragma unroll
                for (int r = 0; r < QN; r++) q[r] = 0;
                for (int sp = warp; sp < splits; sp += kConsumerWarps) {
                    const int64_t sl = (int64_t) row * splits + sp;
                    const int n = __ldcg(sa.part_n + sl);
                    uint64_t t[QN];
#pragma unroll
                    for (int r = 0; r < QN; r++) {
                        const int i = r * 32 + lane;
                        t[r] = i < n ? __ldcg(reinterpret_cast<const unsigned long long *>(sa.part_cand) + sl * sa.r.k_bound + i)
                                     : 0ull;
                    }
                    warp_merge_sorted<QN>(q, t);
                }
#pragma unroll
                for (int r = 0; r < QN; r++) s_wbuf[warp * kWarpBuf + r * 32 + lane] = q[r];
            }
            __syncthreads();
            if (warp == 0) {
                uint64_t q[QN];
#pragma unroll
                for (int r = 0; r < QN; r++) q[r] = s_wbuf[r * 32 + lane];
                for (int w = 1; w < kConsumerWarps; w++) {
                    uint64_t t[QN];
#pragma unroll
                    for (int r = 0; r < QN; r++) t[r] = s_wbuf[w * kWarpBuf + r * 32 + lane];
                    warp_merge_sorted<QN>(q, t);
                }
#pragma unroll
                for (int r = 0; r < QN; r++) s_sel[r * 32 + lane] = q[r];
            }
            __syncthreads();
            int nz = 0;
            for (int i = 0; i < 32 * QN && s_sel[i] != 0; i++) nz++;
            kk = nz < k ? nz : k;
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
    if (greedy_row) {
        if (KW > 0) best = s_sel[0];
        if (threadIdx.x == 0) {
            *id_out = (int32_t) composite_index(best), *st_out = SSB_ROW_OK;
            if (out.count) *out.count = 1;
            if (out.tokens && out.cap > 0) out.tokens[0] = *id_out, out.weights[0] = 1.0;
        }
        return;
    }
    const double u = a.u ? a.u[row] : 0.0;
    finalize_draw(s_sel, kk, p, u, reinterpret_cast<double *>(s_wbuf), out);
}

template <typename TIn, int KW, bool kDebug>
void * kernel_ptr() {
    return reinterpret_cast<void *>(select_rows_kernel<TIn, KW, kDebug>);
}

void * pick_kernel(int kw, bool bf16, bool debug) {
#define SSB_KW(T)                                                                                       \
    switch (kw) {                                                                                      \
        case 0: return debug ? kernel_ptr<T, 0, true>() : kernel_ptr<T, 0, false>();                   \
        case 1: return debug ? kernel_ptr<T, 1, true>() : kernel_ptr<T, 1, false>();                   \
        case 2: return debug ? kernel_ptr<T, 2, true>() : kernel_ptr<T, 2, false>();                   \
        default: return debug ? kernel_ptr<T, 4, true>() : kernel_ptr<T, 4, false>();                  \
    }
    if (bf16) SSB_KW(uint16_t)
    SSB_KW(float)
#undef SSB_KW
}

}  // namespace

int select_kw(int k_bound, bool all_greedy) {
    if (all_greedy) return 0;
    return k_bound <= 32 ? 1 : (k_bound <= 64 ? 2 : 4);
}

size_t select_smem_bytes(int kw, int chunk, int hist_slots, int sel_slots) {
    const size_t hwords = (size_t) ((((chunk + 31) >> 5) + 3) & ~3);
    const int qn = kw > 0 ? kw : 1;
    return (size_t) kStages * kStageBytes + hwords * 4 + (size_t) hist_slots * 8 +
           (size_t) kConsumerWarps * kWarpBuf * 8 + (size_t) 32 * qn * 8 +
           (size_t) (sel_slots > 32 * qn ? sel_slots : 32 * qn) * 8 + (size_t) kConsumerWarps * kDefer * (16 + 4);
}

int select_blocks_per_sm(int kw, bool bf16, size_t smem) {
    void * kern = pick_kernel(kw, bf16, false);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem) != cudaSuccess) return 0;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kThreads, smem) != cudaSuccess) return 0;
    return n;
}

cudaError_t launch_select(const StreamArgs & a, int kw, bool bf16, bool debug, cudaStream_t stream) {
    const size_t smem = select_smem_bytes(kw, a.chunk, a.hist_slots, a.sel_slots);
    void * kern = pick_kernel(kw, bf16, debug);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (e != cudaSuccess) return e;
    void * args[] = {const_cast<StreamArgs *>(&a)};
    return cudaLaunchKernel(kern, dim3((unsigned) (a.r.rows * a.splits)), dim3(kThreads), args, smem, stream);
}

}  // namespace ssb
