// Large-vocabulary all-greedy batches (the Qwen3 text decoders' greedy steps, qwen3-decoder.cpp:422-437,
// 492-510, and the host argmax of qwen3-asr/decoder.cpp:108-113): the first maximum of the restricted
// logits (qwen3-tts/sampler.cpp:105-108), HBM-bound.
//
// One CTA streams `chunk` consecutive columns of one row (several CTAs per row when the batch is small;
// the last to finish merges their results, as in ssb_stream.cu). Warp-specialized: a producer warp
// brings the chunk through a ring of kStages shared-memory stages with TMA bulk copies (cp.async.bulk +
// mbarrier complete_tx), refilling a slot as soon as every consumer warp has copied its part into
// registers. Each of 256 consumer lanes takes four 16-byte groups per stage:
//   fast path: one NaN-propagating max over the lane's groups (packed bf16x2 for bf16), folded into the
//     restricted maximum (qwen3-tts/sampler.cpp:43-49) and compared against the CTA's best value so
//     far (a shared 64-bit composite atomic max). Groups that hold a masked or history token ("special"
//     groups, marked in a per-group bitmap built before the stream) never take the fast path.
//   slow path, for lanes whose maximum reaches the best and for special groups: widen, substitute
//     -inf for masked tokens and the penalized logit for history tokens, and key each element as a
//     composite (value, then lowest index) folded into the CTA's best.
// The first stage seeds the threshold with the warps' largest lane maxima.
#include <climits>
#include <cuda_bf16.h>

#include "ssb_device.cuh"
#include "ssb_kernels.h"
#include "ssb_tma.cuh"

namespace ssb {

namespace {

constexpr int kStages = 3;
constexpr int kGroupWordsPerStage = kConsumerWarps * kGroupsPerThread;  // special-group bitmap words per stage
constexpr int kThreads = kStreamCtaThreads;

// Shared state of the CTA's selection.
struct Shared {
    uint64_t best;      // the largest composite seen
    uint32_t seed_key;  // order key of the largest lane maximum of a warp's first stage
    int abort;
};

// Word of the special-group bitmap that holds group `gi` of the chunk (bit gi & 31): the four words of
// one consumer warp in one stage are adjacent, so a warp reads them with one 16-byte load.
__device__ __forceinline__ int group_word(int gi) {
    const int st = gi / kStageGroups, within = gi - st * kStageGroups;
    const int j = within / kConsumers, w = (within - j * kConsumers) >> 5;
    return st * kGroupWordsPerStage + w * kGroupsPerThread + j;
}

struct Ctx {
    int c0;
    int mask_kind;
    const uint32_t * mrow;
    bool penal;
    const uint32_t * hbits;
    const int32_t * hkey;
    const int32_t * hcnt;
    int hbits_n;
    float tscale;
    bool fast;
    bool scale;
    float * processed;
};

// Occurrences of history token t in the row (t is in the table).
__device__ __forceinline__ int history_count(const Ctx & c, int32_t t) {
    const uint32_t mask = (1u << c.hbits_n) - 1u;
    uint32_t h = hash_token(t, c.hbits_n);
    for (uint32_t n = 0; n <= mask && c.hkey[h] != t; n++) h = (h + 1) & mask;
    return c.hcnt[h];
}

// Masked (bits 0..G-1) and history (bits 16..16+G-1) columns among col0 .. col0+G-1.
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

// The restricted logit of column `col` whose raw value is x: -inf where masked, the penalized logit
// (qwen3-tts/sampler.cpp:36-38, then presence/frequency) for a history token, else x.
__device__ __forceinline__ float restrict1(const Ctx & c, const RowParams & p, float x, int col, uint32_t sb, int e) {
    if ((sb >> e) & 1u) return -kInf;
    if ((sb >> (16 + e)) & 1u) return penalize(x, history_count(c, col), p);
    return x;
}

template <typename TIn, bool kDebug>
__global__ void __launch_bounds__(kThreads, 2) select_rows_kernel(const StreamArgs sa) {
    const RowsArgs & a = sa.r;
    constexpr int G = Elem<TIn>::kVec;
    constexpr int kStageElems = kStageBytes / (int) sizeof(TIn);
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
    const int c0 = split * sa.chunk;
    const int c1 = min(vocab, c0 + sa.chunk);
    const int len = c1 - c0;
    const int nvec = len / G;  // whole 16-byte groups; the rest are tail columns
    const int nstages = (nvec + kStageGroups - 1) / kStageGroups;

    // ---- shared memory: [ring] [history bitmap] [special-group bitmap] [hash keys] [hash counts]
    unsigned char * ring = smem;
    const int hw_alloc = (((sa.chunk + 31) >> 5) + 3) & ~3;
    const int gw_alloc = ((sa.chunk * (int) sizeof(TIn) + kStageBytes - 1) / kStageBytes) * kGroupWordsPerStage;
    uint32_t * s_hbits = reinterpret_cast<uint32_t *>(smem + kStages * kStageBytes);
    uint32_t * s_gbits = s_hbits + hw_alloc;
    int32_t * s_hkey = reinterpret_cast<int32_t *>(s_gbits + gw_alloc);
    int32_t * s_hcnt = s_hkey + sa.hist_slots;

    const TIn * src = reinterpret_cast<const TIn *>(a.logits) + (int64_t) row * a.ld;
    const char * gsrc = reinterpret_cast<const char *>(src + c0);

    if (threadIdx.x == 0) {
        sh.best = 0;
        sh.seed_key = 0;
        sh.abort = 0;
        for (int q = 0; q < kStages; q++) mbar_init(&s_full[q], 1), mbar_init(&s_empty[q], kConsumerWarps);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int q = 0; q < kStages && q < nstages; q++) {
            const uint32_t bytes = (uint32_t) min(kStageBytes, (nvec - q * kStageGroups) * 16);
            mbar_expect(&s_full[q], bytes);
            bulk_load(ring + q * kStageBytes, gsrc + (size_t) q * kStageBytes, bytes, &s_full[q]);
        }
    }

    // ---- special groups: history tokens (hash table of distinct ids with their counts, per-column
    //      bitmap) and masked tokens, marked per 16-byte group for the fast path
    const int32_t * hist = a.history ? a.history + (int64_t) row * a.history_ld : nullptr;
    int hlen = 0;
    if (hist) {
        hlen = a.history_len ? a.history_len[row] : (int) a.history_ld;
        hlen = hlen < 0 ? 0 : (hlen > (int) a.history_ld ? (int) a.history_ld : hlen);
    }
    const bool penal = p.history_applies && hlen > 0;
    const uint32_t * mrow = (a.mask && a.mask_kind != SSB_MASK_NONE) ? a.mask + (int64_t) row * a.mask_ld : nullptr;
    const bool special = mrow != nullptr || penal;
    const int hbits_n = sa.hist_slots > 1 ? 31 - __clz(sa.hist_slots) : 1;
    if (special) {
        for (int i = threadIdx.x; i < nstages * kGroupWordsPerStage; i += blockDim.x) s_gbits[i] = 0;
        if (penal) {
            const int nw = (sa.chunk + 31) >> 5;
            for (int i = threadIdx.x; i < nw; i += blockDim.x) s_hbits[i] = 0;
            for (int i = threadIdx.x; i < sa.hist_slots; i += blockDim.x) s_hkey[i] = -1, s_hcnt[i] = 0;
        }
        __syncthreads();
        if (penal) {
            const uint32_t hmask = (uint32_t) sa.hist_slots - 1u;
            for (int base = 0; base < hlen; base += 4 * kThreads) {  // warp-uniform trip count
                int32_t t[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {  // four independent loads in flight
                    const int i = base + q * kThreads + (int) threadIdx.x;
                    t[q] = i < hlen ? __ldg(hist + i) : -1;
                }
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const bool in = t[q] >= c0 && t[q] < c1;
                    const unsigned m = __ballot_sync(0xffffffffu, in);
                    if (in) {
                        const unsigned peers = __match_any_sync(m, t[q]);  // duplicates within the warp
                        if (lane == __ffs(peers) - 1) {
                            uint32_t h = hash_token(t[q], hbits_n);
                            for (uint32_t n = 0; n <= hmask; n++) {
                                const int32_t old = atomicCAS(&s_hkey[h], -1, t[q]);
                                if (old == -1 || old == t[q]) {
                                    atomicAdd(&s_hcnt[h], __popc(peers));
                                    break;
                                }
                                h = (h + 1) & hmask;
                            }
                            const int rel = t[q] - c0;
                            atomicOr(&s_hbits[rel >> 5], 1u << (rel & 31));
                            const int gi = rel / G;
                            if (gi < nvec) atomicOr(&s_gbits[group_word(gi)], 1u << (gi & 31));
                        }
                    }
                }
            }
        }
        if (mrow) {
            // one mask word covers 32/G whole groups (c0 is a multiple of 32)
            constexpr int kGroupsPerWord = 32 / G;
            constexpr uint32_t gfull = (1u << G) - 1u;
            const int w0 = c0 >> 5, nw = (len + 31) >> 5;
            for (int base = 0; base < nw; base += 4 * kThreads) {
                uint32_t mw[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int i = base + q * kThreads + (int) threadIdx.x;
                    mw[q] = i < nw ? __ldg(mrow + w0 + i) : 0u;
                }
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int i = base + q * kThreads + (int) threadIdx.x;
                    const int gi0 = i * kGroupsPerWord;
                    if (i < nw && gi0 < nvec) {
                        uint32_t sb = 0;
#pragma unroll
                        for (int gg = 0; gg < kGroupsPerWord; gg++) {
                            const uint32_t bits = (mw[q] >> (gg * G)) & gfull;
                            sb |= (uint32_t) (a.mask_kind == SSB_MASK_BAN ? bits != 0u : bits != gfull) << gg;
                        }
                        if (gi0 + kGroupsPerWord > nvec) sb &= (1u << (nvec - gi0)) - 1u;
                        if (sb) atomicOr(&s_gbits[group_word(gi0)], sb << (gi0 & 31));
                    }
                }
            }
        }
    }
    __syncthreads();

    Ctx c;
    c.c0 = c0;
    c.mask_kind = a.mask_kind;
    c.mrow = mrow;
    c.penal = penal;
    c.hbits = s_hbits;
    c.hkey = s_hkey;
    c.hcnt = s_hcnt;
    c.hbits_n = hbits_n;
    c.processed = (kDebug && a.dbg_processed) ? a.dbg_processed + (int64_t) row * vocab : nullptr;

    float acc = -kInf;
    uint64_t theta = 0;  // the best composite so far
    float thr = -kInf;   // raw logits below thr cannot reach theta

    // raises theta/thr to the shared state
    auto refresh = [&]() {
        const uint64_t t = *reinterpret_cast<volatile uint64_t *>(&sh.best);
        if (t > theta) {
            theta = t;
            const float b = composite_value(theta);
            thr = b > thr ? b : thr;
        }
        const uint32_t sk = *reinterpret_cast<volatile uint32_t *>(&sh.seed_key);
        if (sk) {
            const float b = key_value(sk);
            thr = b > thr ? b : thr;
        }
    };
    // one flagged group per lane (has): widen, restrict, fold into the statistics; the lane's best
    auto process_item = [&](bool has, const uint4 & raw, int col0) {
        float v[G];
        uint32_t sb = 0;
        if (has) {
            Elem<TIn>::unpack(raw, v);
            sb = special ? special_bits<G>(c, col0) : 0u;
        }
        uint64_t lbest = 0;
#pragma unroll
        for (int e = 0; e < G; e++) {
            if (has) {
                if (special) v[e] = restrict1(c, p, v[e], col0 + e, sb, e);
                acc = max_nan(acc, v[e]);
                if (kDebug && c.processed) c.processed[col0 + e] = v[e];
                if (v[e] == v[e] && v[e] >= thr) {
                    const uint64_t cv = composite(v[e], (uint32_t) (col0 + e));
                    lbest = cv > lbest ? cv : lbest;
                }
            }
        }
        return lbest;
    };
    // folds each lane's best composite of an item into the CTA's best, once per warp
    auto greedy_fold = [&](uint64_t lbest) {
        const uint64_t m = warp_max_u64(lbest);
        if (m > theta) {
            if (lane == 0) atomicMax(reinterpret_cast<unsigned long long *>(&sh.best), (unsigned long long) m);
            theta = m;
            const float b = composite_value(m);
            thr = b > thr ? b : thr;
        }
    };

    if (producer) {
        if (lane == 0) {
            for (int st = kStages; st < nstages; st++) {
                const int slot = st % kStages;
                if (!mbar_wait(&s_empty[slot], (uint32_t) ((st / kStages) - 1) & 1u)) sh.abort = 1;
                const uint32_t bytes = (uint32_t) min(kStageBytes, (nvec - st * kStageGroups) * 16);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_expect(&s_full[slot], bytes);
                bulk_load(ring + slot * kStageBytes, gsrc + (size_t) st * kStageBytes, bytes, &s_full[slot]);
            }
        }
    } else {
        const int tid = (int) threadIdx.x;  // 0 .. kConsumers-1
        const uint4 * gb4 = reinterpret_cast<const uint4 *>(s_gbits);
        int slot = 0;
        uint32_t phase = 0;
        for (int st = 0; st < nstages; st++) {
            const uint4 * stage = reinterpret_cast<const uint4 *>(ring + slot * kStageBytes);
            if (!mbar_wait(&s_full[slot], phase)) sh.abort = 1;
            const int sgroups = min(kStageGroups, nvec - st * kStageGroups);
            uint4 rv[kGroupsPerThread];
            uint32_t live = 0;
#pragma unroll
            for (int j = 0; j < kGroupsPerThread; j++) {
                const int g = j * kConsumers + tid;
                if (g < sgroups) {
                    rv[j] = stage[g];
                    live |= 1u << j;
                } else {
                    rv[j] = neg_inf_group<TIn>();
                }
            }
            uint32_t sp = 0;
            if (special) {
                const uint4 gw = gb4[st * kConsumerWarps + warp];
                sp = (((gw.x >> lane) & 1u) | (((gw.y >> lane) & 1u) << 1) | (((gw.z >> lane) & 1u) << 2) |
                      (((gw.w >> lane) & 1u) << 3)) & live;
            }
            // the lane's part of the stage is in registers: release the slot to the producer
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_empty[slot]);
            if (++slot == kStages) slot = 0, phase ^= 1u;
            refresh();
            const int sbase = c0 + st * kStageElems;
            const uint32_t plain = live & ~sp;  // groups whose raw values are their restricted values
            float lm;
            if (plain == 0xFu) {
                lm = lane_max<TIn>(rv);
            } else {
                lm = -kInf;
#pragma unroll
                for (int j = 0; j < kGroupsPerThread; j++)
                    if ((plain >> j) & 1u) lm = max_nan(lm, group_max<TIn>(rv[j]));
            }
            acc = max_nan(acc, lm);
            if (st == 0) {
                // the warp's largest lane maximum is a value the row's maximum reaches
                float wm = lm == lm ? lm : -kInf;
#pragma unroll
                for (int o = 16; o; o >>= 1) wm = fmaxf(wm, __shfl_xor_sync(0xffffffffu, wm, o));
                if (wm > thr) {
                    if (lane == 0) atomicMax(&sh.seed_key, order_key(wm));
                    thr = wm;
                }
            }
            const bool hit = kDebug ? live != 0u : (sp != 0u || lm >= thr);
            if (__any_sync(0xffffffffu, hit)) {
                uint32_t fl = 0;
                if (hit) {
                    if (kDebug) {
                        fl = live;
                    } else {
                        fl = sp;
                        if (lm >= thr) {
#pragma unroll
                            for (int j = 0; j < kGroupsPerThread; j++)
                                if (((plain >> j) & 1u) && group_max<TIn>(rv[j]) >= thr) fl |= 1u << j;
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < kGroupsPerThread; j++)
                    if (__any_sync(0xffffffffu, (fl >> j) & 1u))
                        greedy_fold(process_item((fl >> j) & 1u, rv[j], sbase + (j * kConsumers + tid) * G));
            }
        }
        // columns past the last whole 16-byte group: one per lane
        for (int base = c0 + nvec * G; base < c1; base += kConsumers) {  // warp-uniform trip count
            const int col = base + tid;
            const bool ok = col < c1;
            float v = -kInf;
            if (ok) {
                v = Elem<TIn>::load1(src, col);
                if (special) v = restrict1(c, p, v, col, special_bits<1>(c, col), 0);
                acc = max_nan(acc, v);
                if (kDebug && c.processed) c.processed[col] = v;
            }
            refresh();
            greedy_fold(ok && v == v && v >= thr ? composite(v, (uint32_t) col) : 0ull);
        }
        if (lane == 0) atomicMax(reinterpret_cast<unsigned long long *>(&sh.best), (unsigned long long) theta);
    }

    // ---- this CTA's result
    __syncthreads();
    const float rmax = block_max_nan(acc, s_redf);
    const int nanf = sh.abort ? 2 : 0;
    uint64_t best = sh.best;

    float row_max = rmax;
    int row_flags = nanf;
    if (splits > 1) {
        const int64_t slot = (int64_t) row * splits + split;
        if (threadIdx.x == 0) {
            sa.part_cand[slot * sa.r.k_bound] = best;
            sa.part_n[slot] = 1;
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
        uint64_t b = 0;
        for (int q = threadIdx.x; q < splits; q += blockDim.x) {
            m = max_nan(m, __ldcg(sa.part_max + (int64_t) row * splits + q));
            f |= __ldcg(sa.part_flags + (int64_t) row * splits + q);
            const uint64_t cv = __ldcg(reinterpret_cast<const unsigned long long *>(sa.part_cand) +
                                       ((int64_t) row * splits + q) * sa.r.k_bound);
            b = cv > b ? cv : b;
        }
        row_max = block_max_nan(m, s_redf);
        row_flags = block_or(f & 2, s_redi) ? 2 : 0;
        best = block_max_u64(b, s_red64);
    }

    // ---- finalize the row (one CTA)
    int32_t * id_out = a.ids + row;
    int32_t * st_out = a.status + row;
    const int stt = (row_flags & 2) ? SSB_ROW_DEVICE_TIMEOUT : restricted_status(row_max, p.rep);
    if (threadIdx.x == 0) {
        const int32_t id = stt == SSB_ROW_OK ? (int32_t) composite_index(best) : -1;
        *id_out = id, *st_out = stt;
        if (kDebug) {
            if (a.dbg_count) a.dbg_count[row] = stt == SSB_ROW_OK ? 1 : 0;
            if (stt == SSB_ROW_OK && a.dbg_tokens && a.dbg_cap > 0) {
                a.dbg_tokens[(int64_t) row * a.dbg_cap] = id;
                a.dbg_weights[(int64_t) row * a.dbg_cap] = 1.0;
            }
        }
    }
}

template <typename TIn, bool kDebug>
void * kernel_ptr() {
    return reinterpret_cast<void *>(select_rows_kernel<TIn, kDebug>);
}

void * pick_kernel(bool bf16, bool debug) {
    if (bf16) return debug ? kernel_ptr<uint16_t, true>() : kernel_ptr<uint16_t, false>();
    return debug ? kernel_ptr<float, true>() : kernel_ptr<float, false>();
}

}  // namespace

int select_kw(int k_bound, bool all_greedy) {
    if (all_greedy) return 0;
    return k_bound <= 32 ? 1 : (k_bound <= 64 ? 2 : 4);
}

int select_max_chunk(int kw, bool bf16) { return kw > 0 ? topk_max_chunk(bf16) : 262144; }

size_t select_smem_bytes(int kw, bool bf16, int chunk, int hist_slots, int sel_slots) {
    if (kw > 0) return topk_smem_bytes(kw, bf16, chunk, hist_slots, sel_slots);
    const size_t hwords = (size_t) ((((chunk + 31) >> 5) + 3) & ~3);
    const int64_t chunk_bytes = (int64_t) chunk * (bf16 ? 2 : 4);
    const size_t gwords = (size_t) ((chunk_bytes + kStageBytes - 1) / kStageBytes) * kGroupWordsPerStage;
    return (size_t) kStages * kStageBytes + hwords * 4 + gwords * 4 + (size_t) hist_slots * 8;
}

int select_blocks_per_sm(int kw, bool bf16, size_t smem) {
    if (kw > 0) return topk_blocks_per_sm(kw, bf16, smem);
    void * kern = pick_kernel(bf16, false);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem) != cudaSuccess) return 0;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kThreads, smem) != cudaSuccess) return 0;
    return n;
}

cudaError_t launch_select(const StreamArgs & a, int kw, bool bf16, bool debug, cudaStream_t stream) {
    if (kw > 0) return launch_topk(a, kw, bf16, debug, stream);
    const size_t smem = select_smem_bytes(0, bf16, a.chunk, a.hist_slots, a.sel_slots);
    void * kern = pick_kernel(bf16, debug);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (e != cudaSuccess) return e;
    void * args[] = {const_cast<StreamArgs *>(&a)};
    return cudaLaunchKernel(kern, dim3((unsigned) (a.r.rows * a.splits)), dim3(kThreads), args, smem, stream);
}

}  // namespace ssb
