// Large-vocabulary rows with top-k <= 128 (every drawing configuration of the Qwen3 text decoders and
// the talker): the HBM-bound hot path of a drawing step.
//
// One CTA streams `chunk` consecutive columns of one row (several CTAs per row when the batch is small;
// the last to finish merges their lists, as in ssb_stream.cu). Two passes:
//
// Pass 1, the stream (warp-specialized). A producer warp brings the chunk through a ring of kStages
// 16 KB shared-memory stages with TMA bulk copies (cp.async.bulk + mbarrier complete_tx) and refills a
// slot as soon as every consumer warp has copied its part into registers. Each of 256 consumer lanes
// takes four 16-byte groups per stage (a "block" of 32 bf16 or 16 fp32 logits) and only
//   * stores the block's NaN-propagating maximum, rounded up to bf16 (an upper bound of every logit
//     in it), and
//   * keeps its own two largest block maxima among blocks without a masked or history token ("plain"
//     blocks: their raw logits are their restricted logits, qwen3-tts/sampler.cpp:29-51).
// No thresholds, no data-dependent branches: the stream runs at the rate the ring is filled.
//
// End phase (block-wide, short loops).
//   E1  bound: radix select (two 8-bit digits) of the k-th largest of the lanes' kept maxima. They are
//       restricted logits of distinct tokens, so k tokens reach the selected prefix s_b, and for a
//       positive temperature (which keeps the order) k scaled logits reach c = fl(s_b / T) — so the k
//       best all have a scaled logit >= c.
//   E2  history tokens (their penalized and masked logits were computed by the producer warp during the
//       stream, from the logits the stream had just brought into L2): candidates if they reach c.
//   E3  pass 2: the blocks whose maximum can reach c are read again (from L2) and every element that is
//       not a history token is restricted (-inf where masked), divided by the temperature exactly as
//       the reference does (qwen3-tts/sampler.cpp:73) and keyed as a composite (value, then lowest
//       index: the order of qwen3-tts/sampler.cpp:78-79 with haru/sampler.cpp:39's tie-break).
//       Composites >= the threshold go to a candidate array (the ring's memory); an array that could
//       overflow is cut to its k best by a radix select, which also raises the threshold.
//   E4  columns past the last whole 16-byte group.
//   E5  the candidates are sorted (bitonic, or radix-selected to k first), and finalize_draw replays
//       the reference's double-precision softmax, top-p cut and pick.
// The restricted maximum (for the row statuses, qwen3-tts/sampler.cpp:43-49) is exact: the largest
// restricted logit lies in a block whose maximum reaches c, or is a history token.
// Temperatures that do not keep the order (<= 0 or NaN) make every block a pass-2 block.
#include <climits>
#include <cuda_bf16.h>

#include "ssb_device.cuh"
#include "ssb_kernels.h"
#include "ssb_tma.cuh"

namespace ssb {

namespace {

constexpr int kTkStages = 4;
constexpr int kCap = kTkStages * kStageBytes / 8;  // candidate composites the ring's memory holds
constexpr int kHistChunk = 8;                      // history slots per thread between overflow checks
constexpr int kRoom = 2304;                        // most candidates one E2 chunk or E3 round adds
static_assert(kRoom >= kStreamCtaThreads * kHistChunk && kRoom >= kConsumerWarps * 32 * 8, "room for one round");

// bf16 bits of the smallest bf16 >= x (NaN stays NaN): block maxima kept in 16 bits as upper bounds.
__device__ __forceinline__ uint16_t bf16_up(float x) {
    if (x != x) return 0x7FC0u;
    const uint32_t b = __float_as_uint(x);
    uint32_t hi = b >> 16;
    if ((b & 0xFFFFu) && !(b >> 31)) hi += 1u;  // positive with dropped bits: the next bf16 up
    return (uint16_t) hi;
}

// Word of the special-block bitmap for 16-byte group `gi` of the chunk; the bit is gi & 31. Block
// (stage, consumer lane t) holds the groups j * kConsumers + t of the stage.
__device__ __forceinline__ int block_word(int gi) {
    const int st = gi / kStageGroups;
    const int t = gi % kConsumers;
    return st * kConsumerWarps + (t >> 5);
}

// Slot of history token t in the table, or -1.
__device__ __forceinline__ int hist_slot(const int32_t * keys, int bits, int32_t t) {
    const uint32_t mask = (1u << bits) - 1u;
    uint32_t h = hash_token(t, bits);
    for (uint32_t n = 0; n <= mask; n++) {
        const int32_t key = keys[h];
        if (key == t) return (int) h;
        if (key == -1) return -1;
        h = (h + 1) & mask;
    }
    return -1;
}

template <typename TIn, int KW, bool kDebug>
__global__ void __launch_bounds__(kStreamCtaThreads, 2) topk_rows_kernel(const StreamArgs sa) {
    const RowsArgs & a = sa.r;
    constexpr int G = Elem<TIn>::kVec;
    constexpr int kStageElems = kStageBytes / (int) sizeof(TIn);
    constexpr int QN = KW;  // registers per lane of a sorted list of 32*QN
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t s_full[kTkStages];
    __shared__ __align__(8) uint64_t s_empty[kTkStages];
    __shared__ SelectState sel;
    __shared__ float s_redf[32];
    __shared__ int s_redi[32];
    __shared__ int s_count, s_gather, s_abort, s_last, s_n0;

    const int tid = (int) threadIdx.x;
    const int warp = warp_id(), lane = lane_id();
    const bool producer = warp == kConsumerWarps;
    const int splits = sa.splits;
    const int row = blockIdx.x / splits;
    const int split = blockIdx.x - row * splits;
    const int vocab = a.vocab;
    const ssb_params pp = a.row_params ? a.row_params[row] : a.params;
    const RowParams p = resolve_params(pp, vocab);
    const bool greedy_row = p.greedy != 0;
    const int k = greedy_row ? 1 : p.k;
    if (a.row_params && !p.greedy && p.k > a.k_bound) {
        if (split == 0 && tid == 0) {
            a.ids[row] = -1, a.status[row] = SSB_ROW_INVALID_ROW;
            if (kDebug && a.dbg_count) a.dbg_count[row] = 0;
        }
        return;
    }
    const int c0 = split * sa.chunk;
    const int c1 = min(vocab, c0 + sa.chunk);
    const int len = c1 - c0;
    const int nvec = len / G;  // whole 16-byte groups; the rest are tail columns
    const int nstages = (nvec + kStageGroups - 1) / kStageGroups;

    // ---- shared memory: [ring = candidates later] [block maxima, bf16] [special-block bitmap]
    //                     [hash keys] [hash counts -> penalized logits] [selected]
    const int nst_alloc = (sa.chunk * (int) sizeof(TIn) + kStageBytes - 1) / kStageBytes;
    unsigned char * ring = smem;
    uint64_t * s_cand = reinterpret_cast<uint64_t *>(smem);  // [kCap], once the stream is over
    float * s_keep = reinterpret_cast<float *>(smem);        // [2 * kConsumers], E1 only
    uint16_t * s_up = reinterpret_cast<uint16_t *>(smem + kTkStages * kStageBytes);  // [nst_alloc][kConsumers]
    uint32_t * s_bb = reinterpret_cast<uint32_t *>(s_up + nst_alloc * kConsumers);  // [nst_alloc][kConsumerWarps]
    int32_t * s_hkey = reinterpret_cast<int32_t *>(s_bb + nst_alloc * kConsumerWarps);
    int32_t * s_hval = s_hkey + sa.hist_slots;
    uint64_t * s_sel = reinterpret_cast<uint64_t *>(s_hval + sa.hist_slots);  // [max(sel_slots, 32*QN)]

    const TIn * src = reinterpret_cast<const TIn *>(a.logits) + (int64_t) row * a.ld;
    const char * gsrc = reinterpret_cast<const char *>(src + c0);

    if (tid == 0) {
        s_count = 0;
        s_abort = 0;
        for (int q = 0; q < kTkStages; q++) mbar_init(&s_full[q], 1), mbar_init(&s_empty[q], kConsumerWarps);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int q = 0; q < kTkStages && q < nstages; q++) {
            const uint32_t bytes = (uint32_t) min(kStageBytes, (nvec - q * kStageGroups) * 16);
            mbar_expect(&s_full[q], bytes);
            bulk_load(ring + q * kStageBytes, gsrc + (size_t) q * kStageBytes, bytes, &s_full[q]);
        }
    }

    // ---- special blocks: history tokens (hash table of distinct ids with their counts) and masked
    //      tokens, marked per block for pass 1
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
        for (int i = tid; i < nstages * kConsumerWarps; i += blockDim.x) s_bb[i] = 0;
        if (penal)
            for (int i = tid; i < sa.hist_slots; i += blockDim.x) s_hkey[i] = -1, s_hval[i] = 0;
        __syncthreads();
        if (penal) {
            const uint32_t hmask = (uint32_t) sa.hist_slots - 1u;
            for (int base = 0; base < hlen; base += 4 * kStreamCtaThreads) {  // warp-uniform trip count
                int32_t t[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {  // four independent loads in flight
                    const int i = base + q * kStreamCtaThreads + tid;
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
                                    atomicAdd(&s_hval[h], __popc(peers));
                                    break;
                                }
                                h = (h + 1) & hmask;
                            }
                            const int gi = (t[q] - c0) / G;
                            if (gi < nvec) atomicOr(&s_bb[block_word(gi)], 1u << (gi & 31));
                        }
                    }
                }
            }
        }
        if (mrow) {
            // one mask word covers 32/G whole groups (c0 is a multiple of 32), in one bitmap word
            constexpr int kGroupsPerWord = 32 / G;
            constexpr uint32_t gfull = (1u << G) - 1u;
            const int w0 = c0 >> 5, nw = (len + 31) >> 5;
            for (int base = 0; base < nw; base += 4 * kStreamCtaThreads) {
                uint32_t mw[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int i = base + q * kStreamCtaThreads + tid;
                    mw[q] = i < nw ? __ldg(mrow + w0 + i) : 0u;
                }
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int i = base + q * kStreamCtaThreads + tid;
                    const int gi0 = i * kGroupsPerWord;
                    if (i < nw && gi0 < nvec) {
                        uint32_t sb = 0;
#pragma unroll
                        for (int gg = 0; gg < kGroupsPerWord; gg++) {
                            const uint32_t bits = (mw[q] >> (gg * G)) & gfull;
                            sb |= (uint32_t) (a.mask_kind == SSB_MASK_BAN ? bits != 0u : bits != gfull) << gg;
                        }
                        if (gi0 + kGroupsPerWord > nvec) sb &= (1u << (nvec - gi0)) - 1u;
                        if (sb) atomicOr(&s_bb[block_word(gi0)], sb << (gi0 & 31));
                    }
                }
            }
        }
    }
    __syncthreads();

    // is column col masked?
    auto masked = [&](int col) {
        if (!mrow) return false;
        const uint32_t w = __ldg(mrow + (col >> 5));
        return masked_bit(w >> (col & 31), a.mask_kind);
    };

    // ---- pass 1
    float keep0 = -kInf, keep1 = -kInf;  // the lane's two largest plain block maxima
    if (producer) {
        if (lane == 0) {
            for (int st = kTkStages; st < nstages; st++) {
                const int slot = st % kTkStages;
                if (!mbar_wait(&s_empty[slot], (uint32_t) ((st / kTkStages) - 1) & 1u)) s_abort = 1;
                const uint32_t bytes = (uint32_t) min(kStageBytes, (nvec - st * kStageGroups) * 16);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_expect(&s_full[slot], bytes);
                bulk_load(ring + slot * kStageBytes, gsrc + (size_t) st * kStageBytes, bytes, &s_full[slot]);
            }
        }
        __syncwarp();
        // every stage is issued: the penalized (and masked) logits of the history tokens, from the
        // logits the stream has brought into L2
        if (penal) {
            for (int base = 0; base < sa.hist_slots; base += 32 * 8) {
                int32_t t[8];
                float raw[8];
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    const int i = base + q * 32 + lane;
                    t[q] = i < sa.hist_slots ? s_hkey[i] : -1;
                }
#pragma unroll
                for (int q = 0; q < 8; q++) raw[q] = t[q] >= 0 ? Elem<TIn>::load1(src, t[q]) : 0.0f;
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    if (t[q] >= 0) {
                        const int i = base + q * 32 + lane;
                        const float v = masked(t[q]) ? -kInf : penalize(raw[q], s_hval[i], p);
                        s_hval[i] = __float_as_int(v);
                    }
                }
            }
        }
    } else {
        int slot = 0;
        uint32_t phase = 0;
        for (int st = 0; st < nstages; st++) {
            const uint4 * stage = reinterpret_cast<const uint4 *>(ring + slot * kStageBytes);
            if (!mbar_wait(&s_full[slot], phase)) s_abort = 1;
            const int sgroups = min(kStageGroups, nvec - st * kStageGroups);
            uint4 rv[kGroupsPerThread];
#pragma unroll
            for (int j = 0; j < kGroupsPerThread; j++) {
                const int g = j * kConsumers + tid;
                rv[j] = g < sgroups ? stage[g] : neg_inf_group<TIn>();
            }
            const bool spb = special && ((s_bb[st * kConsumerWarps + warp] >> lane) & 1u);
            // the lane's part of the stage is in registers: release the slot to the producer
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_empty[slot]);
            if (++slot == kTkStages) slot = 0, phase ^= 1u;
            const float lm = lane_max<TIn>(rv);
            s_up[st * kConsumers + tid] = bf16_up(lm);
            const float v = (spb || lm != lm) ? -kInf : lm;
            if (v > keep1) {
                keep1 = v > keep0 ? keep0 : v;
                keep0 = v > keep0 ? v : keep0;
            }
        }
    }

    // ---- end phase (all threads)
    __syncthreads();
    if (!producer) s_keep[tid] = keep0, s_keep[kConsumers + tid] = keep1;
    __syncthreads();
    // E1: a bound that k restricted logits reach
    radix_select(2 * kConsumers, k, [&](int i) { return (uint64_t) order_key(s_keep[i]) << 32; }, sel, 2);
    const uint32_t sb_key = (uint32_t) (sel.prefix >> 32);
    const float s_b = sb_key <= order_key(-kInf) ? -kInf : key_value(sb_key);
    __syncthreads();  // s_keep is ring memory, about to hold candidates
    const float T = greedy_row ? 1.0f : p.temperature;
    const bool scale = !greedy_row;
    const bool fast = greedy_row ? true : p.fast_scale;
    const bool monotone = greedy_row || T > 0.0f;
    uint64_t theta = composite(monotone && scale ? __fdiv_rn(s_b, T) : (monotone ? s_b : -kInf), 0xFFFFFFFFu);
    float cs = composite_value(theta);  // scaled logits below cs cannot be among the k best
    float rb = scale ? raw_bound(cs, T, fast) : cs;  // raw logits below rb cannot reach cs
    auto raise = [&](uint64_t t) {
        if (t > theta) {
            theta = t;
            cs = composite_value(theta);
            const float b = scale ? raw_bound(cs, T, fast) : cs;
            rb = b > rb ? b : rb;
        }
    };
    auto qualifies = [&](float up) {
        if (up != up || rb > -kInf || !monotone || cs == -kInf) return up != up || up >= rb;
        const float su = scale ? __fdiv_rn(up, T) : up;
        return !(su < cs);
    };

    float acc = -kInf;  // restricted maximum
    int nan_scaled = 0;
    // one candidate per lane where `has`, appended by one shared atomic per warp
    auto append = [&](bool has, uint64_t cv) {
        const unsigned m = __ballot_sync(0xffffffffu, has);
        if (!m) return;
        const int leader = __ffs(m) - 1;
        int base = 0;
        if (lane == leader) base = atomicAdd(&s_count, __popc(m));
        base = __shfl_sync(0xffffffffu, base, leader);
        if (has) s_cand[base + __popc(m & ((1u << lane) - 1u))] = cv;
    };
    // restricted logit v of column col: statistics, and a candidate if its composite reaches theta
    auto consider = [&](bool valid, float v, int col) {
        bool has = false;
        uint64_t cv = 0;
        if (valid) {
            acc = max_nan(acc, v);
            if (v >= rb) {
                const float sc = scale ? __fdiv_rn(v, T) : v;
                nan_scaled |= sc != sc;
                cv = composite(sc, (uint32_t) col);
                has = cv >= theta;
            }
        }
        append(has, cv);
    };
    // cuts the candidates to their k best (block-wide) and raises the threshold to the k-th
    auto cut = [&]() {
        const int n = s_count;
        radix_select(n, k, [&](int i) { return s_cand[i]; }, sel, 8);
        if (tid == 0) s_gather = 0;
        __syncthreads();
        for (int i = tid; i < n; i += blockDim.x) {
            const uint64_t cv = s_cand[i];
            if (selected(cv, sel)) s_sel[atomicAdd(&s_gather, 1)] = cv;
        }
        __syncthreads();
        const int m = s_gather;
        for (int i = tid; i < m; i += blockDim.x) s_cand[i] = s_sel[i];
        raise(sel.prefix);
        __syncthreads();
        if (tid == 0) s_count = m;
        __syncthreads();
    };

    // E2: history tokens
    if (penal) {
        for (int base = 0; base < sa.hist_slots; base += kHistChunk * (int) blockDim.x) {
#pragma unroll 1
            for (int q = 0; q < kHistChunk; q++) {
                const int i = base + q * (int) blockDim.x + tid;
                const int32_t t = i < sa.hist_slots ? s_hkey[i] : -1;
                consider(t >= 0, t >= 0 ? __int_as_float(s_hval[i]) : 0.0f, t);
            }
            __syncthreads();
            if (s_count > kCap - kRoom) cut();
        }
    }

    // E3: pass 2 over the blocks whose maximum can reach the threshold; each consumer warp walks its
    // own blocks, eight per round (lane l takes group l & 3 of block l >> 2)
    int gst = 0, gqst = 0;
    unsigned gq = 0;
    bool more = !producer && nstages > 0;
    while (__syncthreads_or(more)) {
        if (more) {
            int n = 0, my_blk = 0;
            while (n < 8) {  // warp-uniform
                if (gq == 0) {
                    if (gst >= nstages) break;
                    const float up = __uint_as_float((uint32_t) s_up[gst * kConsumers + warp * 32 + lane] << 16);
                    gq = __ballot_sync(0xffffffffu, qualifies(up));
                    gqst = gst++;
                    continue;
                }
                const int b = __ffs(gq) - 1;
                gq &= gq - 1u;
                if (lane == n) my_blk = (gqst << 5) | b;
                n++;
            }
            more = gq != 0 || gst < nstages;
            const int blk = __shfl_sync(0xffffffffu, my_blk, lane >> 2);
            const int bst = blk >> 5, bl = blk & 31;
            const int g = (lane & 3) * kConsumers + warp * 32 + bl;
            const bool has = (lane >> 2) < n && g < min(kStageGroups, nvec - bst * kStageGroups);
            const int col0 = c0 + bst * kStageElems + g * G;
            float v[G];
            uint32_t hist_e = 0;  // history elements: taken in E2
            if (has) {
                Elem<TIn>::unpack(__ldcg(reinterpret_cast<const uint4 *>(src + col0)), v);
                if (special && ((s_bb[bst * kConsumerWarps + warp] >> bl) & 1u)) {
#pragma unroll
                    for (int e = 0; e < G; e++) {
                        if (penal && hist_slot(s_hkey, hbits_n, col0 + e) >= 0) hist_e |= 1u << e;
                        else if (masked(col0 + e)) v[e] = -kInf;
                    }
                }
            }
#pragma unroll
            for (int e = 0; e < G; e++) consider(has && !((hist_e >> e) & 1u), has ? v[e] : 0.0f, col0 + e);
        }
        __syncthreads();
        if (s_count > kCap - kRoom) cut();
    }

    // E4: columns past the last whole 16-byte group (fewer than G)
    if (warp == 0) {
        const int col = c0 + nvec * G + lane;
        bool ok = col < c1;
        float v = 0.0f;
        if (ok) {
            if (penal && hist_slot(s_hkey, hbits_n, col) >= 0) ok = false;
            else v = masked(col) ? -kInf : Elem<TIn>::load1(src, col);
        }
        consider(ok, v, col);
    }
    if (kDebug && a.dbg_processed) {
        float * processed = a.dbg_processed + (int64_t) row * vocab;
        for (int col = c0 + tid; col < c1; col += blockDim.x) {
            const int hs = penal ? hist_slot(s_hkey, hbits_n, col) : -1;
            processed[col] = hs >= 0 ? __int_as_float(s_hval[hs]) : (masked(col) ? -kInf : Elem<TIn>::load1(src, col));
        }
    }
    __syncthreads();

    // E5: this CTA's best, sorted
    int nc = s_count;
    if (nc > 256 && nc > k) {
        cut();
        nc = s_count;
    }
    int np2 = 2;
    while (np2 < nc) np2 <<= 1;
    for (int i = nc + tid; i < np2; i += blockDim.x) s_cand[i] = 0ull;
    __syncthreads();
    bitonic_sort_desc(s_cand, np2);
    int kk = nc < k ? nc : k;
    const float rmax = block_max_nan(acc, s_redf);
    const int nanf = block_or(nan_scaled, s_redi) | (s_abort ? 2 : 0);

    const uint64_t * sorted = s_cand;
    float row_max = rmax;
    int row_flags = nanf;
    if (splits > 1) {
        const int64_t slot = (int64_t) row * splits + split;
        for (int i = tid; i < kk; i += blockDim.x) sa.part_cand[slot * sa.r.k_bound + i] = s_cand[i];
        if (tid == 0) {
            sa.part_n[slot] = kk;
            sa.part_max[slot] = rmax;
            sa.part_flags[slot] = nanf;
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) s_last = atomicAdd(&sa.counters[row], 1u) == (unsigned) (splits - 1);
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        if (tid == 0) sa.counters[row] = 0;  // ready for the next launch
        float m = -kInf;
        int f = 0;
        for (int q = tid; q < splits; q += blockDim.x) {
            m = max_nan(m, __ldcg(sa.part_max + (int64_t) row * splits + q));
            f |= __ldcg(sa.part_flags + (int64_t) row * splits + q);
        }
        row_max = block_max_nan(m, s_redf);
        row_flags = block_or(f & 1, s_redi) | (block_or(f & 2, s_redi) ? 2 : 0);
        // each consumer warp merges the lists of splits w, w+8, ...; warp 0 merges the warps' results
        uint64_t * lists = s_cand;  // [kConsumerWarps][32*QN]
        __syncthreads();
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
                    t[r] = i < n ? __ldcg(reinterpret_cast<const unsigned long long *>(sa.part_cand) + sl * sa.r.k_bound + i) : 0ull;
                }
                warp_merge_sorted<QN>(q, t);
            }
#pragma unroll
            for (int r = 0; r < QN; r++) lists[warp * 32 * QN + r * 32 + lane] = q[r];
        }
        __syncthreads();
        if (warp == 0) {
            uint64_t q[QN];
#pragma unroll
            for (int r = 0; r < QN; r++) q[r] = lists[r * 32 + lane];
            for (int w = 1; w < kConsumerWarps; w++) {
                uint64_t t[QN];
#pragma unroll
                for (int r = 0; r < QN; r++) t[r] = lists[w * 32 * QN + r * 32 + lane];
                warp_merge_sorted<QN>(q, t);
            }
            int nz = 0;
#pragma unroll
            for (int r = 0; r < QN; r++) {
                s_sel[r * 32 + lane] = q[r];
                nz += __popc(__ballot_sync(0xffffffffu, q[r] != 0ull));
            }
            if (lane == 0) s_n0 = nz;
        }
        __syncthreads();
        const int nz = s_n0;
        kk = nz < k ? nz : k;
        sorted = s_sel;
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
        if (tid == 0) {
            *id_out = -1, *st_out = stt;
            if (out.count) *out.count = 0;
        }
        return;
    }
    if (greedy_row) {
        if (tid == 0) {
            *id_out = (int32_t) composite_index(sorted[0]), *st_out = SSB_ROW_OK;
            if (out.count) *out.count = 1;
            if (out.tokens && out.cap > 0) out.tokens[0] = *id_out, out.weights[0] = 1.0;
        }
        return;
    }
    const double u = a.u ? a.u[row] : 0.0;
    // scratch for the weights: candidate memory past the sorted list (the split path sorted into s_sel)
    finalize_draw(sorted, kk, p, u, reinterpret_cast<double *>(s_cand + (splits > 1 ? kConsumerWarps * 32 * QN : np2)), out);
}

template <typename TIn, int KW, bool kDebug>
void * kernel_ptr() {
    return reinterpret_cast<void *>(topk_rows_kernel<TIn, KW, kDebug>);
}

void * pick_kernel(int kw, bool bf16, bool debug) {
#define SSB_KW(T)                                                                                       \
    switch (kw) {                                                                                      \
        case 1: return debug ? kernel_ptr<T, 1, true>() : kernel_ptr<T, 1, false>();                   \
        case 2: return debug ? kernel_ptr<T, 2, true>() : kernel_ptr<T, 2, false>();                   \
        default: return debug ? kernel_ptr<T, 4, true>() : kernel_ptr<T, 4, false>();                  \
    }
    if (bf16) SSB_KW(uint16_t)
    SSB_KW(float)
#undef SSB_KW
}

}  // namespace

size_t topk_smem_bytes(int kw, bool bf16, int chunk, int hist_slots, int sel_slots) {
    const int64_t nst = ((int64_t) chunk * (bf16 ? 2 : 4) + kStageBytes - 1) / kStageBytes;
    const int qn = kw;
    return (size_t) kTkStages * kStageBytes + (size_t) nst * kConsumers * 2 + (size_t) nst * kConsumerWarps * 4 +
           (size_t) hist_slots * 8 + (size_t) (sel_slots > 32 * qn ? sel_slots : 32 * qn) * 8;
}

int topk_blocks_per_sm(int kw, bool bf16, size_t smem) {
    void * kern = pick_kernel(kw, bf16, false);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem) != cudaSuccess) return 0;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kStreamCtaThreads, smem) != cudaSuccess) return 0;
    return n;
}

cudaError_t launch_topk(const StreamArgs & a, int kw, bool bf16, bool debug, cudaStream_t stream) {
    const size_t smem = topk_smem_bytes(kw, bf16, a.chunk, a.hist_slots, a.sel_slots);
    void * kern = pick_kernel(kw, bf16, debug);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (e != cudaSuccess) return e;
    void * args[] = {const_cast<StreamArgs *>(&a)};
    return cudaLaunchKernel(kern, dim3((unsigned) (a.r.rows * a.splits)), dim3(kStreamCtaThreads), args, smem, stream);
}

}  // namespace ssb
