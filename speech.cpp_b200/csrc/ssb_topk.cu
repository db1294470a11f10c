// Large-vocabulary rows with top-k <= 128 (every drawing configuration of the Qwen3 text decoders and
// the talker): the HBM-bound hot path of a drawing step.
//
// One CTA streams `chunk` consecutive columns of one row (several CTAs per row when the batch is small;
// the last to finish merges their lists, as in ssb_stream.cu). Two passes:
//
// Before the stream: the row's history table (distinct ids with their counts, built in one pass of
// insert-or-find and count) and a bitmap of the blocks holding a history or a masked token ("special"
// blocks; every other block's raw logits are its restricted logits, qwen3-tts/sampler.cpp:29-51),
// built by all threads while the first stages load.
//
// Pass 1, the stream. A producer warp brings the chunk through a ring of kTkStages 16 KB shared-memory
// stages with TMA bulk copies (cp.async.bulk + mbarrier complete_tx) and refills a slot as soon as every
// consumer warp has copied its part into registers. Each of 256 consumer lanes takes four 16-byte groups
// per stage (a "block" of 32 bf16 or 16 fp32 logits), stores the block's NaN-propagating maximum
// rounded up to bf16 (an upper bound of every logit in it) and keeps its two largest plain block maxima.
//
// End phase (short, mostly warp-local).
//   E1  bound: the lanes' kept maxima are restricted logits of distinct tokens (for fp32 rows the
//       largest bf16 at or below each). A two-digit radix select (histograms of the keys' high bytes,
//       then of the low bytes within the chosen one) gives their exact k-th largest, s_b. k tokens
//       reach s_b, so for a positive temperature (which keeps the order) every one of the k best has a
//       scaled logit >= c = fl(s_b / T).
//   E2  history tokens: penalized (and masked) logits computed now, from the logits the stream has just
//       brought into L2; candidates if they reach c.
//   E3  pass 2: every lane keeps its best block's logits in registers through the stream; its other
//       blocks whose maximum can reach c (only when its second best can) form a list, read again
//       from L2 one 16-byte group per lane, eight blocks per warp and round. Every element that
//       is not a history token is restricted (-inf where masked), divided by the temperature exactly as
//       the reference does (qwen3-tts/sampler.cpp:73) and keyed as a composite (value, then lowest
//       index: the order of qwen3-tts/sampler.cpp:78-79 with haru/sampler.cpp:39's tie-break).
//       A special best block is taken only if its maximum outside the history (masked tokens at -inf)
//       can reach c, computed from its registers: a history token's raw logit alone does not qualify it.
//       Composites >= the threshold go to a candidate array in the ring's memory. When the qualifying
//       blocks could overflow it (or the list), the rounds are synchronized and the array is cut to
//       its k best by a radix select (which also raises the threshold) between them.
//   E4  columns past the last whole 16-byte group.
//   E5  the candidates are ranked (each against all: they are few and distinct), and draw_row replays
//       the reference's double-precision softmax, top-p cut and pick.
// The restricted maximum (for the row statuses, qwen3-tts/sampler.cpp:43-49) is exact: the largest
// restricted logit lies in a block whose maximum reaches c, or is a history token.
// Temperatures that do not keep the order (<= 0 or NaN) make every block a pass-2 block.
#include <climits>
#include <type_traits>
#include <cuda_bf16.h>

#include "ssb_device.cuh"
#include "ssb_kernels.h"
#include "ssb_tma.cuh"

namespace ssb {

namespace {

constexpr int kTkStages = 3;
constexpr int kTkThreads = kStreamCtaThreads;      // 8 consumer warps + the producer warp
constexpr int kStageArea = kConsumers * 64;                     // staged best blocks: 64 bytes per lane
constexpr int kCap = (kTkStages * kStageBytes - kStageArea) / 8;  // candidate composites in the ring's memory
constexpr int kMaxStages = 64;                     // stages of one chunk (a lane's pass-2 mask is 64-bit)
constexpr int kRankMax = kTkThreads;               // candidates ranked directly (one per thread)
constexpr int kListMax = 1024;                     // pass-2 blocks listed for the cooperative rounds
constexpr int kRoundBlocks = kConsumerWarps * 8;   // blocks per cooperative round

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

// A group with the elements of bit mask ex (element order) set to -inf.
template <typename TIn> __device__ __forceinline__ uint4 exclude_group(const uint4 & g, uint32_t ex);
template <> __device__ __forceinline__ uint4 exclude_group<uint16_t>(const uint4 & g, uint32_t ex) {
    auto f = [](uint32_t w, uint32_t b) {
        const uint32_t sel = ((b & 1u) ? 0x0000FFFFu : 0u) | ((b & 2u) ? 0xFFFF0000u : 0u);
        return (w & ~sel) | (0xFF80FF80u & sel);
    };
    return make_uint4(f(g.x, ex), f(g.y, ex >> 2), f(g.z, ex >> 4), f(g.w, ex >> 6));
}
template <> __device__ __forceinline__ uint4 exclude_group<float>(const uint4 & g, uint32_t ex) {
    return make_uint4((ex & 1u) ? 0xFF800000u : g.x, (ex & 2u) ? 0xFF800000u : g.y, (ex & 4u) ? 0xFF800000u : g.z,
                      (ex & 8u) ? 0xFF800000u : g.w);
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
__global__ void __launch_bounds__(kTkThreads, 2) topk_rows_kernel(const StreamArgs sa) {
    const RowsArgs & a = sa.r;
    constexpr int G = Elem<TIn>::kVec;
    constexpr int kStageElems = kStageBytes / (int) sizeof(TIn);
    constexpr int kBlockElems = kGroupsPerThread * G;
    constexpr int QN = KW;  // registers per lane of a sorted list of 32*QN
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t s_full[kTkStages];
    __shared__ __align__(8) uint64_t s_empty[kTkStages];
    __shared__ SelectState sel;
    __shared__ float s_redf[32];
    __shared__ int s_redi[32];
    __shared__ int s_count, s_gather, s_abort, s_last, s_n0, s_qn, s_issued;
    __shared__ __align__(16) uint32_t s_f1[256];  // bound: histogram of the kept keys' high bytes
    __shared__ __align__(16) uint32_t s_f2[256];  // and of their low bytes within the chosen high byte
    __shared__ int s_qlist[kListMax];

    const int tid = (int) threadIdx.x;
    const int warp = warp_id(), lane = lane_id();
    const bool consumer = warp < kConsumerWarps;
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

    // ---- shared memory: [ring = candidates once the stream is over] [block maxima, bf16] [special-block bitmap]
    //                     [history-column bitmap] [hash keys] [hash counts] [selected]
    const int nst_alloc = (sa.chunk * (int) sizeof(TIn) + kStageBytes - 1) / kStageBytes;
    unsigned char * ring = smem;
    uint64_t * s_cand = reinterpret_cast<uint64_t *>(smem);  // [kCap], once the stream is over
    uint4 * s_stage = reinterpret_cast<uint4 *>(smem + kCap * 8);  // [kConsumers][4], E3
    uint16_t * s_up = reinterpret_cast<uint16_t *>(smem + kTkStages * kStageBytes);  // [nst_alloc][kConsumers]
    uint32_t * s_bb = reinterpret_cast<uint32_t *>(s_up + nst_alloc * kConsumers);  // [nst_alloc][kConsumerWarps]
    const int hw_alloc = sa.hist_slots > 0 ? ((((sa.chunk + 31) >> 5) + 3) & ~3) : 0;
    uint32_t * s_hbits = s_bb + nst_alloc * kConsumerWarps;  // [hw_alloc] history columns of the chunk
    int32_t * s_hkey = reinterpret_cast<int32_t *>(s_hbits + hw_alloc);
    int32_t * s_hcnt = s_hkey + sa.hist_slots;
    uint64_t * s_sel = reinterpret_cast<uint64_t *>(s_hcnt + sa.hist_slots);  // [max(sel_slots, 32*QN)]

    const TIn * src = reinterpret_cast<const TIn *>(a.logits) + (int64_t) row * a.ld;
    const char * gsrc = reinterpret_cast<const char *>(src + c0);

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

    // each thread's first history ids, requested before the first stages' copies
    int32_t hpre[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const int i = q * kTkThreads + tid;
        hpre[q] = penal && i < hlen ? __ldg(hist + i) : -1;
    }
    for (int i = tid; i < 256; i += blockDim.x) s_f1[i] = 0, s_f2[i] = 0;
    if (tid == 0) {
        s_count = 0;
        s_qn = 0;
        s_abort = 0;
        for (int q = 0; q < kTkStages; q++) mbar_init(&s_full[q], 1), mbar_init(&s_empty[q], kConsumerWarps);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        int q = 0;
        for (; q < kTkStages && q < nstages; q++) {
            const uint32_t bytes = (uint32_t) min(kStageBytes, (nvec - q * kStageGroups) * 16);
            mbar_expect(&s_full[q], bytes);
            bulk_load(ring + q * kStageBytes, gsrc + (size_t) q * kStageBytes, bytes, &s_full[q]);
        }
        s_issued = q;
    }

    // ---- special blocks (all threads, while the first stages load)
    if (special) {
        for (int i = tid; i < nstages * kConsumerWarps; i += blockDim.x) s_bb[i] = 0;
        if (penal) {
            for (int i = tid; i < sa.hist_slots; i += blockDim.x) s_hkey[i] = -1, s_hcnt[i] = 0;
            for (int i = tid; i < ((sa.chunk + 31) >> 5); i += blockDim.x) s_hbits[i] = 0;
        }
        __syncthreads();
        if (penal) {
            // one pass: every occurrence of an id finds or takes its slot and counts itself there; the
            // column bit and the block bit are set by every occurrence alike
            const uint32_t hmask = (uint32_t) sa.hist_slots - 1u;
            for (int base = 0; base < hlen; base += 4 * kTkThreads) {  // uniform trip count
                int32_t t[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {  // four independent loads in flight
                    const int i = base + q * kTkThreads + tid;
                    t[q] = base == 0 ? hpre[q] : (i < hlen ? __ldg(hist + i) : -1);
                }
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    if (t[q] >= c0 && t[q] < c1) {
                        const int rel = t[q] - c0;
                        atomicOr(&s_hbits[rel >> 5], 1u << (rel & 31));
                        const int gi = rel / G;
                        if (gi < nvec) atomicOr(&s_bb[block_word(gi)], 1u << (gi & 31));
                        uint32_t h = hash_token(t[q], hbits_n);
                        for (uint32_t n = 0; n <= hmask; n++) {
                            const int32_t old = atomicCAS(&s_hkey[h], -1, t[q]);
                            if (old == -1 || old == t[q]) {
                                atomicAdd(&s_hcnt[h], 1);
                                break;
                            }
                            h = (h + 1) & hmask;
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
            for (int base = 0; base < nw; base += 4 * kTkThreads) {
                uint32_t mw[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int i = base + q * kTkThreads + tid;
                    mw[q] = i < nw ? __ldg(mrow + w0 + i) : 0u;
                }
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int i = base + q * kTkThreads + tid;
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
        __syncwarp();
    }
    __syncthreads();

    // is column col masked?
    auto masked = [&](int col) {
        if (!mrow) return false;
        const uint32_t w = __ldg(mrow + (col >> 5));
        return masked_bit(w >> (col & 31), a.mask_kind);
    };

    // ---- pass 1
    uint32_t key0 = 0, key1 = 0;  // the lane's two largest plain block maxima (16-bit order keys; 0: none)
    // the lane's best block (largest maximum, NaN first) with its logits, and the second largest maximum
    float best_v = -kInf, second_v = -kInf;
    int best_st = -1;
    uint4 best_rv[kGroupsPerThread];
#pragma unroll
    for (int j = 0; j < kGroupsPerThread; j++) best_rv[j] = make_uint4(0, 0, 0, 0);
    if (!consumer) {
        // producer: a slot is refilled once every consumer warp has released it; a release that does not
        // come within the bounded wait stops the producer (no further copy is issued)
        if (lane == 0) {
            int st = kTkStages;
            for (; st < nstages; st++) {
                const int slot = st % kTkStages;
                if (!mbar_wait(&s_empty[slot], (uint32_t) ((st / kTkStages) - 1) & 1u)) {
                    atomicOr(&s_abort, 1);
                    break;
                }
#ifdef SSB_WAIT_TEST
                // the wait-limit test build: row 0's first refill is never issued, so its consumers'
                // bounded wait runs out (a stage that nothing fills)
                if (row == 0 && split == 0 && st == kTkStages) continue;
#endif
                const uint32_t bytes = (uint32_t) min(kStageBytes, (nvec - st * kStageGroups) * 16);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_expect(&s_full[slot], bytes);
                bulk_load(ring + slot * kStageBytes, gsrc + (size_t) st * kStageBytes, bytes, &s_full[slot]);
            }
            if (st > kTkStages) s_issued = st;
        }
    } else {
        int slot = 0;
        uint32_t phase = 0;
        for (int st = 0; st < nstages; st++) {
            const uint4 * stage = reinterpret_cast<const uint4 *>(ring + slot * kStageBytes);
            if (!mbar_wait(&s_full[slot], phase)) atomicOr(&s_abort, 1);
            const int sgroups = min(kStageGroups, nvec - st * kStageGroups);
            uint4 rv[kGroupsPerThread];
#pragma unroll
            for (int j = 0; j < kGroupsPerThread; j++) {
                const int g = j * kConsumers + tid;
                rv[j] = g < sgroups ? stage[g] : neg_inf_group<TIn>();
            }
            // the lane's part of the stage is in registers: release the slot to the producer
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_empty[slot]);
            if (++slot == kTkStages) slot = 0, phase ^= 1u;
            const float lm = lane_max<TIn>(rv);
            const uint16_t up = bf16_up(lm);
            s_up[st * kConsumers + tid] = up;
            const bool plain = !(special && ((s_bb[st * kConsumerWarps + warp] >> lane) & 1u)) && lm == lm;
            // a plain block's maximum, as the key of a bf16 at or below it (fp32 maxima were rounded up)
            const uint32_t kb = (order_key(__uint_as_float((uint32_t) up << 16)) >> 16) -
                                ((sizeof(TIn) == 4 && lm > -kInf) ? 1u : 0u);
            if (plain && kb > key1) {
                key1 = kb > key0 ? key0 : kb;
                key0 = kb > key0 ? kb : key0;
            }
            const float bv = lm == lm ? lm : kInf;
            if (best_st < 0 || bv > best_v) {
                second_v = best_st < 0 ? -kInf : best_v;
                best_v = bv;
                best_st = st;
#pragma unroll
                for (int j = 0; j < kGroupsPerThread; j++) best_rv[j] = rv[j];
            } else if (bv > second_v) {
                second_v = bv;
            }
        }
    }
    __syncwarp();

    // ---- end phase (all threads)
    // E1: the exact k-th largest of the lanes' kept keys, by a two-digit radix select (a histogram of the
    // high bytes, then of the low bytes within the chosen one; every warp reads each after its barrier,
    // the second of which also frees the ring's memory for the candidates)
    red_bin(s_f1, consumer && key0 != 0, key0 >> 8);
    red_bin(s_f1, consumer && key1 != 0, key1 >> 8);
    __syncthreads();
    if (tid == 0 && s_abort) {
        // a wait ran out: before the ring's memory is reused (and before the CTA exits), wait (bounded)
        // for the last copy issued into every slot
        const int issued = s_issued;
        for (int st = issued - kTkStages; st < issued; st++)
            if (st >= 0) (void) mbar_wait(&s_full[st % kTkStages], (uint32_t) (st / kTkStages) & 1u);
    }
    uint32_t above1 = 0;
    const int b1 = top_bin(s_f1, (uint32_t) k, &above1);
    red_bin(s_f2, consumer && b1 >= 0 && key0 != 0 && (int) (key0 >> 8) == b1, key0 & 255u);
    red_bin(s_f2, consumer && b1 >= 0 && key1 != 0 && (int) (key1 >> 8) == b1, key1 & 255u);
    __syncthreads();
    uint32_t P = 0;
    if (b1 >= 0) {
        uint32_t above2 = 0;
        const int b2 = top_bin(s_f2, (uint32_t) k - above1, &above2);
        if (b2 >= 0) P = ((uint32_t) b1 << 8) | (uint32_t) b2;
    }
    // P <= key of -inf (no k keys): no bound; else the value of key P << 16 is at or below k restricted
    // logits
    const float s_b = (P << 16) <= order_key(-kInf) ? -kInf : key_value(P << 16);
    const float T = greedy_row ? 1.0f : p.temperature;
    const bool scale = !greedy_row;
    const bool fast = greedy_row ? true : p.fast_scale;
    const bool monotone = greedy_row || T > 0.0f;
    float c_init = monotone ? (scale ? __fdiv_rn(s_b, T) : s_b) : -kInf;
    if (c_init != c_init) c_init = -kInf;
    uint64_t theta = composite(c_init, 0xFFFFFFFFu);
    float cs = composite_value(theta);               // scaled logits below cs cannot be among the k best
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
    // each lane's candidates (cv[i] where bit i of vm is set), appended by one shared atomic per warp
    auto append_m = [&](uint32_t vm, const uint64_t * cv, auto n_tag) {
        constexpr int N = decltype(n_tag)::value;
        const int n = __popc(vm);
        int incl = n;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        const int total = __shfl_sync(0xffffffffu, incl, 31);
        int base = 0;
        if (lane == 31) base = atomicAdd(&s_count, total);
        base = __shfl_sync(0xffffffffu, base, 31) + incl - n;
#pragma unroll
        for (int i = 0; i < N; i++)
            if ((vm >> i) & 1u) s_cand[base + __popc(vm & ((1u << i) - 1u))] = cv[i];
    };
    // restricted logit v of column col: whether its composite reaches theta
    auto test = [&](float v, int col, uint64_t & cv) {
        if (!(v >= rb)) return false;
        const float sc = scale ? __fdiv_rn(v, T) : v;
        nan_scaled |= sc != sc;
        cv = composite(sc, (uint32_t) col);
        return cv >= theta;
    };
    // one 16-byte group: its restricted logits into the maximum, its candidates appended (history elements
    // are skipped: taken in E2). A plain group below the raw bound has no candidate.
    auto take_group = [&](bool live, const uint4 & raw, int col0, bool blk_special) {
        uint64_t cv[G];
        uint32_t vm = 0;
        if (live) {
            const float gm = group_max<TIn>(raw);
            if (!blk_special) acc = max_nan(acc, gm);
            if (blk_special || gm >= rb) {
                float v[G];
                Elem<TIn>::unpack(raw, v);
#pragma unroll
                for (int e = 0; e < G; e++) {
                    bool skip = false;
                    if (blk_special) {
                        if (penal && ((s_hbits[(col0 + e - c0) >> 5] >> ((col0 + e - c0) & 31)) & 1u)) skip = true;
                        else if (masked(col0 + e)) v[e] = -kInf;
                        if (!skip) acc = max_nan(acc, v[e]);
                    }
                    if (!skip && test(v[e], col0 + e, cv[e])) vm |= 1u << e;
                }
            }
        }
        if (__any_sync(0xffffffffu, vm != 0)) append_m(vm, cv, std::integral_constant<int, G>());
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
        for (int base = 0; base < sa.hist_slots; base += 8 * kTkThreads) {  // uniform
            int32_t t[8];
            float raw[8];
#pragma unroll
            for (int q = 0; q < 8; q++) {
                const int i = base + q * kTkThreads + tid;
                t[q] = i < sa.hist_slots ? s_hkey[i] : -1;
            }
#pragma unroll
            for (int q = 0; q < 8; q++) raw[q] = t[q] >= 0 ? Elem<TIn>::load1(src, t[q]) : 0.0f;
            uint64_t cv[8];
            uint32_t vm = 0;
#pragma unroll
            for (int q = 0; q < 8; q++) {
                if (t[q] >= 0) {
                    const int i = base + q * kTkThreads + tid;
                    const float v = masked(t[q]) ? -kInf : penalize(raw[q], s_hcnt[i], p);
                    acc = max_nan(acc, v);
                    if (test(v, t[q], cv[q])) vm |= 1u << q;
                }
            }
            if (__any_sync(0xffffffffu, vm != 0)) append_m(vm, cv, std::integral_constant<int, 8>());
            __syncwarp();
            __syncthreads();
            if (s_count > kCap - 8 * kTkThreads) cut();
        }
    }

    // E3: pass 2 over the blocks whose maximum can reach the threshold. A lane's best block is still in
    // its registers: it is staged in shared memory; its other qualifying blocks (only when its second
    // best can qualify) are read again from L2. All of them are listed and taken cooperatively, one
    // 16-byte group per lane, eight blocks per warp and round.
    const bool lane_q = consumer && best_st >= 0 && qualifies(best_v);  // the lane has a qualifying block
    bool best_q = lane_q;  // its best block is taken
    if (best_q && special && ((s_bb[best_st * kConsumerWarps + warp] >> lane) & 1u)) {
        // a special best block (still in registers) is taken only if its maximum over the tokens outside
        // the history (masked ones at -inf) can reach the threshold: its history tokens are E2's
        float lx = -kInf;
#pragma unroll
        for (int j = 0; j < kGroupsPerThread; j++) {
            const int g = j * kConsumers + tid;
            if (g < min(kStageGroups, nvec - best_st * kStageGroups)) {
                const int col0 = c0 + best_st * kStageElems + g * G, rel0 = col0 - c0;
                uint32_t ex = penal ? (s_hbits[rel0 >> 5] >> (rel0 & 31)) & ((1u << G) - 1u) : 0u;
                if (mrow) {
                    const uint32_t mw = (__ldg(mrow + (col0 >> 5)) >> (col0 & 31)) & ((1u << G) - 1u);
                    ex |= a.mask_kind == SSB_MASK_BAN ? mw : (~mw & ((1u << G) - 1u));
                }
                lx = max_nan(lx, group_max<TIn>(exclude_group<TIn>(best_rv[j], ex)));
            }
        }
        best_q = qualifies(lx);
    }
    uint64_t qmask = 0;  // stages of this lane's other qualifying blocks
    if (lane_q && qualifies(second_v))
        for (int st = 0; st < nstages; st++)
            if (st != best_st && qualifies(__uint_as_float((uint32_t) s_up[st * kConsumers + tid] << 16))) qmask |= 1ull << st;
    const int nq = __popcll(qmask);
    if (best_q) {
#pragma unroll
        for (int j = 0; j < kGroupsPerThread; j++) s_stage[tid * kGroupsPerThread + j] = best_rv[j];
    }
    if (best_q || nq > 0) {
        const int at = atomicAdd(&s_qn, nq + (best_q ? 1 : 0));
        int i = 0;
        if (best_q && at < kListMax) s_qlist[at] = (1 << 30) | (best_st << 9) | tid, i = 1;  // bit 30: staged
        uint64_t m = qmask;
        for (; i < nq + (best_q ? 1 : 0) && at + i < kListMax; i++) {
            const int st = __ffsll((long long) m) - 1;
            m &= m - 1;
            s_qlist[at + i] = (st << 9) | tid;
        }
    }
    __syncwarp();
    __syncthreads();
    const int qtotal = s_qn;
    const bool synced = s_count + qtotal * kBlockElems + G > kCap;
    if (synced && s_count > kCap - kConsumers * G) cut();
    if (qtotal <= kListMax) {
        const int rounds = (qtotal + kRoundBlocks - 1) / kRoundBlocks;
        for (int r = 0; r < rounds; r++) {  // CTA-uniform
            if (consumer) {
                const int e = r * kRoundBlocks + warp * 8 + (lane >> 2);
                const int j = lane & 3;
                bool live = false;
                uint4 raw = make_uint4(0, 0, 0, 0);
                int col0 = c0;
                bool blk_special = false;
                if (e < qtotal) {
                    const int ent = s_qlist[e];
                    const int st = (ent >> 9) & 0x1FFFF, t = ent & 511;
                    const int g = j * kConsumers + t;
                    col0 = c0 + st * kStageElems + g * G;
                    live = g < min(kStageGroups, nvec - st * kStageGroups);
                    if (live) raw = (ent >> 30) ? s_stage[t * kGroupsPerThread + j] : __ldcg(reinterpret_cast<const uint4 *>(src + col0));
                    blk_special = special && ((s_bb[st * kConsumerWarps + (t >> 5)] >> (t & 31)) & 1u);
                }
                take_group(live, raw, col0, blk_special);
            }
            if (synced) {
                __syncwarp();
                __syncthreads();
                if (s_count > kCap - kConsumers * G) cut();
            }
        }
    } else {
        // a list that long (no useful bound): each lane takes its own blocks, one group per round
        if (best_q) qmask |= 1ull << best_st;
        const int passes = block_max_int(__popcll(qmask), s_redi);
        for (int pass = 0; pass < passes; pass++) {  // CTA-uniform
            const bool has = qmask != 0;
            const int st = has ? __ffsll((long long) qmask) - 1 : 0;
            qmask &= qmask - 1;
            const bool blk_special = has && special && ((s_bb[st * kConsumerWarps + warp] >> lane) & 1u);
            for (int j = 0; j < kGroupsPerThread; j++) {
                const int g = j * kConsumers + tid;
                const int col0 = c0 + st * kStageElems + g * G;
                const bool live = has && g < min(kStageGroups, nvec - st * kStageGroups);
                const uint4 raw = live ? __ldcg(reinterpret_cast<const uint4 *>(src + col0)) : make_uint4(0, 0, 0, 0);
                if (consumer) take_group(live, raw, col0, blk_special);
                __syncwarp();
                __syncthreads();
                if (s_count > kCap - kConsumers * G) cut();
            }
        }
    }

    // E4: columns past the last whole 16-byte group (fewer than G)
    if (warp == 0) {
        const int col = c0 + nvec * G + lane;
        uint64_t cv[1];
        uint32_t vm = 0;
        if (col < c1 && !(penal && ((s_hbits[(col - c0) >> 5] >> ((col - c0) & 31)) & 1u))) {
            const float v = masked(col) ? -kInf : Elem<TIn>::load1(src, col);
            acc = max_nan(acc, v);
            if (test(v, col, cv[0])) vm = 1u;
        }
        if (__any_sync(0xffffffffu, vm != 0)) append_m(vm, cv, std::integral_constant<int, 1>());
    }
    if (kDebug && a.dbg_processed) {
        float * processed = a.dbg_processed + (int64_t) row * vocab;
        for (int col = c0 + tid; col < c1; col += blockDim.x) {
            const int hs = penal ? hist_slot(s_hkey, hbits_n, col) : -1;
            float v = Elem<TIn>::load1(src, col);
            if (hs >= 0) v = penalize(v, s_hcnt[hs], p);
            processed[col] = masked(col) ? -kInf : v;
        }
    }
    __syncwarp();
    __syncthreads();

    // E5: this CTA's best min(k, n) candidates, sorted, by rank (composites are distinct)
    if (s_count > kRankMax) cut();
    const int nc = s_count;
    const int kk0 = nc < k ? nc : k;
    if (tid < nc) {
        const uint64_t mine = s_cand[tid];
        int rank = 0;
        for (int j = 0; j < nc; j++) rank += s_cand[j] > mine;
        if (rank < kk0) s_sel[rank] = mine;
    }
    const float rmax = block_max_nan(acc, s_redf);
    const int nanf = block_or(nan_scaled, s_redi) | (s_abort ? 2 : 0);
    int kk = kk0;

    float row_max = rmax;
    int row_flags = nanf;
    if (splits > 1) {
        const int64_t slot = (int64_t) row * splits + split;
        for (int i = tid; i < kk; i += blockDim.x) sa.part_cand[slot * sa.r.k_bound + i] = s_sel[i];
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
        if (consumer) {
            uint64_t q[QN];
#pragma unroll
            for (int r = 0; r < QN; r++) q[r] = 0;
            // four lists at a time: their counts and entries requested together (entries up to k_bound, the
            // slot's own storage, then cut to the count), so a list costs no dependent round trip of its own
            for (int sp0 = warp; sp0 < splits; sp0 += 4 * kConsumerWarps) {
                uint64_t t[4][QN];
                int n[4];
#pragma unroll
                for (int g = 0; g < 4; g++) {
                    const int sp = sp0 + g * kConsumerWarps;
                    const int64_t sl = (int64_t) row * splits + sp;
                    n[g] = sp < splits ? __ldcg(sa.part_n + sl) : 0;
#pragma unroll
                    for (int r = 0; r < QN; r++) {
                        const int i = r * 32 + lane;
                        t[g][r] = sp < splits && i < sa.r.k_bound
                                      ? __ldcg(reinterpret_cast<const unsigned long long *>(sa.part_cand) + sl * sa.r.k_bound + i)
                                      : 0ull;
                    }
                }
#pragma unroll
                for (int g = 0; g < 4; g++) {
#pragma unroll
                    for (int r = 0; r < QN; r++)
                        if (r * 32 + lane >= n[g]) t[g][r] = 0ull;
                    if (sp0 + g * kConsumerWarps < splits) warp_merge_sorted<QN>(q, t[g]);  // warp-uniform
                }
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
            *id_out = (int32_t) composite_index(s_sel[0]), *st_out = SSB_ROW_OK;
            if (out.count) *out.count = 1;
            if (out.tokens && out.cap > 0) out.tokens[0] = *id_out, out.weights[0] = 1.0;
        }
        return;
    }
    const double u = a.u ? a.u[row] : 0.0;
    if (warp == 0) draw_row(s_sel, kk, p, u, reinterpret_cast<double *>(s_cand), out);  // candidate memory as scratch
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

int topk_kw(int k_bound) { return k_bound <= 32 ? 1 : (k_bound <= 64 ? 2 : 4); }

int topk_max_chunk(bool bf16) { return kMaxStages * kStageBytes / (bf16 ? 2 : 4); }

size_t topk_smem_bytes(int kw, bool bf16, int chunk, int hist_slots, int sel_slots) {
    const int64_t nst = ((int64_t) chunk * (bf16 ? 2 : 4) + kStageBytes - 1) / kStageBytes;
    const int qn = kw;
    const size_t hwords = hist_slots > 0 ? (size_t) ((((chunk + 31) >> 5) + 3) & ~3) : 0;
    return (size_t) kTkStages * kStageBytes + (size_t) nst * kConsumers * 2 + (size_t) nst * kConsumerWarps * 4 +
           hwords * 4 + (size_t) hist_slots * 8 + (size_t) (sel_slots > 32 * qn ? sel_slots : 32 * qn) * 8;
}

int topk_blocks_per_sm(int kw, bool bf16, size_t smem) {
    void * kern = pick_kernel(kw, bf16, false);
    if (ssb::set_max_dynamic_smem((const void *) kern, smem) != cudaSuccess) return 0;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kTkThreads, smem) != cudaSuccess) return 0;
    return n;
}

cudaError_t launch_topk(const StreamArgs & a, int kw, bool bf16, bool debug, cudaStream_t stream) {
    const size_t smem = topk_smem_bytes(kw, bf16, a.chunk, a.hist_slots, a.sel_slots);
    void * kern = pick_kernel(kw, bf16, debug);
    cudaError_t e = ssb::set_max_dynamic_smem((const void *) kern, smem);
    if (e != cudaSuccess) return e;
    void * args[] = {const_cast<StreamArgs *>(&a)};
    return cudaLaunchKernel(kern, dim3((unsigned) (a.r.rows * a.splits)), dim3(kTkThreads), args, smem, stream);
}

}  // namespace ssb
