// Large-vocabulary rows whose top-k keeps more than kStreamMaxK tokens (top-k 0 = every token, as in
// constrained decoding with an allow mask and top-p): the candidates of qwen3-tts/sampler.cpp:69-101
// with k = V, then pick() (sampling.cpp:9-19).
//
// The reference sorts every token, sums exp(s - max) over all of them in that order (double), cuts at the
// first running share >= top_p and draws with pick(). Its answer is two positions in the sorted order:
// where the running share first reaches top_p (keep) and where pick()'s running sum first exceeds u
// (chosen). Only the order near those two positions matters, and only if a running sum is within
// rounding error of its limit. So, per row (one CTA; a CTA loops over rows):
//   pass 1  the row: restricted (penalties, mask) and scaled logits; every token with a finite scaled
//           logit goes to a per-CTA list in global memory as its composite key (value, then lowest index).
//   pass 2  the list: w = exp(s - max) in double, its total, and a histogram of that mass (and of the
//           token counts) over buckets linear in max - s (1/64 wide; mass_bucket).
//   cut     scanning the histogram from the top finds the bucket where the running share reaches top_p;
//           its tokens are sorted in shared memory and scanned, which gives keep and pick()'s total;
//   draw    the same for the running sum u * total: its bucket, sorted and scanned, gives chosen.
// Every running sum here is summed in another order than the reference's; the error of either is at most
// (2n + 2) ulp of the total for n tokens, so a crossing whose margin exceeds kMargin (relative) is the
// reference's. A crossing closer than that, a crossing bucket too large for shared memory, a top_p that
// no running share reaches, and every debug export take the exact path instead: the whole list sorted
// in global memory (bitonic) and the reference's sequential sums, in the reference's order.
#include <climits>
#include <cuda_bf16.h>

#include "ssb_device.cuh"
#include "ssb_kernels.h"
#include "ssb_tma.cuh"  // hash_token

namespace ssb {

namespace {

constexpr int kNThreads = 512;
constexpr int kNWarps = kNThreads / 32;
constexpr int kBucketBits = 12;
constexpr int kBuckets = 1 << kBucketBits;
constexpr int kBucketShift = 32 - kBucketBits;
constexpr int kListMaxN = 4096;     // tokens of one crossing bucket sorted in shared memory
constexpr int kQueue = 256;         // pass 1's per-warp queue of a sparse round (kNWarps x kQueue <= 2 kListMaxN)
constexpr double kMargin = 1e-9;    // relative margin that decides a crossing without the exact path
constexpr int kChunk = 256;         // exact path: values computed per step by the warp for lane 0's sums
constexpr int kScanUnroll = 8;      // list entries requested together per thread by the list scans
constexpr int kMergedScanMin = 16384;  // candidates from which one scan loads both crossings' buckets

__device__ __forceinline__ uint32_t bucket_of(uint64_t c) { return (uint32_t) (c >> 32) >> kBucketShift; }

// Bucket of a candidate's mass: linear in the distance of its scaled logit below the row's maximum mxf,
// 1/64 per bucket from the top bucket down (every candidate 64 or more below shares bucket 0). Like
// bucket_of it never decreases along the composite order, and it is far finer where the mass lies: the
// top 12 key bits hold only 3 mantissa bits, so logits of a few units spread over a few dozen buckets.
__device__ __forceinline__ uint32_t mass_bucket(uint64_t c, float mxf) {
    const float d = __fmul_rn(__fsub_rn(mxf, composite_value(c)), 64.0f);
    return d >= (float) (kBuckets - 1) ? 0u : (uint32_t) (kBuckets - 1) - (uint32_t) d;
}

// Block-wide inclusive scan of one double per thread (blockDim = kNThreads); `s` holds kNWarps doubles.
__device__ __forceinline__ double block_scan_incl(double v, double * s) {
    const int lane = lane_id(), warp = warp_id();
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
    }
    __syncthreads();
    if (lane == 31) s[warp] = v;
    __syncthreads();
    double before = 0.0;
    for (int w = 0; w < warp; w++) before += s[w];
    return v + before;
}

__device__ __forceinline__ double block_sum_double(double v, double * s) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane_id() == 0) s[warp_id()] = v;
    __syncthreads();
    double t = 0.0;
    for (int w = 0; w < kNWarps; w++) t += s[w];
    return t;
}

// Descending bitonic sort of n (a power of two) u64 in global memory, block-wide.
__device__ void global_bitonic_desc(uint64_t * x, int n) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < (n >> 1); i += blockDim.x) {
                const int lo = 2 * stride * (i / stride) + (i % stride);
                const int hi = lo + stride;
                const bool desc = (lo & size) == 0;
                const uint64_t a = __ldcg(reinterpret_cast<const unsigned long long *>(x + lo));
                const uint64_t b = __ldcg(reinterpret_cast<const unsigned long long *>(x + hi));
                if ((a < b) == desc) x[lo] = b, x[hi] = a;
            }
            __threadfence_block();
            __syncthreads();
        }
    }
}

template <typename TIn, bool kDebug>
__global__ void __launch_bounds__(kNThreads, 1) nucleus_rows_kernel(const NucleusArgs na) {
    const RowsArgs & a = na.r;
    extern __shared__ __align__(16) unsigned char smem[];
    double * s_hmass = reinterpret_cast<double *>(smem);                 // [kBuckets]
    int * s_hcount = reinterpret_cast<int *>(s_hmass + kBuckets);        // [kBuckets]
    uint64_t * s_list = reinterpret_cast<uint64_t *>(s_hcount + kBuckets);  // [kListMaxN]
    const int hw = na.hist_slots > 0 ? (((a.vocab + 31) >> 5) + 3) & ~3 : 0;
    uint32_t * s_hbits = reinterpret_cast<uint32_t *>(s_list + kListMaxN);  // [hw] history columns
    int32_t * s_hkey = reinterpret_cast<int32_t *>(s_hbits + hw);           // [hist_slots]
    int32_t * s_hcnt = s_hkey + na.hist_slots;                              // [hist_slots]
    __shared__ double s_red[kNWarps];
    __shared__ float s_redf[32];
    __shared__ int s_redi[32];
    __shared__ uint64_t s_red64[32];
    __shared__ int s_n, s_lc, s_lc2;
    __shared__ double s_d0, s_d1;
    __shared__ int s_i0, s_i1;

    const int tid = (int) threadIdx.x, lane = lane_id();
    const int vocab = a.vocab;
    uint64_t * list = na.scratch + (int64_t) blockIdx.x * na.scratch_ld;
    const int hbits_n = na.hist_slots > 1 ? 31 - __clz(na.hist_slots) : 1;

    for (int row = blockIdx.x; row < a.rows; row += gridDim.x) {
        const ssb_params pp = a.row_params ? a.row_params[row] : a.params;
        const RowParams p = resolve_params(pp, vocab);
        const bool greedy_row = p.greedy != 0;
        int32_t * id_out = a.ids + row;
        int32_t * st_out = a.status + row;
        if (a.row_params && !p.greedy && p.k > a.k_bound) {
            if (tid == 0) {
                *id_out = -1, *st_out = SSB_ROW_INVALID_ROW;
                if (kDebug && a.dbg_count) a.dbg_count[row] = 0;
            }
            continue;
        }
        const TIn * src = reinterpret_cast<const TIn *>(a.logits) + (int64_t) row * a.ld;
        const uint32_t * mrow = (a.mask && a.mask_kind != SSB_MASK_NONE) ? a.mask + (int64_t) row * a.mask_ld : nullptr;
        const int32_t * hist = a.history ? a.history + (int64_t) row * a.history_ld : nullptr;
        int hlen = 0;
        if (hist) {
            hlen = a.history_len ? a.history_len[row] : (int) a.history_ld;
            hlen = hlen < 0 ? 0 : (hlen > (int) a.history_ld ? (int) a.history_ld : hlen);
        }
        const bool penal = p.history_applies && hlen > 0;
        const float T = greedy_row ? 1.0f : p.temperature;

        // ---- history table: distinct ids with their counts, and the history columns
        if (tid == 0) s_n = 0;
        if (penal) {
            for (int i = tid; i < na.hist_slots; i += kNThreads) s_hkey[i] = -1, s_hcnt[i] = 0;
            for (int i = tid; i < hw; i += kNThreads) s_hbits[i] = 0;
            __syncthreads();
            const uint32_t hmask = (uint32_t) na.hist_slots - 1u;
            for (int i = tid; i < hlen; i += kNThreads) {
                const int32_t t = __ldg(hist + i);
                if (t < 0 || t >= vocab) continue;
                uint32_t h = hash_token(t, hbits_n);
                for (uint32_t n = 0; n <= hmask; n++) {
                    const int32_t old = atomicCAS(&s_hkey[h], -1, t);
                    if (old == -1 || old == t) {
                        atomicAdd(&s_hcnt[h], 1);
                        break;
                    }
                    h = (h + 1) & hmask;
                }
                atomicOr(&s_hbits[t >> 5], 1u << (t & 31));
            }
        }
        __syncthreads();
        // penalized logit of history column col (raw logit v)
        auto penalized = [&](int col, float v) {
            const uint32_t hmask = (uint32_t) na.hist_slots - 1u;
            uint32_t h = hash_token(col, hbits_n);
            for (uint32_t n = 0; n <= hmask && s_hkey[h] != col; n++) h = (h + 1) & hmask;
            return penalize(v, s_hcnt[h], p);
        };
        // restricted logit of column col
        auto restricted = [&](int col) {
            float v = Elem<TIn>::load1(src, col);
            if (penal && ((s_hbits[col >> 5] >> (col & 31)) & 1u)) v = penalized(col, v);
            if (mrow && masked_bit(__ldg(mrow + (col >> 5)) >> (col & 31), a.mask_kind)) v = -kInf;
            return v;
        };

        // ---- pass 1: the row, one mask word (32 columns) per thread and round; the finite scaled logits go
        // to the list as composites, counted per bucket. A chunk of 8 columns that the mask bans whole is
        // -inf without being read (the debug export reads every column, for the restricted logits).
        for (int i = tid; i < kBuckets; i += kNThreads) s_hcount[i] = 0;
        __syncthreads();
        float acc = -kInf;
        int nan_scaled = 0;
        uint64_t best = 0;
        const bool vec = (reinterpret_cast<uintptr_t>(src) & 15u) == 0;  // 16-byte loads of whole chunks
        // a temperature that is a power of two scales exactly by its reciprocal: fl(x * 2^-e) is the
        // correctly rounded x / 2^e, the same number __fdiv_rn gives
        const bool pow2 = T > 0.0f && T < kInf && (__float_as_uint(T) & 0x007FFFFFu) == 0u;
        const float inv_t = pow2 ? __fdiv_rn(1.0f, T) : 0.0f;
        const int nwords = (vocab + 31) >> 5;
        uint32_t next_mw = mrow && tid < nwords ? __ldg(mrow + tid) : 0u;  // the next round's mask word, read ahead
        for (int wbase = 0; wbase < nwords; wbase += kNThreads) {  // uniform trip count
            const int w = wbase + tid;
            const int col0 = w << 5;
            const uint32_t mw = next_mw;
            if (mrow && w + kNThreads < nwords) next_mw = __ldg(mrow + w + kNThreads);
            uint32_t live = 0, allowed = 0, hbw = 0;
            if (w < nwords) {
                live = vocab - col0 >= 32 ? 0xFFFFFFFFu : ((1u << (vocab - col0)) - 1u);
                allowed = live;
                if (mrow) allowed &= a.mask_kind == SSB_MASK_BAN ? ~mw : mw;
                if (penal) hbw = s_hbits[w];
            }
            const uint32_t visit = kDebug ? live : allowed;
            // a sparse round (an allow mask of low density): the warp's visited columns are queued (at most
            // kQueue, in the still unused list buffer) and taken 32 at a time, one per lane, so that no lane
            // idles through a chunk that only one lane of the warp has a token in
            if (!kDebug) {
                const int nv = __popc(visit);
                int incl = nv;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int t = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += t;
                }
                const int total = __shfl_sync(0xffffffffu, incl, 31);
                if (total <= kQueue) {
                    int32_t * q = reinterpret_cast<int32_t *>(s_list) + warp_id() * kQueue;
                    int pos = incl - nv;
                    for (uint32_t bits = visit; bits; bits &= bits - 1u) q[pos++] = col0 + __ffs(bits) - 1;
                    __syncwarp();
                    for (int t0 = 0; t0 < total; t0 += 32) {  // warp-uniform
                        const int t = t0 + lane;
                        uint64_t cv = 0;
                        bool has = false;
                        if (t < total) {
                            const int col = q[t];
                            float v = Elem<TIn>::load1(src, col);
                            if (penal && ((s_hbits[col >> 5] >> (col & 31)) & 1u)) v = penalized(col, v);
                            acc = max_nan(acc, v);
                            const float sc = greedy_row ? v : (pow2 ? __fmul_rn(v, inv_t) : __fdiv_rn(v, T));
                            nan_scaled |= sc != sc;
                            if (sc == sc && sc > -kInf) {
                                cv = composite(sc, (uint32_t) col);
                                has = true;
                                best = cv > best ? cv : best;
                                atomicAdd(&s_hcount[bucket_of(cv)], 1);
                            }
                        }
                        const unsigned m = __ballot_sync(0xffffffffu, has);
                        if (m) {
                            int at = 0;
                            if (lane == __ffs(m) - 1) at = atomicAdd(&s_n, __popc(m));
                            at = __shfl_sync(0xffffffffu, at, __ffs(m) - 1);
                            if (has) list[at + __popc(m & ((1u << lane) - 1u))] = cv;
                        }
                    }
                    __syncwarp();
                    continue;
                }
            }
            // the chunks' logits, read together (16-byte loads where the chunk is whole and aligned)
            constexpr int kPerChunk = 8 * (int) sizeof(TIn) / 16;  // 16-byte loads per 8 columns
            uint4 raw[4 * kPerChunk];
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const bool load = ((visit >> (8 * c)) & 0xFFu) != 0 && vec && ((live >> (8 * c)) & 0xFFu) == 0xFFu;
#pragma unroll
                for (int q = 0; q < kPerChunk; q++)
                    raw[c * kPerChunk + q] = load ? ld_stream(src + col0 + 8 * c + q * (16 / (int) sizeof(TIn))) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const uint32_t vis = (visit >> (8 * c)) & 0xFFu;
                const bool whole = vec && ((live >> (8 * c)) & 0xFFu) == 0xFFu;
                uint64_t cv[8];
                uint32_t has = 0;
                if (vis) {
                    float x[8];
                    if (whole) {
#pragma unroll
                        for (int q = 0; q < kPerChunk; q++) Elem<TIn>::unpack(raw[c * kPerChunk + q], x + q * (8 / kPerChunk));
                    }
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        const int bit = 8 * c + e, col = col0 + bit;
                        if ((vis >> e) & 1u) {
                            float v = whole ? x[e] : Elem<TIn>::load1(src, col);
                            if (!((allowed >> bit) & 1u)) v = -kInf;
                            else if ((hbw >> bit) & 1u) v = penalized(col, v);
                            if (kDebug && a.dbg_processed) a.dbg_processed[(int64_t) row * vocab + col] = v;
                            acc = max_nan(acc, v);
                            if ((allowed >> bit) & 1u) {
                                const float sc = greedy_row ? v : (pow2 ? __fmul_rn(v, inv_t) : __fdiv_rn(v, T));
                                nan_scaled |= sc != sc;
                                if (sc == sc && sc > -kInf) {
                                    cv[e] = composite(sc, (uint32_t) col);
                                    has |= 1u << e;
                                    best = cv[e] > best ? cv[e] : best;
                                    atomicAdd(&s_hcount[bucket_of(cv[e])], 1);
                                }
                            }
                        }
                    }
                }
                if (__any_sync(0xffffffffu, has != 0)) {
                    // one shared atomic per warp: a scan of the lanes' counts gives each its place
                    const int n = __popc(has);
                    int incl = n;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const int t = __shfl_up_sync(0xffffffffu, incl, o);
                        if (lane >= o) incl += t;
                    }
                    int at = 0;
                    if (lane == 31) at = atomicAdd(&s_n, incl);
                    at = __shfl_sync(0xffffffffu, at, 31) + incl - n;
#pragma unroll
                    for (int e = 0; e < 8; e++)
                        if ((has >> e) & 1u) list[at + __popc(has & ((1u << e) - 1u))] = cv[e];
                }
            }
        }
        const float row_max = block_max_nan(acc, s_redf);
        const int nanf = block_or(nan_scaled, s_redi);
        best = block_max_u64(best, s_red64);
        __threadfence_block();
        __syncthreads();
        const int n = s_n;
        int stt = restricted_status(row_max, p.rep);
        if (stt == SSB_ROW_OK && !greedy_row && nanf) stt = SSB_ROW_TEMPERATURE_OVERFLOW;
        if (stt == SSB_ROW_OK && !greedy_row && !(n > 0 && composite_value(best) < kInf)) stt = SSB_ROW_TEMPERATURE_OVERFLOW;
        if (stt != SSB_ROW_OK) {
            if (tid == 0) {
                *id_out = -1, *st_out = stt;
                if (kDebug && a.dbg_count) a.dbg_count[row] = 0;
            }
            __syncthreads();
            continue;
        }
        if (greedy_row) {
            if (tid == 0) {
                *id_out = (int32_t) composite_index(best), *st_out = SSB_ROW_OK;
                if (kDebug && a.dbg_count) a.dbg_count[row] = 1;
                if (kDebug && a.dbg_tokens && a.dbg_cap > 0) a.dbg_tokens[(int64_t) row * a.dbg_cap] = *id_out, a.dbg_weights[(int64_t) row * a.dbg_cap] = 1.0;
            }
            __syncthreads();
            continue;
        }
        const double mx = (double) composite_value(best);
        const float mxf = composite_value(best);
        const double u = a.u ? a.u[row] : 0.0;
        const double tp = p.top_p < 1.0f ? (double) p.top_p : 2.0;  // 2: no cut
        const int kk = p.k;  // the candidates: the kk best (kk may exceed n: the rest are -inf)
        double total = 0.0;

        // In place, from the top bucket down: the tokens (and, with `mass`, the mass) strictly above each.
        auto prefix_above = [&](bool mass) {
            constexpr int kPer = kBuckets / kNThreads;  // buckets per thread, descending from the top
            double m[kPer];
            int c[kPer];
            double ms = 0.0;
            int cs = 0;
#pragma unroll
            for (int j = 0; j < kPer; j++) {
                const int b = kBuckets - 1 - (tid * kPer + j);
                m[j] = mass ? s_hmass[b] : 0.0, c[j] = s_hcount[b];
                ms += m[j], cs += c[j];
            }
            const double mincl = block_scan_incl(ms, s_red);
            const double cdincl = block_scan_incl((double) cs, s_red);  // counts: exact in doubles
            double mb = mincl - ms;
            double cb = cdincl - (double) cs;
            __syncthreads();
#pragma unroll
            for (int j = 0; j < kPer; j++) {
                const int b = kBuckets - 1 - (tid * kPer + j);
                if (mass) s_hmass[b] = mb;
                s_hcount[b] = (int) cb;
                mb += m[j], cb += (double) c[j];
            }
            __syncthreads();
        };
        // The bucket in which the running mass (from the top) first reaches `target` (strict: exceeds),
        // or -1 (needs prefix_above(true)).
        auto crossing_bucket = [&](double target, bool strict) {
            if (tid == 0) s_i0 = -1;
            __syncthreads();
            for (int b = tid; b < kBuckets; b += kNThreads) {
                const double above = s_hmass[b];
                const double incl = b > 0 ? s_hmass[b - 1] : total;  // the next lower bucket's "above"
                const bool in = strict ? (above <= target && incl > target) : (above < target && incl >= target);
                if (in) atomicMax(&s_i0, b);
            }
            __syncthreads();
            const int r = s_i0;
            __syncthreads();  // every thread holds the result before a following call resets s_i0
            return r;
        };
        // Sorts bucket b's tokens of the list (descending) into s_list; returns their count, or -1 if too
        // many for shared memory.
        auto load_bucket = [&](int b, uint64_t floor, bool by_mass) {
            if (tid == 0) s_lc = 0;
            __syncthreads();
            // uniform trip count (the ballot needs every lane); kScanUnroll entries in flight per thread
            for (int base = 0; base < n; base += kNThreads * kScanUnroll) {
                uint64_t cs[kScanUnroll];
#pragma unroll
                for (int q = 0; q < kScanUnroll; q++) {
                    const int i = base + q * kNThreads + tid;
                    cs[q] = i < n ? __ldcg(reinterpret_cast<const unsigned long long *>(list + i)) : 0ull;
                }
#pragma unroll
                for (int q = 0; q < kScanUnroll; q++) {
                    const int i = base + q * kNThreads + tid;
                    const uint64_t c = cs[q];
                    const bool in = i < n && (int) (by_mass ? mass_bucket(c, mxf) : bucket_of(c)) == b && c >= floor;
                    const unsigned m = __ballot_sync(0xffffffffu, in);
                    if (m) {
                        int at = 0;
                        if (lane == __ffs(m) - 1) at = atomicAdd(&s_lc, __popc(m));
                        at = __shfl_sync(0xffffffffu, at, __ffs(m) - 1);
                        const int pos = at + __popc(m & ((1u << lane) - 1u));
                        if (in && pos < kListMaxN) s_list[pos] = c;
                    }
                }
            }
            __syncthreads();
            const int cnt = s_lc;
            if (cnt > kListMaxN) return -1;
            int np2 = 1;
            while (np2 < cnt) np2 <<= 1;
            for (int i = cnt + tid; i < np2; i += kNThreads) s_list[i] = 0ull;
            __syncthreads();
            if (np2 > 1) bitonic_sort_desc(s_list, np2);
            return cnt;
        };
        // One scan for both crossings: the tokens of mass bucket b1 into the first half of s_list and those
        // of buckets lo..hi into the second, each half sorted; a count is -1 when its half overflows.
        auto load_two = [&](int b1, int lo, int hi, uint64_t floor, int & c1, int & c2) {
            constexpr int kHalf = kListMaxN / 2;
            uint64_t * A = s_list;
            uint64_t * B = s_list + kHalf;
            if (tid == 0) s_lc = 0, s_lc2 = 0;
            __syncthreads();
            auto put = [&](bool in, uint64_t c, uint64_t * dst, int * counter) {
                const unsigned m = __ballot_sync(0xffffffffu, in);
                if (m) {
                    int at = 0;
                    if (lane == __ffs(m) - 1) at = atomicAdd(counter, __popc(m));
                    at = __shfl_sync(0xffffffffu, at, __ffs(m) - 1);
                    const int pos = at + __popc(m & ((1u << lane) - 1u));
                    if (in && pos < kHalf) dst[pos] = c;
                }
            };
            for (int base = 0; base < n; base += kNThreads * kScanUnroll) {  // uniform trip count
                uint64_t cs[kScanUnroll];
#pragma unroll
                for (int q = 0; q < kScanUnroll; q++) {
                    const int i = base + q * kNThreads + tid;
                    cs[q] = i < n ? __ldcg(reinterpret_cast<const unsigned long long *>(list + i)) : 0ull;
                }
#pragma unroll
                for (int q = 0; q < kScanUnroll; q++) {
                    const int i = base + q * kNThreads + tid;
                    const uint64_t c = cs[q];
                    const int bk = (i < n && c >= floor) ? (int) mass_bucket(c, mxf) : -1;
                    put(bk == b1, c, A, &s_lc);
                    put(bk >= lo && bk <= hi, c, B, &s_lc2);
                }
            }
            __syncthreads();
            c1 = s_lc <= kHalf ? s_lc : -1;
            c2 = s_lc2 <= kHalf ? s_lc2 : -1;
            __syncthreads();  // every thread holds the counts before load_bucket may reset s_lc
            for (int h = 0; h < 2; h++) {  // block-uniform
                const int cnt = h == 0 ? c1 : c2;
                if (cnt < 0) continue;
                uint64_t * x = h == 0 ? A : B;
                int np2 = 1;
                while (np2 < cnt) np2 <<= 1;
                for (int i = cnt + tid; i < np2; i += kNThreads) x[i] = 0ull;
                __syncthreads();
                if (np2 > 1) bitonic_sort_desc(x, np2);
                __syncthreads();
            }
        };
        // In the sorted bucket list (cnt tokens, mass `above` before it): the first position whose running
        // mass reaches `target` (strict: exceeds it), with the running mass there (s_d0) and just before it
        // (s_d1); -1 when none in the list.
        auto crossing_in_list = [&](const uint64_t * L, int cnt, double above, double target, bool strict) {
            for (int base = 0; base < cnt; base += kNThreads) {  // uniform
                const int i = base + tid;
                const double e = i < cnt ? exp((double) composite_value(L[i]) - mx) : 0.0;
                const double incl = block_scan_incl(e, s_red) + above;
                if (tid == 0) s_i1 = INT_MAX;
                __syncthreads();
                if (i < cnt && (strict ? incl > target : incl >= target)) atomicMin(&s_i1, i);
                __syncthreads();
                const int at = s_i1;
                if (at != INT_MAX) {
                    if (i == at) s_d0 = incl, s_d1 = incl - e;
                    __syncthreads();
                    return at;
                }
                if (tid == kNThreads - 1) s_d1 = incl;  // the running mass through this chunk
                __syncthreads();
                above = s_d1;
                __syncthreads();
            }
            return -1;
        };

        bool exact = kDebug || !(mxf > -kInf && mxf < kInf);  // the mass buckets need a finite maximum
        // the kk-th best composite: the candidates are those at or above it (every finite one when kk >= n)
        uint64_t kth = 0;
        if (!exact && kk < n) {
            prefix_above(false);
            if (tid == 0) s_i0 = -1;
            __syncthreads();
            for (int b = tid; b < kBuckets; b += kNThreads) {
                const int above = s_hcount[b];
                const int incl = b > 0 ? s_hcount[b - 1] : n;
                if (above < kk && incl >= kk) atomicMax(&s_i0, b);
            }
            __syncthreads();
            const int bk = s_i0;
            const int above = bk >= 0 ? s_hcount[bk] : 0;
            const int cnt = bk >= 0 ? load_bucket(bk, 0ull, false) : -1;
            if (cnt < 0 || kk - above - 1 >= cnt) exact = true;
            else kth = s_list[kk - above - 1];
            __syncthreads();
        }

        if (!exact) {
            // ---- pass 2: the candidates' mass, its total and its histogram over the top bits of the key
            for (int i = tid; i < kBuckets; i += kNThreads) s_hmass[i] = 0.0, s_hcount[i] = 0;
            __syncthreads();
            double part = 0.0;
            for (int base = 0; base < n; base += kNThreads * kScanUnroll) {  // kScanUnroll entries in flight
                uint64_t cs[kScanUnroll];
#pragma unroll
                for (int q = 0; q < kScanUnroll; q++) {
                    const int i = base + q * kNThreads + tid;
                    cs[q] = i < n ? __ldcg(reinterpret_cast<const unsigned long long *>(list + i)) : 0ull;
                }
#pragma unroll
                for (int q = 0; q < kScanUnroll; q++) {
                    const uint64_t c = cs[q];
                    if (base + q * kNThreads + tid >= n || c < kth) continue;
                    const double e = exp((double) composite_value(c) - mx);
                    part += e;
                    const uint32_t b = mass_bucket(c, mxf);
                    atomicAdd(&s_hmass[b], e);
                    atomicAdd(&s_hcount[b], 1);
                }
            }
            total = block_sum_double(part, s_red);
            __syncthreads();
            prefix_above(true);
        }

        int keep = 0;
        int32_t chosen_id = -1;
        if (!exact) {
            // the cut: running share >= top_p, i.e. running mass >= tp * total
            int b1 = tp <= 1.0 ? crossing_bucket(tp * total, false) : -2;
            double T1 = total;  // pick()'s total (as running mass)
            int posk = n - 1;   // sorted position of the last kept token
            // the draw's buckets are bounded before the cut is found: pick()'s total T1 lies in b1's share
            // of the running mass, (above(b1), above(b1 - 1)], so the draw's target u * T1 lies between u
            // times those two; for a long list one scan then loads b1 and that range (a short list is
            // scanned twice more cheaply than the two bucket searches this costs)
            int lo2 = -1, hi2 = -1, cnt2 = -1;
            const uint64_t * L2 = s_list + kListMaxN / 2;
            if (b1 >= 0 && n >= kMergedScanMin) {
                const double a1 = s_hmass[b1], i1 = b1 > 0 ? s_hmass[b1 - 1] : total;
                hi2 = crossing_bucket(u * a1, true);
                lo2 = crossing_bucket(u * i1, true);
            }
            if (b1 == -1) {
                exact = true;
            } else if (b1 >= 0) {
                int cnt = -1;
                if (lo2 >= 0 && hi2 >= lo2) load_two(b1, lo2, hi2, kth, cnt, cnt2);
                if (cnt < 0) {
                    cnt2 = -1;
                    cnt = load_bucket(b1, kth, true);
                }
                if (cnt < 0) {
                    exact = true;
                } else {
                    const int j = crossing_in_list(s_list, cnt, s_hmass[b1], tp * total, false);
                    if (j < 0) {
                        exact = true;
                    } else {
                        const double at = s_d0 / total, before = s_d1 / total;
                        if (!(at - tp > kMargin && tp - before > kMargin)) exact = true;
                        T1 = s_d0;
                        posk = s_hcount[b1] + j;
                    }
                }
            } else {
                // no cut (top_p >= 1): every finite token is kept; the -inf ones add nothing, but pick()
                // runs over all of them and the last is its fallback: the exact path handles that
                exact = true;
            }
            if (!exact) {
                keep = posk + 1;
                // the draw: pick()'s running sum over the first keep - 1 > u, i.e. running mass > u * T1
                const double target = u * T1;
                const int b2 = crossing_bucket(target, true);
                if (b2 < 0) {
                    exact = true;
                } else {
                    // the range loaded with b1 when it holds b2, else b2 alone (over b1's list: the cut is done)
                    const bool ranged = cnt2 >= 0 && b2 >= lo2 && b2 <= hi2;
                    const int top = ranged ? hi2 : b2;
                    const uint64_t * L = ranged ? L2 : s_list;
                    const int cnt = ranged ? cnt2 : load_bucket(b2, kth, true);
                    if (cnt < 0) {
                        exact = true;
                    } else {
                        const int j = crossing_in_list(L, cnt, s_hmass[top], target, true);
                        if (j < 0) {
                            exact = true;
                        } else {
                            const double at = s_d0 / T1, before = s_d1 / T1;
                            if (!(at - u > kMargin && u - before > kMargin)) exact = true;
                            const int pos = s_hcount[top] + j;
                            if (pos >= keep - 1) {
                                // no running sum of the first keep - 1 exceeds u: the last kept token
                                if (posk == pos) chosen_id = (int32_t) composite_index(L[j]);
                                else exact = true;  // the last kept token lies in another bucket
                            } else {
                                chosen_id = (int32_t) composite_index(L[j]);
                            }
                        }
                    }
                }
            }
        }

        if (exact) {
            // ---- the exact path: the whole list sorted, the reference's sums in its order
            int np2 = 1;
            while (np2 < n) np2 <<= 1;
            for (int i = n + tid; i < np2; i += kNThreads) list[i] = 0ull;
            __threadfence_block();
            __syncthreads();
            global_bitonic_desc(list, np2);
            double * w = reinterpret_cast<double *>(s_hmass);  // [kChunk] values of the current chunk
            const int mk = min(kk, n);  // the finite candidates
            // softmax total over the candidates in order (the -inf ones add exactly 0)
            double S = 0.0;
            for (int base = 0; base < mk; base += kChunk) {
                const int m = min(kChunk, mk - base);
                for (int i = tid; i < m; i += kNThreads)
                    w[i] = exp((double) composite_value(__ldcg(reinterpret_cast<const unsigned long long *>(list + base + i))) - mx);
                __syncthreads();
                if (tid == 0) {
                    double unused;
                    (void) unused;
                    for (int i = 0; i < m; i++) S = __dadd_rn(S, w[i]);
                }
                __syncthreads();
            }
            if (tid == 0) s_d0 = S;
            __syncthreads();
            S = s_d0;
            // top-p cut: first running share >= top_p (keep = all when none)
            double C = 0.0;
            int kp = -1;
            for (int base = 0; base < mk && kp < 0; base += kChunk) {
                const int m = min(kChunk, mk - base);
                for (int i = tid; i < m; i += kNThreads) {
                    const double wi = __ddiv_rn(exp((double) composite_value(__ldcg(reinterpret_cast<const unsigned long long *>(list + base + i))) - mx), S);
                    w[i] = wi;
                    if (kDebug && a.dbg_tokens && base + i < a.dbg_cap) {
                        a.dbg_tokens[(int64_t) row * a.dbg_cap + base + i] =
                            (int32_t) composite_index(__ldcg(reinterpret_cast<const unsigned long long *>(list + base + i)));
                        a.dbg_weights[(int64_t) row * a.dbg_cap + base + i] = wi;
                    }
                }
                __syncthreads();
                if (tid == 0) {
                    for (int i = 0; i < m; i++) {
                        C = __dadd_rn(C, w[i]);
                        if (p.top_p < 1.0f && C >= (double) p.top_p) {
                            s_i0 = base + i;
                            break;
                        }
                    }
                    if (!(p.top_p < 1.0f && C >= (double) p.top_p)) s_i0 = -1;
                    s_d0 = C;
                }
                __syncthreads();
                kp = s_i0;
                C = s_d0;
                __syncthreads();
            }
            // keep: through the cut, or every candidate (the -inf ones too) when no share reaches top_p
            keep = kp >= 0 ? kp + 1 : kk;
            const double Tk = C;  // the running sum through keep - 1 (zeros change nothing)
            // pick() over the first keep - 1: first running sum > u, else the last kept token
            double D = 0.0;
            int ch = -1;
            const int lim = min(keep - 1, mk);
            for (int base = 0; base < lim && ch < 0; base += kChunk) {
                const int m = min(kChunk, lim - base);
                for (int i = tid; i < m; i += kNThreads)
                    w[i] = __ddiv_rn(__ddiv_rn(exp((double) composite_value(__ldcg(reinterpret_cast<const unsigned long long *>(list + base + i))) - mx), S), Tk);
                __syncthreads();
                if (tid == 0) {
                    s_i1 = -1;
                    for (int i = 0; i < m; i++) {
                        D = __dadd_rn(D, w[i]);
                        if (D > u) {
                            s_i1 = base + i;
                            break;
                        }
                    }
                }
                __syncthreads();
                ch = s_i1;
                __syncthreads();
            }
            const int pos = ch >= 0 ? ch : keep - 1;
            if (pos < n) {
                chosen_id = (int32_t) composite_index(__ldcg(reinterpret_cast<const unsigned long long *>(list + pos)));
            } else {
                // a token whose scaled logit is -inf: the (pos - n)-th of them by index
                const int want = pos - n;
                if (tid == 0) s_i0 = -1, s_lc = 0;
                __syncthreads();
                for (int base = 0; base < vocab; base += kNThreads) {
                    const int col = base + tid;
                    bool ninf = false;
                    if (col < vocab) {
                        const float v = restricted(col);
                        const float sc = __fdiv_rn(v, T);
                        ninf = !(sc == sc && sc > -kInf);
                    }
                    const int before = s_lc;
                    const double incl = block_scan_incl(ninf ? 1.0 : 0.0, s_red);
                    const int r = before + (int) incl - 1;
                    if (ninf && r == want) s_i0 = col;
                    __syncthreads();
                    if (tid == kNThreads - 1) s_lc = before + (int) incl;
                    __syncthreads();
                    if (s_i0 >= 0) break;
                }
                chosen_id = s_i0;
            }
            if (kDebug && a.dbg_count && tid == 0) a.dbg_count[row] = keep;
        }
        if (tid == 0) {
            *id_out = chosen_id, *st_out = SSB_ROW_OK;
            if (kDebug && a.dbg_count && !exact) a.dbg_count[row] = keep;
        }
        __syncthreads();
    }
}

template <typename TIn, bool kDebug>
void * kernel_ptr() {
    return reinterpret_cast<void *>(nucleus_rows_kernel<TIn, kDebug>);
}

void * pick_kernel(bool bf16, bool debug) {
    if (bf16) return debug ? kernel_ptr<uint16_t, true>() : kernel_ptr<uint16_t, false>();
    return debug ? kernel_ptr<float, true>() : kernel_ptr<float, false>();
}

}  // namespace

size_t nucleus_smem_bytes(int vocab, int hist_slots) {
    const size_t hw = hist_slots > 0 ? (size_t) ((((vocab + 31) >> 5) + 3) & ~3) : 0;
    return (size_t) kBuckets * 12 + (size_t) kListMaxN * 8 + hw * 4 + (size_t) hist_slots * 8;
}

int64_t nucleus_scratch_ld(int vocab) {
    int64_t np2 = 1;
    while (np2 < vocab) np2 <<= 1;
    return np2;
}

int nucleus_threads() { return kNThreads; }

int nucleus_blocks_per_sm(bool bf16, size_t smem) {
    void * kern = pick_kernel(bf16, false);
    if (ssb::set_max_dynamic_smem((const void *) kern, smem) != cudaSuccess) return 0;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kNThreads, smem) != cudaSuccess) return 0;
    return n;
}

cudaError_t launch_nucleus(const NucleusArgs & a, int grid, bool bf16, bool debug, cudaStream_t stream) {
    const size_t smem = nucleus_smem_bytes(a.r.vocab, a.hist_slots);
    void * kern = pick_kernel(bf16, debug);
    cudaError_t e = ssb::set_max_dynamic_smem((const void *) kern, smem);
    if (e != cudaSuccess) return e;
    void * args[] = {const_cast<NucleusArgs *>(&a)};
    return cudaLaunchKernel(kern, dim3((unsigned) grid), dim3(kNThreads), args, smem, stream);
}

}  // namespace ssb
