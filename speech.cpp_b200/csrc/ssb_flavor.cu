// The other families' candidate rules on the device: Haru's text sampler (haru::candidates,
// src/families/haru/sampler.cpp:18-61) and Drama 3's (drama3::candidates, src/families/drama3/sampler.cpp:30-60),
// each followed by pick() (src/common/sampling.cpp:9-19) with the row's replayed uniform. One CTA per row,
// at most kFlavorMaxK candidates.
//
// Per row: the restricted logits (the engine's penalties and mask, qwen3-tts/sampler.cpp:29-42 and the
// extensions, applied before the family's rule; with none given they are the stored logits), then the
// family's checks, then the k best by scaled logit (falling, ties by lowest index: both families'
// comparators) by radix select over the row (read again from L2), sorted in shared memory, then the
// family's weights and the draw:
//
//   Haru    NaN or +inf anywhere -> NON_FINITE_INPUT (:21-23); T <= 0 -> the first maximum (:26-30);
//           scaled = l / T, a finite logit scaled beyond float -> TEMPERATURE_OVERFLOW (:31-35);
//           k = top_k if 0 < top_k < V else V; the float32 softmax: exp(s_i - s_0) summed in order,
//           each divided by the sum (:43-49); where 0 < top_p < 1, a weight whose running float sum
//           less itself does not stay below top_p becomes 0 (:52-59).
//   Drama3  any non-finite logit -> NON_FINITE_INPUT (:35-37); t = max(T, 1e-5); k = min(max(top_k, 1), V);
//           top = the largest scaled logit, non-finite -> TEMPERATURE_OVERFLOW (:46-47); the double sum
//           of exp(s - top) over every token in index order (:48-49); the tokens by falling scaled logit
//           are kept while the running share of exp(s - top) / sum stays at most top_p, the first always
//           (:50-58), with weight exp(s - top). Tokens the mask bans are not candidates (the reference's
//           rows hold no -inf), a row with none left is NO_FINITE_LOGIT.
//
// Drama 3's sum runs over the whole row; it is summed in parallel, and each top-p comparison of the
// running share is decided when it clears top_p by a margin (1e-9 plus V times the double epsilon:
// above the largest difference between any two orders of adding V positive terms); otherwise warp 0
// recomputes the sum in the reference's index order. Haru's float32 exponentials are exp in double
// rounded once to float; the reference's expf is within an ulp of that, which its own check allows for
// ((k + 64) 2^-24, checks/haru/haru-sampling-check.cpp:36). The double exponentials of Drama 3 and the
// qwen3-tts path agree with the host's exp to an ulp in the same way.
#include <climits>
#include <cuda_bf16.h>

#include "ssb_device.cuh"
#include "ssb_kernels.h"
#include "ssb_tma.cuh"  // hash_token

namespace ssb {

namespace {

constexpr int kFlThreads = 512;
constexpr double kFlMargin = 1e-9;
constexpr double kFlEps = 0x1p-52;  // the double epsilon

// Slot of token t in the history table (keys -1 = empty), or -1.
__device__ __forceinline__ int fl_find(const int32_t * keys, int slots, int bits, int32_t t) {
    const uint32_t mask = (uint32_t) slots - 1u;
    uint32_t h = hash_token(t, bits);
    for (uint32_t n = 0; n <= mask; n++) {
        const int32_t key = keys[h];
        if (key == t) return (int) h;
        if (key == -1) return -1;
        h = (h + 1) & mask;
    }
    return -1;
}

// pick() (sampling.cpp:9-19) over w[0 .. n), n >= 1, by the whole block: the ordered sum (one thread),
// each share w_i / sum (every thread; w is overwritten), then the first running share > u among the
// first n - 1, else the last (one thread). Every thread returns the index.
__device__ int fl_pick(double * w, int n, double u, double * s_sum, int * s_at) {
    if (threadIdx.x == 0) {
        double sum;
        chain_reach(w, n, kInf, true, &sum);
        *s_sum = sum;
    }
    __syncthreads();
    const double sum = *s_sum;
    for (int i = (int) threadIdx.x; i < n - 1; i += kFlThreads) w[i] = __ddiv_rn(w[i], sum);
    __syncthreads();
    if (threadIdx.x == 0) {
        double unused;
        *s_at = chain_reach(w, n - 1, u, true, &unused);
    }
    __syncthreads();
    return *s_at;
}

// The running float sum of x[0 .. n) in index order (one thread), eight loads issued ahead of the adds.
__device__ float fl_sum_f32(const float * x, int n) {
    float s = 0.0f;
    for (int i0 = 0; i0 < n; i0 += 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = i0 + j < n ? x[i0 + j] : 0.0f;
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (i0 + j < n) s = __fadd_rn(s, v[j]);
    }
    return s;
}

template <typename TIn, bool kDebug>
__global__ void __launch_bounds__(kFlThreads) flavor_rows_kernel(const __grid_constant__ FlavorArgs fa) {
    const RowsArgs & a = fa.r;
    extern __shared__ __align__(16) unsigned char smem[];
    const int cap = fa.cap;
    uint64_t * s_cand = reinterpret_cast<uint64_t *>(smem);                // [cap] the k best, falling
    double * s_w = reinterpret_cast<double *>(s_cand + cap);               // [cap] weights
    float * s_pf = reinterpret_cast<float *>(s_w + cap);                   // [cap] Haru's float32 softmax
    uint32_t * s_bits = reinterpret_cast<uint32_t *>(s_pf + cap);          // [bit_words] history columns
    int32_t * s_hkey = reinterpret_cast<int32_t *>(s_bits + fa.bit_words);
    int32_t * s_hcnt = s_hkey + fa.hist_slots;
    __shared__ SelectState sel;
    __shared__ int s_redi[32];
    __shared__ uint64_t s_red64[32];
    __shared__ double s_redd[32];
    __shared__ int s_n, s_i0;
    __shared__ double s_d0;

    const int row = blockIdx.x, tid = (int) threadIdx.x, lane = lane_id(), warp = warp_id();
    const int vocab = a.vocab;
    const ssb_params pp = a.row_params ? a.row_params[row] : a.params;
    const RowParams p = resolve_params(pp, vocab);
    int32_t * const id_out = a.ids + row;
    int32_t * const st_out = a.status + row;
    int32_t * const cnt_out = kDebug && a.dbg_count ? a.dbg_count + row : nullptr;
    int32_t * const tok_out = kDebug && a.dbg_tokens ? a.dbg_tokens + (int64_t) row * a.dbg_cap : nullptr;
    double * const w_out = kDebug && a.dbg_weights ? a.dbg_weights + (int64_t) row * a.dbg_cap : nullptr;
    auto finish = [&](int id, int st, int count) {
        if (tid == 0) {
            *id_out = id, *st_out = st;
            if (cnt_out) *cnt_out = count;
        }
    };
    auto export_entries = [&](int n) {  // the candidate export: tokens and weights, falling
        if (tok_out)
            for (int i = tid; i < n && i < a.dbg_cap; i += kFlThreads)
                tok_out[i] = (int32_t) composite_index(s_cand[i]), w_out[i] = s_w[i];
    };
    const bool haru = pp.flavor == SSB_FLAVOR_HARU;
    const float T = pp.temperature;
    const bool greedy = pp.greedy || (haru && T <= 0.0f);
    // Haru: k = top_k where 0 < top_k < V, else V (:36); Drama 3: min(max(top_k, 1), V) (:40)
    int k = haru ? (pp.top_k > 0 && pp.top_k < vocab ? pp.top_k : vocab) : min(max(pp.top_k, 1), vocab);
    // a row of another family, or one whose candidates exceed the launch's capacity
    if (pp.flavor != fa.flavor || (!greedy && k > cap)) {
        finish(-1, SSB_ROW_INVALID_ROW, 0);
        return;
    }
    const TIn * src = reinterpret_cast<const TIn *>(a.logits) + (int64_t) row * a.ld;
    const int32_t * hist = a.history ? a.history + (int64_t) row * a.history_ld : nullptr;
    int hlen = 0;
    if (hist) {
        hlen = a.history_len ? a.history_len[row] : (int) a.history_ld;
        hlen = hlen < 0 ? 0 : (hlen > (int) a.history_ld ? (int) a.history_ld : hlen);
    }
    const bool penal = p.history_applies && hlen > 0;
    const uint32_t * mrow = (a.mask && a.mask_kind != SSB_MASK_NONE) ? a.mask + (int64_t) row * a.mask_ld : nullptr;
    const int slots = fa.hist_slots;
    const int hbits_n = slots > 1 ? 31 - __clz(slots) : 1;
    const bool use_bits = penal && fa.bit_words >= ((vocab + 31) >> 5);

    // ---- history table (distinct ids with counts) and the history-column bitmap
    if (penal) {
        for (int i = tid; i < slots; i += kFlThreads) s_hkey[i] = -1, s_hcnt[i] = 0;
        if (use_bits)
            for (int i = tid; i < fa.bit_words; i += kFlThreads) s_bits[i] = 0;
        __syncthreads();
        const uint32_t hmask = (uint32_t) slots - 1u;
        for (int i = tid; i < hlen; i += kFlThreads) {
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
            if (use_bits) atomicOr(&s_bits[t >> 5], 1u << (t & 31));
        }
    }
    __syncthreads();
    // the restricted logit of column `col` whose stored logit is v: the history's penalties, then the mask
    auto restrict_col = [&](float v, int col) {
        if (penal && (!use_bits || ((s_bits[col >> 5] >> (col & 31)) & 1u))) {
            const int s = fl_find(s_hkey, slots, hbits_n, col);
            if (s >= 0) v = penalize(v, s_hcnt[s], p);
        }
        if (mrow && masked_bit(__ldg(mrow + (col >> 5)) >> (col & 31), a.mask_kind)) v = -kInf;
        return v;
    };
    auto restricted = [&](int col) { return restrict_col(Elem<TIn>::load1(src, col), col); };
    const float t_div = haru ? T : fmaxf(T, 1e-5f);  // Drama 3 divides by 1e-5 at the least (:31)
    auto scaled = [&](float r) { return __fdiv_rn(r, t_div); };

    // ---- pass A: the family's checks and, for greedy rows, the first maximum. Haru refuses NaN and +inf
    // among the logits it is given (the restricted ones, where -inf is a banned token); Drama 3 refuses
    // a stored logit that is not finite, and a penalty that made one NaN or +inf (a mask's -inf bans).
    int bad = 0, ovf = 0;
    uint64_t best = 0;
    for (int base = 0; base < vocab; base += 4 * kFlThreads) {
        float x4[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int col = base + q * kFlThreads + tid;
            x4[q] = col < vocab ? Elem<TIn>::load1(src, col) : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int col = base + q * kFlThreads + tid;
            if (col >= vocab) continue;
            const float r = restrict_col(x4[q], col);
            if (kDebug && a.dbg_processed) a.dbg_processed[(int64_t) row * vocab + col] = r;
            bad |= (r != r || r == kInf) || (!haru && !(x4[q] > -kInf && x4[q] < kInf));
            if (greedy) {
                const uint64_t c = composite(r, (uint32_t) col);
                best = c > best ? c : best;
            } else if (haru) {
                const float s = scaled(r);
                ovf |= (r > -kInf && r < kInf) && !(s > -kInf && s < kInf);
            }
        }
    }
    bad = block_or(bad, s_redi);
    ovf = block_or(ovf, s_redi);
    best = block_max_u64(best, s_red64);
    if (bad) {
        finish(-1, SSB_ROW_NON_FINITE_INPUT, 0);
        return;
    }
    if (greedy) {
        const int id = (int) composite_index(best);
        finish(id, SSB_ROW_OK, 1);
        if (tid == 0 && tok_out && a.dbg_cap > 0) tok_out[0] = id, w_out[0] = 1.0;
        return;
    }
    if (ovf) {
        finish(-1, SSB_ROW_TEMPERATURE_OVERFLOW, 0);
        return;
    }

    // ---- the k best scaled logits, falling, ties by lowest index
    auto key_of = [&](int col) { return composite(scaled(restricted(col)), (uint32_t) col); };
    if (k < vocab) radix_select(vocab, k, key_of, sel);
    const int kp2 = next_pow2(k);
    for (int i = tid; i < kp2; i += kFlThreads) s_cand[i] = 0ull;
    if (tid == 0) s_n = 0;
    __syncthreads();
    for (int base = 0; base < vocab; base += kFlThreads) {  // uniform trip count: the ballot needs every lane
        const int col = base + tid;
        const uint64_t c = col < vocab ? key_of(col) : 0ull;
        const bool take = col < vocab && (k >= vocab || selected(c, sel));
        const unsigned m = __ballot_sync(0xffffffffu, take);
        if (m) {
            int at = 0;
            if (lane == __ffs(m) - 1) at = atomicAdd(&s_n, __popc(m));
            at = __shfl_sync(0xffffffffu, at, __ffs(m) - 1) + __popc(m & ((1u << lane) - 1u));
            if (take && at < kp2) s_cand[at] = c;
        }
    }
    __syncthreads();
    bitonic_sort_desc(s_cand, kp2);
    const double u = a.u ? a.u[row] : 0.0;
    const float s0 = composite_value(s_cand[0]);

    if (haru) {
        // float32 softmax (haru/sampler.cpp:43-49): exp of s_i - s_0 rounded once to float, their float
        // sum in order, each divided by it
        for (int i = tid; i < k; i += kFlThreads) s_pf[i] = (float) exp((double) __fsub_rn(composite_value(s_cand[i]), s0));
        __syncthreads();
        if (tid == 0) s_d0 = (double) fl_sum_f32(s_pf, k);
        __syncthreads();
        const float sum = (float) s_d0;
        for (int i = tid; i < k; i += kFlThreads) s_pf[i] = __fdiv_rn(s_pf[i], sum);
        __syncthreads();
        // top-p (:52-59): a weight whose running float sum less itself is not below top_p becomes 0
        if (pp.top_p > 0.0f && pp.top_p < 1.0f) {
            if (tid == 0) {
                float cumulative = 0.0f;
                for (int i0 = 0; i0 < k; i0 += 8) {
                    float v[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) v[j] = i0 + j < k ? s_pf[i0 + j] : 0.0f;
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        if (i0 + j < k) {
                            cumulative = __fadd_rn(cumulative, v[j]);
                            s_w[i0 + j] = __fsub_rn(cumulative, v[j]) < pp.top_p ? (double) v[j] : 0.0;
                        }
                    }
                }
            }
        } else {
            for (int i = tid; i < k; i += kFlThreads) s_w[i] = (double) s_pf[i];
        }
        __syncthreads();
        export_entries(k);
        __syncthreads();
        const int chosen = fl_pick(s_w, k, u, &s_d0, &s_i0);
        finish((int) composite_index(s_cand[chosen]), SSB_ROW_OK, k);
        return;
    }

    // ---- Drama 3 (drama3/sampler.cpp:46-58)
    if (!(s0 > -kInf && s0 < kInf)) {
        finish(-1, s0 == -kInf ? SSB_ROW_NO_FINITE_LOGIT : SSB_ROW_TEMPERATURE_OVERFLOW, 0);
        return;
    }
    // Tokens the mask banned (or a penalty took to -inf, which the reference's rows never hold) are no
    // candidates: k stops before the first -inf, which sorts after every finite value.
    if (tid == 0) s_n = k;
    __syncthreads();
    for (int i = tid; i < k; i += kFlThreads)
        if (composite_value(s_cand[i]) == -kInf && composite_value(s_cand[i - 1]) != -kInf) s_n = i;  // i >= 1: s_cand[0] is finite
    __syncthreads();
    k = s_n;
    __syncthreads();
    const double top = (double) s0;
    // the sum of exp(s - top) over every token, in parallel
    double part = 0.0;
    for (int base = 0; base < vocab; base += 4 * kFlThreads) {
        float r4[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int col = base + q * kFlThreads + tid;
            r4[q] = col < vocab ? restricted(col) : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < 4; q++)
            if (base + q * kFlThreads + tid < vocab) part += exp((double) scaled(r4[q]) - top);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (lane == 0) s_redd[warp] = part;
    // the weights exp(s - top) of the k best
    for (int i = tid; i < k; i += kFlThreads) s_w[i] = exp((double) composite_value(s_cand[i]) - top);
    __syncthreads();
    // the kept count: the first r > 0 whose running share w_0 / S + ... + w_r / S passes top_p (all k when
    // none). With the parallel S each comparison must clear top_p by the margin; otherwise the reference's
    // index-order S decides.
    const double margin = kFlMargin + (double) vocab * kFlEps;
    auto kept_with = [&](double S, bool check, bool * sure) {
        double cum = 0.0;
        for (int r0 = 0; r0 < k; r0 += 8) {
            double q[8];
#pragma unroll
            for (int j = 0; j < 8; j++) q[j] = r0 + j < k ? __ddiv_rn(s_w[r0 + j], S) : 0.0;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int r = r0 + j;
                if (r >= k) break;
                cum = __dadd_rn(cum, q[j]);
                if (r > 0) {
                    if (check && fabs(cum - (double) pp.top_p) <= margin) *sure = false;
                    if (cum > (double) pp.top_p) return r;
                }
            }
        }
        return k;
    };
    if (tid == 0) {
        double S = 0.0;
        for (int w = 0; w < kFlThreads / 32; w++) S += s_redd[w];
        bool sure = true;
        const int kept = kept_with(S, true, &sure);
        s_i0 = sure ? kept : -1;
    }
    __syncthreads();
    if (s_i0 < 0) {
        // too close to call: the reference's sum in its order (warp 0 computes 32 terms at a time, every
        // lane adds them in order), then the same comparisons
        if (warp == 0) {
            double S = 0.0;
            for (int base = 0; base < vocab; base += 32) {
                const int col = base + lane;
                const double e = col < vocab ? exp((double) scaled(restricted(col)) - top) : 0.0;
                const int n = min(32, vocab - base);
                for (int j = 0; j < n; j++) S = __dadd_rn(S, __shfl_sync(0xffffffffu, e, j));
            }
            if (lane == 0) {
                bool unused = true;
                s_i0 = kept_with(S, false, &unused);
            }
        }
        __syncthreads();
    }
    const int kept = s_i0;
    export_entries(kept);
    __syncthreads();
    const int chosen = fl_pick(s_w, kept, u, &s_d0, &s_n);
    finish((int) composite_index(s_cand[chosen]), SSB_ROW_OK, kept);
}

template <typename TIn, bool kDebug>
cudaError_t launch_t(const FlavorArgs & a, size_t smem, cudaStream_t stream) {
    auto kern = flavor_rows_kernel<TIn, kDebug>;
    cudaError_t e = ssb::set_max_dynamic_smem((const void *) kern, smem);
    if (e != cudaSuccess) return e;
    kern<<<a.r.rows, kFlThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace

size_t flavor_smem_bytes(int cap, int bit_words, int hist_slots) {
    return (size_t) cap * 20 + (size_t) bit_words * 4 + (size_t) hist_slots * 8;
}

cudaError_t launch_flavor(const FlavorArgs & a, bool bf16, bool debug, cudaStream_t stream) {
    const size_t smem = flavor_smem_bytes(a.cap, a.bit_words, a.hist_slots);
    if (bf16) return debug ? launch_t<uint16_t, true>(a, smem, stream) : launch_t<uint16_t, false>(a, smem, stream);
    return debug ? launch_t<float, true>(a, smem, stream) : launch_t<float, false>(a, smem, stream);
}

}  // namespace ssb
