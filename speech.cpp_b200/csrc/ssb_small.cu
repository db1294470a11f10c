// Small-vocabulary rows (vocab <= SSB_SMALL_VOCAB): one CTA samples one row entirely from shared
// memory. This is the path of the Qwen3-TTS talker (3072 codes) and code predictor (2048 codes).
//
// Per row, in the reference's order (src/families/qwen3-tts/sampler.cpp):
//   1. load the row into shared memory as fp32 (bf16 widened exactly);
//   2. repetition penalty once per distinct in-range history id (:33-39; a shared count table plays the
//      reference's `seen` bitmap), then the presence/frequency extension;
//   3. ban/allow mask -> -inf (:40-42);
//   4. max -> PENALTY_OVERFLOW / NO_FINITE_LOGIT (:43-49), NaN -> NON_FINITE_INPUT (steps 2-5's per-element
//      work is one pass; the row's statistics meet in one shared atomic per warp);
//   5. greedy: first maximum (:105-108); else scale by the temperature (:73), top-k (k <= 128: the k-th
//      largest 16-bit key from two histograms, the composites reaching it ranked; otherwise a radix select
//      on composite keys and a sort of the k), softmax in double, top-p, pick (:76-99, sampling.cpp:9-19).
#include "ssb_device.cuh"
#include "ssb_kernels.h"

namespace ssb {

namespace {

constexpr int kSmallThreads = 512;
constexpr int kFastK = 128;                // top-k of the histogram path
constexpr int kFastCand = kSmallThreads;   // candidates it ranks (one per thread); more take the general path

template <typename TIn, bool kDebug>
__global__ void __launch_bounds__(kSmallThreads) small_rows_kernel(const SmallArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ SelectState sel;

    const int row = blockIdx.x;
    const int vocab = a.vocab;
    const ssb_params pp = a.row_params ? a.row_params[row] : a.params;
    const RowParams p = resolve_params(pp, vocab);
    int32_t * id_out = a.ids + row;
    int32_t * status_out = a.status + row;
    RowOut out{id_out, status_out, nullptr, nullptr, nullptr, 0};
    if (kDebug) {
        out.tokens = a.dbg_tokens ? a.dbg_tokens + (int64_t) row * a.dbg_cap : nullptr;
        out.weights = a.dbg_weights ? a.dbg_weights + (int64_t) row * a.dbg_cap : nullptr;
        out.count = a.dbg_count ? a.dbg_count + row : nullptr;
        out.cap = a.dbg_cap;
    }
    if (a.row_params && !p.greedy && p.k > a.k_bound) {
        if (threadIdx.x == 0) *id_out = -1, *status_out = SSB_ROW_INVALID_ROW;
        if (kDebug && out.count && threadIdx.x == 0) *out.count = 0;
        return;
    }

    float * s_val = reinterpret_cast<float *>(smem);                       // [vocab]
    unsigned char * s_after = smem + (((size_t) vocab * 4 + 15) & ~(size_t) 15);
    uint32_t * s_cnt = reinterpret_cast<uint32_t *>(s_after);               // [vocab], aliased below

    const TIn * src = reinterpret_cast<const TIn *>(a.logits) + (int64_t) row * a.ld;
    const int32_t * hist = a.history ? a.history + (int64_t) row * a.history_ld : nullptr;
    int hlen = 0;
    if (hist) {
        hlen = a.history_len ? a.history_len[row] : (int) a.history_ld;
        hlen = hlen < 0 ? 0 : (hlen > (int) a.history_ld ? (int) a.history_ld : hlen);
    }
    const bool penal = p.history_applies && hlen > 0;
    // each thread's first history id is requested with the logits, eight of which are in flight per thread
    const int32_t h_first = penal && (int) threadIdx.x < hlen ? __ldg(hist + threadIdx.x) : -1;
    for (int base = 0; base < vocab; base += 8 * kSmallThreads) {
        float v[8];
#pragma unroll
        for (int q = 0; q < 8; q++) {
            const int i = base + q * kSmallThreads + (int) threadIdx.x;
            v[q] = i < vocab ? Elem<TIn>::load1(src, i) : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < 8; q++) {
            const int i = base + q * kSmallThreads + (int) threadIdx.x;
            if (i < vocab) s_val[i] = v[q];
        }
    }

    const bool fastk = !p.greedy && p.k <= kFastK;
    __shared__ __align__(16) uint32_t s_h1[256];
    __shared__ __align__(16) uint32_t s_h2[256];
    __shared__ uint32_t s_rawkey;           // the largest order key of a non-NaN restricted logit (0: none)
    __shared__ int s_flags;                 // bit 0: a NaN restricted logit; bit 1: a NaN scaled logit
    __shared__ unsigned long long s_best;   // greedy: the largest composite of the restricted logits
    __shared__ int s_nc;
    for (int i = threadIdx.x; i < 256; i += blockDim.x) s_h1[i] = 0, s_h2[i] = 0;
    if (threadIdx.x == 0) s_rawkey = 0, s_flags = 0, s_best = 0ull, s_nc = 0;

    // ---- penalties over the history
    if (penal) {
        for (int i = threadIdx.x; i < vocab; i += blockDim.x) s_cnt[i] = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < hlen; i += blockDim.x) {
            const int32_t t = i == (int) threadIdx.x ? h_first : hist[i];
            if (t >= 0 && t < vocab) atomicAdd(&s_cnt[t], 1u);
        }
    }
    __syncthreads();

    // ---- one pass: penalties, mask, processed output and the row's statistics; for a drawing row the
    // logits scaled by the temperature (qwen3-tts/sampler.cpp:73, every logit, -inf included, divided in
    // fp32) and counted in the first key histogram. The statistics meet in one shared atomic per warp.
    const uint32_t * mrow = (a.mask && a.mask_kind != SSB_MASK_NONE) ? a.mask + (int64_t) row * a.mask_ld : nullptr;
    uint32_t mkey = 0;
    int flags = 0;
    uint64_t best = 0;  // greedy: composite of the unscaled value (first maximum = lowest index on ties)
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
        float v = s_val[i];
        if (penal) {
            const uint32_t c = s_cnt[i];
            if (c) v = penalize(v, (int) c, p);
        }
        if (mrow && masked_bit(mrow[i >> 5] >> (i & 31), a.mask_kind)) v = -kInf;
        if (kDebug && a.dbg_processed) a.dbg_processed[(int64_t) row * vocab + i] = v;
        if (v != v) flags |= 1;
        else mkey = max(mkey, order_key(v));
        if (p.greedy) {
            const uint64_t c = composite(v, (uint32_t) i);
            best = c > best ? c : best;
        } else {
            const float sc = __fdiv_rn(v, p.temperature);
            if (sc != sc) flags |= 2;
            s_val[i] = sc;
            if (fastk) red_bin(s_h1, true, order_key(sc) >> 24);
        }
    }
    mkey = __reduce_max_sync(0xffffffffu, mkey);
    flags = (int) __reduce_or_sync(0xffffffffu, (unsigned) flags);
    if (p.greedy) best = warp_max_u64(best);
    if (lane_id() == 0) {
        atomicMax(&s_rawkey, mkey);
        if (flags) atomicOr(&s_flags, flags);
        if (p.greedy) atomicMax(&s_best, (unsigned long long) best);
    }
    __syncthreads();
    const int row_flags = s_flags;
    const float raw_max = (row_flags & 1) ? __uint_as_float(0x7FC00000u) : key_value(s_rawkey);
    const int st = restricted_status(raw_max, p.rep);
    if (st != SSB_ROW_OK) {
        if (threadIdx.x == 0) {
            *id_out = -1, *status_out = st;
            if (out.count) *out.count = 0;
        }
        return;
    }
    if (p.greedy) {
        if (threadIdx.x == 0) {
            *id_out = (int32_t) composite_index(s_best), *status_out = SSB_ROW_OK;
            if (out.count) *out.count = 1;
            if (out.tokens && out.cap > 0) out.tokens[0] = *id_out, out.weights[0] = 1.0;
        }
        return;
    }
    if (row_flags & 2) {
        if (threadIdx.x == 0) {
            *id_out = -1, *status_out = SSB_ROW_TEMPERATURE_OVERFLOW;
            if (out.count) *out.count = 0;
        }
        return;
    }

    const int k = p.k;
    const double u = a.u ? a.u[row] : 0.0;
    if (fastk) {
        // ---- top-k by the k-th largest 16-bit key (two 256-bin histograms: high byte, counted above,
        // then low byte), the composites whose key reaches it (the k best and their ties at 16 bits),
        // ranked (s_cnt's space)
        uint32_t above1 = 0;
        const int b1 = top_bin(s_h1, (uint32_t) k, &above1);  // the histogram holds vocab >= k keys
        for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
            const uint32_t key = order_key(s_val[i]) >> 16;
            red_bin(s_h2, (int) (key >> 8) == b1, key & 255u);
        }
        __syncthreads();
        uint32_t above2 = 0;
        const int b2 = top_bin(s_h2, (uint32_t) k - above1, &above2);
        const uint32_t P = ((uint32_t) b1 << 8) | (uint32_t) (b2 < 0 ? 0 : b2);
        uint64_t * s_c = reinterpret_cast<uint64_t *>(s_after);  // [kFastCand] candidates, then draw scratch
        uint64_t * s_sorted = s_c + kFastCand;                    // [k]
        for (int base = 0; base < vocab; base += blockDim.x) {  // warp-uniform trip count
            const int i = base + threadIdx.x;
            const bool take = i < vocab && (order_key(s_val[i]) >> 16) >= P;
            const unsigned m = __ballot_sync(0xffffffffu, take);
            if (m) {
                int at = 0;
                if (lane_id() == __ffs(m) - 1) at = atomicAdd(&s_nc, __popc(m));
                at = __shfl_sync(0xffffffffu, at, __ffs(m) - 1) + __popc(m & ((1u << lane_id()) - 1));
                if (take && at < kFastCand) s_c[at] = composite(s_val[i], (uint32_t) i);
            }
        }
        __syncthreads();
        const int nc = s_nc;
        if (nc <= kFastCand) {  // block-uniform
            if ((int) threadIdx.x < nc) {
                const uint64_t mine = s_c[threadIdx.x];
                int rank = 0;
                for (int j = 0; j < nc; j++) rank += s_c[j] > mine;
                if (rank < k) s_sorted[rank] = mine;
            }
            __syncthreads();
            if (warp_id() == 0) draw_row(s_sorted, k, p, u, reinterpret_cast<double *>(s_c), out);
            return;
        }
        __syncthreads();  // too many ties at the bound: the general path below
    }

    // ---- top-k by radix select, then sort the k (s_cnt's space is reused for the candidates)
    radix_select(vocab, k, [&](int i) { return composite(s_val[i], (uint32_t) i); }, sel);
    const int kp2 = next_pow2(k);
    uint64_t * s_cand = reinterpret_cast<uint64_t *>(s_after);      // [kp2]
    double * s_w = reinterpret_cast<double *>(s_cand + kp2);         // [k]
    __shared__ int s_n;
    if (threadIdx.x == 0) s_n = 0;
    for (int i = kp2 - 1 - threadIdx.x; i >= k; i -= blockDim.x) s_cand[i] = 0;
    __syncthreads();
    for (int base = 0; base < vocab; base += blockDim.x) {
        const int i = base + threadIdx.x;
        const uint64_t c = i < vocab ? composite(s_val[i], (uint32_t) i) : 0;
        const bool take = i < vocab && selected(c, sel);
        const unsigned m = __ballot_sync(0xffffffffu, take);
        if (m) {
            int slot = 0;
            if (lane_id() == __ffs(m) - 1) slot = atomicAdd(&s_n, __popc(m));
            slot = __shfl_sync(0xffffffffu, slot, __ffs(m) - 1);
            const int at = slot + __popc(m & ((1u << lane_id()) - 1));
            if (take && at < kp2) s_cand[at] = c;
        }
    }
    __syncthreads();
    bitonic_sort_desc(s_cand, kp2);
    if (warp_id() == 0) draw_row(s_cand, k, p, u, s_w, out);
}

template <typename TIn, bool kDebug>
cudaError_t launch_small_t(const SmallArgs & a, size_t smem, cudaStream_t stream) {
    auto kern = small_rows_kernel<TIn, kDebug>;
    cudaError_t e = ssb::set_max_dynamic_smem((const void *) kern, smem);
    if (e != cudaSuccess) return e;
    kern<<<a.rows, kSmallThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace

size_t small_smem_bytes(int vocab, int k_bound) {
    const size_t vals = ((size_t) vocab * 4 + 15) & ~(size_t) 15;
    const int kp2 = next_pow2(k_bound < 1 ? 1 : k_bound);
    const size_t cnt = (size_t) vocab * 4;
    size_t cand = (size_t) kp2 * 8 + (size_t) k_bound * 8;
    const size_t fast = (size_t) (kFastCand + kFastK) * 8;  // the histogram path's candidates and sorted k
    cand = cand > fast ? cand : fast;
    return vals + (cnt > cand ? cnt : cand);
}

cudaError_t launch_small(const SmallArgs & a, bool bf16, bool debug, cudaStream_t stream) {
    const size_t smem = small_smem_bytes(a.vocab, a.k_bound);
    if (bf16) return debug ? launch_small_t<uint16_t, true>(a, smem, stream) : launch_small_t<uint16_t, false>(a, smem, stream);
    return debug ? launch_small_t<float, true>(a, smem, stream) : launch_small_t<float, false>(a, smem, stream);
}

}  // namespace ssb
