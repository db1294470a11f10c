// Large-vocabulary rows (vocab > SSB_SMALL_VOCAB, e.g. Qwen3's 151936): the logits row is streamed
// once from HBM in 16-byte vectors and reduced on the fly. This is the HBM-bound hot path.
//
// Work decomposition: `splits` CTAs per row, each owning `chunk` consecutive columns; with one split
// a CTA finishes its row alone, otherwise the last CTA to arrive (per-row counter) merges the
// partial results the others left in global scratch. No CTA ever waits on another.
//
// Per element the stream does only what every element needs: widen to fp32, substitute -inf for a
// masked token and the penalized value for a history token (both rare, flagged by bitmaps), fold into
// a NaN-propagating maximum (the restricted max of qwen3-tts/sampler.cpp:43-49), and compare against
// a running threshold. Two modes:
//   mode 0 (greedy rows): first maximum, qwen3-tts/sampler.cpp:105-108 — a per-thread composite max.
//   mode 1 (top-k draws): a shared candidate buffer fed by a running threshold. Until the buffer has
//     held k entries every element enters; afterwards only elements whose composite beats the k-th
//     best seen so far. Columns are visited in increasing order, iteration by iteration, so a later
//     element equal in value to the threshold loses on index and the strict comparison is exact.
//     The comparison runs on raw logits against a bound below which no logit can scale past the
//     threshold (raw_bound), so the fp32 division by the temperature (qwen3-tts/sampler.cpp:73) is
//     done exactly, but only for the few elements near the top.
// The row's top-k composites are then sorted and finalize_draw replays the reference's double-
// precision softmax, top-p cut and pick.
#include <climits>

#include "ssb_device.cuh"
#include "ssb_kernels.h"

namespace ssb {

namespace {

constexpr int kPrefetch = 4;  // 16-byte vectors in flight per thread

__device__ __forceinline__ int lower_bound_i32(const int32_t * a, int n, int32_t t) {
    int lo = 0, hi = n;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (a[mid] < t) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

// Everything a CTA keeps while it streams its columns.
struct Stream {
    int c0;
    int mask_kind;
    const uint32_t * mrow;
    bool penal;
    const uint32_t * hbits;
    const int32_t * htok;
    const float * hval;
    int nh;
    float tscale;
    bool fast;
    bool scale;
    float * processed;  // debug: the restricted logits of this row
    // running state
    float acc;
    int nan_scaled;
    uint64_t best;
    uint64_t theta;
    int theta_valid;
    float theta_lo;
    int over;
    uint64_t * buf;
    int * count;
    int high;
};

// One group of G consecutive columns starting at col0 (col0 % G == 0), nvalid of them real.
// Called by every thread of the CTA at the same time (warp-uniform control around the vote).
template <int G, int kMode, bool kDebug>
__device__ __forceinline__ void stream_group(Stream & s, float (&v)[G], const int col0, const int nvalid) {
    const uint32_t vmask = nvalid >= G ? (uint32_t) ((1ull << G) - 1) : (uint32_t) ((1ull << nvalid) - 1);
    if (vmask) {
        uint32_t mb = 0, hb = 0;
        if (s.mrow) {
            const uint32_t w = __ldg(s.mrow + (col0 >> 5)) >> (col0 & 31);
            mb = (s.mask_kind == SSB_MASK_BAN ? w : ~w) & vmask;
        }
        if (s.penal) hb = (s.hbits[(col0 - s.c0) >> 5] >> ((col0 - s.c0) & 31)) & vmask;
        if (mb | hb) {
#pragma unroll
            for (int e = 0; e < G; e++) {
                if ((mb >> e) & 1u) v[e] = -kInf;
                else if ((hb >> e) & 1u) v[e] = s.hval[lower_bound_i32(s.htok, s.nh, col0 + e)];
            }
        }
        if (kDebug && s.processed) {
#pragma unroll
            for (int e = 0; e < G; e++)
                if ((vmask >> e) & 1u) s.processed[col0 + e] = v[e];
        }
    }
    float lm = -kInf;
#pragma unroll
    for (int e = 0; e < G; e++)
        if ((vmask >> e) & 1u) lm = max_nan(lm, v[e]);
    s.acc = max_nan(s.acc, lm);
    if (kMode == 0) {
        if (vmask && order_key(lm) >= (uint32_t) (s.best >> 32)) {
#pragma unroll
            for (int e = 0; e < G; e++) {
                if ((vmask >> e) & 1u) {
                    const uint64_t c = composite(v[e], (uint32_t) (col0 + e));
                    s.best = c > s.best ? c : s.best;
                }
            }
        }
    } else {
        uint32_t cm = 0;
        uint64_t ck[G];
#pragma unroll
        for (int e = 0; e < G; e++) ck[e] = 0;
        if (vmask && lm >= s.theta_lo) {
#pragma unroll
            for (int e = 0; e < G; e++) {
                if (((vmask >> e) & 1u) && v[e] >= s.theta_lo) {
                    const float sc = s.scale ? __fdiv_rn(v[e], s.tscale) : v[e];
                    s.nan_scaled |= sc != sc;
                    const uint64_t c = composite(sc, (uint32_t) (col0 + e));
                    if (!s.theta_valid || c > s.theta) {
                        ck[e] = c;
                        cm |= 1u << e;
                    }
                }
            }
        }
        if (__any_sync(0xffffffffu, cm != 0)) {
            const int lane = lane_id();
#pragma unroll
            for (int e = 0; e < G; e++) {
                const bool b = (cm >> e) & 1u;
                const unsigned m = __ballot_sync(0xffffffffu, b);
                if (m) {
                    const int leader = __ffs(m) - 1;
                    int slot = 0;
                    if (lane == leader) {
                        slot = atomicAdd(s.count, __popc(m));
                        if (slot + __popc(m) > s.high) s.over = 1;
                    }
                    slot = __shfl_sync(0xffffffffu, slot, leader);
                    if (b) s.buf[slot + __popc(m & ((1u << lane) - 1u))] = ck[e];
                }
            }
        }
    }
}

// Shared state of the candidate buffer.
struct BufShared {
    int count;
    int nsel;
    int theta_valid;
    uint64_t theta;
    float theta_lo;
};

// Keeps the k best of the buffer (all of them when it holds fewer) in sel[0..kk), kk returned, and
// the threshold for what may still enter. Block-wide; buffer contents are stable during the call.
__device__ int compact_buffer(uint64_t * buf, uint64_t * sel, int k, bool copy_back, float tscale, bool fast,
                              BufShared & bs, SelectState & st, uint64_t * s_red64) {
    const int n = bs.count;
    const int kk = n < k ? n : k;
    if (threadIdx.x == 0) bs.nsel = 0;
    if (kk < n) {
        radix_select(n, kk, [&](int i) { return buf[i]; }, st);
        for (int base = 0; base < n; base += blockDim.x) {
            const int i = base + threadIdx.x;
            const uint64_t c = i < n ? buf[i] : 0;
            const bool take = i < n && selected(c, st);
            const unsigned m = __ballot_sync(0xffffffffu, take);
            if (m) {
                const int leader = __ffs(m) - 1;
                int slot = 0;
                if (lane_id() == leader) slot = atomicAdd(&bs.nsel, __popc(m));
                slot = __shfl_sync(0xffffffffu, slot, leader);
                const int at = slot + __popc(m & ((1u << lane_id()) - 1u));
                if (take && at < kk) sel[at] = c;
            }
        }
    } else {
        for (int i = threadIdx.x; i < n; i += blockDim.x) sel[i] = buf[i];
    }
    __syncthreads();
    if (copy_back) {
        for (int i = threadIdx.x; i < kk; i += blockDim.x) buf[i] = sel[i];
    }
    uint64_t mn = ~0ull;
    for (int i = threadIdx.x; i < kk; i += blockDim.x) mn = sel[i] < mn ? sel[i] : mn;
    mn = block_min_u64(mn, s_red64);
    if (threadIdx.x == 0) {
        bs.count = kk;
        if (kk == k) {
            bs.theta_valid = 1;
            bs.theta = mn;
            bs.theta_lo = raw_bound(composite_value(mn), tscale, fast);
        }
    }
    __syncthreads();
    return kk;
}

template <typename TIn, int kMode, bool kVec, bool kDebug>
__global__ void __launch_bounds__(kStreamThreads, 3) stream_rows_kernel(const StreamArgs sa) {
    const RowsArgs & a = sa.r;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ SelectState sel;
    __shared__ BufShared bs;
    __shared__ float s_redf[32];
    __shared__ uint64_t s_red64[32];
    __shared__ int s_redi[32];
    __shared__ int s_nh, s_last;

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

    const int hw_alloc = (((sa.chunk + 31) >> 5) + 3) & ~3;  // bitmap words, padded to 16 bytes
    uint32_t * s_hbits = reinterpret_cast<uint32_t *>(smem);
    int32_t * s_htok = reinterpret_cast<int32_t *>(s_hbits + hw_alloc);
    float * s_hval = reinterpret_cast<float *>(s_htok + sa.hist_slots);
    uint64_t * s_buf = reinterpret_cast<uint64_t *>(s_hval + sa.hist_slots);  // hist_slots is even
    uint64_t * s_sel = s_buf + sa.cap;

    const TIn * src = reinterpret_cast<const TIn *>(a.logits) + (int64_t) row * a.ld;

    // ---- history: distinct in-range ids, their counts and penalized values, and a bitmap of them
    const int32_t * hist = a.history ? a.history + (int64_t) row * a.history_ld : nullptr;
    int hlen = 0;
    if (hist) {
        hlen = a.history_len ? a.history_len[row] : (int) a.history_ld;
        hlen = hlen < 0 ? 0 : (hlen > (int) a.history_ld ? (int) a.history_ld : hlen);
    }
    const bool penal = p.history_applies && hlen > 0;
    int nh = 0;
    if (penal) {
        const int nw = (sa.chunk + 31) >> 5;
        for (int i = threadIdx.x; i < nw; i += blockDim.x) s_hbits[i] = 0;
        if (threadIdx.x == 0) s_nh = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < hlen; i += blockDim.x) {
            const int32_t t = hist[i];
            if (t >= c0 && t < c1) s_htok[atomicAdd(&s_nh, 1)] = t;
        }
        __syncthreads();
        nh = s_nh;
        const int np2 = next_pow2(nh < 1 ? 1 : nh);
        for (int i = nh + threadIdx.x; i < np2; i += blockDim.x) s_htok[i] = INT_MAX;
        __syncthreads();
        bitonic_sort_asc_i32(s_htok, np2);
        for (int j = threadIdx.x; j < nh; j += blockDim.x) {
            const int32_t t = s_htok[j];
            if (j == 0 || s_htok[j - 1] != t) {
                int e = j + 1;
                while (e < nh && s_htok[e] == t) e++;
                s_hval[j] = penalize(Elem<TIn>::load1(src, t), e - j, p);
                atomicOr(&s_hbits[(t - c0) >> 5], 1u << ((t - c0) & 31));
            }
        }
    }
    if (kMode == 1 && threadIdx.x == 0) {
        bs.count = 0;
        bs.theta_valid = 0;
        bs.theta = 0;
        bs.theta_lo = -kInf;
    }
    __syncthreads();

    Stream s;
    s.c0 = c0;
    s.mask_kind = a.mask_kind;
    s.mrow = (a.mask && a.mask_kind != SSB_MASK_NONE) ? a.mask + (int64_t) row * a.mask_ld : nullptr;
    s.penal = penal;
    s.hbits = s_hbits;
    s.htok = s_htok;
    s.hval = s_hval;
    s.nh = nh;
    s.scale = !greedy_row;
    s.tscale = greedy_row ? 1.0f : p.temperature;
    s.fast = greedy_row ? true : p.fast_scale;
    s.processed = (kDebug && a.dbg_processed) ? a.dbg_processed + (int64_t) row * vocab : nullptr;
    s.acc = -kInf;
    s.nan_scaled = 0;
    s.best = 0;
    s.theta = 0;
    s.theta_valid = 0;
    s.theta_lo = -kInf;
    s.over = 0;
    s.buf = s_buf;
    s.count = &bs.count;

    auto iteration_end = [&]() {
        if (kMode == 1) {
            if (__syncthreads_or(s.over)) {
                compact_buffer(s_buf, s_sel, k, true, s.tscale, s.fast, bs, sel, s_red64);
                s.over = 0;
                s.theta_valid = bs.theta_valid;
                s.theta = bs.theta;
                s.theta_lo = bs.theta_lo;
            }
        }
    };

    if (kVec) {
        constexpr int G = Elem<TIn>::kVec;
        s.high = sa.cap - kStreamThreads * G;
        const int nvec = len / G;
        const int iters = (nvec + kStreamThreads - 1) / kStreamThreads;
        const char * base = reinterpret_cast<const char *>(src + c0);
        uint4 ring[kPrefetch];
#pragma unroll
        for (int q = 0; q < kPrefetch; q++) {
            const int j = q * kStreamThreads + threadIdx.x;
            ring[q] = j < nvec ? ld_stream(base + (size_t) j * 16) : make_uint4(0, 0, 0, 0);
        }
        for (int it0 = 0; it0 < iters; it0 += kPrefetch) {
#pragma unroll
            for (int q = 0; q < kPrefetch; q++) {
                const int it = it0 + q;
                if (it < iters) {
                    const uint4 cur = ring[q];
                    const int jn = (it + kPrefetch) * kStreamThreads + threadIdx.x;
                    if (jn < nvec) ring[q] = ld_stream(base + (size_t) jn * 16);
                    const int j = it * kStreamThreads + threadIdx.x;
                    float v[G];
                    Elem<TIn>::unpack(cur, v);
                    stream_group<G, kMode, kDebug>(s, v, c0 + j * G, j < nvec ? G : 0);
                    iteration_end();
                }
            }
        }
        const int tail = len - nvec * G;
        if (tail > 0) {
            const int col = c0 + nvec * G + (int) threadIdx.x;
            const bool ok = (int) threadIdx.x < tail;
            float v1[1] = {ok ? Elem<TIn>::load1(src, col) : -kInf};
            stream_group<1, kMode, kDebug>(s, v1, col, ok ? 1 : 0);
            iteration_end();
        }
    } else {
        s.high = sa.cap - kStreamThreads;
        const int iters = (len + kStreamThreads - 1) / kStreamThreads;
        for (int it = 0; it < iters; it++) {
            const int col = c0 + it * kStreamThreads + (int) threadIdx.x;
            const bool ok = col < c1;
            float v1[1] = {ok ? Elem<TIn>::load1(src, col) : -kInf};
            stream_group<1, kMode, kDebug>(s, v1, col, ok ? 1 : 0);
            iteration_end();
        }
    }

    // ---- this CTA's result
    __syncthreads();
    int kk = 1;
    if (kMode == 1) kk = compact_buffer(s_buf, s_sel, k, false, s.tscale, s.fast, bs, sel, s_red64);
    const float rmax = block_max_nan(s.acc, s_redf);
    const int nanf = block_or(s.nan_scaled, s_redi);
    uint64_t best = 0;
    if (kMode == 0) best = block_max_u64(s.best, s_red64);

    float row_max = rmax;
    int row_nan = nanf;
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
        row_nan = block_or(f, s_redi);
        if (kMode == 0) {
            uint64_t b = 0;
            for (int q = threadIdx.x; q < splits; q += blockDim.x) {
                const uint64_t c = __ldcg(reinterpret_cast<const unsigned long long *>(sa.part_cand) +
                                          ((int64_t) row * splits + q) * sa.r.k_bound);
                b = c > b ? c : b;
            }
            best = block_max_u64(b, s_red64);
        } else {
            // gather every split's candidates into the buffer, compacting whenever it could overflow
            const int total_slots = splits * sa.r.k_bound;
            const int room = sa.cap - k;  // entries that may be appended after a compaction
            if (threadIdx.x == 0) bs.count = 0;
            __syncthreads();
            for (int b0 = 0; b0 < total_slots; b0 += room) {
                const int nb = min(room, total_slots - b0);
                for (int i0 = 0; i0 < nb; i0 += blockDim.x) {  // warp-uniform trip count
                    const int ii = i0 + (int) threadIdx.x;
                    bool take = false;
                    uint64_t c = 0;
                    if (ii < nb) {
                        const int i = b0 + ii;
                        const int q = i / sa.r.k_bound, j = i - q * sa.r.k_bound;
                        const int64_t sl = (int64_t) row * splits + q;
                        if (j < __ldcg(sa.part_n + sl)) {
                            take = true;
                            c = __ldcg(reinterpret_cast<const unsigned long long *>(sa.part_cand) + sl * sa.r.k_bound + j);
                        }
                    }
                    const unsigned mm = __ballot_sync(0xffffffffu, take);
                    if (mm) {
                        const int leader = __ffs(mm) - 1;
                        int sl2 = 0;
                        if (lane_id() == leader) sl2 = atomicAdd(&bs.count, __popc(mm));
                        sl2 = __shfl_sync(0xffffffffu, sl2, leader);
                        if (take) s_buf[sl2 + __popc(mm & ((1u << lane_id()) - 1u))] = c;
                    }
                }
                __syncthreads();
                const bool more = b0 + nb < total_slots;
                kk = compact_buffer(s_buf, s_sel, k, more, s.tscale, s.fast, bs, sel, s_red64);
            }
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
    int st = restricted_status(row_max, p.rep);
    if (st == SSB_ROW_OK && !greedy_row && row_nan) st = SSB_ROW_TEMPERATURE_OVERFLOW;
    if (st != SSB_ROW_OK) {
        if (threadIdx.x == 0) {
            *id_out = -1, *st_out = st;
            if (out.count) *out.count = 0;
        }
        return;
    }
    if (kMode == 0 || greedy_row) {
        if (kMode == 1) {
            uint64_t b = 0;
            for (int i = threadIdx.x; i < kk; i += blockDim.x) b = s_sel[i] > b ? s_sel[i] : b;
            best = block_max_u64(b, s_red64);
        }
        if (threadIdx.x == 0) {
            *id_out = (int32_t) composite_index(best), *st_out = SSB_ROW_OK;
            if (out.count) *out.count = 1;
            if (out.tokens && out.cap > 0) out.tokens[0] = *id_out, out.weights[0] = 1.0;
        }
        return;
    }
    const int kp2 = next_pow2(kk);
    for (int i = kk + threadIdx.x; i < kp2; i += blockDim.x) s_sel[i] = 0;
    __syncthreads();
    bitonic_sort_desc(s_sel, kp2);
    const double u = a.u ? a.u[row] : 0.0;
    finalize_draw(s_sel, kk, p, u, reinterpret_cast<double *>(s_buf), out);
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

size_t stream_smem_bytes(int mode, int chunk, int hist_slots, int cap, int sel_slots) {
    const size_t hwords = (size_t) ((((chunk + 31) >> 5) + 3) & ~3);
    size_t bytes = hwords * 4 + (size_t) hist_slots * 8;
    if (mode == 1) bytes += (size_t) cap * 8 + (size_t) sel_slots * 8;
    return bytes;
}

int stream_blocks_per_sm(int mode, bool bf16, bool vec, size_t smem) {
    void * kern = select_kernel(mode, bf16, vec, false);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem) != cudaSuccess) return 0;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kStreamThreads, smem) != cudaSuccess) return 0;
    return n;
}

cudaError_t launch_stream(const StreamArgs & a, int mode, bool bf16, bool vec, bool debug, cudaStream_t stream) {
    const size_t smem = stream_smem_bytes(mode, a.chunk, a.hist_slots, a.cap, a.sel_slots);
    void * kern = select_kernel(mode, bf16, vec, debug);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (e != cudaSuccess) return e;
    void * args[] = {const_cast<StreamArgs *>(&a)};
    return cudaLaunchKernel(kern, dim3((unsigned) (a.r.rows * a.splits)), dim3(kStreamThreads), args, smem, stream);
}

}  // namespace ssb
