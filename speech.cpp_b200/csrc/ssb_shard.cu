// The vocabulary-sharded draw: a row whose columns are split over several GPUs (a tensor-parallel LM head
// leaves its logits that way) is sampled from a small exchange of candidates instead of the whole row.
//
//   shard_select_kernel  (every rank, on its slice [col_offset, col_offset + width) of each row) the
//                        restricted logits of the slice (the history ids that fall in it, translated; the
//                        slice's mask words), their NaN-propagating maximum, whether a scaled logit is NaN,
//                        and the slice's k best composites (scaled logit, or the restricted logit for a
//                        greedy row, with the token's GLOBAL index), sorted, into one record per row:
//                        k_cap composites (0 = none) and a word (max bits << 32 | flags). Two passes over
//                        the slice: a 4096-bin histogram of the keys' top 12 bits gives the bin of the k-th
//                        key; the keys at or above it (at most 4096, else a radix select) are sorted.
//   (the records of all ranks are all-gathered: one collective of rows * (k_cap + 1) * 8 bytes per rank)
//   shard_merge_kernel   (every rank, identically) per row: the global maximum and flags give the row's
//                        status exactly as the whole-row kernels decide it (restricted_status, then a NaN
//                        scaled logit = TEMPERATURE_OVERFLOW); the world x k_cap composites sorted; the first
//                        is a greedy row's id, the first k are a drawing row's candidates and draw_row()
//                        replays the reference's softmax, top-p and pick() on them.
//
// Exact for every row whose effective top-k is at most k_cap: the k best composites of the row are among
// the union of each slice's k best, and the draw depends on nothing else. Rows that keep more (top-k 0)
// are INVALID_ROW here; they take the restricted-slice exchange instead.
#include <cstdint>

#include "ssb_device.cuh"
#include "ssb_kernels.h"
#include "ssb_tma.cuh"  // hash_token

namespace ssb {

namespace {

constexpr int kShardThreads = 512;
constexpr int kShardUnroll = 8;  // logits loads in flight per thread in the passes over the slice
constexpr int kShardBins = 4096;  // histogram of the top 12 bits of the keys
constexpr int kShardList = 4096;  // candidates kept for the exact sort (>= k_cap)

__device__ __forceinline__ int sh_find(const int32_t * keys, int slots, int bits, int32_t t) {
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

template <typename TIn>
__global__ void __launch_bounds__(kShardThreads) shard_select_kernel(const __grid_constant__ ShardArgs sa) {
    const RowsArgs & a = sa.r;
    extern __shared__ __align__(16) unsigned char smem[];
    uint64_t * s_list = reinterpret_cast<uint64_t *>(smem);                 // [kShardList] candidates
    uint32_t * s_hist = reinterpret_cast<uint32_t *>(s_list + kShardList);  // [kShardBins]
    uint32_t * s_bits = s_hist + kShardBins;                                // [bit_words] history columns
    int32_t * s_hkey = reinterpret_cast<int32_t *>(s_bits + sa.bit_words);  // [hist_slots]
    int32_t * s_hcnt = s_hkey + sa.hist_slots;
    __shared__ SelectState sel;
    __shared__ float s_redf[32];
    __shared__ int s_redi[32];
    __shared__ uint32_t s_scan[kShardThreads];
    __shared__ int s_n, s_bin;

    const int row = blockIdx.x, tid = (int) threadIdx.x, lane = lane_id();
    const int width = a.vocab;
    const ssb_params pp = a.row_params ? a.row_params[row] : a.params;
    const RowParams p = resolve_params(pp, sa.vocab_total);
    const bool greedy = p.greedy != 0;
    const int want = greedy ? 1 : p.k;
    const int kk = want < width ? want : width;
    uint64_t * rec = sa.records + (int64_t) row * (sa.k_cap + 1);
    const TIn * src = reinterpret_cast<const TIn *>(a.logits) + (int64_t) row * a.ld;
    const int32_t * hist = a.history ? a.history + (int64_t) row * a.history_ld : nullptr;
    int hlen = 0;
    if (hist) {
        hlen = a.history_len ? a.history_len[row] : (int) a.history_ld;
        hlen = hlen < 0 ? 0 : (hlen > (int) a.history_ld ? (int) a.history_ld : hlen);
    }
    const bool penal = p.history_applies && hlen > 0 && sa.hist_slots > 0;
    const uint32_t * mrow = (a.mask && a.mask_kind != SSB_MASK_NONE) ? a.mask + (int64_t) row * a.mask_ld : nullptr;
    const int slots = sa.hist_slots;
    const int hbits = slots > 1 ? 31 - __clz(slots) : 1;
    const bool use_bits = penal && sa.bit_words >= ((width + 31) >> 5);

    // the history ids inside the slice, as slice columns, with their counts, and a bitmap of them
    for (int i = tid; i < kShardBins; i += kShardThreads) s_hist[i] = 0u;
    if (penal) {
        for (int i = tid; i < slots; i += kShardThreads) s_hkey[i] = -1, s_hcnt[i] = 0;
        if (use_bits)
            for (int i = tid; i < sa.bit_words; i += kShardThreads) s_bits[i] = 0u;
        __syncthreads();
        const uint32_t hmask = (uint32_t) slots - 1u;
        for (int i = tid; i < hlen; i += kShardThreads) {
            const int32_t g = __ldg(hist + i), t = g - sa.col_offset;
            if (t < 0 || t >= width || g >= sa.vocab_total) continue;
            uint32_t h = hash_token(t, hbits);
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
    auto restrict_v = [&](float v, int col) {
        if (penal && (!use_bits || ((s_bits[col >> 5] >> (col & 31)) & 1u))) {
            const int s = sh_find(s_hkey, slots, hbits, col);
            if (s >= 0) v = penalize(v, s_hcnt[s], p);
        }
        if (mrow && masked_bit(__ldg(mrow + (col >> 5)) >> (col & 31), a.mask_kind)) v = -kInf;
        return v;
    };
    auto restricted = [&](int col) { return restrict_v(Elem<TIn>::load1(src, col), col); };
    auto key_from = [&](float r, int col) {
        return composite(greedy ? r : __fdiv_rn(r, p.temperature), (uint32_t) (sa.col_offset + col));
    };
    auto key_of = [&](int col) { return key_from(restricted(col), col); };
    // kShardUnroll columns per thread and step (col = base + j * threads + tid), their loads issued together
    auto load_step = [&](int base, float (&v)[kShardUnroll]) {
#pragma unroll
        for (int j = 0; j < kShardUnroll; j++) {
            const int col = base + j * kShardThreads + tid;
            v[j] = col < width ? Elem<TIn>::load1(src, col) : 0.0f;
        }
    };
    constexpr int kStep = kShardUnroll * kShardThreads;

    // pass 1: the restricted maximum, whether a scaled logit is NaN, and a histogram of the top 12 bits
    // of every key
    // (most keys share a few bins: the lanes of a warp with the same bin add once, through their leader)
    float mx = -kInf;
    int nan_scaled = 0;
    for (int base = 0; base < width; base += kStep) {  // uniform trip count for the match
        float v[kShardUnroll];
        load_step(base, v);
#pragma unroll
        for (int j = 0; j < kShardUnroll; j++) {
            const int col = base + j * kShardThreads + tid;
            const bool live = col < width;
            uint32_t b = 0xFFFFFFFFu;
            if (live) {
                const float r = restrict_v(v[j], col);
                mx = max_nan(mx, r);
                const float sc = greedy ? r : __fdiv_rn(r, p.temperature);
                nan_scaled |= !greedy && sc != sc;
                b = order_key(sc) >> 20;
            }
            const unsigned peers = __match_any_sync(0xffffffffu, b);
            if (live && lane == __ffs(peers) - 1) atomicAdd(&s_hist[b], (uint32_t) __popc(peers));
        }
    }
    mx = block_max_nan(mx, s_redf);
    nan_scaled = block_or(nan_scaled, s_redi);
    const int take = kk <= sa.k_cap ? kk : 0;  // larger rows are refused by the merge

    // the bin holding the take-th largest key: thread t sums bins [kPer t, kPer t + kPer) from the top
    constexpr int kPer = kShardBins / kShardThreads;
    uint32_t mine = 0;
    for (int j = 0; j < kPer; j++) mine += s_hist[kShardBins - 1 - (tid * kPer + j)];
    s_scan[tid] = mine;
    if (tid == 0) s_bin = 0, s_n = 0;
    __syncthreads();
    if (tid == 0 && take > 0) {
        uint32_t above = 0;
        int t = 0;
        while (t < kShardThreads && above + s_scan[t] < (uint32_t) take) above += s_scan[t++];
        int b = kShardBins - 1 - t * kPer;
        for (int j = 0; j < kPer && b >= 0; j++, b--) {
            above += s_hist[b];
            if (above >= (uint32_t) take) break;
        }
        s_bin = b < 0 ? 0 : b;
        s_scan[0] = above;  // keys in bins >= s_bin
    }
    __syncthreads();
    const int bin = s_bin;
    const bool fits = take > 0 && s_scan[0] <= (uint32_t) kShardList;
    __syncthreads();
    if (take > 0 && fits) {
        // pass 2: every key in a bin at or above the bound, then sorted: the first `take` are the best
        for (int base = 0; base < width; base += kStep) {  // uniform trip count for the ballot
            float v[kShardUnroll];
            load_step(base, v);
#pragma unroll
            for (int j = 0; j < kShardUnroll; j++) {
                const int col = base + j * kShardThreads + tid;
                const uint64_t c = col < width ? key_from(restrict_v(v[j], col), col) : 0ull;
                const bool in = col < width && (int) (uint32_t) (c >> 52) >= bin;
                const unsigned m = __ballot_sync(0xffffffffu, in);
                if (m) {
                    int at = 0;
                    if (lane == __ffs(m) - 1) at = atomicAdd(&s_n, __popc(m));
                    at = __shfl_sync(0xffffffffu, at, __ffs(m) - 1) + __popc(m & ((1u << lane) - 1u));
                    if (in && at < kShardList) s_list[at] = c;
                }
            }
        }
        __syncthreads();
        const int n = s_n < kShardList ? s_n : kShardList;
        const int np2 = next_pow2(n);
        for (int i = n + tid; i < np2; i += kShardThreads) s_list[i] = 0ull;
        __syncthreads();
        bitonic_sort_desc(s_list, np2);
    } else if (take > 0) {
        // too many keys share the bound's bin: radix select over the row, then the selected keys
        if (take < width) radix_select(width, take, key_of, sel);
        for (int base = 0; base < width; base += kShardThreads) {
            const int col = base + tid;
            const uint64_t c = col < width ? key_of(col) : 0ull;
            const bool in = col < width && (take >= width || selected(c, sel));
            const unsigned m = __ballot_sync(0xffffffffu, in);
            if (m) {
                int at = 0;
                if (lane == __ffs(m) - 1) at = atomicAdd(&s_n, __popc(m));
                at = __shfl_sync(0xffffffffu, at, __ffs(m) - 1) + __popc(m & ((1u << lane) - 1u));
                if (in && at < kShardList) s_list[at] = c;
            }
        }
        __syncthreads();
        const int np2 = next_pow2(take);
        for (int i = take + tid; i < np2; i += kShardThreads) s_list[i] = 0ull;
        __syncthreads();
        bitonic_sort_desc(s_list, np2);
    }
    for (int i = tid; i < sa.k_cap; i += kShardThreads) rec[i] = i < take ? s_list[i] : 0ull;
    if (tid == 0) rec[sa.k_cap] = ((uint64_t) __float_as_uint(mx) << 32) | (uint32_t) nan_scaled;
}

__global__ void __launch_bounds__(kShardThreads) shard_merge_kernel(const __grid_constant__ ShardArgs sa) {
    const RowsArgs & a = sa.r;
    extern __shared__ __align__(16) unsigned char smem[];
    const int n = sa.world * sa.k_cap;
    const int np2 = next_pow2(n);
    uint64_t * s_all = reinterpret_cast<uint64_t *>(smem);   // [np2]
    double * s_w = reinterpret_cast<double *>(s_all + np2);  // [k_cap] draw scratch
    __shared__ float s_max;
    __shared__ int s_flags;

    const int row = blockIdx.x, tid = (int) threadIdx.x, warp = warp_id();
    const ssb_params pp = a.row_params ? a.row_params[row] : a.params;
    const RowParams p = resolve_params(pp, sa.vocab_total);
    const bool greedy = p.greedy != 0;
    const int k = greedy ? 1 : p.k;
    int32_t * id_out = a.ids + row;
    int32_t * st_out = a.status + row;
    if (k > sa.k_cap) {
        if (tid == 0) *id_out = -1, *st_out = SSB_ROW_INVALID_ROW;
        return;
    }
    const int64_t stride = (int64_t) a.rows * (sa.k_cap + 1);  // one rank's records
    for (int i = tid; i < np2; i += kShardThreads) {
        uint64_t c = 0ull;
        if (i < n) {
            const int rank = i / sa.k_cap, j = i - rank * sa.k_cap;
            c = sa.records[rank * stride + (int64_t) row * (sa.k_cap + 1) + j];
        }
        s_all[i] = c;
    }
    if (tid == 0) {
        float mx = -kInf;
        int fl = 0;
        for (int r = 0; r < sa.world; r++) {
            const uint64_t w = sa.records[r * stride + (int64_t) row * (sa.k_cap + 1) + sa.k_cap];
            mx = max_nan(mx, __uint_as_float((uint32_t) (w >> 32)));
            fl |= (int) (uint32_t) w;
        }
        s_max = mx, s_flags = fl;
    }
    __syncthreads();
    int stt = restricted_status(s_max, p.rep);
    if (stt == SSB_ROW_OK && !greedy && (s_flags & 1)) stt = SSB_ROW_TEMPERATURE_OVERFLOW;
    if (stt != SSB_ROW_OK) {
        if (tid == 0) *id_out = -1, *st_out = stt;
        return;
    }
    bitonic_sort_desc(s_all, np2);
    if (greedy) {
        if (tid == 0) *id_out = (int32_t) composite_index(s_all[0]), *st_out = SSB_ROW_OK;
        return;
    }
    const double u = a.u ? a.u[row] : 0.0;
    RowOut out{id_out, st_out, nullptr, nullptr, nullptr, 0};
    if (warp == 0) draw_row(s_all, k, p, u, s_w, out);
}

}  // namespace

size_t shard_select_smem_bytes(int bit_words, int hist_slots) {
    return (size_t) kShardList * 8 + (size_t) kShardBins * 4 + (size_t) bit_words * 4 + (size_t) hist_slots * 8;
}
size_t shard_merge_smem_bytes(int world, int k_cap) {
    return (size_t) next_pow2(world * k_cap) * 8 + (size_t) k_cap * 8;
}

cudaError_t launch_shard_select(const ShardArgs & a, bool bf16, cudaStream_t stream) {
    const size_t smem = shard_select_smem_bytes(a.bit_words, a.hist_slots);
    auto kern = bf16 ? shard_select_kernel<uint16_t> : shard_select_kernel<float>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (e != cudaSuccess) return e;
    kern<<<a.r.rows, kShardThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_shard_merge(const ShardArgs & a, cudaStream_t stream) {
    const size_t smem = shard_merge_smem_bytes(a.world, a.k_cap);
    cudaError_t e = cudaFuncSetAttribute(shard_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (e != cudaSuccess) return e;
    shard_merge_kernel<<<a.r.rows, kShardThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace ssb
