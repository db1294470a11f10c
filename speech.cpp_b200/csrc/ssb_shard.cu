// The vocabulary-sharded draw: a row whose columns are split over several GPUs (a tensor-parallel LM head
// leaves its logits that way) is sampled from a small exchange of candidates instead of the whole row.
//
//   shard_select_kernel  (every rank, on its slice [col_offset, col_offset + width) of each row) the
//                        restricted logits of the slice (the history ids that fall in it, translated; the
//                        slice's mask words), their NaN-propagating maximum, whether a scaled logit is NaN,
//                        and the slice's k best composites (scaled logit, or the restricted logit for a
//                        greedy row, with the token's GLOBAL index), sorted, into one record per row:
//                        k_cap composites (0 = none) and a word (max bits << 32 | flags). Two passes over
//                        the slice with eight loads in flight per thread and no atomics on the bulk: each
//                        thread's two best composites give a floor (the k-th largest of them, by a radix
//                        select, below which none of the k best lies); the composites at or above it (a
//                        few times k, at most 4096, else a radix select over the slice) are ranked by
//                        counting (up to one per thread) or sorted.
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
constexpr int kShardList = 4096;  // candidates kept for the exact sort (>= 2 x threads >= k_cap)

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

template <typename TIn, bool kVecLoad>
__global__ void __launch_bounds__(kShardThreads) shard_select_kernel(const __grid_constant__ ShardArgs sa) {
    const RowsArgs & a = sa.r;
    extern __shared__ __align__(16) unsigned char smem[];
    uint64_t * s_list = reinterpret_cast<uint64_t *>(smem);                 // [kShardList] candidates
    uint32_t * s_bits = reinterpret_cast<uint32_t *>(s_list + kShardList);  // [bit_words] history columns
    int32_t * s_hkey = reinterpret_cast<int32_t *>(s_bits + sa.bit_words);  // [hist_slots]
    int32_t * s_hcnt = s_hkey + sa.hist_slots;
    __shared__ SelectState sel;
    __shared__ float s_redf[32];
    __shared__ int s_redi[32];
    __shared__ int s_n, s_last;

    // this CTA's part of the slice row: columns [c0, c0 + width) of the slice (the whole slice when the
    // rows are not split)
    const int split = blockIdx.x, row = blockIdx.y, tid = (int) threadIdx.x, lane = lane_id();
    const int c0 = split * sa.chunk;
    const int width = min(a.vocab, c0 + sa.chunk) - c0;
    const int col_base = sa.col_offset + c0;  // the global index of the part's first column
    const ssb_params pp = a.row_params ? a.row_params[row] : a.params;
    const RowParams p = resolve_params(pp, sa.vocab_total);
    const bool greedy = p.greedy != 0;
    const int want = greedy ? 1 : p.k;
    const int kk = want < width ? want : width;  // this part's best
    const int kk_row = want < a.vocab ? want : a.vocab;  // the slice row's best
    uint64_t * rec = sa.records + (int64_t) row * (sa.k_cap + 1);
    const TIn * src = reinterpret_cast<const TIn *>(a.logits) + (int64_t) row * a.ld + c0;
    const int32_t * hist = a.history ? a.history + (int64_t) row * a.history_ld : nullptr;
    int hlen = 0;
    if (hist) {
        hlen = a.history_len ? a.history_len[row] : (int) a.history_ld;
        hlen = hlen < 0 ? 0 : (hlen > (int) a.history_ld ? (int) a.history_ld : hlen);
    }
    const bool penal = p.history_applies && hlen > 0 && sa.hist_slots > 0;
    const uint32_t * mrow =
        (a.mask && a.mask_kind != SSB_MASK_NONE) ? a.mask + (int64_t) row * a.mask_ld + (c0 >> 5) : nullptr;
    const int slots = sa.hist_slots;
    const int hbits = slots > 1 ? 31 - __clz(slots) : 1;
    const bool use_bits = penal && sa.bit_words >= ((width + 31) >> 5);

    // the history ids inside the slice, as slice columns, with their counts, and a bitmap of them
    if (penal) {
        for (int i = tid; i < slots; i += kShardThreads) s_hkey[i] = -1, s_hcnt[i] = 0;
        if (use_bits)
            for (int i = tid; i < sa.bit_words; i += kShardThreads) s_bits[i] = 0u;
        __syncthreads();
        const uint32_t hmask = (uint32_t) slots - 1u;
        for (int i = tid; i < hlen; i += kShardThreads) {
            const int32_t g = __ldg(hist + i), t = g - col_base;
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
        return composite(greedy ? r : __fdiv_rn(r, p.temperature), (uint32_t) (col_base + col));
    };
    auto key_of = [&](int col) { return key_from(restricted(col), col); };
    // kPerStep columns per thread and step, their loads issued together: kShardUnroll scalar loads
    // (column base + j * threads + tid), or on 16-byte-aligned slices kShardUnroll / 2 vector loads of
    // Elem::kVec columns each (column base + (j * threads + tid) * kVec + e)
    constexpr int kVecN = kVecLoad ? Elem<TIn>::kVec : 1;
    constexpr int kLoads = kVecLoad ? kShardUnroll / 2 : kShardUnroll;
    constexpr int kPerStep = kLoads * kVecN;
    auto col_of = [&](int base, int i) {  // the column of the thread's i-th value of a step
        return kVecLoad ? base + ((i / kVecN) * kShardThreads + tid) * kVecN + (i % kVecN) : base + i * kShardThreads + tid;
    };
    auto load_step = [&](int base, float (&v)[kPerStep]) {
        if constexpr (kVecLoad) {
#pragma unroll
            for (int j = 0; j < kLoads; j++) {
                const int c = base + (j * kShardThreads + tid) * kVecN;
                if (c + kVecN <= width) {
                    float u[kVecN];
                    Elem<TIn>::unpack(ld_stream(src + c), u);
#pragma unroll
                    for (int e = 0; e < kVecN; e++) v[j * kVecN + e] = u[e];
                } else {
#pragma unroll
                    for (int e = 0; e < kVecN; e++) v[j * kVecN + e] = c + e < width ? Elem<TIn>::load1(src, c + e) : 0.0f;
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < kPerStep; j++) {
                const int col = base + j * kShardThreads + tid;
                v[j] = col < width ? Elem<TIn>::load1(src, col) : 0.0f;
            }
        }
    };
    constexpr int kStep = kPerStep * kShardThreads;

    // pass 1: the restricted maximum, whether a scaled logit is NaN, and each thread's two largest values
    // to order by: the restricted logits themselves where the scaled order is theirs (greedy rows, and
    // temperatures that are normal positive floats: x -> fl(x / T) does not fall), else the scaled ones
    const bool raw_order = greedy || p.fast_scale;
    float mx = -kInf;
    int nan_scaled = 0;
    float b0 = -kInf, b1 = -kInf;
    for (int base = 0; base < width; base += kStep) {
        float v[kPerStep];
        load_step(base, v);
#pragma unroll 1
        for (int j = 0; j < kPerStep; j++) {
            const int col = col_of(base, j);
            if (col >= width) continue;
            const float r = restrict_v(v[j], col);
            mx = max_nan(mx, r);
            float o = r;
            if (!raw_order) {
                o = __fdiv_rn(r, p.temperature);
                nan_scaled |= o != o;
                o = o != o ? kInf : o;  // a NaN row is refused anyway; keep the floor finite-ordered
            }
            if (o > b1) {
                if (o > b0) b1 = b0, b0 = o;
                else b1 = o;
            }
        }
    }
    mx = block_max_nan(mx, s_redf);
    // with raw order, a scaled logit is NaN only where the restricted one is (a NaN row) or x / T of an
    // infinite x with a finite T (never NaN): the flag of the other rows is 0
    if (raw_order && !greedy) nan_scaled = mx != mx;
    nan_scaled = block_or(nan_scaled, s_redi);
    const int take = kk <= sa.k_cap ? kk : 0;  // larger rows are refused by the merge

    // the floor: the take-th largest of the threads' 2 x threads values. take threads hold a value at or
    // above it, so at least take of the row's elements do: the row's take best are all at or above it
    // (take <= k_cap <= 1024 <= 2 x threads). Elements whose restricted logit lies below `rb` cannot reach
    // it (raw_bound) and are not divided at all.
    // (a radix select over the 32-bit keys: at least take of them reach its prefix, so the prefix's value
    // is at or below the take-th largest)
    s_list[2 * tid] = (uint64_t) order_key(b0) << 32, s_list[2 * tid + 1] = (uint64_t) order_key(b1) << 32;
    if (tid == 0) s_n = 0;
    __syncthreads();
    float fv = -kInf;
    if (take > 0) {  // block-uniform
        radix_select(2 * kShardThreads, take, [&](int i) { return s_list[i]; }, sel, 4);
        fv = key_value((uint32_t) (sel.prefix >> 32));
    }
    uint64_t floor_key;
    float rb;
    if (take == 0) {
        floor_key = ~0ull, rb = kInf;
    } else if (raw_order) {
        const float sf = greedy ? fv : __fdiv_rn(fv, p.temperature);
        floor_key = composite(sf, 0xFFFFFFFFu);  // the least composite of that value
        rb = greedy ? fv : raw_bound(sf, p.temperature, true);
    } else {
        floor_key = composite(fv, 0xFFFFFFFFu), rb = -kInf;
    }
    __syncthreads();
    // pass 2: every composite at or above the floor (usually a few times take), then sorted
    for (int base = 0; base < width && take > 0; base += kStep) {  // uniform trip count for the ballot
        float v[kPerStep];
        load_step(base, v);
#pragma unroll 1
        for (int j = 0; j < kPerStep; j++) {
            const int col = col_of(base, j);
            bool in = false;
            uint64_t c = 0ull;
            if (col < width) {
                const float r = restrict_v(v[j], col);
                if (r >= rb || r != r || !raw_order) {
                    c = key_from(r, col);
                    in = c >= floor_key;
                }
            }
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
    const bool fits = s_n <= kShardList;
    const uint64_t * sorted = s_list;  // the record's first entries, best first
    int nsorted = take;                // how many of them are valid (the rest are written as 0)
    if (take > 0 && fits && s_n <= kShardThreads) {
        // one candidate per thread: each ranked against all (composites are distinct), the take best
        // written to their places in the upper half of the list
        const int n = s_n;
        uint64_t * out = s_list + kShardList / 2;
        if (tid < n) {
            const uint64_t mine = s_list[tid];
            int rank = 0;
            for (int j = 0; j < n; j++) rank += s_list[j] > mine;
            if (rank < take) out[rank] = mine;
        }
        __syncthreads();
        sorted = out;
        nsorted = n < take ? n : take;
    } else if (take > 0 && fits) {
        const int n = s_n;
        const int np2 = next_pow2(n);
        for (int i = n + tid; i < np2; i += kShardThreads) s_list[i] = 0ull;
        __syncthreads();
        bitonic_sort_desc(s_list, np2);
        nsorted = n < take ? n : take;
    } else if (take > 0) {
        // too many composites at the floor (a row of many equal logits): radix select, then the selected
        __syncthreads();
        if (tid == 0) s_n = 0;
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
    const uint64_t word = ((uint64_t) __float_as_uint(mx) << 32) | (uint32_t) nan_scaled;
    if (sa.splits == 1) {
        for (int i = tid; i < sa.k_cap; i += kShardThreads) rec[i] = i < nsorted ? sorted[i] : 0ull;
        if (tid == 0) rec[sa.k_cap] = word;
        return;
    }
    // split rows: this part's record into the scratch; the row's last CTA to arrive merges the parts'
    // records (splits x k_cap composites, sorted) into the row's record and leaves the counter at 0
    uint64_t * part = sa.parts + ((int64_t) row * sa.splits + split) * (sa.k_cap + 1);
    for (int i = tid; i < sa.k_cap; i += kShardThreads) part[i] = i < nsorted ? sorted[i] : 0ull;
    __syncthreads();
    if (tid == 0) {
        part[sa.k_cap] = word;
        __threadfence();
        s_last = atomicAdd(&sa.counters[row], 1u) == (unsigned) (sa.splits - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int total = sa.splits * sa.k_cap;  // <= kShardList (host)
    const int tp2 = next_pow2(total);
    const uint64_t * parts = sa.parts + (int64_t) row * sa.splits * (sa.k_cap + 1);
    for (int i = tid; i < tp2; i += kShardThreads) {
        uint64_t c = 0ull;
        if (i < total) {
            const int q = i / sa.k_cap, j = i - q * sa.k_cap;
            c = __ldcg(reinterpret_cast<const unsigned long long *>(parts) + (int64_t) q * (sa.k_cap + 1) + j);
        }
        s_list[i] = c;
    }
    float gmx = -kInf;
    int gfl = 0;
    for (int q = tid; q < sa.splits; q += kShardThreads) {
        const uint64_t w = __ldcg(reinterpret_cast<const unsigned long long *>(parts) + (int64_t) q * (sa.k_cap + 1) + sa.k_cap);
        gmx = max_nan(gmx, __uint_as_float((uint32_t) (w >> 32)));
        gfl |= (int) (uint32_t) w;
    }
    gmx = block_max_nan(gmx, s_redf);
    gfl = block_or(gfl, s_redi);
    bitonic_sort_desc(s_list, tp2);
    const int take_row = kk_row <= sa.k_cap ? kk_row : 0;
    for (int i = tid; i < sa.k_cap; i += kShardThreads) rec[i] = i < take_row ? s_list[i] : 0ull;
    if (tid == 0) {
        rec[sa.k_cap] = ((uint64_t) __float_as_uint(gmx) << 32) | (uint32_t) gfl;
        sa.counters[row] = 0;
    }
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
    return (size_t) kShardList * 8 + (size_t) bit_words * 4 + (size_t) hist_slots * 8;
}
size_t shard_merge_smem_bytes(int world, int k_cap) {
    return (size_t) next_pow2(world * k_cap) * 8 + (size_t) k_cap * 8;
}

cudaError_t launch_shard_select(const ShardArgs & a, bool bf16, cudaStream_t stream) {
    const size_t smem = shard_select_smem_bytes(a.bit_words, a.hist_slots);
    const bool vec = reinterpret_cast<uintptr_t>(a.r.logits) % 16 == 0 && (a.r.ld * (bf16 ? 2 : 4)) % 16 == 0;
    auto kern = bf16 ? (vec ? shard_select_kernel<uint16_t, true> : shard_select_kernel<uint16_t, false>)
                     : (vec ? shard_select_kernel<float, true> : shard_select_kernel<float, false>);
    cudaError_t e = ssb::set_max_dynamic_smem((const void *) kern, smem);
    if (e != cudaSuccess) return e;
    kern<<<dim3(a.splits, a.r.rows), kShardThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_shard_merge(const ShardArgs & a, cudaStream_t stream) {
    const size_t smem = shard_merge_smem_bytes(a.world, a.k_cap);
    cudaError_t e = ssb::set_max_dynamic_smem((const void *) shard_merge_kernel, smem);
    if (e != cudaSuccess) return e;
    shard_merge_kernel<<<a.r.rows, kShardThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace ssb
