// The vocabulary-sharded draw: a row whose columns are split over several GPUs (a tensor-parallel LM head
// leaves its logits that way) is sampled from a small exchange of candidates instead of the whole row.
//
//   shard_select_kernel  (every rank, on its slice [col_offset, col_offset + width) of each row) the
//                        restricted logits of the slice (the history ids that fall in it, translated; the
//                        slice's mask words), their NaN-propagating maximum, whether a scaled logit is NaN,
//                        and the slice's k best composites (scaled logit, or the restricted logit for a
//                        greedy row, with the token's GLOBAL index), sorted, into one record per row:
//                        k_cap composites (0 = none) and a word (max bits << 32 | flags).
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

constexpr int kShardThreads = 256;

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
    uint64_t * s_sel = reinterpret_cast<uint64_t *>(smem);             // [k_cap]
    int32_t * s_hkey = reinterpret_cast<int32_t *>(s_sel + sa.k_cap);  // [hist_slots]
    int32_t * s_hcnt = s_hkey + sa.hist_slots;
    __shared__ SelectState sel;
    __shared__ float s_redf[32];
    __shared__ int s_redi[32];
    __shared__ int s_n;

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

    // the history ids inside the slice, as slice columns, with their counts
    if (penal) {
        for (int i = tid; i < slots; i += kShardThreads) s_hkey[i] = -1, s_hcnt[i] = 0;
        __syncthreads();
        const uint32_t hmask = (uint32_t) slots - 1u;
        for (int i = tid; i < hlen; i += kShardThreads) {
            const int32_t t = __ldg(hist + i) - sa.col_offset;
            if (t < 0 || t >= width || __ldg(hist + i) >= sa.vocab_total) continue;
            uint32_t h = hash_token(t, hbits);
            for (uint32_t n = 0; n <= hmask; n++) {
                const int32_t old = atomicCAS(&s_hkey[h], -1, t);
                if (old == -1 || old == t) {
                    atomicAdd(&s_hcnt[h], 1);
                    break;
                }
                h = (h + 1) & hmask;
            }
        }
    }
    __syncthreads();
    auto restricted = [&](int col) {
        float v = Elem<TIn>::load1(src, col);
        if (penal) {
            const int s = sh_find(s_hkey, slots, hbits, col);
            if (s >= 0) v = penalize(v, s_hcnt[s], p);
        }
        if (mrow && masked_bit(__ldg(mrow + (col >> 5)) >> (col & 31), a.mask_kind)) v = -kInf;
        return v;
    };
    auto key_of = [&](int col) {
        const float r = restricted(col);
        return composite(greedy ? r : __fdiv_rn(r, p.temperature), (uint32_t) (sa.col_offset + col));
    };

    // the slice's restricted maximum and whether a scaled logit is NaN
    float mx = -kInf;
    int nan_scaled = 0;
    for (int col = tid; col < width; col += kShardThreads) {
        const float r = restricted(col);
        mx = max_nan(mx, r);
        if (!greedy) {
            const float sc = __fdiv_rn(r, p.temperature);
            nan_scaled |= sc != sc;
        }
    }
    mx = block_max_nan(mx, s_redf);
    nan_scaled = block_or(nan_scaled, s_redi);

    // the slice's kk best composites, sorted (kk <= k_cap: larger rows are refused by the merge)
    const int take = kk <= sa.k_cap ? kk : 0;
    if (take > 0 && take < width) radix_select(width, take, key_of, sel);
    for (int i = tid; i < sa.k_cap; i += kShardThreads) s_sel[i] = 0ull;
    if (tid == 0) s_n = 0;
    __syncthreads();
    if (take > 0) {
        for (int base = 0; base < width; base += kShardThreads) {  // uniform trip count for the ballot
            const int col = base + tid;
            const uint64_t c = col < width ? key_of(col) : 0ull;
            const bool in = col < width && (take >= width || selected(c, sel));
            const unsigned m = __ballot_sync(0xffffffffu, in);
            if (m) {
                int at = 0;
                if (lane == __ffs(m) - 1) at = atomicAdd(&s_n, __popc(m));
                at = __shfl_sync(0xffffffffu, at, __ffs(m) - 1) + __popc(m & ((1u << lane) - 1u));
                if (in && at < sa.k_cap) s_sel[at] = c;
            }
        }
    }
    __syncthreads();
    bitonic_sort_desc(s_sel, sa.k_cap);
    for (int i = tid; i < sa.k_cap; i += kShardThreads) rec[i] = s_sel[i];
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

size_t shard_select_smem_bytes(int k_cap, int hist_slots) { return (size_t) k_cap * 8 + (size_t) hist_slots * 8; }
size_t shard_merge_smem_bytes(int world, int k_cap) {
    return (size_t) next_pow2(world * k_cap) * 8 + (size_t) k_cap * 8;
}

cudaError_t launch_shard_select(const ShardArgs & a, bool bf16, cudaStream_t stream) {
    const size_t smem = shard_select_smem_bytes(a.k_cap, a.hist_slots);
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
