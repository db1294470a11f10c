// The restricted logits of a batch of rows on their own (the reference's restricted(),
// qwen3-tts/sampler.cpp:29-51): the repetition penalty and the presence/frequency extension over each
// row's distinct history ids, then the mask, before the temperature. Two launches on one stream:
//   restrict_copy_kernel     every column: the raw logit widened to f32, -inf where masked (HBM-bound:
//                            2 or 4 bytes read and 4 written per column);
//   restrict_history_kernel  one CTA per row: the row's history table in shared memory (distinct ids
//                            with their counts, one pass of insert-or-find and count), then each
//                            history token's penalized logit (-inf where masked) over the copy.
// The values are those every sampling kernel computes for the same row (the same penalize() and
// masked_bit()), so a row assembled from restricted slices samples to the whole row's id.
#include <algorithm>
#include <cuda_bf16.h>

#include "ssb_device.cuh"
#include "ssb_kernels.h"
#include "ssb_tma.cuh"

namespace ssb {
namespace {

constexpr int kRestrictThreads = 256;

template <typename TIn>
__global__ void __launch_bounds__(kRestrictThreads) restrict_copy_kernel(const RowsArgs a, float * out, int64_t out_ld) {
    for (int row = blockIdx.y; row < a.rows; row += gridDim.y) {
        const TIn * src = reinterpret_cast<const TIn *>(a.logits) + (int64_t) row * a.ld;
        const uint32_t * mrow = a.mask ? a.mask + (int64_t) row * a.mask_ld : nullptr;
        float * dst = out + (int64_t) row * out_ld;
        for (int col = blockIdx.x * blockDim.x + threadIdx.x; col < a.vocab; col += gridDim.x * blockDim.x) {
            float v = Elem<TIn>::load1(src, col);
            if (mrow && masked_bit(__ldg(mrow + (col >> 5)) >> (col & 31), a.mask_kind)) v = -kInf;
            dst[col] = v;
        }
    }
}

template <typename TIn>
__global__ void __launch_bounds__(kRestrictThreads) restrict_history_kernel(const RowsArgs a, int hist_slots, float * out,
                                                                            int64_t out_ld, int col_offset, int vocab_total) {
    extern __shared__ int32_t s_table[];
    int32_t * s_key = s_table;               // [hist_slots] ids, -1 empty
    int32_t * s_cnt = s_table + hist_slots;  // [hist_slots] occurrences
    const int bits = 31 - __clz(hist_slots);
    const uint32_t hmask = (uint32_t) hist_slots - 1u;
    for (int row = blockIdx.x; row < a.rows; row += gridDim.x) {
        const ssb_params pp = a.row_params ? a.row_params[row] : a.params;
        const RowParams p = resolve_params(pp, a.vocab);
        int hlen = a.history_len ? a.history_len[row] : (int) a.history_ld;
        hlen = hlen < 0 ? 0 : (hlen > (int) a.history_ld ? (int) a.history_ld : hlen);
        if (!p.history_applies || hlen == 0) continue;  // uniform in the CTA
        const int32_t * hist = a.history + (int64_t) row * a.history_ld;
        const TIn * src = reinterpret_cast<const TIn *>(a.logits) + (int64_t) row * a.ld;
        const uint32_t * mrow = a.mask ? a.mask + (int64_t) row * a.mask_ld : nullptr;
        for (int i = threadIdx.x; i < hist_slots; i += blockDim.x) s_key[i] = -1, s_cnt[i] = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < hlen; i += blockDim.x) {
            // history ids are the whole row's; the rows here may be a slice starting at col_offset
            const int32_t g = __ldg(hist + i), t = g - col_offset;
            if (g < 0 || g >= vocab_total || t < 0 || t >= a.vocab) continue;
            uint32_t h = hash_token(t, bits);
            for (uint32_t n = 0; n <= hmask; n++) {
                const int32_t old = atomicCAS(&s_key[h], -1, t);
                if (old == -1 || old == t) {
                    atomicAdd(&s_cnt[h], 1);
                    break;
                }
                h = (h + 1) & hmask;
            }
        }
        __syncthreads();
        for (int i = threadIdx.x; i < hist_slots; i += blockDim.x) {
            const int32_t t = s_key[i];
            if (t < 0) continue;
            const bool m = mrow && masked_bit(__ldg(mrow + (t >> 5)) >> (t & 31), a.mask_kind);
            out[(int64_t) row * out_ld + t] = m ? -kInf : penalize(Elem<TIn>::load1(src, t), s_cnt[i], p);
        }
        __syncthreads();
    }
}

}  // namespace

size_t restrict_smem_bytes(int hist_slots) { return (size_t) hist_slots * 8; }

cudaError_t launch_restrict(const RowsArgs & a, int hist_slots, bool bf16, float * out, int64_t out_ld, int sm_count,
                            cudaStream_t stream, int col_offset, int vocab_total) {
    if (vocab_total <= 0) vocab_total = a.vocab;
    const int col_blocks = (int) std::min<int64_t>((a.vocab + kRestrictThreads - 1) / kRestrictThreads, 4 * sm_count);
    const dim3 grid((unsigned) std::max(1, col_blocks), (unsigned) std::min(a.rows, 65535));
    if (bf16) restrict_copy_kernel<uint16_t><<<grid, kRestrictThreads, 0, stream>>>(a, out, out_ld);
    else restrict_copy_kernel<float><<<grid, kRestrictThreads, 0, stream>>>(a, out, out_ld);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || !a.history || hist_slots == 0) return e;
    const size_t smem = restrict_smem_bytes(hist_slots);
    void * kern = bf16 ? reinterpret_cast<void *>(restrict_history_kernel<uint16_t>)
                       : reinterpret_cast<void *>(restrict_history_kernel<float>);
    e = ssb::set_max_dynamic_smem((const void *) kern, smem);
    if (e != cudaSuccess) return e;
    const int blocks = std::min(a.rows, 4 * sm_count);
    if (bf16) restrict_history_kernel<uint16_t><<<blocks, kRestrictThreads, smem, stream>>>(a, hist_slots, out, out_ld, col_offset, vocab_total);
    else restrict_history_kernel<float><<<blocks, kRestrictThreads, smem, stream>>>(a, hist_slots, out, out_ld, col_offset, vocab_total);
    return cudaGetLastError();
}

}  // namespace ssb
