// All-greedy batches over large vocabularies (config 1: the ASR text head, Qwen3Readback::Pick / verify,
// src/common/qwen3-decoder.cpp:422-437, 492-510; host max_element, qwen3-asr/decoder.cpp:108-113): the first
// maximum of each row's restricted logits (qwen3-tts/sampler.cpp:103-107) and its status.
//
// Grid (splits, rows). Each CTA reads one chunk of a row with 16-byte loads (one per thread when the
// batch is small: 1024 fp32 or 2048 bf16 columns per CTA, the next one in flight otherwise), applies
// the row's ban/allow mask word, and reduces to (the maximum
// composite order_key(l) << 32 | ~column, the NaN-propagating maximum). History tokens of the chunk, where
// a penalty applies, are taken out of the vector pass (a bitmap of the chunk's history columns) and
// added penalized, with their occurrence counts. The CTA's pair goes to the context's split-row scratch;
// the last CTA of the row to arrive (a per-row counter, left at 0 again) merges the row's pairs, decides
// the status from the maximum (restricted_status) and writes the id. Two dependent global round trips
// after the read, and no block-wide list work.
#include <cstdint>

#include "ssb_device.cuh"
#include "ssb_kernels.h"
#include "ssb_tma.cuh"  // hash_token

namespace ssb {

namespace {

constexpr int kArgThreads = 256;

template <typename TIn>
__global__ void __launch_bounds__(kArgThreads) argmax_rows_kernel(const __grid_constant__ StreamArgs sa) {
    const RowsArgs & a = sa.r;
    extern __shared__ __align__(16) unsigned char smem[];
    uint32_t * s_bits = reinterpret_cast<uint32_t *>(smem);      // [chunk / 32] history columns of the chunk
    int32_t * s_hkey = reinterpret_cast<int32_t *>(s_bits + (sa.chunk >> 5));
    int32_t * s_hcnt = s_hkey + sa.hist_slots;
    __shared__ float s_redf[32];
    __shared__ uint64_t s_red64[32];
    __shared__ int s_any, s_last;

    const int split = blockIdx.x, row = blockIdx.y, tid = (int) threadIdx.x;
    const int vocab = a.vocab;
    const ssb_params pp = a.row_params ? a.row_params[row] : a.params;
    const RowParams p = resolve_params(pp, vocab);
    const int c0 = split * sa.chunk;
    const int c1 = min(vocab, c0 + sa.chunk);
    const TIn * src = reinterpret_cast<const TIn *>(a.logits) + (int64_t) row * a.ld;
    const uint32_t * mrow = (a.mask && a.mask_kind != SSB_MASK_NONE) ? a.mask + (int64_t) row * a.mask_ld : nullptr;
    const int32_t * hist = a.history ? a.history + (int64_t) row * a.history_ld : nullptr;
    int hlen = 0;
    if (hist) {
        hlen = a.history_len ? a.history_len[row] : (int) a.history_ld;
        hlen = hlen < 0 ? 0 : (hlen > (int) a.history_ld ? (int) a.history_ld : hlen);
    }
    const bool penal = p.history_applies && hlen > 0 && sa.hist_slots > 0;

    // the first vector read is issued first; the history of the chunk is sorted out while it is in flight
    constexpr int kV = Elem<TIn>::kVec;
    constexpr int kStride = kArgThreads * kV;
    auto load_vec = [&](int col, float (&v)[kV], uint32_t & mword) {
        if (col + kV <= c1) {
            Elem<TIn>::unpack(ld_stream(src + col), v);
        } else {
#pragma unroll
            for (int j = 0; j < kV; j++) v[j] = col + j < c1 ? Elem<TIn>::load1(src, col + j) : -kInf;
        }
        mword = (mrow && col < c1) ? __ldg(mrow + (col >> 5)) : 0u;
    };
    float v[kV];
    uint32_t mword = 0;
    int col = c0 + tid * kV;
    if (col < c1) load_vec(col, v, mword);

    int slots = sa.hist_slots, hbits = 1;
    if (penal) {
        hbits = 31 - __clz(slots);
        for (int i = tid; i < (sa.chunk >> 5); i += kArgThreads) s_bits[i] = 0u;
        for (int i = tid; i < slots; i += kArgThreads) s_hkey[i] = -1, s_hcnt[i] = 0;
        if (tid == 0) s_any = 0;
        __syncthreads();
        const uint32_t hmask = (uint32_t) slots - 1u;
        for (int i = tid; i < hlen; i += kArgThreads) {
            const int32_t t = __ldg(hist + i);
            if (t < c0 || t >= c1) continue;
            s_any = 1;
            atomicOr(&s_bits[(t - c0) >> 5], 1u << ((t - c0) & 31));
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
        __syncthreads();
    }

    float mx = -kInf;
    uint64_t best = 0ull;
    for (; col < c1; col += kStride) {
        float nv[kV];
        uint32_t nword = 0;
        if (col + kStride < c1) load_vec(col + kStride, nv, nword);  // the next vector in flight
#pragma unroll
        for (int j = 0; j < kV; j++) {
            const int cj = col + j;
            if (cj >= c1) break;
            float l = v[j];
            if (penal && ((s_bits[(cj - c0) >> 5] >> ((cj - c0) & 31)) & 1u)) continue;  // taken below, penalized
            if (mrow && masked_bit(mword >> (cj & 31), a.mask_kind)) l = -kInf;
            mx = max_nan(mx, l);
            const uint64_t c = composite(l, (uint32_t) cj);
            best = c > best ? c : best;
        }
#pragma unroll
        for (int j = 0; j < kV; j++) v[j] = nv[j];
        mword = nword;
    }
    if (penal && s_any) {
        for (int h = tid; h < slots; h += kArgThreads) {
            const int32_t t = s_hkey[h];
            if (t < 0) continue;
            float l = penalize(Elem<TIn>::load1(src, t), s_hcnt[h], p);
            if (mrow && masked_bit(__ldg(mrow + (t >> 5)) >> (t & 31), a.mask_kind)) l = -kInf;
            mx = max_nan(mx, l);
            const uint64_t c = composite(l, (uint32_t) t);
            best = c > best ? c : best;
        }
    }
    mx = block_max_nan(mx, s_redf);
    best = block_max_u64(best, s_red64);

    if (sa.splits > 1) {
        const int64_t slot = (int64_t) row * sa.splits + split;
        if (tid == 0) {
            sa.part_cand[slot] = best;
            sa.part_max[slot] = mx;
            __threadfence();
            s_last = atomicAdd(&sa.counters[row], 1u) == (unsigned) (sa.splits - 1);
        }
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        mx = -kInf;
        best = 0ull;
        for (int q = tid; q < sa.splits; q += kArgThreads) {
            mx = max_nan(mx, __ldcg(sa.part_max + (int64_t) row * sa.splits + q));
            const uint64_t c = __ldcg(reinterpret_cast<const unsigned long long *>(sa.part_cand) + (int64_t) row * sa.splits + q);
            best = c > best ? c : best;
        }
        mx = block_max_nan(mx, s_redf);
        best = block_max_u64(best, s_red64);
        if (tid == 0) sa.counters[row] = 0;  // ready for the next launch
    }
    if (tid == 0) {
        const int st = restricted_status(mx, p.rep);
        a.ids[row] = st == SSB_ROW_OK ? (int32_t) composite_index(best) : -1;
        a.status[row] = st;
        if (a.dbg_count) a.dbg_count[row] = st == SSB_ROW_OK ? 1 : 0;
        if (a.dbg_tokens && a.dbg_cap > 0 && st == SSB_ROW_OK) {
            a.dbg_tokens[(int64_t) row * a.dbg_cap] = (int32_t) composite_index(best);
            a.dbg_weights[(int64_t) row * a.dbg_cap] = 1.0;
        }
    }
}

}  // namespace

int argmax_unit(bool bf16) { return kArgThreads * (bf16 ? 8 : 4); }

size_t argmax_smem_bytes(int chunk, int hist_slots) { return (size_t) (chunk >> 5) * 4 + (size_t) hist_slots * 8; }

cudaError_t launch_argmax(const StreamArgs & a, bool bf16, cudaStream_t stream) {
    const size_t smem = argmax_smem_bytes(a.chunk, a.hist_slots);
    const void * kern = bf16 ? (const void *) argmax_rows_kernel<uint16_t> : (const void *) argmax_rows_kernel<float>;
    cudaError_t e = set_max_dynamic_smem(kern, smem);
    if (e != cudaSuccess) return e;
    const dim3 grid(a.splits, a.r.rows);
    if (bf16) argmax_rows_kernel<uint16_t><<<grid, kArgThreads, smem, stream>>>(a);
    else argmax_rows_kernel<float><<<grid, kArgThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace ssb
