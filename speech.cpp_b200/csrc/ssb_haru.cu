// Haru's logit shaping and its DRY repetition penalty on the device (src/families/haru/sampler.cpp:82-124):
//
//   dry_update_kernel  Dry::update(token) (:86-110) for every text stream, one CTA per stream: the token
//                      (unless exempt) joins the stream's ring of its last lookback + max_match_length + 1
//                      tokens; for every earlier occurrence j of the last token within the lookback, the
//                      length of the match ending there (at most max_match_length) is counted by one
//                      thread; a match of at least allowed_length proposes the token after it; per
//                      proposed token the longest match wins, and the non-exempt ones get the penalty
//                      min(max_penalty, multiplier * base^(length - allowed_length)) in double, by rising
//                      token, as std::map orders them.
//   haru_shape_kernel  shape_logits() (:116-124) for f32 rows in place, one CTA per row: each DRY penalty
//                      rounded to float subtracted from its token's logit, then PAD's and EOP's logits
//                      replaced by the silent head's, the EOP bias added, and PAD, EOP and EOS set to -inf
//                      where the row must speak.
//
// Both touch a few hundred values per stream; they exist so that a decode loop keeps the drawn token on
// the device: sample (ssb_sample_rows, Haru family) -> dry update -> next frame's shape, all queued on
// one stream, no readback.
#include <cstdint>

#include "ssb_device.cuh"
#include "ssb_kernels.h"

namespace ssb {

namespace {

constexpr int kDryThreads = 256;
constexpr int kShapeThreads = 128;

__device__ __forceinline__ bool is_exempt(const int32_t * ex, int n, int32_t t) {
    for (int i = 0; i < n; i++)
        if (ex[i] == t) return true;
    return false;
}

__global__ void __launch_bounds__(kDryThreads) dry_update_kernel(const __grid_constant__ DryArgs a, const int32_t * tokens) {
    extern __shared__ __align__(16) unsigned char smem[];
    uint64_t * s_rec = reinterpret_cast<uint64_t *>(smem);            // [next_pow2(window)] (token, length)
    int32_t * s_h = reinterpret_cast<int32_t *>(s_rec + a.rec_slots);  // [window] the stream's tokens, oldest first
    __shared__ int32_t s_ex[SSB_DRY_MAX_EXEMPT];
    __shared__ int s_m, s_base[kDryThreads + 1];

    const int s = blockIdx.x, tid = (int) threadIdx.x;
    const int32_t token = tokens[s];
    if (token < 0) return;
    for (int i = tid; i < a.n_exempt; i += kDryThreads) s_ex[i] = a.exempt[i];
    __syncthreads();
    if (is_exempt(s_ex, a.n_exempt, token)) return;  // Dry::update returns before touching anything (:87)

    const int window = a.window;
    int32_t * ring = a.hist + (int64_t) s * window;
    const int head0 = a.head[s], count0 = a.count[s];
    // the token joins the ring; the oldest drops out once the ring is full (:88-90)
    const int count = count0 < window ? count0 + 1 : window;
    const int head = count0 < window ? head0 : (head0 + 1) % window;
    const int at = (head0 + count0) % window;  // the slot of the token (the oldest one's when full)
    for (int i = tid; i < count; i += kDryThreads) {
        const int idx = (head + i) % window;
        s_h[i] = idx == at ? token : ring[idx];
    }
    if (tid == 0) s_m = 0;
    __syncthreads();
    if (tid == 0) {
        ring[at] = token;
        a.head[s] = head;
        a.count[s] = count;
    }
    const int n = count;
    const DryConfigD & c = a.cfg;
    if (n < max(1, c.allowed_length)) {  // (:92-93)
        if (tid == 0) a.pen_n[s] = 0;
        return;
    }
    // every earlier occurrence of the last token within the lookback: the match ending there (:95-104)
    const int32_t last = s_h[n - 1];
    const int jlo = max(0, n - 1 - c.lookback);
    for (int j = n - 2 - tid; j >= jlo; j -= kDryThreads) {
        if (s_h[j] != last) continue;
        int length = 1;
        while (length < c.max_match_length && j - length >= 0 && s_h[j - length] == s_h[n - 1 - length]) length++;
        if (length >= c.allowed_length) {
            const int slot = atomicAdd(&s_m, 1);
            s_rec[slot] = ((uint64_t) (uint32_t) s_h[j + 1] << 32) | (uint32_t) length;
        }
    }
    __syncthreads();
    const int m = s_m;
    if (m == 0) {
        if (tid == 0) a.pen_n[s] = 0;
        return;
    }
    const int mp2 = next_pow2(m);
    for (int i = m + tid; i < mp2; i += kDryThreads) s_rec[i] = 0ull;  // below every record (sorted last)
    __syncthreads();
    bitonic_sort_desc(s_rec, mp2);  // by falling token, the longest match first within a token
    // the first record of each token = its longest match; exempt tokens get no penalty (:106-108).
    // Thread t takes records [t*per, (t+1)*per); the kept ones are numbered by a block scan.
    const int per = (m + kDryThreads - 1) / kDryThreads;
    const int lo = min(m, tid * per), hi = min(m, lo + per);
    auto keep = [&](int i) {
        const int32_t t = (int32_t) (s_rec[i] >> 32);
        return (i == 0 || (int32_t) (s_rec[i - 1] >> 32) != t) && !is_exempt(s_ex, a.n_exempt, t);
    };
    int mine = 0;
    for (int i = lo; i < hi; i++) mine += keep(i) ? 1 : 0;
    s_base[tid + 1] = mine;
    __syncthreads();
    if (tid == 0) {
        s_base[0] = 0;
        for (int t = 1; t <= kDryThreads; t++) s_base[t] += s_base[t - 1];
    }
    __syncthreads();
    const int total = s_base[kDryThreads];
    int32_t * pt = a.pen_tok + (int64_t) s * a.pen_cap;
    double * pv = a.pen_val + (int64_t) s * a.pen_cap;
    int r = s_base[tid];
    for (int i = lo; i < hi; i++) {
        if (!keep(i)) continue;
        const int32_t t = (int32_t) (s_rec[i] >> 32);
        const int length = (int) (uint32_t) s_rec[i];
        const double pen = fmin(c.max_penalty, c.multiplier * pow(c.base, (double) (length - c.allowed_length)));
        const int out = total - 1 - r;  // records fall by token; the penalties rise by token
        pt[out] = t;
        pv[out] = pen;
        r++;
    }
    if (tid == 0) a.pen_n[s] = total;
}

__global__ void __launch_bounds__(kShapeThreads) haru_shape_kernel(const __grid_constant__ ShapeArgs a) {
    const int r = blockIdx.x, tid = (int) threadIdx.x;
    float * row = a.logits + (int64_t) r * a.ld;
    if (a.pen_n) {
        const int n = a.pen_n[r];
        const int32_t * pt = a.pen_tok + (int64_t) r * a.pen_cap;
        const double * pv = a.pen_val + (int64_t) r * a.pen_cap;
        for (int i = tid; i < n; i += kShapeThreads) {  // distinct tokens: no two threads write one logit
            const int32_t t = pt[i];
            if (t >= 0 && t < a.vocab) row[t] = __fsub_rn(row[t], (float) pv[i]);
        }
    }
    __syncthreads();  // the replacements come after the penalties (:117-119)
    if (tid == 0) {
        const float * sil = a.silent + (int64_t) r * a.silent_ld;
        row[a.pad] = sil[0];
        row[a.eop] = sil[1];
        if (a.eop_bias != 0.0f) row[a.eop] = __fadd_rn(row[a.eop], a.eop_bias);
        if (a.must_speak && a.must_speak[r]) row[a.pad] = -kInf, row[a.eop] = -kInf, row[a.eos] = -kInf;
    }
}

}  // namespace

size_t dry_smem_bytes(int window) { return (size_t) next_pow2(window) * 8 + (size_t) window * 4; }

cudaError_t launch_dry_update(const DryArgs & a, const int32_t * tokens, cudaStream_t stream) {
    const size_t smem = dry_smem_bytes(a.window);
    cudaError_t e = ssb::set_max_dynamic_smem((const void *) dry_update_kernel, smem);
    if (e != cudaSuccess) return e;
    dry_update_kernel<<<a.streams, kDryThreads, smem, stream>>>(a, tokens);
    return cudaGetLastError();
}

cudaError_t launch_haru_shape(const ShapeArgs & a, cudaStream_t stream) {
    haru_shape_kernel<<<a.rows, kShapeThreads, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace ssb
