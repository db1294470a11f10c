// Device building blocks shared by the sampler kernels (sm_100a).
//
// Candidate order. The reference's candidates() orders tokens by falling scaled logit
// (src/families/qwen3-tts/sampler.cpp:78-79) and this engine breaks ties by lowest index, Haru's
// comparator (src/families/haru/sampler.cpp:39). Both are encoded in one 64-bit "composite" key:
//     composite = order_key(scaled) << 32 | ~index
// where order_key maps floats to uint32 monotonically (with -0 folded onto +0, since the reference
// compares with `>` and -0 == +0). A larger composite comes first; all composites of a row differ.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "speech_sampler_b200.h"

namespace ssb {

constexpr float kInf = __builtin_huge_valf();

// ---------------------------------------------------------------- keys and values
__device__ __forceinline__ uint32_t order_key(float f) {
    uint32_t b = __float_as_uint(f);
    if ((b << 1) == 0) b = 0;  // -0 -> +0
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float key_value(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__device__ __forceinline__ uint64_t composite(float s, uint32_t index) {
    return ((uint64_t) order_key(s) << 32) | (uint32_t) ~index;
}

__device__ __forceinline__ uint32_t composite_index(uint64_t c) { return ~(uint32_t) c; }
__device__ __forceinline__ float composite_value(uint64_t c) { return key_value((uint32_t) (c >> 32)); }

// NaN-propagating max (PTX max.NaN, sm_80+): a NaN anywhere in a reduction survives to its end.
__device__ __forceinline__ float max_nan(float a, float b) {
    float d;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}

// bf16 halves of a 32-bit word, widened exactly.
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

template <typename TIn> struct Elem;
template <> struct Elem<float> {
    static constexpr int kVec = 4;  // elements per 16-byte vector
    __device__ static __forceinline__ float load1(const float * p, int64_t i) { return __ldg(p + i); }
    __device__ static __forceinline__ void unpack(const uint4 & v, float * out) {
        out[0] = __uint_as_float(v.x), out[1] = __uint_as_float(v.y);
        out[2] = __uint_as_float(v.z), out[3] = __uint_as_float(v.w);
    }
};
template <> struct Elem<uint16_t> {
    static constexpr int kVec = 8;
    __device__ static __forceinline__ float load1(const uint16_t * p, int64_t i) {
        return __uint_as_float((uint32_t) __ldg(p + i) << 16);
    }
    __device__ static __forceinline__ void unpack(const uint4 & v, float * out) {
        out[0] = bf16_lo(v.x), out[1] = bf16_hi(v.x), out[2] = bf16_lo(v.y), out[3] = bf16_hi(v.y);
        out[4] = bf16_lo(v.z), out[5] = bf16_hi(v.z), out[6] = bf16_lo(v.w), out[7] = bf16_hi(v.w);
    }
};

// Streaming 16-byte load that does not allocate in L1 (each logits byte is read once).
__device__ __forceinline__ uint4 ld_stream(const void * p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// ---------------------------------------------------------------- per-row settings
struct RowParams {
    int greedy;
    float temperature;
    int k;  // effective top-k: min(top_k, vocab), or vocab for top_k <= 0
    float top_p;
    float rep, presence, frequency;
    bool history_applies;  // a repetition, presence or frequency penalty is active
    bool fast_scale;       // temperature is a normal positive float within [2^-100, 2^100]
};

__device__ __forceinline__ RowParams resolve_params(const ssb_params & p, int vocab) {
    RowParams r;
    r.greedy = p.greedy != 0;
    r.temperature = p.temperature;
    r.k = p.top_k > 0 ? (p.top_k < vocab ? p.top_k : vocab) : vocab;
    r.top_p = p.top_p;
    r.rep = p.repetition_penalty;
    r.presence = p.presence_penalty;
    r.frequency = p.frequency_penalty;
    const bool ext = p.presence_penalty != 0.0f || p.frequency_penalty != 0.0f;
    r.history_applies = p.repetition_penalty != 1.0f || ext;
    const float t = p.temperature;
    r.fast_scale = t >= 0x1p-100f && t <= 0x1p100f;  // false for NaN, <= 0, inf, tiny or huge
    return r;
}

// The penalties of one history token with `count` occurrences (qwen3-tts/sampler.cpp:36-38, then the
// presence/frequency extension). Explicit _rn intrinsics keep every step a single rounding, as the
// CPU restatement computes it with -ffp-contract=off.
__device__ __forceinline__ float penalize(float l, int count, const RowParams & p) {
    if (p.rep != 1.0f) l = l < 0.0f ? __fmul_rn(l, p.rep) : __fdiv_rn(l, p.rep);
    if (p.presence != 0.0f || p.frequency != 0.0f) {
        l = __fsub_rn(l, __fmul_rn(p.frequency, (float) count));
        l = __fsub_rn(l, p.presence);
    }
    return l;
}

__device__ __forceinline__ bool masked_bit(uint32_t word_bits, int mask_kind) {
    return mask_kind == SSB_MASK_BAN ? (word_bits & 1u) : (mask_kind == SSB_MASK_ALLOW ? !(word_bits & 1u) : false);
}

// Status of a row from the maximum of its restricted logits (qwen3-tts/sampler.cpp:43-49), with NaN
// refused first (a NaN max means a NaN among them).
__device__ __forceinline__ int restricted_status(float raw_max, float rep) {
    if (raw_max != raw_max) return SSB_ROW_NON_FINITE_INPUT;
    if (raw_max == kInf && rep != 1.0f) return SSB_ROW_PENALTY_OVERFLOW;
    if (!(raw_max > -kInf && raw_max < kInf)) return SSB_ROW_NO_FINITE_LOGIT;
    return SSB_ROW_OK;
}

// A raw-logit bound for the stream filter: every x whose scaled value x/T can reach the scaled value
// s satisfies x >= bound. Valid when T is a normal positive float and s is normal; -inf otherwise
// (no filtering: every element then takes the exact path).
//   fl(x/T) >= s  =>  x/T >= s - ulp(s)/2  =>  x >= T*s*(1 - 2^-23) (s > 0) or T*s*(1 + 2^-23) (s < 0),
// and y = fl(s*T) is within a factor (1 +- 2^-24) of T*s, so y - |y|*2^-20 lies below both.
__device__ __forceinline__ float raw_bound(float s, float t, bool fast_scale) {
    if (!fast_scale) return -kInf;
    const float a = fabsf(s);
    if (!(a >= 0x1p-100f && a <= 0x1p100f)) return -kInf;
    const float y = __fmul_rn(s, t);
    return __fsub_rn(y, __fmul_rn(fabsf(y), 0x1p-20f));
}

// ---------------------------------------------------------------- warp / block helpers
__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }
__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }

template <typename T> __device__ __forceinline__ T shfl_xor(T v, int m) { return __shfl_xor_sync(0xffffffffu, v, m); }

__device__ __forceinline__ float warp_max_nan(float v) {
#pragma unroll
    for (int m = 16; m; m >>= 1) v = max_nan(v, shfl_xor(v, m));
    return v;
}

__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
    for (int m = 16; m; m >>= 1) {
        const uint64_t o = shfl_xor(v, m);
        v = o > v ? o : v;
    }
    return v;
}

__device__ __forceinline__ uint64_t warp_min_u64(uint64_t v) {
#pragma unroll
    for (int m = 16; m; m >>= 1) {
        const uint64_t o = shfl_xor(v, m);
        v = o < v ? o : v;
    }
    return v;
}

// Block reductions through a 32-entry shared scratch; every thread gets the result.
__device__ __forceinline__ float block_max_nan(float v, float * scratch) {
    v = warp_max_nan(v);
    __syncthreads();
    if (lane_id() == 0) scratch[warp_id()] = v;
    __syncthreads();
    const int nw = blockDim.x >> 5;
    float r = lane_id() < nw ? scratch[lane_id()] : -kInf;
    r = warp_max_nan(r);
    return r;
}

__device__ __forceinline__ uint64_t block_max_u64(uint64_t v, uint64_t * scratch) {
    v = warp_max_u64(v);
    __syncthreads();
    if (lane_id() == 0) scratch[warp_id()] = v;
    __syncthreads();
    const int nw = blockDim.x >> 5;
    uint64_t r = lane_id() < nw ? scratch[lane_id()] : 0ull;
    return warp_max_u64(r);
}

__device__ __forceinline__ uint64_t block_min_u64(uint64_t v, uint64_t * scratch) {
    v = warp_min_u64(v);
    __syncthreads();
    if (lane_id() == 0) scratch[warp_id()] = v;
    __syncthreads();
    const int nw = blockDim.x >> 5;
    uint64_t r = lane_id() < nw ? scratch[lane_id()] : ~0ull;
    return warp_min_u64(r);
}

__device__ __forceinline__ int block_or(int v, int * scratch) {
    v = __any_sync(0xffffffffu, v);
    __syncthreads();
    if (lane_id() == 0) scratch[warp_id()] = v;
    __syncthreads();
    const int nw = blockDim.x >> 5;
    return __any_sync(0xffffffffu, lane_id() < nw ? scratch[lane_id()] : 0);
}

__device__ __forceinline__ int block_sum_int(int v, int * scratch) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane_id() == 0) scratch[warp_id()] = v;
    __syncthreads();
    const int nw = blockDim.x >> 5;
    int t = lane_id() < nw ? scratch[lane_id()] : 0;
#pragma unroll
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return t;
}

__device__ __forceinline__ int block_max_int(int v, int * scratch) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane_id() == 0) scratch[warp_id()] = v;
    __syncthreads();
    const int nw = blockDim.x >> 5;
    int t = lane_id() < nw ? scratch[lane_id()] : INT_MIN;
#pragma unroll
    for (int o = 16; o; o >>= 1) t = max(t, __shfl_xor_sync(0xffffffffu, t, o));
    return t;
}

// ---------------------------------------------------------------- 16-bit key histograms
// Adds one to bin `bin` of a shared histogram for every lane with `take` (plain shared atomics: cheaper
// here than aggregating equal bins first).
__device__ __forceinline__ void red_bin(uint32_t * hist, bool take, uint32_t bin) {
    if (take) atomicAdd(&hist[bin], 1u);
}

// In a 256-bin histogram (a larger bin holds larger keys), the bin holding the need-th key from the top,
// with the number of keys in the bins above it; -1 when the histogram holds fewer than `need` keys.
// Warp-wide; the result is the same on every lane.
__device__ __forceinline__ int top_bin(const uint32_t * hist, uint32_t need, uint32_t * above) {
    const int lane = lane_id();
    // lane L takes bins 255 - 8L down to 248 - 8L
    const uint4 h0 = reinterpret_cast<const uint4 *>(hist)[63 - 2 * lane];
    const uint4 h1 = reinterpret_cast<const uint4 *>(hist)[62 - 2 * lane];
    const uint32_t c[8] = {h0.w, h0.z, h0.y, h0.x, h1.w, h1.z, h1.y, h1.x};
    uint32_t sum = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) sum += c[i];
    uint32_t incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    const unsigned hit = __ballot_sync(0xffffffffu, incl >= need);
    if (!hit) return -1;
    const int fl = __ffs(hit) - 1;
    uint32_t run = incl - sum;  // keys in the bins above this lane's
    int bin = -1;
    uint32_t ab = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        if (bin < 0 && run + c[i] >= need) bin = 255 - 8 * lane - i, ab = run;
        run += c[i];
    }
    *above = __shfl_sync(0xffffffffu, ab, fl);
    return __shfl_sync(0xffffffffu, bin, fl);
}

// ---------------------------------------------------------------- radix select on composites
// Shared state of one selection.
struct SelectState {
    uint32_t hist[256];
    uint64_t prefix;
    int shift;      // bits below the decided prefix
    int remaining;  // how many still to take from the prefix's bucket
    int done;
};

// Selects the `k` largest composites among n produced by key_of(i) (i in [0, n)), 1 <= k <= n.
// Afterwards an element is selected iff (key >> st.shift) >= (st.prefix >> st.shift), equivalently
// key >= st.prefix (its bits below st.shift are zero): digits of 8 bits from the top, stopping as soon
// as the bucket holding the k-th is taken whole, or after `max_rounds` digits — then the selection
// holds at least k elements (the k best and the rest of their bucket). Block-wide.
template <typename KeyOf>
__device__ inline void radix_select(int n, int k, KeyOf key_of, SelectState & st, int max_rounds = 8) {
    if (threadIdx.x == 0) {
        st.prefix = 0;
        st.shift = 64;
        st.remaining = k;
        st.done = 0;
    }
    __syncthreads();
    while (true) {
        const int shift = st.shift - 8;
        const uint64_t prefix = st.prefix;
        const uint64_t hi_mask = shift + 8 >= 64 ? 0ull : (~0ull << (shift + 8));
        for (int i = threadIdx.x; i < 256; i += blockDim.x) st.hist[i] = 0;
        if (threadIdx.x == 0) st.done = 1;  // a round in which no lane claims a digit ends the loop
        __syncthreads();
        for (int base = 0; base < n; base += blockDim.x) {  // warp-uniform trip count
            const int i = base + threadIdx.x;
            uint64_t c = 0;
            bool match = false;
            if (i < n) {
                c = key_of(i);
                match = ((c ^ prefix) & hi_mask) == 0;
            }
            const uint32_t bin = (uint32_t) (c >> shift) & 255u;
            const unsigned m = __ballot_sync(0xffffffffu, match);
            if (match) {
                const unsigned peers = __match_any_sync(m, bin);
                if ((int) (__ffs(peers) - 1) == lane_id()) atomicAdd(&st.hist[bin], (uint32_t) __popc(peers));
            }
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            // lane L owns bins 255-8L .. 248-8L (descending); find the bin where the count from the top
            // reaches `remaining`.
            const int lane = threadIdx.x;
            uint32_t c[8];
            uint32_t sum = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) c[j] = st.hist[255 - 8 * lane - j], sum += c[j];
            uint32_t incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += t;
            }
            const uint32_t excl = incl - sum;
            const int rem = st.remaining;
            const bool mine = excl < (uint32_t) rem && incl >= (uint32_t) rem;
            if (mine) {
                uint32_t above = excl;
                int j = 0;
                for (; j < 8; j++) {
                    if (above + c[j] >= (uint32_t) rem) break;
                    above += c[j];
                }
                const uint32_t digit = 255u - 8u * lane - (uint32_t) j;
                st.prefix = prefix | ((uint64_t) digit << shift);
                st.remaining = rem - (int) above;
                st.shift = shift;
                st.done = (c[j] == (uint32_t) (rem - (int) above)) || shift <= 64 - 8 * max_rounds;
            }
        }
        __syncthreads();
        // read st.done inside a barrier: thread 0 resets it at the start of the next round
        if (__syncthreads_or(threadIdx.x == 0 && st.done)) break;
    }
}

__device__ __forceinline__ bool selected(uint64_t c, const SelectState & st) {
    return st.shift >= 64 ? true : (c >> st.shift) >= (st.prefix >> st.shift);
}

// Descending bitonic sort of the 32*R u64 held by one warp, element r*32 + lane in x[r]. Warp-wide,
// registers and shuffles only.
template <int R>
__device__ __forceinline__ void warp_sort_desc(uint64_t (&x)[R]) {
    const int lane = lane_id();
#pragma unroll
    for (int size = 2; size <= 32 * R; size <<= 1) {
#pragma unroll
        for (int j = size >> 1; j > 0; j >>= 1) {
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int i = r * 32 + lane;
                const bool desc = (i & size) == 0;
                if (j >= 32) {
                    const int rp = r ^ (j >> 5);
                    if (rp > r) {
                        const uint64_t a = x[r], b = x[rp];
                        if ((a < b) == desc) x[r] = b, x[rp] = a;
                    }
                } else {
                    const uint64_t o = shfl_xor(x[r], j);
                    const bool keep_max = ((lane & j) == 0) == desc;
                    x[r] = keep_max ? (x[r] > o ? x[r] : o) : (x[r] < o ? x[r] : o);
                }
            }
        }
    }
}

// Descending bitonic sort of n (a power of two) u64 in shared memory. Block-wide.
__device__ inline void bitonic_sort_desc(uint64_t * x, int n) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < (n >> 1); i += blockDim.x) {
                const int lo = 2 * stride * (i / stride) + (i % stride);
                const int hi = lo + stride;
                const bool desc = (lo & size) == 0;
                const uint64_t a = x[lo], b = x[hi];
                if ((a < b) == desc) x[lo] = b, x[hi] = a;
            }
            __syncthreads();
        }
    }
}

// Ascending bitonic sort of n (a power of two) int32 in shared memory. Block-wide.
__device__ inline void bitonic_sort_asc_i32(int32_t * x, int n) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < (n >> 1); i += blockDim.x) {
                const int lo = 2 * stride * (i / stride) + (i % stride);
                const int hi = lo + stride;
                const bool asc = (lo & size) == 0;
                const int32_t a = x[lo], b = x[hi];
                if ((a > b) == asc) x[lo] = b, x[hi] = a;
            }
            __syncthreads();
        }
    }
}

__host__ __device__ __forceinline__ int next_pow2(int v) {
    int p = 1;
    while (p < v) p <<= 1;
    return p;
}

// ---------------------------------------------------------------- finalize one drawing row
// Outputs of one row; the debug export fields are null in the product path.
struct RowOut {
    int32_t * id;
    int32_t * status;
    int32_t * tokens;   // [cap] or null
    double * weights;   // [cap] or null
    int32_t * count;    // or null
    int cap;
};

// The running sum of w[0 .. n) in index order (the reference's sequential accumulation from 0), one
// thread: the first index at which it reaches `limit` (`strict`: exceeds it) or n, with the sum there
// (or over all n) in *at_sum. `limit` = +inf gives the plain ordered sum. The next 8 values load while
// the current 8 are added, so the chain runs at the latency of the additions.
__device__ __forceinline__ int chain_reach(const double * w, int n, double limit, bool strict, double * at_sum) {
    double s = 0.0;
    int at = n;
    double cur[8], nxt[8];
#pragma unroll
    for (int j = 0; j < 8; j++) cur[j] = j < n ? w[j] : 0.0;
    for (int i = 0; i < n; i += 8) {
#pragma unroll
        for (int j = 0; j < 8; j++) nxt[j] = i + 8 + j < n ? w[i + 8 + j] : 0.0;
        bool done = false;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            if (!done && i + j < n) {
                s = __dadd_rn(s, cur[j]);
                if (strict ? s > limit : s >= limit) {
                    at = i + j;
                    done = true;
                }
            }
        }
        if (done) break;
#pragma unroll
        for (int j = 0; j < 8; j++) cur[j] = nxt[j];
    }
    *at_sum = s;
    return at;
}

// The draw of one row by one warp (warp-synchronous, no block barrier): the reference's softmax, top-p
// cut and pick() over the k candidates sorted by composite (descending), as IEEE double operations in
// the reference's order (qwen3-tts/sampler.cpp:80-99, sampling.cpp:9-19). The parallel steps (exp, the divisions) run across the lanes with all of a lane's operations
// issued together; the three running sums (the softmax total, the top-p cut, pick()) run on lane 0. The
// kept total of pick() is the top-p running sum at the cut (the same additions, from 0, in the same
// order). `w` is shared scratch of k doubles; lane 0 writes the outputs.
__device__ inline void finalize_draw_warp(const uint64_t * sorted, int k, const RowParams & p, double u, double * w,
                                          const RowOut & out) {
    const int lane = lane_id();
    const float max_logit = composite_value(sorted[0]);
    if (!(max_logit > -kInf && max_logit < kInf)) {
        if (lane == 0) {
            *out.id = -1;
            *out.status = SSB_ROW_TEMPERATURE_OVERFLOW;
            if (out.count) *out.count = 0;
        }
        return;
    }
    // softmax (qwen3-tts/sampler.cpp:80-87)
    for (int base = 0; base < k; base += 128) {
        double e[4];
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int i = base + lane + 32 * r;
            e[r] = i < k ? exp((double) composite_value(sorted[i]) - (double) max_logit) : 0.0;
        }
#pragma unroll
        for (int r = 0; r < 4; r++)
            if (base + lane + 32 * r < k) w[base + lane + 32 * r] = e[r];
    }
    __syncwarp();
    double sum = 0.0;
    if (lane == 0) chain_reach(w, k, kInf, true, &sum);
    sum = __shfl_sync(0xffffffffu, sum, 0);
    for (int base = 0; base < k; base += 128) {
        double q[4];
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int i = base + lane + 32 * r;
            q[r] = i < k ? __ddiv_rn(w[i], sum) : 0.0;
        }
#pragma unroll
        for (int r = 0; r < 4; r++)
            if (base + lane + 32 * r < k) w[base + lane + 32 * r] = q[r];
    }
    __syncwarp();
    // top-p cut (:88-99): keep through the first running share >= top_p (all k when none, or top_p >= 1);
    // the running sum there is pick()'s total over the kept weights
    int keep = k;
    double total = 0.0;
    if (lane == 0) {
        const int at = chain_reach(w, k, p.top_p < 1.0f ? (double) p.top_p : kInf, false, &total);
        keep = at < k ? at + 1 : k;
    }
    keep = __shfl_sync(0xffffffffu, keep, 0);
    total = __shfl_sync(0xffffffffu, total, 0);
    if (out.tokens) {
        for (int i = lane; i < keep && i < out.cap; i += 32) {
            out.tokens[i] = (int32_t) composite_index(sorted[i]);
            out.weights[i] = w[i];
        }
    }
    __syncwarp();
    // pick() (sampling.cpp:9-19): the renormalized shares, then the first running sum > u (else the last)
    for (int base = 0; base < keep - 1; base += 128) {
        double q[4];
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int i = base + lane + 32 * r;
            q[r] = i < keep - 1 ? __ddiv_rn(w[i], total) : 0.0;
        }
#pragma unroll
        for (int r = 0; r < 4; r++)
            if (base + lane + 32 * r < keep - 1) w[base + lane + 32 * r] = q[r];
    }
    __syncwarp();
    if (lane == 0) {
        double unused;
        const int chosen = chain_reach(w, keep - 1, u, true, &unused);  // keep - 1 (the last) when none passes
        *out.id = (int32_t) composite_index(sorted[chosen]);
        *out.status = SSB_ROW_OK;
        if (out.count) *out.count = keep;
    }
}

// Margin that separates the crossings of the parallel draw from those of the reference's sequential
// sums. The reference divides each weight by its sequential total, accumulates the shares in order and
// (for pick()) renormalizes by the kept total; the parallel draw compares prefix sums of the same
// exponentials (summed in another order) against top_p times their total, and against u times the kept
// prefix. With n <= 128 terms >= 0, every one of these sums and quotients lies within 8 n u (u = 2^-53)
// of its exact value, relative to the total: under 1.2e-13. Crossings farther than kDrawMargin (times
// the total) from their limits are decided identically.
constexpr double kDrawMargin = 1e-11;

// The draw of one row by one warp without divisions and with warp scans instead of sequential chains
// (k <= 128): e_i = exp(s_i - max) as the reference computes them, E_i their running sums (four per
// lane, then a warp scan), S = E_{k-1}. The top-p cut is the first i with E_i >= top_p S, pick() the
// first i < keep - 1 with E_i > u E_{keep-1} (else keep - 1). The id equals finalize_draw_warp's
// whenever each decided comparison clears its limit by kDrawMargin of the total; otherwise it returns
// false without writing anything and the caller runs finalize_draw_warp. Registers and shuffles only.
__device__ __forceinline__ bool draw_parallel(const uint64_t * sorted, int k, const RowParams & p, double u,
                                              const RowOut & out) {
    const int lane = lane_id();
    const float max_logit = composite_value(sorted[0]);
    if (!(max_logit > -kInf && max_logit < kInf)) return false;
    double e[4];
#pragma unroll
    for (int r = 0; r < 4; r++) {
        const int i = 4 * lane + r;
        e[r] = i < k ? exp((double) composite_value(sorted[i]) - (double) max_logit) : 0.0;
    }
    // running sums in index order: lane-local, then a warp scan of the lanes' totals
    e[1] = __dadd_rn(e[0], e[1]);
    e[2] = __dadd_rn(e[1], e[2]);
    e[3] = __dadd_rn(e[2], e[3]);
    double incl = e[3];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl = __dadd_rn(incl, t);
    }
    const double before = __shfl_up_sync(0xffffffffu, incl, 1);
    if (lane > 0) {
#pragma unroll
        for (int r = 0; r < 4; r++) e[r] = __dadd_rn(before, e[r]);
    }
    auto get = [&](int i) {  // E_i for a warp-uniform i
        const int r = i & 3;
        const double v = r == 0 ? e[0] : (r == 1 ? e[1] : (r == 2 ? e[2] : e[3]));
        return __shfl_sync(0xffffffffu, v, i >> 2);
    };
    auto first = [&](int n, double limit, bool strict) {  // first i < n with E_i >= limit (> when strict), or n
        int f = 4;
#pragma unroll
        for (int r = 3; r >= 0; r--) {
            const int i = 4 * lane + r;
            if (i < n && (strict ? e[r] > limit : e[r] >= limit)) f = r;
        }
        const unsigned hit = __ballot_sync(0xffffffffu, f < 4);
        if (!hit) return n;
        const int fl = __ffs(hit) - 1;
        return 4 * fl + __shfl_sync(0xffffffffu, f, fl);
    };
    const double S = get(k - 1);
    const double m = kDrawMargin * S;
    int keep = k;
    if (p.top_p < 1.0f) {
        const double lim = (double) p.top_p * S;
        const int at = first(k, lim, false);
        if (at < k) {
            if (!(get(at) >= lim + m)) return false;
            if (at > 0 && !(get(at - 1) < lim - m)) return false;
            keep = at + 1;
        } else if (!(get(k - 1) < lim - m)) {
            return false;
        }
    }
    const int n = keep - 1;
    const double kept = get(n);
    const double lim2 = u * kept;
    const int ch = first(n, lim2, true);
    if (ch < n) {
        if (!(get(ch) > lim2 + m)) return false;
        if (ch > 0 && !(get(ch - 1) <= lim2 - m)) return false;
    } else if (n > 0 && !(get(n - 1) <= lim2 - m)) {
        return false;
    }
    if (lane == 0) {
        *out.id = (int32_t) composite_index(sorted[ch]);
        *out.status = SSB_ROW_OK;
        if (out.count) *out.count = keep;
    }
    return true;
}

// The draw of a row by one warp: the parallel draw where it decides the id, else the sequential one
// (always for the candidate export, which needs the weights).
__device__ inline void draw_row(const uint64_t * sorted, int k, const RowParams & p, double u, double * w,
                                const RowOut & out) {
    if (k <= 128 && !out.tokens && draw_parallel(sorted, k, p, u, out)) return;
    finalize_draw_warp(sorted, k, p, u, w, out);
}

}  // namespace ssb
