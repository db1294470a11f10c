// Pieces of the large-vocabulary top-k kernel (ssb_topk.cu): TMA bulk copies into a shared-memory ring
// paced by mbarriers, and the per-lane reductions of the 16-byte groups a consumer lane takes from each
// stage.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>

#include "ssb_device.cuh"

namespace ssb {
namespace {

constexpr int kStageBytes = 16384;
constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kStreamCtaThreads = kConsumers + 32;  // + the producer warp
constexpr int kStageGroups = kStageBytes / 16;      // 16-byte groups per stage
constexpr int kGroupsPerThread = kStageGroups / kConsumers;
// Bounded mbarrier waits: a wait gives up after this many SM clock cycles (about 1 s at 1.9 GHz).
// The wait-limit test build (SSB_WAIT_TEST) shortens it so that its planted missing stage times out
// quickly.
#ifdef SSB_WAIT_TEST
constexpr long long kWaitCycles = 1ll << 22;
#else
constexpr long long kWaitCycles = 1ll << 31;
#endif

static_assert(kGroupsPerThread * kConsumers * 16 == kStageBytes, "stage must split evenly");
static_assert(kGroupsPerThread == 4, "a lane holds four groups of a stage");

__device__ __forceinline__ uint32_t smem_addr(const void * p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect(uint64_t * bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t * bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// One test of phase `parity` of `bar`; the thread may be suspended (not spinning, so it takes no issue
// slots from the warps that work meanwhile) until the phase completes or about kSuspendNs pass.
constexpr uint32_t kSuspendNs = 100000;
__device__ __forceinline__ bool mbar_try_wait(uint64_t * bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendNs)
        : "memory");
    return ok != 0;
}

// Waits for phase `parity` of `bar`, giving up after kWaitCycles clock cycles (returns false).
__device__ __forceinline__ bool mbar_wait(uint64_t * bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (clock64() - t0 > kWaitCycles) return false;
    }
}

// Barrier of `threads` threads (a multiple of 32) on hardware barrier `id` (1..15; 0 is __syncthreads).
__device__ __forceinline__ void bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// One TMA bulk copy global -> shared, completing on `bar` (both addresses and the size are multiples
// of 16 bytes). No cluster multicast.
__device__ __forceinline__ void bulk_load(void * dst, const void * src, uint32_t bytes, uint64_t * bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

// NaN-propagating maximum of one 16-byte group.
template <typename TIn> __device__ __forceinline__ float group_max(const uint4 & r);
template <> __device__ __forceinline__ float group_max<uint16_t>(const uint4 & r) {
    const __nv_bfloat162 a = __hmax2_nan(*reinterpret_cast<const __nv_bfloat162 *>(&r.x),
                                         *reinterpret_cast<const __nv_bfloat162 *>(&r.y));
    const __nv_bfloat162 b = __hmax2_nan(*reinterpret_cast<const __nv_bfloat162 *>(&r.z),
                                         *reinterpret_cast<const __nv_bfloat162 *>(&r.w));
    const __nv_bfloat162 m = __hmax2_nan(a, b);
    const uint32_t w = *reinterpret_cast<const uint32_t *>(&m);
    return max_nan(bf16_lo(w), bf16_hi(w));
}
template <> __device__ __forceinline__ float group_max<float>(const uint4 & r) {
    return max_nan(max_nan(__uint_as_float(r.x), __uint_as_float(r.y)), max_nan(__uint_as_float(r.z), __uint_as_float(r.w)));
}

// The maximum of a lane's four groups, NaN if any element is NaN: one packed reduction for bf16.
template <typename TIn> __device__ __forceinline__ float lane_max(const uint4 (&r)[kGroupsPerThread]);
template <> __device__ __forceinline__ float lane_max<uint16_t>(const uint4 (&r)[kGroupsPerThread]) {
    __nv_bfloat162 m[kGroupsPerThread];
#pragma unroll
    for (int j = 0; j < kGroupsPerThread; j++) {
        const __nv_bfloat162 a = __hmax2_nan(*reinterpret_cast<const __nv_bfloat162 *>(&r[j].x),
                                             *reinterpret_cast<const __nv_bfloat162 *>(&r[j].y));
        const __nv_bfloat162 b = __hmax2_nan(*reinterpret_cast<const __nv_bfloat162 *>(&r[j].z),
                                             *reinterpret_cast<const __nv_bfloat162 *>(&r[j].w));
        m[j] = __hmax2_nan(a, b);
    }
    const __nv_bfloat162 t = __hmax2_nan(__hmax2_nan(m[0], m[1]), __hmax2_nan(m[2], m[3]));
    const uint32_t w = *reinterpret_cast<const uint32_t *>(&t);
    return max_nan(bf16_lo(w), bf16_hi(w));
}
template <> __device__ __forceinline__ float lane_max<float>(const uint4 (&r)[kGroupsPerThread]) {
    return max_nan(max_nan(group_max<float>(r[0]), group_max<float>(r[1])),
                   max_nan(group_max<float>(r[2]), group_max<float>(r[3])));
}

// A group of -inf elements, standing in for the missing groups of a partial stage.
template <typename TIn> __device__ __forceinline__ uint4 neg_inf_group() {
    const uint32_t w = sizeof(TIn) == 2 ? 0xFF80FF80u : 0xFF800000u;
    return make_uint4(w, w, w, w);
}

// Multiplicative hash of a token id into `bits` bits (Knuth's multiplicative method).
__device__ __forceinline__ uint32_t hash_token(int32_t t, int bits) { return ((uint32_t) t * 0x9E3779B1u) >> (32 - bits); }

// Element i (= r * 32 + lane) of a warp-distributed array, for a warp-uniform i.
template <int R>
__device__ __forceinline__ uint64_t warp_get(const uint64_t (&x)[R], int i) {
    uint64_t v = 0;
#pragma unroll
    for (int r = 0; r < R; r++)
        if (r == (i >> 5)) v = x[r];
    return __shfl_sync(0xffffffffu, v, i & 31);
}

// Merges the sorted (descending) 32*KW elements of `q` with the sorted 32*KW elements of `t`, keeping
// the best 32*KW sorted in q: max against t reversed gives a bitonic sequence holding the best half,
// which a bitonic clean-up sorts.
template <int KW>
__device__ __forceinline__ void warp_merge_sorted(uint64_t (&q)[KW], const uint64_t (&t)[KW]) {
    const int lane = lane_id();
#pragma unroll
    for (int r = 0; r < KW; r++) {
        const uint64_t o = __shfl_sync(0xffffffffu, t[KW - 1 - r], 31 - lane);
        q[r] = q[r] > o ? q[r] : o;
    }
#pragma unroll
    for (int j = 16 * KW; j > 0; j >>= 1) {
#pragma unroll
        for (int r = 0; r < KW; r++) {
            if (j >= 32) {
                const int rp = r ^ (j >> 5);
                if (rp > r) {
                    const uint64_t a = q[r], b = q[rp];
                    if (a < b) q[r] = b, q[rp] = a;
                }
            } else {
                const uint64_t o = shfl_xor(q[r], j);
                const bool keep_max = (lane & j) == 0;
                q[r] = keep_max ? (q[r] > o ? q[r] : o) : (q[r] < o ? q[r] : o);
            }
        }
    }
}

}  // namespace
}  // namespace ssb
