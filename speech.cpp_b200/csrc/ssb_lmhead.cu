// The LM head and its greedy pick fused (src/common/qwen3-decoder.cpp:422-437 Qwen3Readback::Pick and
// :492-510 verify): ids[r] = argmax_v (hidden[r] . weight[v]) for bf16 hidden rows [rows, dim] and the bf16
// head [vocab, dim], fp32 accumulation on the 5th-generation tensor cores, and the logits never written.
//
// One persistent CTA per SM walks 128-token tiles of the vocabulary. Warp roles:
//   warp 0     TMA producer: per 64-wide slice of dim, the head tile [128 x 64] and the hidden rows
//              [N x 64] (rows past `rows` zero-filled by the tensor map) into a ring of shared-memory
//              stages, 128-byte swizzled, completing on the stage's mbarrier.
//   warp 1     owns the tensor memory (two accumulators of N fp32 columns); one thread issues
//              tcgen05.mma kind::f16 (M = 128 tokens, N = padded rows, K = 16) per 16 columns of the slice,
//              and tcgen05.commit frees the stage, or marks the accumulator full after the last slice.
//   warps 2-5  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lanes 32 (w % 4) ...), each
//              (row, token) logit folded into a composite key order_key(logit) << 32 | ~token (ties: lowest
//              token, as max_element / ggml_argmax take the first), a warp transpose-reduce per 16 rows,
//              and running maxima in registers across the CTA's tiles; the CTA's maxima go into best[row]
//              with one 64-bit atomicMax per row at the end. The accumulator is handed back while the next
//              tile's MMAs run into the other one.
// lm_finish_kernel turns best[] into ids, the maximum logits and statuses, and clears best[] for the next
// call. Every mbarrier wait is bounded (mbar_wait): a wait that gives up sets the error word, every role
// leaves its loop, the issued copies and MMAs are waited for (bounded again) and the tensor memory is
// freed; the rows then report SSB_ROW_DEVICE_TIMEOUT. No cluster, no multicast.
#include <cstdint>
#include <cuda.h>
#include <cudaTypedefs.h>

#include "ssb_device.cuh"
#include "ssb_kernels.h"
#include "ssb_tma.cuh"

namespace ssb {

namespace {

constexpr int kLmThreads = 192;   // producer, MMA, 4 epilogue warps
constexpr int kLmTileM = 128;     // tokens per tile (MMA M)
constexpr int kLmSliceK = 64;     // dim columns per stage: one 128-byte swizzle row of bf16
constexpr int kLmStageA = kLmTileM * kLmSliceK * 2;  // 16 KB

__device__ __forceinline__ void tma_load_2d(void * dst, const CUtensorMap * map, int x, int y, uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// Shared-memory matrix descriptor of a K-major bf16 tile with 128-byte swizzle: rows of 64 elements
// (128 B), 8-row groups 1024 B apart (stride byte offset), leading byte offset 1 (unused when swizzled),
// version 1 (bits 46-47), layout SWIZZLE_128B = 2 (bits 61-63). `addr` advances by 32 B per K = 16.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    return (uint64_t) ((addr >> 4) & 0x3FFFu) | ((uint64_t) 1 << 16) | ((uint64_t) (1024 >> 4) << 32) |
           ((uint64_t) 1 << 46) | ((uint64_t) 2 << 61);
}

// Instruction descriptor of kind::f16: D f32 (bits 4-5 = 1), A and B bf16 (bits 7-9, 10-12 = 1), both
// K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28.
__host__ __device__ constexpr uint32_t f16_idesc(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t) (n >> 3) << 17) | ((uint32_t) (m >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t * bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 16 consecutive fp32 columns of the warp's 32 TMEM lanes (thread t: lane base + t).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 16; j++) v[j] = __uint_as_float(r[j]);
}

__global__ void __launch_bounds__(kLmThreads, 1)
    lm_argmax_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_h,
                     const __grid_constant__ LmArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // the stages must start on 1024-byte boundaries (the swizzle pattern repeats every 8 rows of 128 B)
    unsigned char * smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
    const int S = a.stages, N = a.n_pad;
    const int stage_b = N * kLmSliceK * 2;
    unsigned char * sa = smem;                           // [S][128 x 64] head tiles
    unsigned char * sb = smem + (size_t) S * kLmStageA;  // [S][N x 64] hidden rows
    __shared__ __align__(8) uint64_t full[16], empty[16], tfull[2], tempty[2], drain;
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    __shared__ uint64_t s_best[kLmMaxRows];  // this CTA's maxima per row, merged into best[] once at the end

    const int tid = (int) threadIdx.x, warp = warp_id(), lane = lane_id();
    auto aborted = [&]() { return *reinterpret_cast<volatile int *>(&s_abort) != 0; };
    const int KB = a.dim / kLmSliceK;
    const int tiles = (a.vocab + kLmTileM - 1) / kLmTileM;
    if (tid == 0) {
        for (int s = 0; s < S; s++) mbar_init(&full[s], 1), mbar_init(&empty[s], 1);
        for (int i = 0; i < 2; i++) mbar_init(&tfull[i], 1), mbar_init(&tempty[i], 4);
        mbar_init(&drain, 1);
        s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    for (int c = tid; c < a.rows; c += kLmThreads) s_best[c] = 0ull;
    if (warp == 1) {  // the whole warp allocates; the address lands in s_tmem
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&s_tmem)),
                     "r"(a.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    if (warp == 0) {
        // ---- producer
        int issued[16];
        for (int s = 0; s < 16; s++) issued[s] = 0;
        if (lane == 0) {
            const uint32_t bytes = (uint32_t) (kLmStageA + stage_b);
            int it = 0;
            for (int t = blockIdx.x; t < tiles && !aborted(); t += gridDim.x) {
                for (int kb = 0; kb < KB; kb++, it++) {
                    const int s = it % S;
                    if (it >= S && !mbar_wait(&empty[s], (uint32_t) ((it / S) - 1) & 1u)) {
                        atomicOr(&s_abort, 1);
                        break;
                    }
                    mbar_expect(&full[s], bytes);
                    tma_load_2d(sa + (size_t) s * kLmStageA, &map_w, kb * kLmSliceK, t * kLmTileM, &full[s]);
                    tma_load_2d(sb + (size_t) s * stage_b, &map_h, kb * kLmSliceK, 0, &full[s]);
                    issued[s] = it / S + 1;  // uses of stage s so far
                }
            }
            if (aborted()) {  // let every issued copy land before the CTA can exit
                for (int s = 0; s < S; s++)
                    if (issued[s] > 0) mbar_wait(&full[s], (uint32_t) (issued[s] - 1) & 1u);
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = f16_idesc(kLmTileM, N);
            int it = 0, tc = 0;
            bool any = false;
            for (int t = blockIdx.x; t < tiles && !aborted(); t += gridDim.x, tc++) {
                const int acc = tc & 1;
                if (tc >= 2 && !mbar_wait(&tempty[acc], (uint32_t) ((tc >> 1) - 1) & 1u)) {
                    atomicOr(&s_abort, 1);
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t) (acc * N);
                bool ok = true;
                for (int kb = 0; kb < KB; kb++, it++) {
                    const int s = it % S;
                    if (!mbar_wait(&full[s], (uint32_t) (it / S) & 1u)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_addr(sa + (size_t) s * kLmStageA), b0 = smem_addr(sb + (size_t) s * stage_b);
#pragma unroll
                    for (int kk = 0; kk < kLmSliceK / 16; kk++)
                        umma_bf16(d, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), idesc, (kb | kk) != 0);
                    umma_commit(&empty[s]);
                    any = true;
                }
                if (!ok) {
                    atomicOr(&s_abort, 1);
                    break;
                }
                umma_commit(&tfull[acc]);
            }
            if (aborted() && any) {  // every issued MMA done before the tensor memory is freed
                umma_commit(&drain);
                mbar_wait(&drain, 0);
            }
        }
    } else {
        // ---- epilogue (warps 2-5: TMEM lanes 32 (warp % 4) ...). Per 16 columns (rows of hidden) a
        // transpose-reduce over the warp leaves lane L with the maximum of column L & 15 over the warp's 32
        // tokens (16 exchanges instead of 5 per column); lane L keeps a running maximum per 16-column chunk
        // across all of the CTA's tiles, merged into s_best once at the end.
        const int q = warp & 3;
        const int chunks = (a.rows + 15) / 16;
        uint64_t run[kLmMaxRows / 16];
#pragma unroll
        for (int ch = 0; ch < kLmMaxRows / 16; ch++) run[ch] = 0ull;
        int tc = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, tc++) {
            const int acc = tc & 1;
            bool ok = false;
            if (lane == 0) ok = mbar_wait(&tfull[acc], (uint32_t) (tc >> 1) & 1u);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok || aborted()) {
                if (lane == 0) atomicOr(&s_abort, 1);
                break;
            }
            tc_fence_after();
            const int token = t * kLmTileM + q * 32 + lane;
            const bool valid = token < a.vocab;
            const uint32_t base = tmem + ((uint32_t) (q * 32) << 16) + (uint32_t) (acc * N);
#pragma unroll
            for (int ch = 0; ch < kLmMaxRows / 16; ch++) {
                if (ch >= chunks) break;
                float v[16];
                tmem_ld16(base + (uint32_t) (ch * 16), v);
                uint64_t k[16];
#pragma unroll
                for (int j = 0; j < 16; j++) k[j] = valid ? composite(v[j], (uint32_t) token) : 0ull;
                // round o (8, 4, 2, 1): a lane with bit o keeps the upper half of its m keys, the other the
                // lower, each taking the partner's copy of the half it keeps
#pragma unroll
                for (int o = 8, m = 16; o >= 1; o >>= 1, m >>= 1) {
                    const bool upper = (lane & o) != 0;
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        if (i >= m / 2) break;
                        const uint64_t send = upper ? k[i] : k[i + m / 2];
                        const uint64_t keep = upper ? k[i + m / 2] : k[i];
                        const uint64_t got = shfl_xor(send, o);
                        k[i] = keep > got ? keep : got;
                    }
                }
                const uint64_t other = shfl_xor(k[0], 16);  // the other half-warp's 16 tokens
                const uint64_t best = k[0] > other ? k[0] : other;
                run[ch] = run[ch] > best ? run[ch] : best;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
        }
        // lane L < 16 holds column ch * 16 + L of every chunk
#pragma unroll
        for (int ch = 0; ch < kLmMaxRows / 16; ch++) {
            const int c = ch * 16 + lane;
            if (ch < chunks && lane < 16 && c < a.rows && run[ch])
                atomicMax(reinterpret_cast<unsigned long long *>(&s_best[c]), (unsigned long long) run[ch]);
        }
    }
    __syncthreads();
    if (tid == 0 && s_abort) atomicOr(a.error, 1);
    for (int c = tid; c < a.rows; c += kLmThreads)
        if (s_best[c]) atomicMax(reinterpret_cast<unsigned long long *>(a.best + c), (unsigned long long) s_best[c]);
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_cols) : "memory");
    }
}

__global__ void lm_finish_kernel(LmArgs a) {
    for (int r = (int) threadIdx.x; r < a.rows; r += blockDim.x) {
        const uint64_t b = a.best[r];
        const bool err = *a.error != 0;
        a.ids[r] = err || b == 0 ? -1 : (int32_t) composite_index(b);
        if (a.max_logit) a.max_logit[r] = err || b == 0 ? __int_as_float(0x7fc00000) : composite_value(b);
        if (a.status) a.status[r] = err ? SSB_ROW_DEVICE_TIMEOUT : (b == 0 ? SSB_ROW_NO_FINITE_LOGIT : SSB_ROW_OK);
        a.best[r] = 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) *a.error = 0;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void * p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

// A 2D bf16 tensor map [rows, cols] (row stride ld elements) with boxes of [box_rows x 64], 128-byte swizzle.
bool make_map(CUtensorMap * m, const void * base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t) cols, (cuuint64_t) rows};
    const cuuint64_t strides[1] = {(cuuint64_t) ld * 2};
    const cuuint32_t box[2] = {(cuuint32_t) kLmSliceK, (cuuint32_t) box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int lm_stages(int n_pad, size_t max_smem) {
    const size_t per = (size_t) kLmStageA + (size_t) n_pad * kLmSliceK * 2;
    const size_t reserve = 1024 + 4096;  // alignment slack + the kernel's static shared memory (about 2.4 KB)
    const size_t avail = max_smem > reserve ? max_smem - reserve : 0;
    int s = (int) (avail / per);
    return s > 8 ? 8 : s;
}

size_t lm_smem_bytes(int n_pad, int stages) {
    return (size_t) stages * ((size_t) kLmStageA + (size_t) n_pad * kLmSliceK * 2) + 1024;
}

cudaError_t launch_lm_argmax(const LmArgs & a, const void * hidden, int64_t hidden_ld, const void * weight,
                             int64_t weight_ld, int grid, cudaStream_t stream) {
    CUtensorMap mw, mh;
    if (!make_map(&mw, weight, a.vocab, a.dim, weight_ld, kLmTileM) ||
        !make_map(&mh, hidden, a.rows, a.dim, hidden_ld, a.n_pad))
        return cudaErrorInvalidValue;
    const size_t smem = lm_smem_bytes(a.n_pad, a.stages);
    cudaError_t e = ssb::set_max_dynamic_smem((const void *) lm_argmax_kernel, smem);
    if (e != cudaSuccess) return e;
    lm_argmax_kernel<<<grid, kLmThreads, smem, stream>>>(mw, mh, a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    lm_finish_kernel<<<1, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace ssb
