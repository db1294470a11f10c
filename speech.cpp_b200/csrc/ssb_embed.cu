// The embedding rows of drawn ids: ggml_get_rows(table, id) of the code predictor's chain
// (src/families/qwen3-tts/talker.cpp:58-64) done on the device right after the draw, so the next step's
// input never leaves HBM. One CTA per (row, slice of dim): the id is read from the sampler's output in
// stream order; 16-byte copies where the table row, the out row and dim allow, else element copies.
#include <cstdint>

#include "ssb_kernels.h"

namespace ssb {

namespace {

constexpr int kEmbedThreads = 128;

template <typename T>
__global__ void __launch_bounds__(kEmbedThreads) embed_kernel(const __grid_constant__ EmbedArgs a) {
    const int r = blockIdx.y;
    const int32_t id = a.ids[r];
    const bool ok = a.status[r] == SSB_ROW_OK && id >= 0 && id < a.table_rows;
    const T * src = static_cast<const T *>(a.table) + (int64_t) (ok ? id : 0) * a.ld;
    T * dst = static_cast<T *>(a.out) + (int64_t) r * a.out_ld;
    constexpr int kVec = 16 / sizeof(T);
    const bool vec = (a.dim % kVec) == 0 && (reinterpret_cast<uintptr_t>(src) % 16) == 0 &&
                     (reinterpret_cast<uintptr_t>(dst) % 16) == 0;
    if (vec) {
        const int n = a.dim / kVec;
        for (int i = blockIdx.x * kEmbedThreads + (int) threadIdx.x; i < n; i += gridDim.x * kEmbedThreads)
            reinterpret_cast<uint4 *>(dst)[i] = ok ? __ldg(reinterpret_cast<const uint4 *>(src) + i) : make_uint4(0, 0, 0, 0);
    } else {
        for (int i = blockIdx.x * kEmbedThreads + (int) threadIdx.x; i < a.dim; i += gridDim.x * kEmbedThreads)
            dst[i] = ok ? src[i] : T(0);
    }
}

}  // namespace

cudaError_t launch_embed(const EmbedArgs & a, bool bf16, cudaStream_t stream) {
    const int per = kEmbedThreads * (bf16 ? 8 : 4);
    const int gx = (a.dim + per - 1) / per;
    const dim3 grid(gx < 8 ? gx : 8, a.rows);
    if (bf16) embed_kernel<uint16_t><<<grid, kEmbedThreads, 0, stream>>>(a);
    else embed_kernel<float><<<grid, kEmbedThreads, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace ssb
