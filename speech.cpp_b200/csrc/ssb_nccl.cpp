// The vocabulary-sharded draw over NCCL (include/speech_sampler_b200_nccl.h): host C++ around the engine's
// two shard steps and one ncclAllGather, all queued on the caller's stream. Built into its own library so
// that the engine itself does not depend on NCCL.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include <cuda_runtime.h>
#include <nccl.h>

#include "speech_sampler_b200_nccl.h"

struct ssb_shard_comm {
    ssb_context * ctx = nullptr;
    ncclComm_t comm = nullptr;
    int world = 0, rank = 0, device = 0;
    uint64_t * local = nullptr;  // [words]
    uint64_t * all = nullptr;    // [world * words]
    int64_t words = 0;
    // the restricted-slice exchange: every rank's (offset, width), learnt once per local layout
    int32_t lay_offset = -1, lay_width = -1, lay_vocab = -1;
    std::vector<int32_t> offsets, widths;
    int32_t * lay_dev = nullptr;  // [2 * world]
    float * f_local = nullptr;    // [rows * wmax]
    float * f_all = nullptr;      // [world * rows * wmax]
    float * f_rows = nullptr;     // [rows * vocab]
    size_t f_local_n = 0, f_all_n = 0, f_rows_n = 0;
};

namespace {

thread_local std::string g_error;

ssb_status fail(ssb_status s, const std::string & m) {
    g_error = m;
    return s;
}

ssb_status engine_fail(ssb_status s, const char * what) { return fail(s, std::string(what) + ": " + ssb_last_error()); }

template <typename T>
ssb_status grow_buf(T ** p, size_t * have, size_t need, const char * what) {
    if (need <= *have) return SSB_OK;
    cudaFree(*p);
    *p = nullptr;
    *have = 0;
    const cudaError_t e = cudaMalloc(p, need * sizeof(T));
    if (e != cudaSuccess) return fail(SSB_OUT_OF_MEMORY, std::string(what) + ": " + cudaGetErrorString(e));
    *have = need;
    return SSB_OK;
}

// The restricted-slice exchange (any row, top-k 0 included): every rank restricts its slice
// (ssb_restrict_slice), one ncclAllGather of the f32 slices padded to the widest, the whole rows laid out
// (one 2D copy per rank), and ssb_sample_rows on them with the rows' settings and u and no history or
// mask (both applied): the whole-row engine's ids and statuses on every rank.
ssb_status sample_full(ssb_shard_comm * c, const ssb_rows * slice, int32_t col_offset, int32_t vocab_total,
                       cudaStream_t stream) {
    const int width = slice->vocab, rows = slice->rows;
    if (c->lay_offset != col_offset || c->lay_width != width || c->lay_vocab != vocab_total) {
        // learn every rank's slice (collective; synchronises the stream once per layout)
        if (!c->lay_dev && cudaMalloc(&c->lay_dev, sizeof(int32_t) * 2 * (size_t) c->world) != cudaSuccess)
            return fail(SSB_OUT_OF_MEMORY, "slice layout");
        const int32_t mine[2] = {col_offset, width};
        cudaError_t e = cudaMemcpyAsync(c->lay_dev + 2 * c->rank, mine, sizeof(mine), cudaMemcpyHostToDevice, stream);
        if (e != cudaSuccess) return fail(SSB_DEVICE, std::string("slice layout: ") + cudaGetErrorString(e));
        const ncclResult_t r = ncclAllGather(c->lay_dev + 2 * c->rank, c->lay_dev, 2, ncclInt32, c->comm, stream);
        if (r != ncclSuccess) return fail(SSB_DEVICE, std::string("ncclAllGather: ") + ncclGetErrorString(r));
        std::vector<int32_t> lay(2 * (size_t) c->world);
        e = cudaMemcpyAsync(lay.data(), c->lay_dev, sizeof(int32_t) * lay.size(), cudaMemcpyDeviceToHost, stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) return fail(SSB_DEVICE, std::string("slice layout: ") + cudaGetErrorString(e));
        c->offsets.assign(c->world, 0);
        c->widths.assign(c->world, 0);
        for (int q = 0; q < c->world; q++) {
            c->offsets[q] = lay[2 * q], c->widths[q] = lay[2 * q + 1];
            if (c->offsets[q] < 0 || c->widths[q] < 1 || (int64_t) c->offsets[q] + c->widths[q] > vocab_total)
                return fail(SSB_INVALID_ARGUMENT, "the ranks' slices do not lie inside [0, vocab_total)");
        }
        c->lay_offset = col_offset, c->lay_width = width, c->lay_vocab = vocab_total;
    }
    const int wmax = *std::max_element(c->widths.begin(), c->widths.end());
    ssb_status s = grow_buf(&c->f_local, &c->f_local_n, (size_t) rows * wmax, "restricted slice");
    if (s == SSB_OK) s = grow_buf(&c->f_all, &c->f_all_n, (size_t) c->world * rows * wmax, "gathered slices");
    if (s == SSB_OK) s = grow_buf(&c->f_rows, &c->f_rows_n, (size_t) rows * vocab_total, "assembled rows");
    if (s != SSB_OK) return s;
    s = ssb_restrict_slice(c->ctx, slice, col_offset, vocab_total, c->f_local, wmax, stream);
    if (s != SSB_OK) return engine_fail(s, "ssb_restrict_slice");
    const ncclResult_t r = ncclAllGather(c->f_local, c->f_all, (size_t) rows * wmax, ncclFloat32, c->comm, stream);
    if (r != ncclSuccess) return fail(SSB_DEVICE, std::string("ncclAllGather: ") + ncclGetErrorString(r));
    for (int q = 0; q < c->world; q++) {
        const cudaError_t e = cudaMemcpy2DAsync(c->f_rows + c->offsets[q], sizeof(float) * vocab_total,
                                                c->f_all + (size_t) q * rows * wmax, sizeof(float) * wmax,
                                                sizeof(float) * c->widths[q], rows, cudaMemcpyDeviceToDevice, stream);
        if (e != cudaSuccess) return fail(SSB_DEVICE, std::string("assembling the rows: ") + cudaGetErrorString(e));
    }
    ssb_rows whole = *slice;
    whole.logits = c->f_rows;
    whole.ld = vocab_total;
    whole.dtype = SSB_F32;
    whole.vocab = vocab_total;
    whole.history = nullptr;
    whole.history_ld = 0;
    whole.history_len = nullptr;
    whole.mask = nullptr;
    whole.mask_ld = 0;
    whole.mask_kind = SSB_MASK_NONE;
    s = ssb_sample_rows(c->ctx, &whole, stream);
    if (s != SSB_OK) return engine_fail(s, "ssb_sample_rows");
    return SSB_OK;
}

ssb_status grow(ssb_shard_comm * c, int64_t words) {
    if (words <= c->words) return SSB_OK;
    cudaFree(c->local);
    cudaFree(c->all);
    c->local = c->all = nullptr;
    c->words = 0;
    cudaError_t e = cudaMalloc(&c->local, (size_t) words * 8);
    if (e == cudaSuccess) e = cudaMalloc(&c->all, (size_t) words * 8 * (size_t) c->world);
    if (e != cudaSuccess) return fail(SSB_OUT_OF_MEMORY, std::string("shard records: ") + cudaGetErrorString(e));
    c->words = words;
    return SSB_OK;
}

}  // namespace

extern "C" {

const char * ssb_nccl_last_error(void) { return g_error.c_str(); }

ssb_status ssb_nccl_unique_id(uint8_t id[128]) {
    if (!id) return fail(SSB_INVALID_ARGUMENT, "id is null");
    ncclUniqueId u;
    const ncclResult_t r = ncclGetUniqueId(&u);
    if (r != ncclSuccess) return fail(SSB_DEVICE, std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
    static_assert(sizeof(u) == 128, "an NCCL unique id is 128 bytes");
    std::memcpy(id, &u, 128);
    return SSB_OK;
}

ssb_status ssb_shard_comm_create(ssb_context * ctx, const uint8_t id[128], int32_t world, int32_t rank,
                                 ssb_shard_comm ** out) {
    if (!ctx || !id || !out) return fail(SSB_INVALID_ARGUMENT, "ctx, id and out are required");
    if (world < 1 || rank < 0 || rank >= world) return fail(SSB_INVALID_ARGUMENT, "rank must lie in [0, world)");
    *out = nullptr;
    int dev = 0;
    cudaGetDevice(&dev);
    ssb_shard_comm * c = new ssb_shard_comm();
    c->ctx = ctx;
    c->world = world;
    c->rank = rank;
    c->device = dev;
    ncclUniqueId u;
    std::memcpy(&u, id, 128);
    const ncclResult_t r = ncclCommInitRank(&c->comm, world, u, rank);
    if (r != ncclSuccess) {
        delete c;
        return fail(SSB_DEVICE, std::string("ncclCommInitRank: ") + ncclGetErrorString(r));
    }
    *out = c;
    return SSB_OK;
}

ssb_status ssb_shard_comm_destroy(ssb_shard_comm * c) {
    if (!c) return SSB_OK;
    if (c->comm) ncclCommDestroy(c->comm);
    cudaFree(c->local);
    cudaFree(c->all);
    cudaFree(c->lay_dev);
    cudaFree(c->f_local);
    cudaFree(c->f_all);
    cudaFree(c->f_rows);
    delete c;
    return SSB_OK;
}

ssb_status ssb_shard_comm_reserve(ssb_shard_comm * c, int32_t rows, int32_t k_cap) {
    if (!c || rows < 0 || k_cap < 1) return fail(SSB_INVALID_ARGUMENT, "comm, rows >= 0 and k_cap >= 1 are required");
    return grow(c, ssb_shard_record_words(rows, k_cap));
}

ssb_status ssb_shard_sample(ssb_shard_comm * c, const ssb_rows * slice, int32_t col_offset, int32_t vocab_total,
                            int32_t k_cap, void * stream) {
    if (!c || !slice) return fail(SSB_INVALID_ARGUMENT, "comm and slice are required");
    if (slice->rows == 0) return SSB_OK;
    // k_cap 0, or (without per-row settings) a drawing row keeping more than k_cap tokens: the
    // restricted-slice exchange
    const ssb_params & q = slice->params;
    const int64_t keff = q.top_k > 0 ? std::min<int64_t>(q.top_k, vocab_total) : vocab_total;
    if (k_cap == 0 || (!slice->row_params && !q.greedy && keff > k_cap))
        return sample_full(c, slice, col_offset, vocab_total, static_cast<cudaStream_t>(stream));
    const int64_t words = ssb_shard_record_words(slice->rows, k_cap);
    ssb_status s = grow(c, words);
    if (s != SSB_OK) return s;
    s = ssb_shard_select(c->ctx, slice, col_offset, vocab_total, k_cap, c->local, stream);
    if (s != SSB_OK) return engine_fail(s, "ssb_shard_select");
    const ncclResult_t r = ncclAllGather(c->local, c->all, (size_t) words, ncclUint64, c->comm,
                                         static_cast<cudaStream_t>(stream));
    if (r != ncclSuccess) return fail(SSB_DEVICE, std::string("ncclAllGather: ") + ncclGetErrorString(r));
    // the gathered records sit rank after rank with `words` per rank: the merge's [world][rows][k_cap + 1]
    s = ssb_shard_merge(c->ctx, slice, vocab_total, c->world, k_cap, c->all, stream);
    if (s != SSB_OK) return engine_fail(s, "ssb_shard_merge");
    return SSB_OK;
}

}  // extern "C"
