// The vocabulary-sharded draw over NCCL (include/speech_sampler_b200_nccl.h): host C++ around the engine's
// two shard steps and one ncclAllGather, all queued on the caller's stream. Built into its own library so
// that the engine itself does not depend on NCCL.
#include <cstdint>
#include <cstring>
#include <string>

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
};

namespace {

thread_local std::string g_error;

ssb_status fail(ssb_status s, const std::string & m) {
    g_error = m;
    return s;
}

ssb_status engine_fail(ssb_status s, const char * what) { return fail(s, std::string(what) + ": " + ssb_last_error()); }

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
