// The C ABI of include/speech_sampler_b200.h: argument checks, the choice of kernel, the context's
// scratch, and the host-buffer entry point. No CPU sampling exists behind it: every row is sampled by
// the CUDA kernels (ssb_small.cu, ssb_topk.cu, ssb_stream.cu, ssb_nucleus.cu), or the call fails.
#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <string>
#include <map>
#include <mutex>
#include <thread>
#include <vector>

#include <cuda_runtime.h>

#include "speech_sampler_b200.h"
#include "ssb_device.cuh"
#include "ssb_kernels.h"

struct ssb_context {
    int device = 0;
    int sm_count = 0;
    int max_smem = 0;   // opt-in shared memory per block
    int max_slots = 0;  // resident CTAs of the streaming kernel the scratch is sized for
    // split-row scratch, sized once at creation (rows * splits never exceeds max_slots)
    uint64_t * part_cand = nullptr;  // [max_slots * kStreamMaxK]
    int32_t * part_n = nullptr;      // [max_slots]
    float * part_max = nullptr;      // [max_slots]
    int32_t * part_flags = nullptr;  // [max_slots]
    uint32_t * counters = nullptr;   // [max_slots]
    // rows that keep more than kStreamMaxK tokens: one region of the list per resident CTA, grown on use
    uint64_t * nuc_scratch = nullptr;
    size_t nuc_bytes = 0;
    // host-call staging
    unsigned char * stage = nullptr;
    size_t stage_bytes = 0;
    cudaEvent_t done = nullptr;
    // occupancy of the streaming kernel per (mode, bf16, vec), measured at the row's full width
    int occupancy[2][2][2] = {};
    // occupancy of the top-k kernel per (warp-list width class, bf16)
    int occ_topk[3][2] = {};
    size_t occ_topk_smem[3][2] = {};  // the shared memory each was measured at
    // device copies of caller masks (ssb_context_mask), freed with the context
    std::vector<void *> masks;
    // the fused LM-head argmax: per-row composite maxima and the error word, zero between calls
    uint64_t * lm_best = nullptr;  // [kLmMaxRows]
    int32_t * lm_error = nullptr;
};

// The DRY state of Haru's text streams (one device allocation).
struct ssb_dry {
    int device = 0;
    int max_smem = 0;
    void * block = nullptr;
    ssb::DryArgs a{};
};

namespace ssb {

cudaError_t set_max_dynamic_smem(const void * kernel, size_t bytes) {
    static std::mutex mu;
    static std::map<std::pair<int, const void *>, size_t> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    size_t & have = done[{dev, kernel}];
    if (bytes <= have) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) bytes);
    if (e == cudaSuccess) have = bytes;
    return e;
}

}  // namespace ssb

namespace {

thread_local std::string g_error;

ssb_status fail(ssb_status s, const std::string & message) {
    g_error = message;
    return s;
}

ssb_status ok() {
    g_error.clear();
    return SSB_OK;
}

ssb_status cuda_fail(cudaError_t e, const char * what) {
    const ssb_status s = e == cudaErrorMemoryAllocation ? SSB_OUT_OF_MEMORY : SSB_DEVICE;
    return fail(s, std::string(what) + ": " + cudaGetErrorString(e));
}

// Makes the context's device current for the calling thread; restores nothing (CUDA convention).
ssb_status use_device(const ssb_context * ctx) {
    int cur = -1;
    cudaError_t e = cudaGetDevice(&cur);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (cur != ctx->device) {
        e = cudaSetDevice(ctx->device);
        if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    }
    return SSB_OK;
}

int64_t div_up(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Grows the nucleus kernel's candidate lists to `grid` regions of `ld` composites (never shrinks).
ssb_status ensure_nucleus_scratch(ssb_context * ctx, int grid, int64_t ld) {
    const size_t need = (size_t) grid * (size_t) ld * sizeof(uint64_t);
    if (need <= ctx->nuc_bytes) return SSB_OK;
    cudaFree(ctx->nuc_scratch);
    ctx->nuc_scratch = nullptr;
    ctx->nuc_bytes = 0;
    const cudaError_t e = cudaMalloc(&ctx->nuc_scratch, need);
    if (e != cudaSuccess) return cuda_fail(e, "nucleus scratch");
    ctx->nuc_bytes = need;
    return SSB_OK;
}

struct Plan {
    int kernel;  // 0 small, 1 stream (top-k / stream kernels), 2 nucleus (top-k above kStreamMaxK), 3 flavour
    int mode;    // stream: 0 greedy, 1 top-k
    int k_bound;
};

ssb_status check_rows(const ssb_rows * r, bool device_side, Plan * plan) {
    if (!r) return fail(SSB_INVALID_ARGUMENT, "rows is null");
    if (r->rows < 0) return fail(SSB_INVALID_ARGUMENT, "rows is negative");
    if (r->vocab < 1) return fail(SSB_INVALID_ARGUMENT, "vocab must be at least 1");
    if (r->vocab > SSB_MAX_VOCAB) return fail(SSB_OUT_OF_RANGE, "vocab exceeds SSB_MAX_VOCAB (16777216)");
    if (r->ld < r->vocab) return fail(SSB_INVALID_ARGUMENT, "ld is smaller than vocab");
    if (r->dtype != SSB_F32 && r->dtype != SSB_BF16) return fail(SSB_INVALID_ARGUMENT, "dtype is neither SSB_F32 nor SSB_BF16");
    if (r->mask_kind < SSB_MASK_NONE || r->mask_kind > SSB_MASK_ALLOW) return fail(SSB_INVALID_ARGUMENT, "mask_kind is not an ssb_mask_kind");
    if (r->reserved != 0) return fail(SSB_INVALID_ARGUMENT, "reserved fields must be 0");
    if (r->params.flavor < SSB_FLAVOR_QWEN3_TTS || r->params.flavor > SSB_FLAVOR_DRAMA3)
        return fail(SSB_INVALID_ARGUMENT, "params.flavor is not an ssb_flavor");
    if (r->rows == 0) return SSB_OK;
    if (!r->logits) return fail(SSB_INVALID_ARGUMENT, "logits is null");
    if (!r->ids || !r->status) return fail(SSB_INVALID_ARGUMENT, "ids and status are required");
    if (r->mask_kind != SSB_MASK_NONE) {
        if (!r->mask) return fail(SSB_INVALID_ARGUMENT, "mask_kind is set but mask is null");
        if (r->mask_ld < 0) return fail(SSB_INVALID_ARGUMENT, "mask_ld is negative");
        if (r->mask_ld > 0 && r->mask_ld < div_up(r->vocab, 32)) return fail(SSB_INVALID_ARGUMENT, "mask_ld is smaller than ceil(vocab / 32)");
    }
    if (r->history) {
        if (r->history_ld < 0) return fail(SSB_INVALID_ARGUMENT, "history_ld is negative");
        if (r->history_ld > INT32_MAX / 2) return fail(SSB_OUT_OF_RANGE, "history_ld is too large");
    }
    const bool all_greedy = !r->row_params && (r->params.greedy || (r->params.flavor == SSB_FLAVOR_HARU &&
                                                                    r->params.temperature <= 0.0f));
    if (!all_greedy && !r->u) return fail(SSB_INVALID_ARGUMENT, "u is required where a row draws (not greedy)");
    int kb;
    if (r->row_params) {
        if (r->max_top_k < 0) return fail(SSB_INVALID_ARGUMENT, "max_top_k is negative");
        kb = r->max_top_k > 0 ? std::min(r->max_top_k, r->vocab) : r->vocab;
    } else {
        kb = r->params.greedy ? 1 : (r->params.top_k > 0 ? std::min(r->params.top_k, r->vocab) : r->vocab);
    }
    plan->k_bound = kb;
    if (r->params.flavor != SSB_FLAVOR_QWEN3_TTS) {
        // Haru's and Drama 3's candidate rules (ssb_flavor.cu), one CTA per row
        const ssb_params & q = r->params;
        const int keff = q.flavor == SSB_FLAVOR_HARU ? (q.top_k > 0 && q.top_k < r->vocab ? q.top_k : r->vocab)
                                                     : std::min(std::max(q.top_k, 1), r->vocab);
        const bool argmax = q.greedy || (q.flavor == SSB_FLAVOR_HARU && q.temperature <= 0.0f);
        if (!r->row_params && !argmax && keff > ssb::kFlavorMaxK)
            return fail(SSB_OUT_OF_RANGE, "the Haru and Drama 3 families keep at most 8192 candidates (top_k)");
        if (!r->row_params) plan->k_bound = argmax ? 1 : keff;
        plan->k_bound = std::min(plan->k_bound, ssb::kFlavorMaxK);
        if (r->history && r->history_ld > SSB_MAX_STREAM_HISTORY)
            return fail(SSB_OUT_OF_RANGE, "history_ld exceeds SSB_MAX_STREAM_HISTORY (8192)");
        plan->kernel = 3;
        plan->mode = 0;
        return SSB_OK;
    }
    if (r->vocab <= SSB_SMALL_VOCAB) {
        plan->kernel = 0;
        plan->mode = 0;
        return SSB_OK;
    }
    if (r->history && r->history_ld > SSB_MAX_STREAM_HISTORY)
        return fail(SSB_OUT_OF_RANGE, "history_ld exceeds SSB_MAX_STREAM_HISTORY (8192) for a vocabulary of more than 8192 tokens");
    plan->kernel = 1;
    plan->mode = all_greedy ? 0 : 1;
    if (plan->mode == 1 && kb > ssb::kStreamMaxK) plan->kernel = 2;
    (void) device_side;
    return SSB_OK;
}

struct Debug {
    int cap = 0;
    int32_t * tokens = nullptr;
    double * weights = nullptr;
    int32_t * count = nullptr;
    float * processed = nullptr;
};

ssb::RowsArgs rows_args(const ssb_rows * r, int k_bound, const Debug * dbg) {
    ssb::RowsArgs a{};
    a.logits = r->logits;
    a.ld = r->ld;
    a.rows = r->rows;
    a.vocab = r->vocab;
    a.params = r->params;
    a.row_params = r->row_params;
    a.k_bound = k_bound;
    a.history = r->history;
    a.history_ld = r->history ? r->history_ld : 0;
    a.history_len = r->history ? r->history_len : nullptr;
    a.mask = r->mask_kind != SSB_MASK_NONE ? r->mask : nullptr;
    a.mask_ld = r->mask_ld;
    a.mask_kind = r->mask_kind;
    a.u = r->u;
    a.ids = r->ids;
    a.status = r->status;
    if (dbg) {
        a.dbg_cap = dbg->cap;
        a.dbg_tokens = dbg->tokens;
        a.dbg_weights = dbg->weights;
        a.dbg_count = dbg->count;
        a.dbg_processed = dbg->processed;
    }
    return a;
}

ssb_status run(ssb_context * ctx, const ssb_rows * r, const Debug * dbg, cudaStream_t stream) {
    Plan plan{};
    ssb_status s = check_rows(r, true, &plan);
    if (s != SSB_OK) return s;
    if (!ctx) return fail(SSB_INVALID_ARGUMENT, "ctx is null");
    if (r->rows == 0) return ok();
    s = use_device(ctx);
    if (s != SSB_OK) return s;
    const bool bf16 = r->dtype == SSB_BF16;
    const bool debug = dbg != nullptr;
    ssb::RowsArgs a = rows_args(r, plan.k_bound, dbg);
    cudaError_t e;
    if (plan.kernel == 0) {
        e = ssb::launch_small(a, bf16, debug, stream);
        if (e != cudaSuccess) return cuda_fail(e, "small-row kernel launch");
        return ok();
    }
    if (plan.kernel == 3) {
        ssb::FlavorArgs fa{};
        fa.r = a;
        fa.flavor = r->params.flavor;
        fa.cap = ssb::next_pow2(std::max(plan.k_bound, 32));
        fa.hist_slots = r->history ? ssb::next_pow2((int) std::max<int64_t>(4, 2 * r->history_ld)) : 0;
        const int words = (int) div_up(r->vocab, 32);
        fa.bit_words = r->history && words <= 16384 ? words : 0;  // the bitmap where it fits in 64 KB
        if (ssb::flavor_smem_bytes(fa.cap, fa.bit_words, fa.hist_slots) > (size_t) ctx->max_smem) fa.bit_words = 0;
        if (ssb::flavor_smem_bytes(fa.cap, fa.bit_words, fa.hist_slots) > (size_t) ctx->max_smem)
            return fail(SSB_OUT_OF_RANGE, "the candidates and the history need more shared memory than the device has");
        e = ssb::launch_flavor(fa, bf16, debug, stream);
        if (e != cudaSuccess) return cuda_fail(e, "flavour kernel launch");
        return ok();
    }
    if (plan.kernel == 2) {
        ssb::NucleusArgs na{};
        na.r = a;
        na.r.k_bound = plan.k_bound;
        na.hist_slots = r->history ? ssb::next_pow2((int) std::max<int64_t>(4, 2 * r->history_ld)) : 0;
        const size_t smem = ssb::nucleus_smem_bytes(r->vocab, na.hist_slots);
        if (smem > (size_t) ctx->max_smem) return fail(SSB_OUT_OF_RANGE, "the history and vocabulary need more shared memory than the device has");
        const int occ = ssb::nucleus_blocks_per_sm(bf16, smem);
        if (occ <= 0) return fail(SSB_DEVICE, "the nucleus kernel does not fit on this device");
        const int grid = std::min(r->rows, ctx->sm_count * occ);
        na.scratch_ld = ssb::nucleus_scratch_ld(r->vocab);
        const ssb_status gs = ensure_nucleus_scratch(ctx, grid, na.scratch_ld);
        if (gs != SSB_OK) return gs;
        na.scratch = ctx->nuc_scratch;
        e = ssb::launch_nucleus(na, grid, bf16, debug, stream);
        if (e != cudaSuccess) return cuda_fail(e, "nucleus kernel launch");
        return ok();
    }
    const int mode = plan.mode;
    const int es = bf16 ? 2 : 4;
    const bool vec = (reinterpret_cast<uintptr_t>(r->logits) % 16 == 0) && ((r->ld * es) % 16 == 0);
    const int kb = std::max(1, plan.k_bound);
    a.k_bound = kb;
    ssb::StreamArgs sa{};
    sa.r = a;
    sa.hist_slots = r->history ? ssb::next_pow2((int) std::max<int64_t>(4, 2 * r->history_ld)) : 0;  // hash, load <= 1/2
    sa.cap = mode == 1 ? (int) div_up(kb + std::max(1024, kb), 32) * 32 : 0;
    sa.sel_slots = mode == 1 ? ssb::next_pow2(std::max(kb, 2)) : 0;
    // all-greedy batches on aligned rows: the split-row argmax (not for the candidate export, which also
    // wants every restricted logit)
    if (mode == 0 && vec && !debug) {
        const int unit = ssb::argmax_unit(bf16);
        const int64_t units = div_up(r->vocab, unit);
        const int64_t per_row = std::max<int64_t>(1, ctx->max_slots / std::max(1, r->rows));
        const int64_t splits = std::min<int64_t>(units, per_row);
        const int64_t chunk = div_up(units, splits) * unit;
        sa.splits = (int) div_up(r->vocab, chunk);
        sa.chunk = (int) chunk;
        if (ssb::argmax_smem_bytes(sa.chunk, sa.hist_slots) <= (size_t) ctx->max_smem) {
            if (sa.splits > 1) {
                sa.part_cand = ctx->part_cand;
                sa.part_max = ctx->part_max;
                sa.counters = ctx->counters;
            }
            e = ssb::launch_argmax(sa, bf16, stream);
            if (e != cudaSuccess) return cuda_fail(e, "argmax kernel launch");
            return ok();
        }
    }
    // aligned rows with a small top-k (or all greedy: top-1) take the warp-specialized top-k kernel
    bool use_topk = vec && (mode == 0 || kb <= ssb::kTopkMaxK);
    const int kw = use_topk ? ssb::topk_kw(kb) : -1;
    const int kwc = kw == 1 ? 0 : (kw == 2 ? 1 : 2);  // its width class
    const int full_chunk = (int) div_up(r->vocab, 32) * 32;
    // the top-k kernel keeps per-chunk state in shared memory: cap the chunk so that it fits
    int max_chunk = full_chunk;
    if (use_topk) {
        max_chunk = std::min(full_chunk, ssb::topk_max_chunk(bf16));
        while (max_chunk > 4096 && ssb::topk_smem_bytes(kw, bf16, max_chunk, sa.hist_slots, sa.sel_slots) > (size_t) ctx->max_smem)
            max_chunk = (int) div_up(max_chunk / 2, 32) * 32;
        if (ssb::topk_smem_bytes(kw, bf16, max_chunk, sa.hist_slots, sa.sel_slots) > (size_t) ctx->max_smem) use_topk = false;
    }
    int occ_topk_now = 0;
    int & occ = use_topk ? occ_topk_now : ctx->occupancy[mode][bf16][vec];
    if (use_topk) {
        // per history size, so measured for this call's shared memory (a cached value per width class)
        int & cached = ctx->occ_topk[kwc][bf16];
        const size_t smem = ssb::topk_smem_bytes(kw, bf16, max_chunk, sa.hist_slots, sa.sel_slots);
        if (cached == 0 || ctx->occ_topk_smem[kwc][bf16] != smem) {
            cached = ssb::topk_blocks_per_sm(kw, bf16, smem);
            ctx->occ_topk_smem[kwc][bf16] = smem;
        }
        occ = cached;
        if (occ <= 0) return fail(SSB_DEVICE, "the top-k kernel does not fit on this device");
    } else if (occ == 0) {
        occ = ssb::stream_blocks_per_sm(mode, bf16, vec, ssb::stream_smem_bytes(mode, vec, full_chunk, sa.hist_slots, sa.cap, sa.sel_slots));
        if (occ <= 0) return fail(SSB_DEVICE, "the streaming kernel does not fit on this device");
    }
    const int slots = std::min(ctx->max_slots, ctx->sm_count * occ);
    const int min_chunk = mode == 0 ? 2048 : 4096;
    int64_t splits = std::max<int64_t>(1, std::min<int64_t>(div_up(r->vocab, min_chunk), slots / std::max(1, r->rows)));
    // two halves of a row do not pay for their merge in the top-k kernel: one CTA per row streams the
    // whole row instead (128 rows of 151936 bf16: 22.8 us against 24.7 us split in two)
    if (use_topk && splits == 2) splits = 1;
    splits = std::max<int64_t>(splits, div_up(r->vocab, max_chunk));
    int64_t chunk = div_up(div_up(r->vocab, splits), 32) * 32;
    splits = div_up(r->vocab, chunk);
    sa.splits = (int) splits;
    sa.chunk = (int) chunk;
    if (splits > 1) {
        if ((int64_t) r->rows * splits > ctx->max_slots) return fail(SSB_OUT_OF_RANGE, "split-row scratch exceeded");
        sa.part_cand = ctx->part_cand;
        sa.part_n = ctx->part_n;
        sa.part_max = ctx->part_max;
        sa.part_flags = ctx->part_flags;
        sa.counters = ctx->counters;
    }
    if ((int64_t) r->rows * splits > INT32_MAX) return fail(SSB_OUT_OF_RANGE, "too many rows for one launch");
    e = use_topk ? ssb::launch_topk(sa, kw, bf16, debug, stream) : ssb::launch_stream(sa, mode, bf16, vec, debug, stream);
    if (e != cudaSuccess) return cuda_fail(e, "streaming kernel launch");
    return ok();
}

// Waits for `stream` with a bound; a device that stops answering becomes SSB_DEVICE, not a hang.
ssb_status wait_stream(ssb_context * ctx, cudaStream_t stream, double timeout_s) {
    cudaError_t e = cudaEventRecord(ctx->done, stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
    const auto t0 = std::chrono::steady_clock::now();
    for (long spin = 0;; spin++) {
        e = cudaEventQuery(ctx->done);
        if (e == cudaSuccess) return SSB_OK;
        if (e != cudaErrorNotReady) return cuda_fail(e, "waiting for the sampler");
        if (spin > 1000) {
            std::this_thread::sleep_for(std::chrono::microseconds(20));
            if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s)
                return fail(SSB_DEVICE, "the device did not finish sampling within the time limit");
        }
    }
}

}  // namespace

namespace ssb {
// Lets other entry points of the library report through ssb_last_error().
void set_last_error(const std::string & message) { g_error = message; }
}  // namespace ssb

extern "C" {

const char * ssb_version(void) { return "0.1.0"; }

const char * ssb_last_error(void) { return g_error.c_str(); }

ssb_status ssb_context_create(int32_t device, ssb_context ** out) {
    if (!out) return fail(SSB_INVALID_ARGUMENT, "out is null");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= n) return fail(SSB_INVALID_ARGUMENT, "no CUDA device " + std::to_string(device));
    auto * ctx = new ssb_context();
    ctx->device = device;
    ssb_status s = use_device(ctx);
    if (s != SSB_OK) {
        delete ctx;
        return s;
    }
    e = cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&ctx->max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    if (e != cudaSuccess) {
        delete ctx;
        return cuda_fail(e, "cudaDeviceGetAttribute");
    }
    ctx->max_slots = ctx->sm_count * 8;  // 8 CTAs of 256 threads fill an SM's 2048 threads
    const size_t ms = (size_t) ctx->max_slots;
    e = cudaMalloc(&ctx->part_cand, ms * ssb::kStreamMaxK * sizeof(uint64_t));
    if (e == cudaSuccess) e = cudaMalloc(&ctx->part_n, ms * sizeof(int32_t));
    if (e == cudaSuccess) e = cudaMalloc(&ctx->part_max, ms * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&ctx->part_flags, ms * sizeof(int32_t));
    if (e == cudaSuccess) e = cudaMalloc(&ctx->counters, ms * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(ctx->counters, 0, ms * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMalloc(&ctx->lm_best, ssb::kLmMaxRows * sizeof(uint64_t) + 16);
    if (e == cudaSuccess) e = cudaMemset(ctx->lm_best, 0, ssb::kLmMaxRows * sizeof(uint64_t) + 16);
    if (e == cudaSuccess) ctx->lm_error = reinterpret_cast<int32_t *>(ctx->lm_best + ssb::kLmMaxRows);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->done, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        ssb_context_destroy(ctx);
        return cuda_fail(e, "context scratch");
    }
    *out = ctx;
    return ok();
}

ssb_status ssb_context_destroy(ssb_context * ctx) {
    if (!ctx) return ok();
    int cur = -1;
    cudaGetDevice(&cur);
    cudaSetDevice(ctx->device);
    cudaFree(ctx->part_cand);
    cudaFree(ctx->part_n);
    cudaFree(ctx->part_max);
    cudaFree(ctx->part_flags);
    cudaFree(ctx->counters);
    cudaFree(ctx->stage);
    cudaFree(ctx->nuc_scratch);
    for (void * m : ctx->masks) cudaFree(m);
    cudaFree(ctx->lm_best);
    if (ctx->done) cudaEventDestroy(ctx->done);
    if (cur >= 0) cudaSetDevice(cur);
    delete ctx;
    return ok();
}

ssb_status ssb_context_mask(ssb_context * ctx, const uint32_t * host_words, int64_t words, const uint32_t ** device_words) {
    if (!ctx) return fail(SSB_INVALID_ARGUMENT, "ctx is null");
    if (!host_words || !device_words) return fail(SSB_INVALID_ARGUMENT, "host_words and device_words are required");
    if (words < 1 || words > SSB_MAX_VOCAB / 32) return fail(SSB_OUT_OF_RANGE, "words must be in [1, SSB_MAX_VOCAB / 32]");
    ssb_status s = use_device(ctx);
    if (s != SSB_OK) return s;
    void * d = nullptr;
    cudaError_t e = cudaMalloc(&d, (size_t) words * 4);
    if (e != cudaSuccess) return cuda_fail(e, "mask copy");
    e = cudaMemcpy(d, host_words, (size_t) words * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(d);
        return cuda_fail(e, "mask copy");
    }
    ctx->masks.push_back(d);
    *device_words = static_cast<const uint32_t *>(d);
    return ok();
}

ssb_status ssb_context_reserve(ssb_context * ctx, int32_t max_rows, int32_t max_vocab) {
    if (!ctx) return fail(SSB_INVALID_ARGUMENT, "ctx is null");
    if (max_rows < 0 || max_vocab < 0) return fail(SSB_INVALID_ARGUMENT, "negative size");
    // Split-row scratch is allocated at creation; reserving sizes the host-call staging buffer for
    // f32 rows, histories of up to SSB_MAX_STREAM_HISTORY ids and per-row masks, and the candidate
    // lists of rows that keep more than kStreamMaxK tokens.
    ssb_status s = use_device(ctx);
    if (s != SSB_OK) return s;
    const size_t rows = (size_t) max_rows, vocab = (size_t) max_vocab;
    const size_t need = rows * vocab * 4 + rows * SSB_MAX_STREAM_HISTORY * 4 + rows * ((vocab + 31) / 32) * 4 +
                        rows * (8 + 4 + 4 + 4 + sizeof(ssb_params)) + 8 * 256;
    if (need > ctx->stage_bytes) {
        cudaFree(ctx->stage);
        ctx->stage = nullptr;
        ctx->stage_bytes = 0;
        cudaError_t e = cudaMalloc(&ctx->stage, need);
        if (e != cudaSuccess) return cuda_fail(e, "staging buffer");
        ctx->stage_bytes = need;
    }
    // rows that keep more than kStreamMaxK tokens: one list region per resident nucleus CTA (the
    // occupancy without a history table is the largest the launch can have)
    if (max_vocab > SSB_SMALL_VOCAB && max_rows > 0) {
        const size_t smem = ssb::nucleus_smem_bytes(max_vocab, 0);
        const int occ = std::max(ssb::nucleus_blocks_per_sm(true, smem), ssb::nucleus_blocks_per_sm(false, smem));
        if (occ <= 0) return fail(SSB_DEVICE, "the nucleus kernel does not fit on this device");
        s = ensure_nucleus_scratch(ctx, std::min(max_rows, ctx->sm_count * occ), ssb::nucleus_scratch_ld(max_vocab));
        if (s != SSB_OK) return s;
    }
    return ok();
}

ssb_status ssb_sample_rows(ssb_context * ctx, const ssb_rows * rows, void * stream) {
    return run(ctx, rows, nullptr, static_cast<cudaStream_t>(stream));
}

ssb_status ssb_sample_embed_rows(ssb_context * ctx, const ssb_rows * rows, const ssb_embed * e, void * stream) {
    if (!e) return fail(SSB_INVALID_ARGUMENT, "embed is required");
    if (e->reserved != 0) return fail(SSB_INVALID_ARGUMENT, "reserved fields must be 0");
    if (e->dtype != SSB_F32 && e->dtype != SSB_BF16) return fail(SSB_INVALID_ARGUMENT, "embed dtype is neither SSB_F32 nor SSB_BF16");
    if (e->dim < 1 || e->table_rows < 1 || e->ld < e->dim || e->out_ld < e->dim)
        return fail(SSB_INVALID_ARGUMENT, "embed dim, table_rows, ld or out_ld out of order");
    if (!e->table || !e->out) return fail(SSB_INVALID_ARGUMENT, "embed table and out are required");
    const ssb_status s = run(ctx, rows, nullptr, static_cast<cudaStream_t>(stream));
    if (s != SSB_OK || rows->rows == 0) return s;
    ssb::EmbedArgs a{};
    a.table = e->table;
    a.ld = e->ld;
    a.table_rows = e->table_rows;
    a.dim = e->dim;
    a.out = e->out;
    a.out_ld = e->out_ld;
    a.ids = rows->ids;
    a.status = rows->status;
    a.rows = rows->rows;
    const cudaError_t err = ssb::launch_embed(a, e->dtype == SSB_BF16, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "embedding launch");
    return ok();
}

int64_t ssb_shard_record_words(int32_t rows, int32_t k_cap) { return (int64_t) rows * ((int64_t) k_cap + 1); }

static bool shard_kcap_ok(int32_t k_cap) { return k_cap >= 1 && k_cap <= ssb::kShardMaxK && (k_cap & (k_cap - 1)) == 0; }

ssb_status ssb_shard_select(ssb_context * ctx, const ssb_rows * r, int32_t col_offset, int32_t vocab_total,
                            int32_t k_cap, uint64_t * records, void * stream) {
    if (!ctx || !r || !records) return fail(SSB_INVALID_ARGUMENT, "ctx, slice and records are required");
    if (!shard_kcap_ok(k_cap)) return fail(SSB_INVALID_ARGUMENT, "k_cap must be a power of two in [1, 1024]");
    if (col_offset < 0 || col_offset % 32 != 0) return fail(SSB_INVALID_ARGUMENT, "col_offset must be a non-negative multiple of 32");
    if (r->vocab < 1 || (int64_t) col_offset + r->vocab > vocab_total || vocab_total > SSB_MAX_VOCAB)
        return fail(SSB_INVALID_ARGUMENT, "the slice must lie inside [0, vocab_total)");
    if (r->rows < 0 || r->ld < r->vocab) return fail(SSB_INVALID_ARGUMENT, "rows is negative or ld below the slice width");
    if (r->dtype != SSB_F32 && r->dtype != SSB_BF16) return fail(SSB_INVALID_ARGUMENT, "dtype is neither SSB_F32 nor SSB_BF16");
    if (r->mask_kind < SSB_MASK_NONE || r->mask_kind > SSB_MASK_ALLOW) return fail(SSB_INVALID_ARGUMENT, "mask_kind is not an ssb_mask_kind");
    if (r->mask_kind != SSB_MASK_NONE && (!r->mask || (r->mask_ld > 0 && r->mask_ld < div_up(vocab_total, 32))))
        return fail(SSB_INVALID_ARGUMENT, "the mask must hold ceil(vocab_total / 32) words per row");
    if (r->history && (r->history_ld < 0 || r->history_ld > SSB_MAX_STREAM_HISTORY))
        return fail(SSB_OUT_OF_RANGE, "history_ld must lie in [0, SSB_MAX_STREAM_HISTORY]");
    if (r->rows == 0) return ok();
    if (!r->logits) return fail(SSB_INVALID_ARGUMENT, "logits is null");
    ssb_status st = use_device(ctx);
    if (st != SSB_OK) return st;
    ssb::ShardArgs a{};
    a.r = rows_args(r, k_cap, nullptr);
    a.r.mask = r->mask_kind != SSB_MASK_NONE ? r->mask + col_offset / 32 : nullptr;
    a.col_offset = col_offset;
    a.vocab_total = vocab_total;
    a.k_cap = k_cap;
    a.world = 1;
    a.hist_slots = r->history ? ssb::next_pow2((int) std::max<int64_t>(4, 2 * r->history_ld)) : 0;
    a.records = records;
    // several CTAs per slice row when there are few rows: parts of >= 16384 columns (a part costs a fixed
    // ~30 us of table, sorts and merge besides its columns), at most two CTAs per SM in all; the parts'
    // records are merged by the row's last CTA (part records in the split-row scratch, arrivals in the row
    // counters)
    int64_t splits = std::min<int64_t>(div_up(r->vocab, 16384), std::max(1, 2 * ctx->sm_count / std::max(1, r->rows)));
    splits = std::min<int64_t>(splits, ssb::kShardMaxParts / k_cap);
    while (splits > 1 && (int64_t) r->rows * splits * (k_cap + 1) > (int64_t) ctx->max_slots * ssb::kStreamMaxK) splits--;
    splits = std::max<int64_t>(1, splits);
    const int64_t chunk = div_up(div_up(r->vocab, splits), 32) * 32;
    a.splits = (int) div_up(r->vocab, chunk);
    a.chunk = (int) chunk;
    a.parts = ctx->part_cand;
    a.counters = ctx->counters;
    const int words = (int) div_up(chunk, 32);
    a.bit_words = r->history && words <= 8192 ? words : 0;  // the bitmap where it fits in 32 KB
    if (ssb::shard_select_smem_bytes(a.bit_words, a.hist_slots) > (size_t) ctx->max_smem) a.bit_words = 0;
    if (ssb::shard_select_smem_bytes(a.bit_words, a.hist_slots) > (size_t) ctx->max_smem)
        return fail(SSB_OUT_OF_RANGE, "the history needs more shared memory than the device has");
    const cudaError_t e = ssb::launch_shard_select(a, r->dtype == SSB_BF16, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "shard select launch");
    return ok();
}

ssb_status ssb_shard_merge(ssb_context * ctx, const ssb_rows * r, int32_t vocab_total, int32_t world, int32_t k_cap,
                           const uint64_t * records, void * stream) {
    if (!ctx || !r || !records) return fail(SSB_INVALID_ARGUMENT, "ctx, rows and records are required");
    if (!shard_kcap_ok(k_cap)) return fail(SSB_INVALID_ARGUMENT, "k_cap must be a power of two in [1, 1024]");
    if (world < 1 || world > 64) return fail(SSB_INVALID_ARGUMENT, "world must lie in [1, 64]");
    if (vocab_total < 1 || vocab_total > SSB_MAX_VOCAB) return fail(SSB_INVALID_ARGUMENT, "vocab_total out of range");
    if (r->rows < 0) return fail(SSB_INVALID_ARGUMENT, "rows is negative");
    if (r->rows == 0) return ok();
    if (!r->ids || !r->status) return fail(SSB_INVALID_ARGUMENT, "ids and status are required");
    if (!(!r->row_params && r->params.greedy) && !r->u) return fail(SSB_INVALID_ARGUMENT, "u is required where a row draws (not greedy)");
    if (ssb::shard_merge_smem_bytes(world, k_cap) > (size_t) ctx->max_smem)
        return fail(SSB_OUT_OF_RANGE, "world x k_cap composites need more shared memory than the device has");
    ssb_status st = use_device(ctx);
    if (st != SSB_OK) return st;
    ssb::ShardArgs a{};
    a.r = rows_args(r, k_cap, nullptr);
    a.vocab_total = vocab_total;
    a.k_cap = k_cap;
    a.world = world;
    a.records = const_cast<uint64_t *>(records);
    const cudaError_t e = ssb::launch_shard_merge(a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "shard merge launch");
    return ok();
}

ssb_status ssb_lm_head_argmax(ssb_context * ctx, const ssb_lm_head * h, void * stream) {
    if (!ctx || !h) return fail(SSB_INVALID_ARGUMENT, "ctx and head are required");
    if (h->dtype != SSB_BF16) return fail(SSB_INVALID_ARGUMENT, "the LM head takes bf16 hidden rows and weights");
    if (h->rows < 1 || h->rows > ssb::kLmMaxRows) return fail(SSB_OUT_OF_RANGE, "rows must lie in [1, 256]");
    if (h->dim < 64 || h->dim % 64 != 0) return fail(SSB_INVALID_ARGUMENT, "dim must be a positive multiple of 64");
    if (h->vocab < 1 || h->vocab > SSB_MAX_VOCAB) return fail(SSB_OUT_OF_RANGE, "vocab must lie in [1, SSB_MAX_VOCAB]");
    if (h->hidden_ld < h->dim || h->weight_ld < h->dim || h->hidden_ld % 8 != 0 || h->weight_ld % 8 != 0)
        return fail(SSB_INVALID_ARGUMENT, "hidden_ld and weight_ld must be at least dim and multiples of 8");
    if (!h->hidden || !h->weight || !h->ids) return fail(SSB_INVALID_ARGUMENT, "hidden, weight and ids are required");
    if ((reinterpret_cast<uintptr_t>(h->hidden) | reinterpret_cast<uintptr_t>(h->weight)) % 16 != 0)
        return fail(SSB_INVALID_ARGUMENT, "hidden and weight must be 16-byte aligned");
    ssb_status st = use_device(ctx);
    if (st != SSB_OK) return st;
    ssb::LmArgs a{};
    a.rows = h->rows;
    a.vocab = h->vocab;
    a.dim = h->dim;
    a.n_pad = (h->rows + 15) / 16 * 16;
    a.stages = ssb::lm_stages(a.n_pad, (size_t) ctx->max_smem);
    if (a.stages < 2) return fail(SSB_OUT_OF_RANGE, "the LM head's stages need more shared memory than the device has");
    a.tmem_cols = ssb::next_pow2(std::max(32, 2 * a.n_pad));
    a.best = ctx->lm_best;
    a.error = ctx->lm_error;
    a.ids = h->ids;
    a.max_logit = h->max_logit;
    a.status = h->status;
    // every CTA the same number of tiles (a last wave of a few tiles would run with HBM half idle)
    const int tiles = (h->vocab + 127) / 128;
    const int per = (tiles + ctx->sm_count - 1) / ctx->sm_count;
    const int grid = (tiles + per - 1) / per;
    const cudaError_t e = ssb::launch_lm_argmax(a, h->hidden, h->hidden_ld, h->weight, h->weight_ld, grid,
                                                static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "LM-head launch");
    return ok();
}

ssb_status ssb_candidates_rows(ssb_context * ctx, const ssb_rows * rows, int32_t cap, int32_t * tokens, double * weights,
                               int32_t * count, float * processed, void * stream) {
    if (cap < 0) return fail(SSB_INVALID_ARGUMENT, "cap is negative");
    if (cap > 0 && (!tokens || !weights)) return fail(SSB_INVALID_ARGUMENT, "tokens and weights are required when cap > 0");
    if (!count) return fail(SSB_INVALID_ARGUMENT, "count is required");
    Debug dbg;
    dbg.cap = cap;
    dbg.tokens = cap > 0 ? tokens : nullptr;
    dbg.weights = cap > 0 ? weights : nullptr;
    dbg.count = count;
    dbg.processed = processed;
    return run(ctx, rows, &dbg, static_cast<cudaStream_t>(stream));
}

ssb_status ssb_restrict_rows(ssb_context * ctx, const ssb_rows * r, float * out, int64_t out_ld, void * stream) {
    if (!r) return fail(SSB_INVALID_ARGUMENT, "rows is null");
    if (r->rows < 0) return fail(SSB_INVALID_ARGUMENT, "rows is negative");
    if (r->vocab < 1) return fail(SSB_INVALID_ARGUMENT, "vocab must be at least 1");
    if (r->vocab > SSB_MAX_VOCAB) return fail(SSB_OUT_OF_RANGE, "vocab exceeds SSB_MAX_VOCAB (16777216)");
    if (r->ld < r->vocab) return fail(SSB_INVALID_ARGUMENT, "ld is smaller than vocab");
    if (r->dtype != SSB_F32 && r->dtype != SSB_BF16) return fail(SSB_INVALID_ARGUMENT, "dtype is neither SSB_F32 nor SSB_BF16");
    if (r->mask_kind < SSB_MASK_NONE || r->mask_kind > SSB_MASK_ALLOW) return fail(SSB_INVALID_ARGUMENT, "mask_kind is not an ssb_mask_kind");
    if (r->reserved != 0) return fail(SSB_INVALID_ARGUMENT, "reserved fields must be 0");
    if (r->params.flavor < SSB_FLAVOR_QWEN3_TTS || r->params.flavor > SSB_FLAVOR_DRAMA3)
        return fail(SSB_INVALID_ARGUMENT, "params.flavor is not an ssb_flavor");
    if (!ctx) return fail(SSB_INVALID_ARGUMENT, "ctx is null");
    if (r->rows == 0) return ok();
    if (!r->logits) return fail(SSB_INVALID_ARGUMENT, "logits is null");
    if (!out) return fail(SSB_INVALID_ARGUMENT, "out is null");
    if (out_ld < r->vocab) return fail(SSB_INVALID_ARGUMENT, "out_ld is smaller than vocab");
    if (r->mask_kind != SSB_MASK_NONE) {
        if (!r->mask) return fail(SSB_INVALID_ARGUMENT, "mask_kind is set but mask is null");
        if (r->mask_ld < 0) return fail(SSB_INVALID_ARGUMENT, "mask_ld is negative");
        if (r->mask_ld > 0 && r->mask_ld < div_up(r->vocab, 32)) return fail(SSB_INVALID_ARGUMENT, "mask_ld is smaller than ceil(vocab / 32)");
    }
    int hist_slots = 0;
    if (r->history) {
        if (r->history_ld < 0) return fail(SSB_INVALID_ARGUMENT, "history_ld is negative");
        if (r->history_ld > SSB_MAX_STREAM_HISTORY) return fail(SSB_OUT_OF_RANGE, "history_ld exceeds SSB_MAX_STREAM_HISTORY (8192)");
        hist_slots = r->history_ld > 0 ? ssb::next_pow2((int) std::max<int64_t>(4, 2 * r->history_ld)) : 0;
    }
    ssb_status s = use_device(ctx);
    if (s != SSB_OK) return s;
    ssb::RowsArgs a = rows_args(r, 1, nullptr);
    const cudaError_t e = ssb::launch_restrict(a, hist_slots, r->dtype == SSB_BF16, out, out_ld, ctx->sm_count,
                                               static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "restrict launch");
    return ok();
}

ssb_status ssb_restrict_slice(ssb_context * ctx, const ssb_rows * r, int32_t col_offset, int32_t vocab_total, float * out,
                              int64_t out_ld, void * stream) {
    if (!ctx || !r || !out) return fail(SSB_INVALID_ARGUMENT, "ctx, slice and out are required");
    if (col_offset < 0 || col_offset % 32 != 0) return fail(SSB_INVALID_ARGUMENT, "col_offset must be a non-negative multiple of 32");
    if (r->vocab < 1 || (int64_t) col_offset + r->vocab > vocab_total || vocab_total > SSB_MAX_VOCAB)
        return fail(SSB_INVALID_ARGUMENT, "the slice must lie inside [0, vocab_total)");
    if (r->rows < 0 || r->ld < r->vocab || out_ld < r->vocab) return fail(SSB_INVALID_ARGUMENT, "rows, ld or out_ld out of order");
    if (r->dtype != SSB_F32 && r->dtype != SSB_BF16) return fail(SSB_INVALID_ARGUMENT, "dtype is neither SSB_F32 nor SSB_BF16");
    if (r->mask_kind < SSB_MASK_NONE || r->mask_kind > SSB_MASK_ALLOW) return fail(SSB_INVALID_ARGUMENT, "mask_kind is not an ssb_mask_kind");
    if (r->mask_kind != SSB_MASK_NONE && (!r->mask || (r->mask_ld > 0 && r->mask_ld < div_up(vocab_total, 32))))
        return fail(SSB_INVALID_ARGUMENT, "the mask must hold ceil(vocab_total / 32) words per row");
    if (r->history && (r->history_ld < 0 || r->history_ld > SSB_MAX_STREAM_HISTORY))
        return fail(SSB_OUT_OF_RANGE, "history_ld must lie in [0, SSB_MAX_STREAM_HISTORY]");
    if (r->rows == 0) return ok();
    if (!r->logits) return fail(SSB_INVALID_ARGUMENT, "logits is null");
    ssb_status s = use_device(ctx);
    if (s != SSB_OK) return s;
    ssb::RowsArgs a = rows_args(r, 1, nullptr);
    a.mask = r->mask_kind != SSB_MASK_NONE ? r->mask + col_offset / 32 : nullptr;
    const int hist_slots = r->history && r->history_ld > 0 ? ssb::next_pow2((int) std::max<int64_t>(4, 2 * r->history_ld)) : 0;
    const cudaError_t e = ssb::launch_restrict(a, hist_slots, r->dtype == SSB_BF16, out, out_ld, ctx->sm_count,
                                               static_cast<cudaStream_t>(stream), col_offset, vocab_total);
    if (e != cudaSuccess) return cuda_fail(e, "restrict launch");
    return ok();
}

ssb_status ssb_sample_host(ssb_context * ctx, const ssb_rows * rows, void * stream_ptr) {
    Plan plan{};
    ssb_status s = check_rows(rows, false, &plan);
    if (s != SSB_OK) return s;
    if (!ctx) return fail(SSB_INVALID_ARGUMENT, "ctx is null");
    if (rows->rows == 0) return ok();
    s = use_device(ctx);
    if (s != SSB_OK) return s;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    const ssb_rows & h = *rows;
    const size_t n = (size_t) h.rows;
    const size_t es = h.dtype == SSB_BF16 ? 2 : 4;
    const size_t logit_bytes = ((n - 1) * (size_t) h.ld + (size_t) h.vocab) * es;
    const size_t hist_bytes = h.history ? n * (size_t) h.history_ld * 4 : 0;
    const size_t hlen_bytes = h.history && h.history_len ? n * 4 : 0;
    const size_t mask_words = h.mask_kind != SSB_MASK_NONE ? (h.mask_ld ? n * (size_t) h.mask_ld : (size_t) div_up(h.vocab, 32)) : 0;
    const size_t u_bytes = h.u ? n * 8 : 0;
    const size_t rp_bytes = h.row_params ? n * sizeof(ssb_params) : 0;
    auto al = [](size_t b) { return (b + 255) & ~(size_t) 255; };
    const size_t need = al(logit_bytes) + al(hist_bytes) + al(hlen_bytes) + al(mask_words * 4) + al(u_bytes) + al(rp_bytes) +
                        al(n * 4) * 2;
    if (need > ctx->stage_bytes) {
        cudaError_t e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
        cudaFree(ctx->stage);
        ctx->stage = nullptr;
        ctx->stage_bytes = 0;
        e = cudaMalloc(&ctx->stage, need);
        if (e != cudaSuccess) return cuda_fail(e, "staging buffer");
        ctx->stage_bytes = need;
    }
    unsigned char * p = ctx->stage;
    auto take = [&](size_t b) {
        unsigned char * q = p;
        p += al(b);
        return q;
    };
    ssb_rows d = h;
    cudaError_t e = cudaSuccess;
    auto up = [&](const void * src, size_t bytes) -> void * {
        if (!src || bytes == 0) return nullptr;
        void * dst = take(bytes);
        if (e == cudaSuccess) e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, stream);
        return dst;
    };
    d.logits = up(h.logits, logit_bytes);
    d.history = static_cast<const int32_t *>(up(h.history, hist_bytes));
    d.history_len = static_cast<const int32_t *>(up(h.history ? h.history_len : nullptr, hlen_bytes));
    d.mask = static_cast<const uint32_t *>(up(h.mask_kind != SSB_MASK_NONE ? h.mask : nullptr, mask_words * 4));
    d.u = static_cast<const double *>(up(h.u, u_bytes));
    d.row_params = static_cast<const ssb_params *>(up(h.row_params, rp_bytes));
    d.ids = reinterpret_cast<int32_t *>(take(n * 4));
    d.status = reinterpret_cast<int32_t *>(take(n * 4));
    if (e != cudaSuccess) return cuda_fail(e, "copying the inputs to the device");
    s = run(ctx, &d, nullptr, stream);
    if (s != SSB_OK) return s;
    e = cudaMemcpyAsync(h.ids, d.ids, n * 4, cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(h.status, d.status, n * 4, cudaMemcpyDeviceToHost, stream);
    if (e != cudaSuccess) return cuda_fail(e, "copying the ids back");
    s = wait_stream(ctx, stream, 60.0);
    if (s != SSB_OK) return s;
    return ok();
}

// ---------------------------------------------------------------- Haru: DRY and logit shaping

ssb_status ssb_dry_create(ssb_context * ctx, const ssb_dry_config * config, int32_t streams, const int32_t * exempt,
                          int32_t n_exempt, ssb_dry ** out) {
    if (!ctx || !config || !out) return fail(SSB_INVALID_ARGUMENT, "ctx, config and out are required");
    *out = nullptr;
    if (config->reserved != 0) return fail(SSB_INVALID_ARGUMENT, "reserved fields must be 0");
    if (streams < 1) return fail(SSB_INVALID_ARGUMENT, "streams must be at least 1");
    if (config->lookback < 0 || config->max_match_length < 0)
        return fail(SSB_INVALID_ARGUMENT, "lookback and max_match_length must not be negative");
    if ((int64_t) config->lookback + config->max_match_length + 1 > SSB_DRY_MAX_WINDOW)
        return fail(SSB_OUT_OF_RANGE, "lookback + max_match_length + 1 exceeds SSB_DRY_MAX_WINDOW (8192)");
    if (n_exempt < 0 || n_exempt > SSB_DRY_MAX_EXEMPT || (n_exempt > 0 && !exempt))
        return fail(SSB_INVALID_ARGUMENT, "exempt must hold n_exempt ids, at most SSB_DRY_MAX_EXEMPT (64)");
    ssb_status st = use_device(ctx);
    if (st != SSB_OK) return st;
    ssb_dry * d = new ssb_dry();
    d->device = ctx->device;
    d->max_smem = ctx->max_smem;
    ssb::DryArgs & a = d->a;
    a.cfg = ssb::DryConfigD{config->multiplier, config->base, config->max_penalty, config->allowed_length,
                            config->lookback, config->max_match_length};
    a.streams = streams;
    a.window = config->lookback + config->max_match_length + 1;
    a.rec_slots = ssb::next_pow2(a.window);
    a.pen_cap = std::max(1, config->lookback);
    a.n_exempt = n_exempt;
    const size_t n = (size_t) streams;
    const size_t bytes = n * a.window * 4 + 3 * n * 4 + n * a.pen_cap * 4 + n * a.pen_cap * 8 + SSB_DRY_MAX_EXEMPT * 4 + 64;
    cudaError_t e = cudaMalloc(&d->block, bytes);
    if (e == cudaSuccess) e = cudaMemset(d->block, 0, bytes);
    if (e != cudaSuccess) {
        cudaFree(d->block);
        delete d;
        return cuda_fail(e, "DRY state");
    }
    unsigned char * p = static_cast<unsigned char *>(d->block);
    a.pen_val = reinterpret_cast<double *>(p);  // 8-byte aligned first
    p += n * a.pen_cap * 8;
    a.hist = reinterpret_cast<int32_t *>(p);
    p += n * a.window * 4;
    a.head = reinterpret_cast<int32_t *>(p);
    p += n * 4;
    a.count = reinterpret_cast<int32_t *>(p);
    p += n * 4;
    a.pen_n = reinterpret_cast<int32_t *>(p);
    p += n * 4;
    a.pen_tok = reinterpret_cast<int32_t *>(p);
    p += n * a.pen_cap * 4;
    int32_t * ex = reinterpret_cast<int32_t *>(p);
    if (n_exempt > 0) {
        e = cudaMemcpy(ex, exempt, (size_t) n_exempt * 4, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            cudaFree(d->block);
            delete d;
            return cuda_fail(e, "DRY exempt ids");
        }
    }
    a.exempt = ex;
    if (ssb::dry_smem_bytes(a.window) > (size_t) ctx->max_smem) {
        cudaFree(d->block);
        delete d;
        return fail(SSB_OUT_OF_RANGE, "the DRY window needs more shared memory than the device has");
    }
    *out = d;
    return ok();
}

ssb_status ssb_dry_destroy(ssb_dry * d) {
    if (!d) return ok();
    int cur = -1;
    cudaGetDevice(&cur);
    cudaSetDevice(d->device);
    cudaFree(d->block);
    if (cur >= 0) cudaSetDevice(cur);
    delete d;
    return ok();
}

ssb_status ssb_dry_update(ssb_dry * d, const int32_t * tokens, void * stream_ptr) {
    if (!d || !tokens) return fail(SSB_INVALID_ARGUMENT, "dry and tokens are required");
    cudaError_t e = cudaSetDevice(d->device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    e = ssb::launch_dry_update(d->a, tokens, static_cast<cudaStream_t>(stream_ptr));
    if (e != cudaSuccess) return cuda_fail(e, "DRY update launch");
    return ok();
}

ssb_status ssb_dry_penalties(const ssb_dry * d, int32_t s, int32_t * tokens, double * penalties, int32_t cap,
                             int32_t * count, void * stream_ptr) {
    if (!d || !count || (cap > 0 && (!tokens || !penalties)))
        return fail(SSB_INVALID_ARGUMENT, "dry, count and (for cap > 0) tokens and penalties are required");
    if (s < 0 || s >= d->a.streams) return fail(SSB_INVALID_ARGUMENT, "s is not a stream of this state");
    cudaError_t e = cudaSetDevice(d->device);
    if (e == cudaSuccess) e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream_ptr));
    int32_t n = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&n, d->a.pen_n + s, 4, cudaMemcpyDeviceToHost);
    const int32_t c = std::min(n, std::max(cap, 0));
    if (e == cudaSuccess && c > 0)
        e = cudaMemcpy(tokens, d->a.pen_tok + (int64_t) s * d->a.pen_cap, (size_t) c * 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && c > 0)
        e = cudaMemcpy(penalties, d->a.pen_val + (int64_t) s * d->a.pen_cap, (size_t) c * 8, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "reading the DRY penalties");
    *count = n;
    return ok();
}

ssb_status ssb_haru_shape_rows(ssb_context * ctx, const ssb_haru_shape * h, const ssb_dry * d, void * stream_ptr) {
    if (!ctx || !h) return fail(SSB_INVALID_ARGUMENT, "ctx and shape are required");
    if (h->rows < 0 || h->vocab < 1) return fail(SSB_INVALID_ARGUMENT, "rows is negative or vocab below 1");
    if (h->rows == 0) return ok();
    if (!h->logits || !h->silent) return fail(SSB_INVALID_ARGUMENT, "logits and silent are required");
    if (h->ld < h->vocab || h->silent_ld < 2) return fail(SSB_INVALID_ARGUMENT, "ld is below vocab or silent_ld below 2");
    for (int32_t id : {h->pad, h->eop, h->eos})
        if (id < 0 || id >= h->vocab) return fail(SSB_INVALID_ARGUMENT, "pad, eop and eos must lie in [0, vocab)");
    if (d && (d->device != ctx->device || h->rows > d->a.streams))
        return fail(SSB_INVALID_ARGUMENT, "the DRY state has fewer streams than rows, or lives on another device");
    ssb_status st = use_device(ctx);
    if (st != SSB_OK) return st;
    ssb::ShapeArgs a{};
    a.logits = h->logits;
    a.ld = h->ld;
    a.rows = h->rows;
    a.vocab = h->vocab;
    a.silent = h->silent;
    a.silent_ld = h->silent_ld;
    a.pad = h->pad;
    a.eop = h->eop;
    a.eos = h->eos;
    a.eop_bias = h->eop_bias;
    a.must_speak = h->must_speak;
    if (d) {
        a.pen_n = d->a.pen_n;
        a.pen_tok = d->a.pen_tok;
        a.pen_val = d->a.pen_val;
        a.pen_cap = d->a.pen_cap;
    }
    const cudaError_t e = ssb::launch_haru_shape(a, static_cast<cudaStream_t>(stream_ptr));
    if (e != cudaSuccess) return cuda_fail(e, "Haru shaping launch");
    return ok();
}

}  // extern "C"
