// ssb_sample_rows_noalloc: sampling of large-vocabulary rows for callers that cannot allocate device
// memory.
//
// Who needs it: code that runs where cudaMalloc is not an option — a host process that hands the
// sampler device buffers owned by someone else (an inference runtime's memory pool, a caching
// allocator that must not be bypassed), an embedding that is not allowed to grow its footprint after
// start-up, or a caller that must not risk the implicit device synchronization and the failure modes
// of an allocation on its decode path. ssb_sample_rows needs an ssb_context, and creating one
// allocates its split-row scratch with cudaMalloc; this entry point needs no context at all.
//
// How: the scratch that the split-row top-k kernel uses to combine the CTAs of one row lives in a
// fixed-size array in this file, `g_scratch` (kScratchBytes, about 2.03 MiB, held by every GPU that
// loads the library until the process exits). Host code cannot use the array's name as a device
// address, so the first call on each device looks the address up with cudaGetSymbolAddress (with that
// device current), clears the per-row arrival counters once (a synchronous cudaMemset of that array,
// not an allocation) and keeps the address; make that first call before any stream capture. The
// caller still passes every input and output buffer.
//
// Limits: rows of more than SSB_SMALL_VOCAB tokens, 16-byte-aligned rows, and top-k of at most 128
// (or greedy rows) — the rows the top-k kernel (ssb_topk.cu) takes; anything else is refused
// with SSB_OUT_OF_RANGE and a message, never sampled another way. The kernel is launched exactly as
// ssb_sample_rows launches it; only where its scratch comes from differs.
//
// Every call shares the one array: calls that overlap on the GPU (on different streams, or from
// different threads without ordering) race on it and must not be made. The kernel returns each row's
// arrival counter to zero itself (the last CTA of a row resets it), so a call leaves the array ready for
// the next one; the counters are cleared once, when the device is set up.
#include <algorithm>
#include <cstdint>
#include <mutex>
#include <string>

#include <cuda_runtime.h>

#include "speech_sampler_b200.h"
#include "ssb_device.cuh"
#include "ssb_kernels.h"

namespace ssb {
void set_last_error(const std::string & message);  // ssb_capi.cu
}

namespace {

constexpr int kScratchSlots = 2048;  // (row, split) pairs one launch may spread over
constexpr int kScratchMaxK = ssb::kTopkMaxK;
constexpr size_t kCandBytes = (size_t) kScratchSlots * kScratchMaxK * sizeof(uint64_t);
constexpr size_t kScratchBytes = kCandBytes + 4 * (size_t) kScratchSlots * sizeof(uint32_t);
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

struct DeviceSetup {
    bool ready = false;
    unsigned char * scratch = nullptr;  // g_scratch's device address on this device
    int sm_count = 0;
    int max_smem = 0;  // opt-in shared memory per block
    // occupancy of the top-k kernel per (warp-list width class, bf16), and the shared memory it was
    // measured at (measured once per shape, under g_setup_mutex)
    int occ[3][2] = {};
    size_t occ_smem[3][2] = {};
};

DeviceSetup g_setup[kMaxDevices];
std::mutex g_setup_mutex;

ssb_status fail(ssb_status s, const std::string & message) {
    ssb::set_last_error(message);
    return s;
}

ssb_status cuda_fail(cudaError_t e, const char * what) {
    return fail(SSB_DEVICE, std::string(what) + ": " + cudaGetErrorString(e));
}

// Looks up g_scratch's address and the SM count of the current device, once.
ssb_status setup(int device, DeviceSetup ** out) {
    if (device < 0 || device >= kMaxDevices) return fail(SSB_OUT_OF_RANGE, "device index beyond 63");
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    DeviceSetup & d = g_setup[device];
    if (!d.ready) {
        void * p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_scratch)");
        e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, device);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&d.max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
        d.scratch = static_cast<unsigned char *>(p);
        // the arrival counters start at zero; every launch leaves them at zero again
        e = cudaMemset(d.scratch + kCandBytes + (size_t) kScratchSlots * 12, 0, (size_t) kScratchSlots * sizeof(uint32_t));
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_fail(e, "clearing the arrival counters");
        d.ready = true;
    }
    *out = &d;
    return SSB_OK;
}

int64_t div_up(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace

extern "C" ssb_status ssb_sample_rows_noalloc(const ssb_rows * r, void * stream_ptr) {
    if (!r) return fail(SSB_INVALID_ARGUMENT, "rows is null");
    if (r->rows < 0) return fail(SSB_INVALID_ARGUMENT, "rows is negative");
    if (r->vocab < 1) return fail(SSB_INVALID_ARGUMENT, "vocab must be at least 1");
    if (r->vocab > SSB_MAX_VOCAB) return fail(SSB_OUT_OF_RANGE, "vocab exceeds SSB_MAX_VOCAB (16777216)");
    if (r->ld < r->vocab) return fail(SSB_INVALID_ARGUMENT, "ld is smaller than vocab");
    if (r->dtype != SSB_F32 && r->dtype != SSB_BF16) return fail(SSB_INVALID_ARGUMENT, "dtype is neither SSB_F32 nor SSB_BF16");
    if (r->mask_kind < SSB_MASK_NONE || r->mask_kind > SSB_MASK_ALLOW) return fail(SSB_INVALID_ARGUMENT, "mask_kind is not an ssb_mask_kind");
    if (r->reserved != 0) return fail(SSB_INVALID_ARGUMENT, "reserved fields must be 0");
    if (r->params.flavor != SSB_FLAVOR_QWEN3_TTS)
        return fail(SSB_OUT_OF_RANGE, "ssb_sample_rows_noalloc samples the Qwen3-TTS family; use ssb_sample_rows");
    if (r->rows == 0) {
        ssb::set_last_error("");
        return SSB_OK;
    }
    if (!r->logits || !r->ids || !r->status) return fail(SSB_INVALID_ARGUMENT, "logits, ids and status are required");
    if (r->vocab <= SSB_SMALL_VOCAB)
        return fail(SSB_OUT_OF_RANGE, "ssb_sample_rows_noalloc samples rows of more than 8192 tokens; use ssb_sample_rows");
    const int es = r->dtype == SSB_BF16 ? 2 : 4;
    if (reinterpret_cast<uintptr_t>(r->logits) % 16 != 0 || (r->ld * es) % 16 != 0)
        return fail(SSB_OUT_OF_RANGE, "ssb_sample_rows_noalloc needs rows that start on 16-byte boundaries");
    if (r->mask_kind != SSB_MASK_NONE) {
        if (!r->mask) return fail(SSB_INVALID_ARGUMENT, "mask_kind is set but mask is null");
        if (r->mask_ld < 0 || (r->mask_ld > 0 && r->mask_ld < div_up(r->vocab, 32)))
            return fail(SSB_INVALID_ARGUMENT, "mask_ld is negative or smaller than ceil(vocab / 32)");
    }
    if (r->history) {
        if (r->history_ld < 0) return fail(SSB_INVALID_ARGUMENT, "history_ld is negative");
        if (r->history_ld > SSB_MAX_STREAM_HISTORY)
            return fail(SSB_OUT_OF_RANGE, "history_ld exceeds SSB_MAX_STREAM_HISTORY (8192)");
    }
    const bool all_greedy = !r->row_params && r->params.greedy;
    if (!all_greedy && !r->u) return fail(SSB_INVALID_ARGUMENT, "u is required where a row draws (not greedy)");
    int kb;
    if (r->row_params) {
        if (r->max_top_k < 0) return fail(SSB_INVALID_ARGUMENT, "max_top_k is negative");
        kb = r->max_top_k > 0 ? std::min(r->max_top_k, r->vocab) : r->vocab;
    } else {
        kb = r->params.greedy ? 1 : (r->params.top_k > 0 ? std::min(r->params.top_k, r->vocab) : r->vocab);
    }
    if (!all_greedy && kb > kScratchMaxK)
        return fail(SSB_OUT_OF_RANGE, "ssb_sample_rows_noalloc takes a top-k of at most 128; use ssb_sample_rows");

    int device = -1;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    DeviceSetup * d = nullptr;
    ssb_status s = setup(device, &d);
    if (s != SSB_OK) return s;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);

    const bool bf16 = r->dtype == SSB_BF16;
    kb = std::max(1, kb);
    const int kw = ssb::topk_kw(kb);
    ssb::StreamArgs sa{};
    ssb::RowsArgs & a = sa.r;
    a.logits = r->logits;
    a.ld = r->ld;
    a.rows = r->rows;
    a.vocab = r->vocab;
    a.params = r->params;
    a.row_params = r->row_params;
    a.k_bound = kb;
    a.history = r->history;
    a.history_ld = r->history ? r->history_ld : 0;
    a.history_len = r->history ? r->history_len : nullptr;
    a.mask = r->mask_kind != SSB_MASK_NONE ? r->mask : nullptr;
    a.mask_ld = r->mask_ld;
    a.mask_kind = r->mask_kind;
    a.u = r->u;
    a.ids = r->ids;
    a.status = r->status;
    sa.hist_slots = r->history ? ssb::next_pow2((int) std::max<int64_t>(4, 2 * r->history_ld)) : 0;
    sa.sel_slots = ssb::next_pow2(std::max(kb, 2));
    const int full_chunk = (int) div_up(r->vocab, 32) * 32;
    // the kernel keeps per-chunk state in shared memory: a long history leaves less of it, so the chunk
    // is halved until it fits (as ssb_sample_rows does); refused only if even a 4096-column chunk does not
    int max_chunk = std::min(full_chunk, ssb::topk_max_chunk(bf16));
    while (max_chunk > 4096 && ssb::topk_smem_bytes(kw, bf16, max_chunk, sa.hist_slots, sa.sel_slots) > (size_t) d->max_smem)
        max_chunk = (int) div_up(max_chunk / 2, 32) * 32;
    const size_t smem = ssb::topk_smem_bytes(kw, bf16, max_chunk, sa.hist_slots, sa.sel_slots);
    if (smem > (size_t) d->max_smem)
        return fail(SSB_OUT_OF_RANGE, "the history is too long for the top-k kernel's shared memory; use ssb_sample_rows");
    const int kwc = kw == 1 ? 0 : (kw == 2 ? 1 : 2);
    int occ = 0;
    {
        std::lock_guard<std::mutex> lock(g_setup_mutex);
        if (d->occ[kwc][bf16] == 0 || d->occ_smem[kwc][bf16] != smem) {
            d->occ[kwc][bf16] = ssb::topk_blocks_per_sm(kw, bf16, smem);
            d->occ_smem[kwc][bf16] = smem;
        }
        occ = d->occ[kwc][bf16];
    }
    if (occ <= 0) return fail(SSB_DEVICE, "the top-k kernel does not fit on this device");
    const int slots = std::min(kScratchSlots, d->sm_count * occ);
    const int min_chunk = all_greedy ? 2048 : 4096;
    int64_t splits = std::max<int64_t>(1, std::min<int64_t>(div_up(r->vocab, min_chunk), slots / std::max(1, r->rows)));
    // two halves of a row do not pay for their merge in the top-k kernel: one CTA per row streams the
    // whole row instead (128 rows of 151936 bf16: 22.8 us against 24.7 us split in two)
    if (splits == 2) splits = 1;
    splits = std::max<int64_t>(splits, div_up(r->vocab, max_chunk));
    const int64_t chunk = div_up(div_up(r->vocab, splits), 32) * 32;
    splits = div_up(r->vocab, chunk);
    sa.splits = (int) splits;
    sa.chunk = (int) chunk;
    if ((int64_t) r->rows * splits > INT32_MAX) return fail(SSB_OUT_OF_RANGE, "too many rows for one launch");
    if (splits > 1) {
        if ((int64_t) r->rows * splits > kScratchSlots) return fail(SSB_OUT_OF_RANGE, "the batch needs more scratch than the fixed array holds");
        unsigned char * base = d->scratch;
        sa.part_cand = reinterpret_cast<uint64_t *>(base);
        sa.part_n = reinterpret_cast<int32_t *>(base + kCandBytes);
        sa.part_max = reinterpret_cast<float *>(base + kCandBytes + (size_t) kScratchSlots * 4);
        sa.part_flags = reinterpret_cast<int32_t *>(base + kCandBytes + (size_t) kScratchSlots * 8);
        sa.counters = reinterpret_cast<uint32_t *>(base + kCandBytes + (size_t) kScratchSlots * 12);
    }
    e = ssb::launch_topk(sa, kw, bf16, false, stream);
    if (e != cudaSuccess) return cuda_fail(e, "top-k kernel launch");
    ssb::set_last_error("");
    return SSB_OK;
}
