// Launch arguments of the sampler kernels (host <-> device, by value).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "speech_sampler_b200.h"

namespace ssb {

// cudaFuncSetAttribute(kernel, MaxDynamicSharedMemorySize, bytes) once per (device, kernel) and size:
// a launch that needs no more than the kernel already allows costs no attribute call (ssb_capi.cu).
cudaError_t set_max_dynamic_smem(const void * kernel, size_t bytes);

// Fields every kernel reads: the batch (device pointers) plus the optional parity/debug outputs.
struct RowsArgs {
    const void * logits;
    int64_t ld;
    int rows;
    int vocab;
    ssb_params params;
    const ssb_params * row_params;
    int k_bound;  // largest effective top-k of a drawing row (rows beyond it are INVALID_ROW)
    const int32_t * history;
    int64_t history_ld;
    const int32_t * history_len;
    const uint32_t * mask;
    int64_t mask_ld;
    int mask_kind;
    const double * u;
    int32_t * ids;
    int32_t * status;
    // debug / parity export (ssb_candidates_rows); null in the product path
    int dbg_cap;
    int32_t * dbg_tokens;
    double * dbg_weights;
    int32_t * dbg_count;
    float * dbg_processed;
};

using SmallArgs = RowsArgs;

// Split-row streaming kernels: `splits` CTAs per row, each streaming `chunk` columns; with more than
// one split, each CTA leaves its partial result in the part_* scratch and the last CTA of the row
// (by the per-row arrival counter) merges them. Counters return to 0 after every launch.
struct StreamArgs {
    RowsArgs r;
    int splits;
    int chunk;       // columns per split, a multiple of 32
    int cap;         // candidate buffer entries per CTA (top-k mode): k_bound + slack
    int hist_slots;  // shared hash-table slots for in-range history ids (power of two >= 2 history_ld)
    int sel_slots;   // shared slots for the selected candidates (>= k_bound)
    uint64_t * part_cand;  // [rows * splits * k_bound] composites
    int32_t * part_n;      // [rows * splits]
    float * part_max;      // [rows * splits] restricted maximum (NaN-propagating)
    int32_t * part_flags;  // [rows * splits] bit 0: a scaled logit was NaN
    uint32_t * counters;   // [rows]
};

constexpr int kStreamThreads = 256;
constexpr int kStreamMaxK = 1024;  // largest top-k of the streaming path

size_t small_smem_bytes(int vocab, int k_bound);
cudaError_t launch_small(const SmallArgs & a, bool bf16, bool debug, cudaStream_t stream);

// mode 0: every row greedy (argmax); mode 1: top-k draw (greedy rows as top-1 of unscaled logits)
size_t stream_smem_bytes(int mode, bool vec, int chunk, int hist_slots, int cap, int sel_slots);
cudaError_t launch_stream(const StreamArgs & a, int mode, bool bf16, bool vec, bool debug, cudaStream_t stream);
int stream_blocks_per_sm(int mode, bool bf16, bool vec, size_t smem);

// All-greedy batches on aligned rows (ssb_argmax.cu): grid (splits, rows), chunks a multiple of
// argmax_unit columns (one 16-byte load per thread), partial maxima merged by the row's last CTA.
int argmax_unit(bool bf16);
size_t argmax_smem_bytes(int chunk, int hist_slots);
cudaError_t launch_argmax(const StreamArgs & a, bool bf16, cudaStream_t stream);

// Top-k kernel (ssb_topk.cu) for 16-byte-aligned rows with top-k <= kTopkMaxK, greedy rows as the
// top-1 of their unscaled logits: kw = the width of its warp lists in registers (1, 2 or 4: top-k up
// to 32, 64, 128).
constexpr int kTopkMaxK = 128;
int topk_kw(int k_bound);
// the longest chunk (columns) one CTA streams
int topk_max_chunk(bool bf16);
size_t topk_smem_bytes(int kw, bool bf16, int chunk, int hist_slots, int sel_slots);
int topk_blocks_per_sm(int kw, bool bf16, size_t smem);
cudaError_t launch_topk(const StreamArgs & a, int kw, bool bf16, bool debug, cudaStream_t stream);

// Rows whose top-k keeps more than kStreamMaxK tokens (top-k 0 = all) over a large vocabulary
// (ssb_nucleus.cu): one CTA per row at a time (rows looped over the grid), each with its own region of
// `scratch` (scratch_ld composites) for the row's finite scaled logits.
struct NucleusArgs {
    RowsArgs r;
    uint64_t * scratch;
    int64_t scratch_ld;
    int hist_slots;
};
size_t nucleus_smem_bytes(int vocab, int hist_slots);
int64_t nucleus_scratch_ld(int vocab);
int nucleus_threads();
int nucleus_blocks_per_sm(bool bf16, size_t smem);
cudaError_t launch_nucleus(const NucleusArgs & a, int grid, bool bf16, bool debug, cudaStream_t stream);

// The Haru and Drama 3 candidate rules (ssb_flavor.cu): one CTA per row, at most kFlavorMaxK candidates.
constexpr int kFlavorMaxK = 8192;
struct FlavorArgs {
    RowsArgs r;
    int flavor;      // ssb_flavor of the call; a row of another family is INVALID_ROW
    int cap;         // candidate slots (a power of two <= kFlavorMaxK); a drawing row with more is INVALID_ROW
    int hist_slots;  // shared hash-table slots for the history (power of two >= 2 history_ld), or 0
    int bit_words;   // words of the history-column bitmap (ceil(vocab / 32)), or 0 to look up the table
};
size_t flavor_smem_bytes(int cap, int bit_words, int hist_slots);
cudaError_t launch_flavor(const FlavorArgs & a, bool bf16, bool debug, cudaStream_t stream);

// The vocabulary-sharded draw (ssb_shard.cu): per slice, the k_cap best composites and (max, flags) of
// each row as one record of k_cap + 1 words; after the all-gather, the merge of world records per row.
struct ShardArgs {
    RowsArgs r;        // select: the slice (vocab = width, mask at the slice's first word); merge: params, u, ids, status
    int col_offset;    // the slice's first column (a multiple of 32)
    int vocab_total;   // the whole row's width
    int k_cap;         // composites per record (a power of two <= 1024)
    int world;         // merge: records per row
    int hist_slots;
    int bit_words;       // select: words of the history-column bitmap (ceil(chunk / 32)), or 0
    uint64_t * records;  // select: [rows, k_cap + 1] out; merge: [world][rows][k_cap + 1] in
    int splits;          // select: CTAs per slice row (splits x k_cap <= 4096), each `chunk` columns
    int chunk;           //         (a multiple of 32)
    uint64_t * parts;    //         [rows, splits, k_cap + 1] the parts' records (splits > 1)
    uint32_t * counters; //         [rows] arrivals, 0 between launches
};
constexpr int kShardMaxK = 1024;
constexpr int kShardMaxParts = 4096;  // splits x k_cap composites merged in shared memory per slice row
size_t shard_select_smem_bytes(int bit_words, int hist_slots);
size_t shard_merge_smem_bytes(int world, int k_cap);
cudaError_t launch_shard_select(const ShardArgs & a, bool bf16, cudaStream_t stream);
cudaError_t launch_shard_merge(const ShardArgs & a, cudaStream_t stream);

// The LM head fused with its argmax (ssb_lmhead.cu): tcgen05 MMAs over 128-token tiles, the argmax in the
// TMEM epilogue. n_pad = rows rounded up to 16 (the MMA's N); tmem_cols = two accumulators of n_pad.
struct LmArgs {
    int rows, vocab, dim, n_pad, stages, tmem_cols;
    uint64_t * best;    // [n_pad] composite maxima, 0 between calls
    int32_t * error;    // 0 between calls
    int32_t * ids;
    float * max_logit;  // or null
    int32_t * status;   // or null
};
constexpr int kLmMaxRows = 256;
int lm_stages(int n_pad, size_t max_smem);
size_t lm_smem_bytes(int n_pad, int stages);
cudaError_t launch_lm_argmax(const LmArgs & a, const void * hidden, int64_t hidden_ld, const void * weight,
                             int64_t weight_ld, int grid, cudaStream_t stream);

// The embedding rows of drawn ids (ssb_embed.cu): out[r] = table[ids[r]] (zeros for a refused row).
struct EmbedArgs {
    const void * table;
    int64_t ld;
    int table_rows;
    int dim;
    void * out;
    int64_t out_ld;
    const int32_t * ids;
    const int32_t * status;
    int rows;
};
cudaError_t launch_embed(const EmbedArgs & a, bool bf16, cudaStream_t stream);

// Haru's DRY state update and logit shaping (ssb_haru.cu).
struct DryConfigD {
    double multiplier, base, max_penalty;
    int allowed_length, lookback, max_match_length;
};
struct DryArgs {
    DryConfigD cfg;
    int streams;
    int window;     // ring capacity: lookback + max_match_length + 1
    int rec_slots;  // next_pow2(window): shared records of one update
    int32_t * hist;   // [streams, window] ring of drawn tokens
    int32_t * head;   // [streams] slot of the oldest
    int32_t * count;  // [streams] tokens held
    int32_t * pen_tok;  // [streams, pen_cap] penalties by rising token
    double * pen_val;   // [streams, pen_cap]
    int32_t * pen_n;    // [streams]
    int pen_cap;        // max(1, lookback): at most one proposal per earlier position
    const int32_t * exempt;  // [n_exempt] device
    int n_exempt;
};
struct ShapeArgs {
    float * logits;
    int64_t ld;
    int rows, vocab;
    const float * silent;
    int64_t silent_ld;
    int pad, eop, eos;
    float eop_bias;
    const int32_t * must_speak;
    const int32_t * pen_n;  // null: no DRY
    const int32_t * pen_tok;
    const double * pen_val;
    int pen_cap;
};
size_t dry_smem_bytes(int window);
cudaError_t launch_dry_update(const DryArgs & a, const int32_t * tokens, cudaStream_t stream);
cudaError_t launch_haru_shape(const ShapeArgs & a, cudaStream_t stream);

// The restricted logits alone (ssb_restrict.cu): every column widened to f32 with the mask applied,
// then each row's history tokens penalized over it. `a` needs no ids, status or u.
size_t restrict_smem_bytes(int hist_slots);
// col_offset / vocab_total: the rows are columns [col_offset, col_offset + a.vocab) of rows of vocab_total
// tokens whose history holds the whole rows' ids (0 / 0: the whole rows).
cudaError_t launch_restrict(const RowsArgs & a, int hist_slots, bool bf16, float * out, int64_t out_ld, int sm_count,
                            cudaStream_t stream, int col_offset = 0, int vocab_total = 0);

}  // namespace ssb
