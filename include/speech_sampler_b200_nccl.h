/*
 * speech_sampler_b200_nccl — the vocabulary-sharded draw over NCCL (libspeech_sampler_b200_nccl.so, host
 * C++ linked with the engine and NCCL). One process per GPU; every rank holds a slice of each row's
 * columns (a tensor-parallel LM head's logits) and every rank ends with the ids and statuses the
 * single-GPU ssb_sample_rows gives on the whole rows. Per call: ssb_shard_select on the rank's slice,
 * one ncclAllGather of the records (rows * (k_cap + 1) * 8 bytes per rank), ssb_shard_merge; all on the
 * caller's stream, nothing read back. No counterpart in the reference, which samples whole host rows.
 */
#ifndef SPEECH_SAMPLER_B200_NCCL_H
#define SPEECH_SAMPLER_B200_NCCL_H

#include "speech_sampler_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ssb_shard_comm ssb_shard_comm;

/* An NCCL unique id (128 bytes) for rank 0 to share with the others (by any out-of-band channel). */
SSB_API ssb_status ssb_nccl_unique_id(uint8_t id[128]);

/* Joins the communicator of `world` ranks identified by `id` as `rank`, on ctx's device (collective:
 * every rank calls it). The communicator owns the record buffers (grown on first use). */
SSB_API ssb_status ssb_shard_comm_create(ssb_context *ctx, const uint8_t id[128], int32_t world, int32_t rank,
                                         ssb_shard_comm **out);
SSB_API ssb_status ssb_shard_comm_destroy(ssb_shard_comm *comm);

/* Sizes the record buffers for `rows` rows of k_cap (so that a later call allocates nothing and can be
 * captured into a CUDA graph). */
SSB_API ssb_status ssb_shard_comm_reserve(ssb_shard_comm *comm, int32_t rows, int32_t k_cap);

/* The sharded draw of `slice` (as ssb_shard_select takes it; its ids, status, u and params as
 * ssb_shard_merge takes them) on every rank (collective). With k_cap > 0 the candidate exchange (rows of
 * row_params keeping more than k_cap tokens come back SSB_ROW_INVALID_ROW); with k_cap 0, or without
 * row_params a drawing row that keeps more than k_cap tokens (top_k 0), the restricted-slice exchange:
 * ssb_restrict_slice, one ncclAllGather of the f32 slices, the whole rows laid out and ssb_sample_rows on
 * them (the first such call, and any call with another slice layout, synchronises the stream once to
 * learn every rank's slice). */
SSB_API ssb_status ssb_shard_sample(ssb_shard_comm *comm, const ssb_rows *slice, int32_t col_offset,
                                    int32_t vocab_total, int32_t k_cap, void *stream);

/* The message of the last failed call of this library on the calling thread. */
SSB_API const char *ssb_nccl_last_error(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* SPEECH_SAMPLER_B200_NCCL_H */
