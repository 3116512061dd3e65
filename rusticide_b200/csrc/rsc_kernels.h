// Internal launch interface between the C ABI (api.cu) and the kernels.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "rsc_common.cuh"

namespace rsc {

// Survivor sets up to this size are finished in shared memory by the
// streaming kernel; larger ones (top-k disabled on a wide row, or ties)
// go to the large-survivor kernel.
constexpr uint32_t kSmallCap = 512;
// Largest top_k the streaming kernel takes; larger k go to the large kernel.
constexpr uint32_t kSmallTopK = kSmallCap / 4;
// Top-k above kSmallTopK and up to this many: the streaming kernel's two-pass
// epilogue (a histogram pass and a gather into a kSmallCap list).
constexpr uint32_t kTwoPassTopK = kSmallCap - 24;

cudaError_t launch_greedy(const float *logits, size_t rows, uint32_t vocab, size_t row_stride,
                          uint32_t *out_ids, int32_t *out_status, int num_sms,
                          cudaStream_t stream);

// Most CTAs a row is spread over by the streaming kernel.
constexpr uint32_t kStreamMaxSplits = 16;

// Overflowing rows one streaming CTA can defer to its epilogue; a launch
// covers at most kStreamRowsPerCta rows per CTA so that the list never fills
// (a CTA's pieces span at most rows / grid + 3 rows).
constexpr uint32_t kStreamOvfCap = 64;
constexpr uint32_t kStreamRowsPerCta = 48;

// Bytes of one part record when a row is spread over `parts` CTAs (kSmallCap /
// parts entries).
size_t split_record_bytes(uint32_t parts);

// Work schedule of the streaming kernel: its grid, the chunks per row, and
// whether CTAs take balanced chunk ranges (rows spread over up to max_parts
// CTAs) or whole rows round-robin.
struct StreamPlan {
    uint32_t grid;
    uint32_t nch;
    uint32_t streamk;
    uint32_t max_parts;
};

// The schedule for a call; seg_capacity_bytes is the size of the handle's
// part-record buffer (rows * max_parts * split_record_bytes(max_parts) must
// fit, else whole rows are used).
StreamPlan stream_plan(size_t rows, uint32_t vocab, bool topk_active, uint32_t top_k,
                       int num_sms, size_t seg_capacity_bytes);

// Streaming top-k kernel for rows whose survivors fit kSmallCap, launched as
// a programmatic dependent of the previous work on the stream (it writes
// global memory only after that work completes). A row spread over several
// CTAs leaves one record per part in seg_records (rows * max_parts records of
// split_record_bytes(max_parts)); row_arrivals (rows counters, zero on entry
// and on exit) tells the last part to merge them. Rows whose candidates
// overflow are sampled at the end of their CTA with the large-row code, in a
// scratch slot (`slots` regions of 4 * vocab uint32) taken under slot_lock
// (`slots` words, zero when free). rows <= plan.grid * kStreamRowsPerCta.
cudaError_t launch_stream_topk(const float *logits, size_t rows, uint32_t vocab,
                               size_t row_stride, const CallParams &p, uint32_t *out_ids,
                               int32_t *out_status, float *out_probs, const StreamPlan &plan,
                               void *seg_records, uint32_t *row_arrivals, uint32_t *scratch,
                               uint32_t slots, uint32_t *slot_lock, cudaStream_t stream);

// Large-survivor kernel over rows [0, rows), one 512-thread block per row.
// Scratch: `slots` regions of 4 * vocab uint32 each.
// Large-survivor kernel: resident CTAs per SM. Each CTA samples one row at a
// time, with its own scratch slot of 4 * vocab words. Its per-row code is a
// chain of block scans and barriers; two CTAs per SM overlap one's barriers
// with the other's work (cap: 64 registers a thread at 512 threads).
constexpr uint32_t kLargeCtasPerSm = 2;

// Log-probability outputs (lse.cu): lse_rows writes each row's partial
// log-sum-exp into parts[row * stride] (for rows the streaming kernel's
// consumers did not cover); lse_finish combines each row's `stride` parts and
// writes the log-sum-exp, the chosen token's log-probability and the listed
// survivors' log-probabilities (each output nullable).
cudaError_t launch_lse_rows(const float *logits, size_t rows, uint32_t vocab, size_t row_stride,
                            float scale, uint2 *parts, uint32_t stride, cudaStream_t stream);
cudaError_t launch_lse_finish(const float *logits, size_t rows, size_t row_stride, float scale,
                              const uint2 *parts, uint32_t stride, const uint32_t *ids,
                              const int32_t *status, const uint32_t *n_surv, const uint32_t *surv,
                              uint32_t cap, float *out_lse, float *out_logprob,
                              float *out_surv_logp, cudaStream_t stream);

cudaError_t launch_large(const float *logits, size_t rows, uint32_t vocab, size_t row_stride,
                         const CallParams &p, uint32_t *out_ids, int32_t *out_status,
                         float *out_probs, uint32_t *scratch, uint32_t slots, cudaStream_t stream);

// Whole-row kernel (sample_whole.cu): one 1024-thread block per SM, a row at
// a time, for rows with top-p on and top-k off at a normal scale whose
// vocabulary is at most kWholeMaxToppVocab (their survivors are sorted in
// shared memory). Scratch: `slots` regions of 4 * vocab uint32, one per
// block. whole_takes says whether a call's rows go there (sample_logits, no
// argmax, no survivor outputs, one parameter set for every row).
constexpr uint32_t kWholeMaxToppVocab = 45056;
bool whole_takes(const CallParams &p, size_t vocab);
cudaError_t launch_whole(const float *logits, size_t rows, uint32_t vocab, size_t row_stride,
                         const CallParams &p, uint32_t *out_ids, int32_t *out_status,
                         float *out_probs, uint32_t *scratch, uint32_t slots, int num_sms,
                         cudaStream_t stream);

// LM-head GEMM with the sampler fused into its epilogue (lmhead.cu). A part's
// record of a row holds at most kLmheadRowCap candidates, so top_k <=
// kLmheadRowCap - RSC_SHARD_TIE_CAP; a row is spread over at most
// kLmheadMaxParts parts of at most 65536 columns each (vocab <=
// kLmheadMaxVocab), whose records one block per row merges.
constexpr uint32_t kLmheadRowCap = 64;
constexpr uint32_t kLmheadMaxParts = 256;
constexpr uint64_t kLmheadMaxVocab = uint64_t{kLmheadMaxParts} * 65536u;
constexpr uint32_t kLmheadRecordSlots = kLmheadMaxParts;  // one record per part and row
uint32_t lmhead_parts(size_t rows, uint32_t vocab, int num_sms);
// logits != nullptr: writes rows x vocab f32 logits; otherwise writes one
// shard record per (part, row) into records ([parts][rows], rec_bytes each).
// index_offset: added to every record index (the vocabulary offset of a
// weight shard).
cudaError_t launch_lmhead(const void *hidden, const void *weight, size_t rows, uint32_t dim,
                          uint32_t vocab, const CallParams &p, float *logits, void *records,
                          size_t rec_bytes, uint32_t parts, uint32_t *error_flag,
                          cudaStream_t stream, uint32_t index_offset = 0);

// Vocab-sharded record: this header, then uint32 key[k + RSC_SHARD_TIE_CAP]
// and uint32 index[k + RSC_SHARD_TIE_CAP] (global indices), entries sorted by
// (key desc, index asc). Keys are f32::total_cmp keys of the scaled logits.
struct ShardRecordHeader {
    float max_scaled;    // max of the shard's scaled logits, NaN skipped (diagnostic)
    float sum_exp;       // reserved, 0
    uint32_t n_finite;   // reserved, 0
    uint32_t n_cand;     // entries that follow
    uint32_t n_dropped;  // entries at or above the local threshold that did not fit
    uint32_t last_key;   // key of the last entry
    uint32_t flags;      // 0 ok; 1 candidate list overflow; 2 a device wait gave up
    float tau;           // a lower bound of the part's k-th largest scaled value; every
                         // value at or above it is an entry unless n_dropped > 0
};
static_assert(sizeof(ShardRecordHeader) == 32, "record header layout");

inline size_t shard_record_bytes(uint32_t top_k) {
    size_t entries = static_cast<size_t>(top_k) + RSC_SHARD_TIE_CAP;
    size_t b = sizeof(ShardRecordHeader) + 8 * entries;
    return (b + 15) & ~static_cast<size_t>(15);
}

cudaError_t launch_shard_partial(const float *logits, size_t rows, uint32_t shard_vocab,
                                 size_t row_stride, uint32_t shard_offset, const CallParams &p,
                                 void *records, size_t rec_bytes, int num_sms,
                                 cudaStream_t stream);

// The merge reading each rank's records in place (peer memory; see
// rsc_peer_exchange in the C header for the pointers): rows [row_begin,
// row_end) merged here, with n_shards <= 32 and one warp per row (n_shards * (k +
// RSC_SHARD_TIE_CAP) <= kSmallCap). With ready_results_ptrs set, the results go
// to every rank's arrays and the last CTA publishes them.
struct PeerPointers {
    const void *const *records;
    const uint32_t *ready_records;
    uint32_t *const *ready_results_ptrs;
    uint32_t *done_counter;
    uint32_t *const *ids;
    int32_t *const *status;
    float *const *probs;
};
cudaError_t launch_shard_merge_peers(const PeerPointers &x, uint32_t step, size_t n_shards,
                                     size_t my_shard, size_t row_begin, size_t row_end,
                                     size_t rec_bytes, const CallParams &p, cudaStream_t stream);
// Waits (bounded) for every rank's results of `step`, then copies this rank's
// result arrays to the caller's.
cudaError_t launch_shard_collect(const uint32_t *ready_results, uint32_t step, size_t n_shards,
                                 size_t rows, const uint32_t *ids, const int32_t *status,
                                 const float *probs, uint32_t *out_ids, int32_t *out_status,
                                 float *out_probs, cudaStream_t stream);
// Stores `step` into word my_shard of every rank's ready array (d_ready_ptrs: a
// device array of n_shards pointers, peer memory) after a system-wide fence.
cudaError_t launch_shard_publish(uint32_t *const *d_ready_ptrs, size_t n_shards, uint32_t my_shard,
                                 uint32_t step, cudaStream_t stream);
cudaError_t launch_shard_merge(const void *records, size_t n_shards, size_t rows, size_t rec_bytes,
                               const CallParams &p, uint32_t *out_ids, int32_t *out_status,
                               float *out_probs, int num_sms, cudaStream_t stream);
// One block per row over all n_parts records (records of k + RSC_SHARD_TIE_CAP
// entries, [n_parts][rows]): the merge of launch_shard_merge in one step for
// up to 256 parts of at most 64 entries (shared memory
// shard_merge_block_smem bytes).
size_t shard_merge_block_smem(uint32_t n_parts, uint32_t cap_entries);
cudaError_t launch_shard_merge_block(const void *records, size_t n_parts, size_t rows,
                                     size_t rec_bytes, const CallParams &p, uint32_t *out_ids,
                                     int32_t *out_status, float *out_probs, cudaStream_t stream);
// The same merge, writing one record per row of the same format into
// out_records ([rows], rec_bytes each) instead of sampling: the parts of one
// vocabulary shard reduced to the shard's record.
cudaError_t launch_shard_reduce_block(const void *records, size_t n_parts, size_t rows,
                                      size_t rec_bytes, const CallParams &p, void *out_records,
                                      cudaStream_t stream);

cudaError_t launch_penalize(float *logits, size_t rows, uint32_t vocab, size_t row_stride,
                            const uint32_t *tokens, size_t n_tokens, float penalty,
                            cudaStream_t stream);

cudaError_t launch_expf(const float *x, float *y, size_t n, cudaStream_t stream);

cudaError_t launch_rng_seed(const uint64_t *seeds, uint64_t *states, size_t rows,
                            cudaStream_t stream);

// Shared-memory bytes of the streaming kernel (for occupancy queries).
size_t stream_topk_smem_bytes();

}  // namespace rsc
