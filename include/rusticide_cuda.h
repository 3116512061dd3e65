/*
 * rusticide_cuda.h -- C ABI of the B200 token-sampling engine.
 *
 * The engine is a batched, device-resident drop-in for the sampler of the Rust
 * crate rusticide-sampling (platform-cortex/rusticide,
 * crates/rusticide-sampling). Each row of an R x V row-major f32 logit matrix
 * is one independent call of the reference's Sampler, with the same result
 * bit for bit given the same uniform draw.
 *
 * Conventions
 *  - Plain C: no exceptions, no C++ or torch types cross this boundary.
 *  - Pointers named d_* are device pointers of the sampler's device; h_* are
 *    host pointers. Logits are borrowed and never written.
 *  - Calls are asynchronous on `stream` (a cudaStream_t passed as void*; NULL
 *    is the legacy default stream) unless documented otherwise. The return
 *    value reports argument and launch errors only; per-row outcomes land in
 *    the caller's d_out_status array (rsc_row_status).
 *  - One rsc_sampler per host thread or stream: a handle owns scratch memory
 *    that concurrent calls would share.
 *  - No call traps, asserts or waits without bound on the device.
 */
#ifndef RUSTICIDE_CUDA_H
#define RUSTICIDE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RSC_ABI_VERSION 2

#if defined(__GNUC__)
#define RSC_API __attribute__((visibility("default")))
#else
#define RSC_API
#endif

/* Call-level status. */
typedef enum {
    RSC_OK = 0,
    RSC_ERR_INVALID_ARGUMENT = 1, /* null pointer where one is required, bad flag */
    RSC_ERR_INVALID_SHAPE = 2,    /* rows/vocab/stride inconsistent (SamplingError::InvalidShape) */
    RSC_ERR_VOCAB_TOO_LARGE = 3,  /* vocab >= 2^31 (SamplingError::VocabOverflow class) */
    RSC_ERR_CAPACITY = 4,         /* rows or vocab above what the handle was created for */
    RSC_ERR_CUDA = 5,             /* a CUDA runtime call or kernel launch failed */
    RSC_ERR_NOT_INITIALIZED = 6,  /* null or destroyed handle */
    RSC_ERR_NO_DEVICE = 7
} rsc_status;

/* Per-row outcome written to d_out_status (int32 per row).
 * The low byte is the result; higher bits are informational flags. */
enum {
    RSC_ROW_OK = 0,               /* d_out_ids[row] holds the token */
    RSC_ROW_NO_VALID_TOKENS = 1,  /* SamplingError::NoValidTokens, src/error.rs:11-12 */
    RSC_ROW_VOCAB_OVERFLOW = 2,   /* SamplingError::VocabOverflow, src/error.rs:13-14 */
    RSC_ROW_INTERNAL = 3,         /* a bounded device wait gave up; row not sampled */
    RSC_ROW_FLAG_DRAW_NEAR_BOUNDARY = 1 << 8, /* |u - CDF edge| < 1e-6 at the chosen token */
    RSC_ROW_FLAG_LARGE_PATH = 1 << 9          /* the row took the large-survivor-set kernel */
};

/* SamplingParams, crates/rusticide-sampling/src/params.rs:5-12. One set per
 * call; repetition_penalty is carried for layout parity and is not applied by
 * rsc_sample (the reference's sample_logits does not apply it either). */
typedef struct {
    float temperature;
    uint32_t top_k;
    float top_p;
    float repetition_penalty;
    uint64_t seed;
} rsc_params;

typedef struct rsc_sampler rsc_sampler;

/* Human-readable name of a call-level status (static storage). */
RSC_API const char *rsc_status_string(rsc_status status);

/* ABI version of the loaded library (RSC_ABI_VERSION at build time). */
RSC_API int rsc_abi_version(void);

/*
 * Creates a sampler on `device` for batches of up to max_rows rows of up to
 * max_vocab logits. Allocates its scratch memory here, once; the sampling
 * calls allocate nothing. The largest parts, in bytes:
 *   - whole-row sort scratch: min(2 x SMs, max_rows) x max_vocab x 16
 *     (about 720 MB at 296 rows of 151936 on a 148-SM B200);
 *   - staging for rsc_pick_host: max_rows x max_vocab x 4.
 * Replaces `Sampler::new(seed)`
 * (crates/rusticide-sampling/src/sampler.rs:17-23) for a batch: per-row
 * generator states are the caller's d_rng_states array (rsc_rng_seed).
 */
RSC_API rsc_status rsc_sampler_create(int device, size_t max_rows, size_t max_vocab,
                              rsc_sampler **out);
RSC_API rsc_status rsc_sampler_destroy(rsc_sampler *sampler);

/*
 * Batched Sampler::sample_logits (src/sampler.rs:44-54): per row, NaN -> -inf,
 * scale by 1/T (T > 0), keep the top_k largest with every tie of the k-th
 * (src/candidates.rs:24-53), then the top_p nucleus (src/candidates.rs:55-78),
 * softmax (src/filters.rs:5-15), then argmax when T == 0 or top_k == 1, else an
 * inverse-CDF draw (src/sampler.rs:111-121).
 *
 * d_logits    rows x vocab f32, row r at d_logits + r * row_stride (row_stride >= vocab).
 * d_uniforms  per-row uniform in [0,1) for the draw (device), or NULL.
 * d_rng_states per-row generator state (device, updated in place) used when
 *             d_uniforms is NULL; a row's state advances only when the row
 *             consumed a draw, as the reference's rng does.
 *             One of d_uniforms / d_rng_states must be non-NULL unless every
 *             row takes the argmax branch (T == 0 or top_k == 1).
 * d_out_ids   uint32 per row; d_out_status int32 per row (rsc_row_status);
 * d_out_probs float per row, nullable: the softmax probability of the chosen
 *             survivor.
 */
RSC_API rsc_status rsc_sample(rsc_sampler *sampler, const float *d_logits, size_t rows,
                      size_t vocab, size_t row_stride, const rsc_params *params,
                      const float *d_uniforms, uint64_t *d_rng_states,
                      uint32_t *d_out_ids, int32_t *d_out_status,
                      float *d_out_probs, void *stream);

/*
 * rsc_sample with one parameter set per row, as a batch of sequences with
 * their own SamplingParams has it: row r is Sampler::sample_logits(row r,
 * h_params[r]) (src/sampler.rs:44-54), with the same outputs and uniforms as
 * rsc_sample. h_params is a HOST array of rows sets, copied to the device
 * before the call returns (the caller may reuse it at once). One launch: a
 * row whose set the streaming top-k filter cannot serve (top-k off over more
 * than 512 logits, top_k > 128, or T = inf) is sampled whole in the same
 * launch, at the large-survivor path's speed. The first call allocates the
 * handle's parameter buffers; a call waits for the previous call's parameter
 * copy to have left the host.
 */
RSC_API rsc_status rsc_sample_rows(rsc_sampler *sampler, const float *d_logits, size_t rows,
                                   size_t vocab, size_t row_stride, const rsc_params *h_params,
                                   const float *d_uniforms, uint64_t *d_rng_states,
                                   uint32_t *d_out_ids, int32_t *d_out_status,
                                   float *d_out_probs, void *stream);

/*
 * Optional outputs of rsc_sample_ex: the candidate set that survived top-k and
 * top-p (the reference's Candidates after Candidates::filter,
 * src/candidates.rs:16-22), per row, in index order.
 * d_n_survivors   uint32 per row, nullable: size of the set.
 * d_survivor_ids  rows x survivor_cap uint32, nullable: the first
 *                 min(n, survivor_cap) token ids of the set.
 * d_survivor_probs rows x survivor_cap f32, nullable: the probabilities of
 *                 the same survivors, the vector the reference's softmax
 *                 returns for the row (src/filters.rs:5-15, as
 *                 src/sampler.rs:50 computes it); entry i belongs to id i.
 *
 * Log-probabilities over the whole vocabulary (ABI 2; no reference
 * counterpart: the reference's softmax normalises over the survivors only).
 * With v the row's scaled logits as the reference's Candidates hold them
 * (x * (1/T) for T > 0, x for T == 0, NaN read as -inf;
 * src/candidates.rs:25-37):
 * d_row_logsumexp  f32 per row, nullable: log(sum_j exp(v_j)) over the row
 *                  (-inf when every v_j is -inf);
 * d_token_logprob  f32 per row, nullable: v_token - logsumexp for the chosen
 *                  token (NaN on a row whose status is not RSC_ROW_OK);
 * d_survivor_logprobs rows x survivor_cap f32, nullable (needs
 *                  d_survivor_ids): v_id - logsumexp for the listed survivors.
 * They are computed with the fast binary32 exp and logf: within about 1e-6
 * relative of the exact value, not bit-exact. On the streaming path the
 * log-sum-exp is accumulated in the same pass over the logits; other rows
 * take one more pass.
 */
typedef struct {
    uint32_t *d_n_survivors;
    uint32_t *d_survivor_ids;
    size_t survivor_cap;
    float *d_survivor_probs;
    float *d_row_logsumexp;
    float *d_token_logprob;
    float *d_survivor_logprobs;
} rsc_sample_extras;

/* rsc_sample with optional extra outputs (extras may be NULL). */
RSC_API rsc_status rsc_sample_ex(rsc_sampler *sampler, const float *d_logits, size_t rows,
                                 size_t vocab, size_t row_stride, const rsc_params *params,
                                 const float *d_uniforms, uint64_t *d_rng_states,
                                 uint32_t *d_out_ids, int32_t *d_out_status,
                                 float *d_out_probs, const rsc_sample_extras *extras,
                                 void *stream);

/*
 * Batched Sampler::greedy_logits (src/sampler.rs:75-88): index of the largest
 * logit with NaN read as -inf, the LAST one on a tie under f32::total_cmp;
 * RSC_ROW_NO_VALID_TOKENS when no logit is finite.
 */
RSC_API rsc_status rsc_greedy(rsc_sampler *sampler, const float *d_logits, size_t rows,
                      size_t vocab, size_t row_stride, uint32_t *d_out_ids,
                      int32_t *d_out_status, void *stream);

/*
 * Batched Sampler::sample_with_temp after extract_logits (src/sampler.rs:97-105,
 * src/logits.rs:9-23): temperature == 0 is greedy; otherwise every logit is
 * multiplied by 1/temperature and the draw runs over the whole row.
 */
RSC_API rsc_status rsc_sample_with_temp(rsc_sampler *sampler, const float *d_logits,
                                size_t rows, size_t vocab, size_t row_stride,
                                float temperature, const float *d_uniforms,
                                uint64_t *d_rng_states, uint32_t *d_out_ids,
                                int32_t *d_out_status, float *d_out_probs,
                                void *stream);

/*
 * rusticide_model::generate::pick (crates/rusticide-model/src/generate.rs:117-124):
 * temperature == 0 routes to rsc_greedy, anything else to rsc_sample.
 */
RSC_API rsc_status rsc_pick(rsc_sampler *sampler, const float *d_logits, size_t rows,
                    size_t vocab, size_t row_stride, const rsc_params *params,
                    const float *d_uniforms, uint64_t *d_rng_states,
                    uint32_t *d_out_ids, int32_t *d_out_status,
                    float *d_out_probs, void *stream);

/*
 * Host-buffer form of rsc_pick for callers whose logits live in host memory,
 * as the reference's Model::forward returns them
 * (crates/rusticide-model/src/model.rs:17): copies h_logits (rows x vocab,
 * dense) and h_uniforms to the device, samples, and copies ids and statuses
 * back. Synchronous: returns after h_out_* are written. Host buffers may be
 * pageable or pinned (pinned is faster). h_uniforms may be NULL when every
 * row takes the argmax branch.
 */
RSC_API rsc_status rsc_pick_host(rsc_sampler *sampler, const float *h_logits,
                         size_t rows, size_t vocab, const rsc_params *params,
                         const float *h_uniforms, uint32_t *h_out_ids,
                         int32_t *h_out_status, float *h_out_probs);

/*
 * Sampler::penalize / apply_repetition_penalty (src/sampler.rs:107-109,
 * src/filters.rs:24-35) on device rows: for each listed token inside the
 * vocabulary, a positive logit is divided by `penalty`, any other multiplied.
 * d_tokens holds n_tokens uint32 ids applied to every row. In place.
 */
RSC_API rsc_status rsc_penalize(rsc_sampler *sampler, float *d_logits, size_t rows,
                        size_t vocab, size_t row_stride,
                        const uint32_t *d_tokens, size_t n_tokens,
                        float penalty, void *stream);

/*
 * Seeds per-row generator states: state[r] = seeds[r] (device arrays), as
 * fastrand::Rng::with_seed(seed) starts (src/sampler.rs:17-23). A row that
 * draws takes fastrand's Rng::f32() from its state: wyrand with the wyhash
 * v4.2 constants, then the low 32 bits' top 23 as a [1,2) mantissa, minus 1.
 * Restated from fastrand 2.5.0's published source, not checked against the
 * crate's own output (no Rust toolchain on this image).
 */
RSC_API rsc_status rsc_rng_seed(const uint64_t *d_seeds, uint64_t *d_rng_states,
                        size_t rows, void *stream);

/*
 * Vocab-sharded sampling, step 1 of 2 (no reference counterpart: the reference
 * samples a whole row on one CPU thread). Each rank holds columns
 * [shard_offset, shard_offset + shard_vocab) of every row. Writes one
 * fixed-size record per row to d_records (rsc_shard_record_bytes(top_k) bytes
 * each): the shard's scaled row maximum and every logit that can survive
 * the global top-k (at most top_k + RSC_SHARD_TIE_CAP of them, with an
 * overflow count). One streaming pass over the shard (rows whose candidates
 * overflow the pass's list take two more passes in the same launch); the caller
 * all-gathers the records of all ranks (NCCL over NVLink) into a
 * [n_shards][rows] array and calls rsc_shard_merge.
 */
#define RSC_SHARD_TIE_CAP 24
RSC_API size_t rsc_shard_record_bytes(uint32_t top_k);
RSC_API rsc_status rsc_shard_partial(rsc_sampler *sampler, const float *d_logits,
                             size_t rows, size_t shard_vocab, size_t row_stride,
                             size_t shard_offset, size_t global_vocab,
                             const rsc_params *params, void *d_records,
                             void *stream);

/*
 * Vocab-sharded sampling, step 2 of 2: merges the gathered records
 * ([n_shards][rows] records, shard-major) into the same per-row result as
 * rsc_sample on the unsharded row. Every rank that calls it with the same
 * gathered records and uniforms computes identical outputs. Rows whose shards
 * overflowed their record report RSC_ROW_INTERNAL and must be resampled
 * unsharded. Up to 256 shards (RSC_ERR_CAPACITY beyond, or when the shards'
 * records of one row exceed 227 KiB of shared memory).
 */
RSC_API rsc_status rsc_shard_merge(rsc_sampler *sampler, const void *d_records,
                           size_t n_shards, size_t rows, size_t global_vocab,
                           const rsc_params *params, const float *d_uniforms,
                           uint64_t *d_rng_states, uint32_t *d_out_ids,
                           int32_t *d_out_status, float *d_out_probs,
                           void *stream);

/*
 * Allocation-free form of rsc_sample. It has no counterpart in the reference,
 * whose sampler runs on the host.
 *
 * It is meant for callers that cannot let a library allocate device memory.
 * One example is a server that reserves almost all of HBM for its KV cache at
 * start-up, so a later cudaMalloc fails. Another is a runtime that owns
 * device memory through its own pool. A third is a plugin that has no place
 * to free a handle. The function takes no rsc_sampler: it samples on the
 * calling thread's current device, with the same results as rsc_sample, and
 * calls no cudaMalloc, cudaFree or other allocating routine.
 *
 * Its sorting scratch is a fixed array of RSC_NOALLOC_SCRATCH_BYTES inside the
 * library's device image. Every GPU that loads the library holds that array
 * until the process exits. vocab above RSC_NOALLOC_MAX_VOCAB returns
 * RSC_ERR_CAPACITY, and vocab 0 with rows > 0 returns RSC_ERR_INVALID_SHAPE. The first call on a device looks the array's address up
 * (cudaGetSymbolAddress). Make that first call before any stream capture;
 * a set-up that failed is retried by the next call.
 * All calls on a device share the array. Calls whose kernels overlap on the
 * GPU (different streams with no ordering between them) race on it, so order
 * them on one stream or with events. Rows are sampled by the large-survivor
 * kernel, at most RSC_NOALLOC_SCRATCH_BYTES / (16 * vocab) rows at a time, so
 * it is slower than rsc_sample on the streaming top-k path.
 */
#define RSC_NOALLOC_SCRATCH_BYTES (64u << 20)
#define RSC_NOALLOC_MAX_VOCAB (RSC_NOALLOC_SCRATCH_BYTES / 16u)
RSC_API rsc_status rsc_sample_noalloc(const float *d_logits, size_t rows, size_t vocab,
                                      size_t row_stride, const rsc_params *params,
                                      const float *d_uniforms, uint64_t *d_rng_states,
                                      uint32_t *d_out_ids, int32_t *d_out_status,
                                      float *d_out_probs, void *stream);

/*
 * LM-head GEMM (no reference counterpart as one call: the reference computes
 * the logits with a host matvec, crates/rusticide-transformer/src/
 * decoder.rs:104-105, then samples them). d_hidden is rows x dim bf16
 * (row-major), d_weight is vocab x dim bf16 (row-major, the nn.Linear
 * layout); logits = hidden . weight^T with bf16 products accumulated in f32
 * on the tensor cores. dim must be a multiple of 8 and both pointers 16-byte
 * aligned.
 *
 * rsc_lmhead_logits writes the rows x vocab f32 logits (dense).
 * rsc_lmhead_sample samples them without writing them: the same GEMM keeps
 * each row's top-k candidates in its epilogue and a merge finishes every row;
 * the result equals rsc_sample on the logits rsc_lmhead_logits returns, bit
 * for bit. It requires top-k on with top_k <= 40 and a finite T > 0 (else
 * RSC_ERR_INVALID_ARGUMENT), and vocab <= 16777216 (else
 * RSC_ERR_VOCAB_TOO_LARGE). The vocabulary is split into parts of at most
 * 65536 columns; a row where, in one part, more than top_k + 24 logits lie at
 * or above the part's k-th value (heavy ties, e.g. a zero hidden state)
 * reports RSC_ROW_INTERNAL and is sampled with rsc_lmhead_logits + rsc_sample
 * instead. The first call allocates the handle's LM-head records.
 */
RSC_API rsc_status rsc_lmhead_logits(rsc_sampler *sampler, const void *d_hidden,
                                     const void *d_weight, size_t rows, size_t dim, size_t vocab,
                                     float *d_logits, void *stream);
RSC_API rsc_status rsc_lmhead_sample(rsc_sampler *sampler, const void *d_hidden,
                                     const void *d_weight, size_t rows, size_t dim, size_t vocab,
                                     const rsc_params *params, const float *d_uniforms,
                                     uint64_t *d_rng_states, uint32_t *d_out_ids,
                                     int32_t *d_out_status, float *d_out_probs, void *stream);

/*
 * rsc_lmhead_sample for a tensor-parallel LM head: this GPU holds the
 * vocabulary rows [shard_offset, shard_offset + shard_vocab) of W
 * (d_weight_shard, shard_vocab x dim bf16) and the whole batch of hidden
 * states. Writes one shard record per row to d_records (rows x
 * rsc_shard_record_bytes(top_k) bytes), with global token ids, in the format
 * of rsc_shard_partial: all-gather the ranks' records in rank order and call
 * rsc_shard_merge with global_vocab, and every rank gets the tokens that
 * rsc_lmhead_sample returns on the whole W. No counterpart in the reference,
 * whose LM head runs on one host (crates/rusticide-transformer/src/
 * decoder.rs:104-105). Parameter limits as rsc_lmhead_sample, with top-k
 * judged against global_vocab.
 */
RSC_API rsc_status rsc_lmhead_partial(rsc_sampler *sampler, const void *d_hidden,
                                      const void *d_weight_shard, size_t rows, size_t dim,
                                      size_t shard_vocab, size_t shard_offset, size_t global_vocab,
                                      const rsc_params *params, void *d_records, void *stream);

/*
 * Evaluates the library's binary32 exp, the function the sampler applies to
 * v - max (Rust's f32::exp, i.e. glibc expf, src/filters.rs:7 and
 * src/candidates.rs:64), on n device floats: d_y[i] = exp(d_x[i]). Exposed so
 * that callers can verify it against their platform's expf. Asynchronous.
 */
RSC_API rsc_status rsc_expf(const float *d_x, float *d_y, size_t n, void *stream);

/*
 * Vocab-sharded sampling over peer memory (no reference counterpart: the
 * reference samples a whole row on one CPU thread). The same result as
 * rsc_shard_partial + an all-gather + rsc_shard_merge, with the all-gather
 * replaced by reads of the other ranks' record arrays in place, over NVLink,
 * and the merge split across the ranks. Every array below lives in memory
 * that every rank can address (for example a symmetric allocation); pointer
 * arrays are device arrays of n_shards entries in rank order. Per step, on
 * every rank:
 *   1. rsc_shard_partial into this rank's record array;
 *   2. rsc_shard_publish(ready_records_ptrs, n_shards, my_shard, step): after
 *      the stream's earlier work, stores `step` into word my_shard of every
 *      rank's records-ready array, after a system-wide fence;
 *   3. rsc_shard_merge_peers: waits until every word of this rank's
 *      records-ready array has reached `step` (wrap-around compare; bounded by
 *      the library's 2 s wait limit, after which rows report
 *      RSC_ROW_INTERNAL), merges rows [rows * my_shard / n_shards, rows *
 *      (my_shard + 1) / n_shards) exactly as rsc_shard_merge, writes their
 *      results into every rank's result arrays, and stores `step` into word
 *      my_shard of every rank's results-ready array;
 *   4. rsc_shard_collect: waits (bounded) until this rank's results-ready
 *      words have reached `step`, then copies this rank's result arrays into
 *      the caller's outputs.
 * With per-row generator states instead of uniforms, every rank merges every
 * row (d_ready_results_ptrs null; results are not shared; step 4 is skipped and
 * the outputs are this rank's result arrays), so that every rank advances
 * every state.
 * `step` increases by one per call; *d_done_counter (a word of this rank) is
 * zero before the first call and is left zero. Two record arrays and two sets
 * of result arrays used alternately (by step parity) keep a slow rank's reads
 * and writes of one step apart from the next. n_shards <= 32 and n_shards *
 * (top_k + RSC_SHARD_TIE_CAP) <= 512, else RSC_ERR_CAPACITY.
 */
typedef struct rsc_peer_exchange {
    const void *const *d_peer_records;       /* n_shards record arrays ([rows] records each) */
    const uint32_t *d_ready_records;         /* this rank's records-ready words (n_shards) */
    uint32_t *const *d_ready_results_ptrs;   /* every rank's results-ready words; null: not shared */
    uint32_t *d_done_counter;                /* one word of this rank */
    uint32_t *const *d_peer_ids;             /* every rank's result ids ([rows]) */
    int32_t *const *d_peer_status;           /* every rank's result statuses */
    float *const *d_peer_probs;              /* every rank's result probabilities, or null */
} rsc_peer_exchange;

RSC_API rsc_status rsc_shard_merge_peers(rsc_sampler *sampler, const rsc_peer_exchange *exchange,
                                         uint32_t step, size_t n_shards, size_t my_shard,
                                         size_t rows, size_t global_vocab,
                                         const rsc_params *params, const float *d_uniforms,
                                         uint64_t *d_rng_states, void *stream);
RSC_API rsc_status rsc_shard_publish(uint32_t *const *d_ready_ptrs, size_t n_shards,
                                     size_t my_shard, uint32_t step, void *stream);
RSC_API rsc_status rsc_shard_collect(const uint32_t *d_ready_results, uint32_t step,
                                     size_t n_shards, size_t rows, const uint32_t *d_ids,
                                     const int32_t *d_status, const float *d_probs,
                                     uint32_t *d_out_ids, int32_t *d_out_status,
                                     float *d_out_probs, void *stream);

/* Number of kernel launches the library issued since the handle was created
 * (for the benchmark's launch count). */
RSC_API uint64_t rsc_launch_count(const rsc_sampler *sampler);

/*
 * Test hook of the bounded device waits (no counterpart in the reference,
 * whose sampler never waits). Marks every scratch slot of the handle taken
 * (hold != 0) or free (hold == 0), ordered on `stream`. While the slots are
 * held, a row that the streaming kernel must finish with the large-row code
 * (a candidate list overflowed by ties) waits for a slot for the library's
 * wait limit (2 s of the GPU's global timer), gives up, and reports
 * RSC_ROW_INTERNAL; every other row is sampled as usual and the device stays
 * usable. Release the slots before sampling such rows again.
 */
RSC_API rsc_status rsc_debug_hold_scratch(rsc_sampler *sampler, int hold, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* RUSTICIDE_CUDA_H */
