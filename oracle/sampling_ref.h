/*
 * CPU oracle for the token-sampling path: a C restatement of the Rust crate
 * rusticide-sampling (platform-cortex/rusticide, crates/rusticide-sampling).
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA sampler
 * is compared against, and the timed CPU baseline of bench.py. No product code
 * path links, loads or calls it.
 *
 * Arithmetic: IEEE-754 binary32 operations in the same order as the Rust code,
 * compiled without fast-math and with -ffp-contract=off, and glibc's expf, which
 * is what Rust's f32::exp calls on x86_64-unknown-linux-gnu.
 *
 * The reference's seeded generator (the fastrand 2.5.0 crate, absent from the
 * reference tree): every draw takes the uniform `u` the caller supplies, and
 * reports whether a draw was consumed. rso_rng_* below restate fastrand's
 * published Rng::gen_u64 (wyrand with the wyhash v4.2 constants) and Rng::f32;
 * the restatement is not checked against the crate's own output, because no
 * Rust toolchain exists on this image.
 */
#ifndef RUSTICIDE_SAMPLING_ORACLE_H
#define RUSTICIDE_SAMPLING_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* crates/rusticide-sampling/src/params.rs:5-12 */
typedef struct {
    float temperature;
    uint32_t top_k;
    float top_p;
    float repetition_penalty;
    uint64_t seed;
} rso_params;

/* crates/rusticide-sampling/src/error.rs:5-15 (Tensor and InvalidShape are
 * raised above this layer, by the tensor entry points) */
enum {
    RSO_OK = 0,
    RSO_NO_VALID_TOKENS = 1,
    RSO_VOCAB_OVERFLOW = 2,
};

/* Result of one call. `consumed_draw` is 1 when the reference would have
 * called rng.f32() (src/sampler.rs:112), which happens only on the
 * multinomial branch after the validity check passed. `prob` is the
 * probability the reference's softmax gave the chosen survivor (NaN when the
 * call failed or took the greedy branch without a softmax). `n_survivors`
 * is the size of the candidate set after top-k and top-p. */
typedef struct {
    int32_t status;
    uint32_t token;
    int32_t consumed_draw;
    uint32_t position;
    float prob;
    uint32_t n_survivors;
    float cdf_lo; /* running sum before the chosen position (draw branch) */
    float cdf_hi; /* running sum after the chosen position (draw branch) */
} rso_result;

/* Sampler::sample_logits, src/sampler.rs:44-54 */
void rso_sample_logits(const float *logits, size_t n, const rso_params *params,
                       float u, rso_result *out);

/* Sampler::greedy_logits, src/sampler.rs:75-88 */
void rso_greedy_logits(const float *logits, size_t n, rso_result *out);

/* Sampler::sample_with_temp after extract_logits, src/sampler.rs:97-105 */
void rso_sample_with_temp(const float *logits, size_t n, float temperature,
                          float u, rso_result *out);

/* rusticide_model::generate::pick, crates/rusticide-model/src/generate.rs:117-124 */
void rso_pick(const float *logits, size_t n, const rso_params *params, float u,
              rso_result *out);

/* Candidates::filter, src/candidates.rs:16-22: writes the surviving indices in
 * index order and their scaled values; returns the survivor count. */
size_t rso_filter(const float *logits, size_t n, const rso_params *params,
                  uint32_t *out_index, float *out_value);

/* Candidates::top_p's cut-off on one row (src/candidates.rs:55-78), for the
 * benchmark's boundary counter: *before and *after get the running sum before
 * and after the element whose cumulative mass first exceeded top_p (both the
 * final sum when none did; NaN when top-p is off). Returns the size of the
 * kept set. */
size_t rso_topp_edge(const float *logits, size_t n, const rso_params *params,
                     float *before, float *after);

/* kth_largest on the scaled row, src/candidates.rs:38-43,93-97; returns -inf
 * when top-k is disabled (k == 0 or k >= n). */
float rso_topk_threshold(const float *logits, size_t n, float temperature,
                         uint32_t k);

/* softmax, src/filters.rs:5-15 (probs written in place of a copy) */
void rso_softmax(const float *values, size_t n, float *probs);

/* argmax, src/filters.rs:37-43: last maximum under f32::total_cmp; returns
 * (size_t)-1 on an empty slice. */
size_t rso_argmax(const float *values, size_t n);

/* apply_repetition_penalty, src/filters.rs:24-35 */
void rso_apply_repetition_penalty(float *logits, size_t n,
                                  const uint32_t *tokens, size_t n_tokens,
                                  float penalty);

/* Batched helpers for tests and the CPU baseline: rows are independent
 * calls, row r reads logits + r * row_stride and uniform u[r]. `threads` <= 1
 * runs on the calling thread. */
void rso_sample_rows(const float *logits, size_t rows, size_t n,
                     size_t row_stride, const rso_params *params,
                     const float *u, rso_result *out, int threads);
void rso_greedy_rows(const float *logits, size_t rows, size_t n,
                     size_t row_stride, rso_result *out, int threads);
void rso_sample_with_temp_rows(const float *logits, size_t rows, size_t n,
                               size_t row_stride, float temperature,
                               const float *u, rso_result *out, int threads);

/* fastrand::Rng::gen_u64 and Rng::f32, restated (see the header comment). */
uint64_t rso_rng_next_u64(uint64_t *state);
float rso_rng_f32(uint64_t *state);

/* glibc expf, exposed so tests can compare the device exp against it. */
void rso_expf_many(const float *x, size_t n, float *y);

#ifdef __cplusplus
}
#endif

#endif
