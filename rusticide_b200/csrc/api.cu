// C ABI of the sampling engine (include/rusticide_cuda.h): argument checks,
// routing between the kernels, and the handle that owns scratch memory.
//
// Routing of rsc_sample (Sampler::sample_logits):
//  - scale finite and > 0, and top-k on or vocab <= kSmallCap: the streaming
//    top-k kernel; a row whose survivors overflow its shared-memory list is
//    sampled whole in the epilogue of the CTA that finished it (same launch);
//  - otherwise every row goes to the large-survivor kernel.
// rsc_sample_rows (one parameter set per row) always takes the streaming
// kernel: each row reads its own set, and a row the filter cannot serve is
// sampled whole in a CTA epilogue.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>

#include "rsc_kernels.h"

struct rsc_sampler {
    int device = -1;
    size_t max_rows = 0;
    size_t max_vocab = 0;
    int num_sms = 0;
    uint32_t large_slots = 0;
    uint32_t *scratch = nullptr;      // [large_slots][4 * max_vocab]
    uint32_t *slot_lock = nullptr;    // [large_slots], zero when a slot is free
    size_t max_units = 0;             // row segments of the streaming kernel
    rsc::StreamPlan plan{};           // schedule of the last streaming call
    size_t plan_rows = 0;
    uint32_t plan_vocab = 0, plan_topk = 0;
    bool plan_valid = false;
    void *seg_records = nullptr;      // [max_units] records of split_record_bytes(splits >= 2)
    void *lm_records = nullptr;       // [kLmheadMaxParts][max_rows] LM-head records (on first use)
    uint32_t *lm_error = nullptr;     // timeout flag of the LM-head kernel
    uint32_t *row_arrivals = nullptr; // [max_rows], zero between calls
    uint2 *lse_parts = nullptr;       // [max_rows][kStreamMaxSplits] log-sum-exp parts (on first use)
    // Device staging of rsc_pick_host.
    float *stage_logits = nullptr;
    float *stage_uniforms = nullptr;
    uint32_t *stage_ids = nullptr;
    int32_t *stage_status = nullptr;
    float *stage_probs = nullptr;
    cudaStream_t host_stream = nullptr;
    // Per-row parameter sets of rsc_sample_rows (on first use): pinned host
    // staging, its device copy, and an event marking the copy's completion.
    rsc_params *rows_host = nullptr;
    rsc_params *rows_dev = nullptr;
    cudaEvent_t rows_copied = nullptr;
    bool rows_pending = false;
    uint64_t launches = 0;
    bool alive = false;
};

namespace {

constexpr size_t kMaxVocab = (size_t{1} << 31) - 1;

rsc_status cuda_status(cudaError_t e) { return e == cudaSuccess ? RSC_OK : RSC_ERR_CUDA; }

// Makes `device` current for the duration of a call and restores the caller's.
class DeviceGuard {
  public:
    explicit DeviceGuard(int device) {
        cudaGetDevice(&prev_);
        if (prev_ != device) cudaSetDevice(device);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (cur != prev_ && prev_ >= 0) cudaSetDevice(prev_);
    }

  private:
    int prev_ = -1;
};

rsc_status check_shape(const rsc_sampler *s, const void *logits, size_t rows, size_t vocab,
                       size_t row_stride) {
    if (!s || !s->alive) return RSC_ERR_NOT_INITIALIZED;
    if (vocab > kMaxVocab) return RSC_ERR_VOCAB_TOO_LARGE;
    if (rows > 0 && vocab > 0 && row_stride < vocab) return RSC_ERR_INVALID_SHAPE;
    if (rows > s->max_rows || vocab > s->max_vocab) return RSC_ERR_CAPACITY;
    if (rows > 0 && vocab > 0 && !logits) return RSC_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(logits) & 3u) != 0) return RSC_ERR_INVALID_ARGUMENT;
    return RSC_OK;
}

rsc::CallParams make_params(const rsc_params &p, size_t vocab, const float *uniforms,
                            uint64_t *rng_states) {
    rsc::CallParams cp;
    cp.temperature = p.temperature;
    // candidates.rs:25-29: 1/T for T > 0, else 1.
    cp.scale = p.temperature > 0.0f ? 1.0f / p.temperature : 1.0f;
    cp.top_k = p.top_k;
    cp.top_p = p.top_p;
    cp.topk_active = p.top_k != 0 && static_cast<size_t>(p.top_k) < vocab;
    cp.topp_active = p.top_p < 1.0f;
    cp.argmax_branch = p.temperature == 0.0f || p.top_k == 1;
    cp.normal_scale = std::isfinite(cp.scale) && cp.scale > 0.0f;
    cp.mode = rsc::kModeSampleLogits;
    cp.uniforms = uniforms;
    cp.rng_states = rng_states;
    cp.out_nsurv = nullptr;
    cp.out_surv = nullptr;
    cp.surv_cap = 0;
    cp.row_params = nullptr;
    return cp;
}

// The per-row arrays of `cp` from row r0 on (a batch of a larger call).
rsc::CallParams rows_from(const rsc::CallParams &cp, size_t r0) {
    rsc::CallParams b = cp;
    if (b.uniforms) b.uniforms += r0;
    if (b.rng_states) b.rng_states += r0;
    if (b.out_nsurv) b.out_nsurv += r0;
    if (b.out_surv) b.out_surv += r0 * b.surv_cap;
    if (b.out_survp) b.out_survp += r0 * b.surv_cap;
    if (b.row_params) b.row_params += r0;
    if (b.lse_parts) b.lse_parts += r0 * b.lse_stride;
    return b;
}

rsc_status stream_impl(rsc_sampler *s, const float *logits, size_t rows, uint32_t v,
                       size_t row_stride, const rsc::CallParams &cp, uint32_t *ids,
                       int32_t *status, float *probs, cudaStream_t stream);

// Whether a call's rows go to the streaming kernel (else the large kernel).
bool streams_rows(const rsc::CallParams &cp, size_t vocab) {
    return cp.mode == rsc::kModeSampleLogits && cp.normal_scale &&
           ((cp.topk_active && cp.top_k <= rsc::kTwoPassTopK) ||
            (!cp.topk_active && vocab <= rsc::kSmallCap));
}

rsc_status sample_impl(rsc_sampler *s, const float *logits, size_t rows, size_t vocab,
                       size_t row_stride, const rsc::CallParams &cp, uint32_t *ids,
                       int32_t *status, float *probs, cudaStream_t stream) {
    if (rows == 0) return RSC_OK;
    const uint32_t v = static_cast<uint32_t>(vocab);
    const bool small = streams_rows(cp, vocab);
    cudaError_t e;
    if (small) return stream_impl(s, logits, rows, v, row_stride, cp, ids, status, probs, stream);
    if (rsc::whole_takes(cp, vocab))
        e = rsc::launch_whole(logits, rows, v, row_stride, cp, ids, status, probs, s->scratch,
                              s->large_slots, s->num_sms, stream);
    else
        e = rsc::launch_large(logits, rows, v, row_stride, cp, ids, status, probs, s->scratch,
                              s->large_slots, stream);
    ++s->launches;
    return cuda_status(e);
}

// The streaming kernel over a call's rows: one launch per batch of at most
// kStreamRowsPerCta rows per CTA (a single launch for every batch that fits
// the GPU this many times).
rsc_status stream_impl(rsc_sampler *s, const float *logits, size_t rows, uint32_t v,
                       size_t row_stride, const rsc::CallParams &cp, uint32_t *ids,
                       int32_t *status, float *probs, cudaStream_t stream) {
    cudaError_t e;
    {
        const size_t batch = static_cast<size_t>(s->num_sms) * 3u * rsc::kStreamRowsPerCta;
        for (size_t r0 = 0; r0 < rows; r0 += batch) {
            const size_t nr = rows - r0 < batch ? rows - r0 : batch;
            if (!s->plan_valid || s->plan_rows != nr || s->plan_vocab != v ||
                s->plan_topk != (cp.topk_active ? cp.top_k : 0u)) {
                // Rows with k above the streaming filter's are not streamed:
                // whole rows, round robin.
                const bool streamed = cp.topk_active && cp.top_k <= rsc::kSmallTopK;
                s->plan = rsc::stream_plan(nr, v, streamed, cp.top_k, s->num_sms,
                                           s->max_units * rsc::split_record_bytes(2));
                s->plan_rows = nr;
                s->plan_vocab = v;
                s->plan_topk = cp.topk_active ? cp.top_k : 0u;
                s->plan_valid = true;
            }
            const rsc::CallParams bp = rows_from(cp, r0);
            e = rsc::launch_stream_topk(logits + r0 * row_stride, nr, v, row_stride, bp, ids + r0,
                                        status + r0, probs ? probs + r0 : nullptr, s->plan,
                                        s->seg_records, s->row_arrivals, s->scratch, s->large_slots,
                                        s->slot_lock, stream);
            ++s->launches;
            if (e != cudaSuccess) return RSC_ERR_CUDA;
        }
        return RSC_OK;
    }
}

rsc_status greedy_impl(rsc_sampler *s, const float *logits, size_t rows, size_t vocab,
                       size_t row_stride, uint32_t *ids, int32_t *status, cudaStream_t stream) {
    // Grid rows are limited to 65535 per launch.
    for (size_t r0 = 0; r0 < rows; r0 += 65535) {
        size_t nr = rows - r0 < 65535 ? rows - r0 : 65535;
        cudaError_t e = rsc::launch_greedy(logits + r0 * row_stride, nr,
                                           static_cast<uint32_t>(vocab), row_stride, ids + r0,
                                           status + r0, s->num_sms, stream);
        ++s->launches;
        if (e != cudaSuccess) return RSC_ERR_CUDA;
    }
    return RSC_OK;
}

}  // namespace

extern "C" {

const char *rsc_status_string(rsc_status status) {
    switch (status) {
        case RSC_OK: return "ok";
        case RSC_ERR_INVALID_ARGUMENT: return "invalid argument";
        case RSC_ERR_INVALID_SHAPE: return "invalid shape";
        case RSC_ERR_VOCAB_TOO_LARGE: return "vocabulary too large";
        case RSC_ERR_CAPACITY: return "batch above the sampler's capacity";
        case RSC_ERR_CUDA: return "CUDA error";
        case RSC_ERR_NOT_INITIALIZED: return "sampler not initialized";
        case RSC_ERR_NO_DEVICE: return "no CUDA device";
    }
    return "unknown status";
}

int rsc_abi_version(void) { return RSC_ABI_VERSION; }

rsc_status rsc_sampler_create(int device, size_t max_rows, size_t max_vocab, rsc_sampler **out) {
    if (!out) return RSC_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    if (max_vocab > kMaxVocab) return RSC_ERR_VOCAB_TOO_LARGE;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return RSC_ERR_NO_DEVICE;
    if (device < 0 || device >= ndev) return RSC_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(device);
    rsc_sampler *s = new (std::nothrow) rsc_sampler();
    if (!s) return RSC_ERR_INVALID_ARGUMENT;
    s->device = device;
    s->max_rows = max_rows < 1 ? 1 : max_rows;
    s->max_vocab = max_vocab < 1 ? 1 : max_vocab;
    cudaError_t e = cudaDeviceGetAttribute(&s->num_sms, cudaDevAttrMultiProcessorCount, device);
    // kLargeCtasPerSm large-survivor CTAs per SM, at most one per row.
    size_t slots = static_cast<size_t>(s->num_sms) * rsc::kLargeCtasPerSm;
    if (slots > s->max_rows) slots = s->max_rows;
    s->large_slots = static_cast<uint32_t>(slots);
    if (e == cudaSuccess) e = cudaMalloc(&s->slot_lock, s->large_slots * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(s->slot_lock, 0, s->large_slots * sizeof(uint32_t));
    if (e == cudaSuccess)
        e = cudaMalloc(&s->scratch, static_cast<size_t>(s->large_slots) * 4u * s->max_vocab *
                                        sizeof(uint32_t));
    // Segment records: up to 4 segments per row, and up to kStreamMaxSplits
    // per row for batches smaller than the GPU.
    s->max_units = 4 * s->max_rows + rsc::kStreamMaxSplits * static_cast<size_t>(s->num_sms) * 4;
    if (e == cudaSuccess)
        e = cudaMalloc(&s->seg_records, s->max_units * rsc::split_record_bytes(2));
    if (e == cudaSuccess) e = cudaMalloc(&s->row_arrivals, s->max_rows * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(s->row_arrivals, 0, s->max_rows * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMalloc(&s->stage_logits, s->max_rows * s->max_vocab * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&s->stage_uniforms, s->max_rows * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&s->stage_ids, s->max_rows * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMalloc(&s->stage_status, s->max_rows * sizeof(int32_t));
    if (e == cudaSuccess) e = cudaMalloc(&s->stage_probs, s->max_rows * sizeof(float));
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s->host_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        s->alive = true;
        rsc_sampler_destroy(s);
        return RSC_ERR_CUDA;
    }
    s->alive = true;
    *out = s;
    return RSC_OK;
}

rsc_status rsc_sampler_destroy(rsc_sampler *s) {
    if (!s || !s->alive) return RSC_ERR_NOT_INITIALIZED;
    DeviceGuard guard(s->device);
    cudaFree(s->slot_lock);
    cudaFree(s->scratch);
    cudaFree(s->seg_records);
    cudaFree(s->lm_records);
    cudaFree(s->lm_error);
    cudaFree(s->row_arrivals);
    cudaFree(s->lse_parts);
    cudaFree(s->stage_logits);
    cudaFree(s->stage_uniforms);
    cudaFree(s->stage_ids);
    cudaFree(s->stage_status);
    cudaFree(s->stage_probs);
    if (s->host_stream) cudaStreamDestroy(s->host_stream);
    if (s->rows_copied) {
        cudaEventSynchronize(s->rows_copied);
        cudaEventDestroy(s->rows_copied);
    }
    cudaFreeHost(s->rows_host);
    cudaFree(s->rows_dev);
    s->alive = false;
    delete s;
    return RSC_OK;
}

rsc_status rsc_sample_ex(rsc_sampler *s, const float *d_logits, size_t rows, size_t vocab,
                         size_t row_stride, const rsc_params *params, const float *d_uniforms,
                         uint64_t *d_rng_states, uint32_t *d_out_ids, int32_t *d_out_status,
                         float *d_out_probs, const rsc_sample_extras *extras, void *stream) {
    rsc_status st = check_shape(s, d_logits, rows, vocab, row_stride);
    if (st != RSC_OK) return st;
    if (!params || (rows > 0 && (!d_out_ids || !d_out_status))) return RSC_ERR_INVALID_ARGUMENT;
    rsc::CallParams cp = make_params(*params, vocab, d_uniforms, d_rng_states);
    if (!cp.argmax_branch && rows > 0 && !d_uniforms && !d_rng_states) return RSC_ERR_INVALID_ARGUMENT;
    const bool want_lp = extras && (extras->d_row_logsumexp || extras->d_token_logprob ||
                                    extras->d_survivor_logprobs);
    if (extras) {
        if ((extras->d_survivor_ids || extras->d_survivor_probs || extras->d_survivor_logprobs) &&
            (extras->survivor_cap == 0 || extras->survivor_cap > 0xffffffffull))
            return RSC_ERR_INVALID_ARGUMENT;
        if (extras->d_survivor_logprobs && !extras->d_survivor_ids) return RSC_ERR_INVALID_ARGUMENT;
        cp.out_nsurv = extras->d_n_survivors;
        cp.out_surv = extras->d_survivor_ids;
        cp.out_survp = extras->d_survivor_probs;
        cp.surv_cap = static_cast<uint32_t>(extras->survivor_cap);
    }
    DeviceGuard guard(s->device);
    cudaStream_t strm = static_cast<cudaStream_t>(stream);
    if (!want_lp || rows == 0)
        return sample_impl(s, d_logits, rows, vocab, row_stride, cp, d_out_ids, d_out_status,
                           d_out_probs, strm);
    // Log-probabilities: each row's log-sum-exp parts, from the streaming
    // kernel's consumers when it streams the rows, else from one more pass.
    if (!s->lse_parts &&
        cudaMalloc(&s->lse_parts, s->max_rows * rsc::kStreamMaxSplits * sizeof(uint2)) != cudaSuccess)
        return RSC_ERR_CUDA;
    cudaError_t e = cudaMemsetAsync(s->lse_parts, 0, rows * rsc::kStreamMaxSplits * sizeof(uint2), strm);
    if (e != cudaSuccess) return RSC_ERR_CUDA;
    const bool fused = streams_rows(cp, vocab) && !(cp.topk_active && cp.top_k > rsc::kSmallTopK);
    if (!fused) {
        e = rsc::launch_lse_rows(d_logits, rows, static_cast<uint32_t>(vocab), row_stride, cp.scale,
                                 s->lse_parts, rsc::kStreamMaxSplits, strm);
        ++s->launches;
        if (e != cudaSuccess) return RSC_ERR_CUDA;
    } else {
        cp.lse_parts = s->lse_parts;
        cp.lse_stride = rsc::kStreamMaxSplits;
    }
    st = sample_impl(s, d_logits, rows, vocab, row_stride, cp, d_out_ids, d_out_status, d_out_probs,
                     strm);
    if (st != RSC_OK) return st;
    e = rsc::launch_lse_finish(d_logits, rows, row_stride, cp.scale, s->lse_parts,
                               rsc::kStreamMaxSplits, d_out_ids, d_out_status, extras->d_n_survivors,
                               extras->d_survivor_ids, static_cast<uint32_t>(extras->survivor_cap),
                               extras->d_row_logsumexp, extras->d_token_logprob,
                               extras->d_survivor_logprobs, strm);
    ++s->launches;
    return cuda_status(e);
}

rsc_status rsc_sample_rows(rsc_sampler *s, const float *d_logits, size_t rows, size_t vocab,
                           size_t row_stride, const rsc_params *h_params, const float *d_uniforms,
                           uint64_t *d_rng_states, uint32_t *d_out_ids, int32_t *d_out_status,
                           float *d_out_probs, void *stream) {
    rsc_status st = check_shape(s, d_logits, rows, vocab, row_stride);
    if (st != RSC_OK) return st;
    if (rows == 0) return RSC_OK;
    if (!h_params || !d_out_ids || !d_out_status) return RSC_ERR_INVALID_ARGUMENT;
    if (vocab == 0) return RSC_ERR_INVALID_SHAPE;
    // The call-wide schedule is planned for the largest top-k among the rows
    // the streaming filter serves; every other row is sampled whole.
    uint32_t max_k = 0;
    bool draws = false;
    for (size_t r = 0; r < rows; ++r) {
        const rsc::CallParams q = make_params(h_params[r], vocab, nullptr, nullptr);
        if (!q.argmax_branch) draws = true;
        if (q.normal_scale && q.topk_active && q.top_k <= rsc::kSmallTopK && q.top_k > max_k)
            max_k = q.top_k;
    }
    if (draws && !d_uniforms && !d_rng_states) return RSC_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(s->device);
    cudaStream_t strm = static_cast<cudaStream_t>(stream);
    if (!s->rows_host) {
        if (cudaHostAlloc(reinterpret_cast<void **>(&s->rows_host), s->max_rows * sizeof(rsc_params),
                          cudaHostAllocDefault) != cudaSuccess)
            return RSC_ERR_CUDA;
        if (cudaMalloc(&s->rows_dev, s->max_rows * sizeof(rsc_params)) != cudaSuccess)
            return RSC_ERR_CUDA;
        if (cudaEventCreateWithFlags(&s->rows_copied, cudaEventDisableTiming) != cudaSuccess)
            return RSC_ERR_CUDA;
    }
    // The staging buffer is rewritten only once the previous call's copy
    // has read it.
    if (s->rows_pending && cudaEventSynchronize(s->rows_copied) != cudaSuccess) return RSC_ERR_CUDA;
    std::memcpy(s->rows_host, h_params, rows * sizeof(rsc_params));
    if (cudaMemcpyAsync(s->rows_dev, s->rows_host, rows * sizeof(rsc_params),
                        cudaMemcpyHostToDevice, strm) != cudaSuccess ||
        cudaEventRecord(s->rows_copied, strm) != cudaSuccess)
        return RSC_ERR_CUDA;
    s->rows_pending = true;
    rsc_params plan_params{1.0f, max_k, 1.0f, 1.0f, 0};
    rsc::CallParams cp = make_params(plan_params, vocab, d_uniforms, d_rng_states);
    cp.row_params = s->rows_dev;
    return stream_impl(s, d_logits, rows, static_cast<uint32_t>(vocab), row_stride, cp, d_out_ids,
                       d_out_status, d_out_probs, strm);
}

rsc_status rsc_sample(rsc_sampler *s, const float *d_logits, size_t rows, size_t vocab,
                      size_t row_stride, const rsc_params *params, const float *d_uniforms,
                      uint64_t *d_rng_states, uint32_t *d_out_ids, int32_t *d_out_status,
                      float *d_out_probs, void *stream) {
    return rsc_sample_ex(s, d_logits, rows, vocab, row_stride, params, d_uniforms, d_rng_states,
                         d_out_ids, d_out_status, d_out_probs, nullptr, stream);
}

rsc_status rsc_greedy(rsc_sampler *s, const float *d_logits, size_t rows, size_t vocab,
                      size_t row_stride, uint32_t *d_out_ids, int32_t *d_out_status,
                      void *stream) {
    rsc_status st = check_shape(s, d_logits, rows, vocab, row_stride);
    if (st != RSC_OK) return st;
    if (rows > 0 && (!d_out_ids || !d_out_status)) return RSC_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(s->device);
    return greedy_impl(s, d_logits, rows, vocab, row_stride, d_out_ids, d_out_status,
                       static_cast<cudaStream_t>(stream));
}

rsc_status rsc_sample_with_temp(rsc_sampler *s, const float *d_logits, size_t rows, size_t vocab,
                                size_t row_stride, float temperature, const float *d_uniforms,
                                uint64_t *d_rng_states, uint32_t *d_out_ids,
                                int32_t *d_out_status, float *d_out_probs, void *stream) {
    rsc_status st = check_shape(s, d_logits, rows, vocab, row_stride);
    if (st != RSC_OK) return st;
    if (rows > 0 && (!d_out_ids || !d_out_status)) return RSC_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(s->device);
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    if (temperature == 0.0f)  // sampler.rs:98-100
        return greedy_impl(s, d_logits, rows, vocab, row_stride, d_out_ids, d_out_status, cs);
    if (rows > 0 && !d_uniforms && !d_rng_states) return RSC_ERR_INVALID_ARGUMENT;
    rsc_params p{temperature, 0u, 1.0f, 1.0f, 0u};
    rsc::CallParams cp = make_params(p, vocab, d_uniforms, d_rng_states);
    cp.mode = rsc::kModeSampleWithTemp;
    cp.scale = 1.0f / temperature;  // apply_temperature, filters.rs:17-22
    cp.topk_active = false;
    cp.topp_active = false;
    cp.argmax_branch = false;
    return sample_impl(s, d_logits, rows, vocab, row_stride, cp, d_out_ids, d_out_status,
                       d_out_probs, cs);
}

rsc_status rsc_pick(rsc_sampler *s, const float *d_logits, size_t rows, size_t vocab,
                    size_t row_stride, const rsc_params *params, const float *d_uniforms,
                    uint64_t *d_rng_states, uint32_t *d_out_ids, int32_t *d_out_status,
                    float *d_out_probs, void *stream) {
    if (!params) return RSC_ERR_INVALID_ARGUMENT;
    if (params->temperature == 0.0f) {
        rsc_status st = rsc_greedy(s, d_logits, rows, vocab, row_stride, d_out_ids, d_out_status, stream);
        if (st == RSC_OK && d_out_probs && rows > 0) {
            // greedy_logits computes no probability.
            DeviceGuard guard(s->device);
            cudaError_t e = cudaMemsetAsync(d_out_probs, 0xff, rows * sizeof(float),
                                            static_cast<cudaStream_t>(stream));
            if (e != cudaSuccess) return RSC_ERR_CUDA;
        }
        return st;
    }
    return rsc_sample(s, d_logits, rows, vocab, row_stride, params, d_uniforms, d_rng_states,
                      d_out_ids, d_out_status, d_out_probs, stream);
}

rsc_status rsc_pick_host(rsc_sampler *s, const float *h_logits, size_t rows, size_t vocab,
                         const rsc_params *params, const float *h_uniforms, uint32_t *h_out_ids,
                         int32_t *h_out_status, float *h_out_probs) {
    rsc_status st = check_shape(s, h_logits, rows, vocab, vocab);
    if (st != RSC_OK) return st;
    if (!params || (rows > 0 && (!h_out_ids || !h_out_status))) return RSC_ERR_INVALID_ARGUMENT;
    if (rows == 0) return RSC_OK;
    const bool argmax = params->temperature == 0.0f || params->top_k == 1;
    if (!argmax && !h_uniforms) return RSC_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(s->device);
    cudaStream_t cs = s->host_stream;
    cudaError_t e = cudaMemcpyAsync(s->stage_logits, h_logits, rows * vocab * sizeof(float),
                                    cudaMemcpyHostToDevice, cs);
    if (e == cudaSuccess && h_uniforms)
        e = cudaMemcpyAsync(s->stage_uniforms, h_uniforms, rows * sizeof(float),
                            cudaMemcpyHostToDevice, cs);
    if (e != cudaSuccess) return RSC_ERR_CUDA;
    st = rsc_pick(s, s->stage_logits, rows, vocab, vocab, params,
                  h_uniforms ? s->stage_uniforms : nullptr, nullptr, s->stage_ids,
                  s->stage_status, h_out_probs ? s->stage_probs : nullptr, cs);
    if (st != RSC_OK) return st;
    e = cudaMemcpyAsync(h_out_ids, s->stage_ids, rows * sizeof(uint32_t), cudaMemcpyDeviceToHost, cs);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(h_out_status, s->stage_status, rows * sizeof(int32_t),
                            cudaMemcpyDeviceToHost, cs);
    if (e == cudaSuccess && h_out_probs)
        e = cudaMemcpyAsync(h_out_probs, s->stage_probs, rows * sizeof(float),
                            cudaMemcpyDeviceToHost, cs);
    if (e == cudaSuccess) e = cudaStreamSynchronize(cs);
    return cuda_status(e);
}

rsc_status rsc_penalize(rsc_sampler *s, float *d_logits, size_t rows, size_t vocab,
                        size_t row_stride, const uint32_t *d_tokens, size_t n_tokens,
                        float penalty, void *stream) {
    rsc_status st = check_shape(s, d_logits, rows, vocab, row_stride);
    if (st != RSC_OK) return st;
    if (n_tokens > 0 && !d_tokens) return RSC_ERR_INVALID_ARGUMENT;
    if (rows == 0 || n_tokens == 0) return RSC_OK;
    DeviceGuard guard(s->device);
    cudaError_t e = rsc::launch_penalize(d_logits, rows, static_cast<uint32_t>(vocab), row_stride,
                                         d_tokens, n_tokens, penalty,
                                         static_cast<cudaStream_t>(stream));
    ++s->launches;
    return cuda_status(e);
}

rsc_status rsc_rng_seed(const uint64_t *d_seeds, uint64_t *d_rng_states, size_t rows, void *stream) {
    if (rows == 0) return RSC_OK;
    if (!d_seeds || !d_rng_states) return RSC_ERR_INVALID_ARGUMENT;
    return cuda_status(rsc::launch_rng_seed(d_seeds, d_rng_states, rows,
                                            static_cast<cudaStream_t>(stream)));
}

size_t rsc_shard_record_bytes(uint32_t top_k) { return rsc::shard_record_bytes(top_k); }

rsc_status rsc_shard_partial(rsc_sampler *s, const float *d_logits, size_t rows,
                             size_t shard_vocab, size_t row_stride, size_t shard_offset,
                             size_t global_vocab, const rsc_params *params, void *d_records,
                             void *stream) {
    rsc_status st = check_shape(s, d_logits, rows, shard_vocab, row_stride);
    if (st != RSC_OK) return st;
    if (!params || (rows > 0 && !d_records)) return RSC_ERR_INVALID_ARGUMENT;
    if (global_vocab > kMaxVocab) return RSC_ERR_VOCAB_TOO_LARGE;
    if (shard_offset + shard_vocab > global_vocab) return RSC_ERR_INVALID_SHAPE;
    rsc::CallParams cp = make_params(*params, global_vocab, nullptr, nullptr);
    // Only a row whose top-k is on can be reduced to a small record, and the
    // streaming kernel needs a scale that creates no NaN.
    if (!cp.topk_active || !cp.normal_scale || params->top_k > rsc::kSmallTopK)
        return RSC_ERR_INVALID_ARGUMENT;
    if (rows == 0) return RSC_OK;
    DeviceGuard guard(s->device);
    cudaError_t e = rsc::launch_shard_partial(
        d_logits, rows, static_cast<uint32_t>(shard_vocab), row_stride,
        static_cast<uint32_t>(shard_offset), cp, d_records, rsc::shard_record_bytes(params->top_k),
        s->num_sms, static_cast<cudaStream_t>(stream));
    ++s->launches;
    return cuda_status(e);
}

rsc_status rsc_shard_merge(rsc_sampler *s, const void *d_records, size_t n_shards, size_t rows,
                           size_t global_vocab, const rsc_params *params, const float *d_uniforms,
                           uint64_t *d_rng_states, uint32_t *d_out_ids, int32_t *d_out_status,
                           float *d_out_probs, void *stream) {
    if (!s || !s->alive) return RSC_ERR_NOT_INITIALIZED;
    if (!params || n_shards == 0) return RSC_ERR_INVALID_ARGUMENT;
    if (global_vocab > kMaxVocab) return RSC_ERR_VOCAB_TOO_LARGE;
    if (rows > s->max_rows) return RSC_ERR_CAPACITY;
    if (rows > 0 && (!d_records || !d_out_ids || !d_out_status)) return RSC_ERR_INVALID_ARGUMENT;
    rsc::CallParams cp = make_params(*params, global_vocab, d_uniforms, d_rng_states);
    if (!cp.topk_active || !cp.normal_scale) return RSC_ERR_INVALID_ARGUMENT;
    // One warp merges a row when the shards' records fit its candidate list;
    // more shards (or a larger k) take one block per row, up to
    // kLmheadMaxParts records whose union fits its shared memory.
    const size_t cap = static_cast<size_t>(params->top_k) + RSC_SHARD_TIE_CAP;
    const bool warp_merge = n_shards * cap <= rsc::kSmallCap;
    if (!warp_merge && (n_shards > rsc::kLmheadMaxParts ||
                        rsc::shard_merge_block_smem(static_cast<uint32_t>(n_shards),
                                                    static_cast<uint32_t>(cap)) > 232448))
        return RSC_ERR_CAPACITY;
    if (!cp.argmax_branch && rows > 0 && !d_uniforms && !d_rng_states) return RSC_ERR_INVALID_ARGUMENT;
    if (rows == 0) return RSC_OK;
    DeviceGuard guard(s->device);
    const size_t rec_bytes = rsc::shard_record_bytes(params->top_k);
    cudaStream_t strm = static_cast<cudaStream_t>(stream);
    cudaError_t e = warp_merge
                        ? rsc::launch_shard_merge(d_records, n_shards, rows, rec_bytes, cp, d_out_ids,
                                                  d_out_status, d_out_probs, s->num_sms, strm)
                        : rsc::launch_shard_merge_block(d_records, n_shards, rows, rec_bytes, cp,
                                                        d_out_ids, d_out_status, d_out_probs, strm);
    ++s->launches;
    return cuda_status(e);
}

namespace {

rsc_status check_lmhead(const rsc_sampler *s, const void *d_hidden, const void *d_weight,
                        size_t rows, size_t dim, size_t vocab) {
    if (!s || !s->alive) return RSC_ERR_NOT_INITIALIZED;
    if (vocab > kMaxVocab || vocab > rsc::kLmheadMaxVocab) return RSC_ERR_VOCAB_TOO_LARGE;
    if (rows > s->max_rows) return RSC_ERR_CAPACITY;
    if (rows > 0 && (vocab == 0 || dim == 0 || dim % 8 != 0)) return RSC_ERR_INVALID_SHAPE;
    if (dim > (size_t{1} << 30)) return RSC_ERR_INVALID_SHAPE;
    if (rows > 0 && (!d_hidden || !d_weight)) return RSC_ERR_INVALID_ARGUMENT;
    if (((reinterpret_cast<uintptr_t>(d_hidden) | reinterpret_cast<uintptr_t>(d_weight)) & 15u) != 0)
        return RSC_ERR_INVALID_ARGUMENT;
    return RSC_OK;
}

// The LM-head records and the timeout flag, allocated on the first LM-head
// call of the handle.
rsc_status ensure_lm_records(rsc_sampler *s) {
    if (s->lm_records) return RSC_OK;
    // One record per vocabulary part and row.
    const size_t bytes = static_cast<size_t>(rsc::kLmheadRecordSlots) * s->max_rows *
                         rsc::shard_record_bytes(rsc::kLmheadRowCap - RSC_SHARD_TIE_CAP);
    if (cudaMalloc(&s->lm_records, bytes) != cudaSuccess) return RSC_ERR_CUDA;
    if (cudaMalloc(&s->lm_error, sizeof(uint32_t)) != cudaSuccess) return RSC_ERR_CUDA;
    if (cudaMemset(s->lm_error, 0, sizeof(uint32_t)) != cudaSuccess) return RSC_ERR_CUDA;
    return RSC_OK;
}

}  // namespace

rsc_status rsc_lmhead_logits(rsc_sampler *s, const void *d_hidden, const void *d_weight,
                             size_t rows, size_t dim, size_t vocab, float *d_logits, void *stream) {
    rsc_status st = check_lmhead(s, d_hidden, d_weight, rows, dim, vocab);
    if (st != RSC_OK) return st;
    if (rows == 0) return RSC_OK;
    if (!d_logits) return RSC_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(s->device);
    st = ensure_lm_records(s);
    if (st != RSC_OK) return st;
    const uint32_t v = static_cast<uint32_t>(vocab);
    rsc_params prm{1.0f, 0, 1.0f, 1.0f, 0};
    const rsc::CallParams cp = make_params(prm, vocab, nullptr, nullptr);
    const uint32_t parts = rsc::lmhead_parts(rows, v, s->num_sms);
    cudaError_t e = rsc::launch_lmhead(d_hidden, d_weight, rows, static_cast<uint32_t>(dim), v, cp,
                                       d_logits, nullptr, 0, parts, s->lm_error,
                                       static_cast<cudaStream_t>(stream));
    ++s->launches;
    return cuda_status(e);
}

rsc_status rsc_lmhead_sample(rsc_sampler *s, const void *d_hidden, const void *d_weight,
                             size_t rows, size_t dim, size_t vocab, const rsc_params *params,
                             const float *d_uniforms, uint64_t *d_rng_states, uint32_t *d_out_ids,
                             int32_t *d_out_status, float *d_out_probs, void *stream) {
    rsc_status st = check_lmhead(s, d_hidden, d_weight, rows, dim, vocab);
    if (st != RSC_OK) return st;
    if (!params) return RSC_ERR_INVALID_ARGUMENT;
    if (rows == 0) return RSC_OK;
    if (!d_out_ids || !d_out_status) return RSC_ERR_INVALID_ARGUMENT;
    const rsc::CallParams cp = make_params(*params, vocab, d_uniforms, d_rng_states);
    if (!cp.topk_active || !cp.normal_scale ||
        params->top_k + RSC_SHARD_TIE_CAP > rsc::kLmheadRowCap)
        return RSC_ERR_INVALID_ARGUMENT;
    if (!cp.argmax_branch && !d_uniforms && !d_rng_states) return RSC_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(s->device);
    st = ensure_lm_records(s);
    if (st != RSC_OK) return st;
    const uint32_t v = static_cast<uint32_t>(vocab);
    const uint32_t parts = rsc::lmhead_parts(rows, v, s->num_sms);
    const size_t rec_bytes = rsc::shard_record_bytes(params->top_k);
    cudaStream_t strm = static_cast<cudaStream_t>(stream);
    cudaError_t e = rsc::launch_lmhead(d_hidden, d_weight, rows, static_cast<uint32_t>(dim), v, cp,
                                       nullptr, s->lm_records, rec_bytes, parts, s->lm_error, strm);
    ++s->launches;
    if (e != cudaSuccess) return RSC_ERR_CUDA;
    // One block per row merges all parts' records (at most 256 parts of at
    // most 64 entries).
    e = rsc::launch_shard_merge_block(s->lm_records, parts, rows, rec_bytes, cp, d_out_ids,
                                      d_out_status, d_out_probs, strm);
    ++s->launches;
    return cuda_status(e);
}

rsc_status rsc_lmhead_partial(rsc_sampler *s, const void *d_hidden, const void *d_weight_shard,
                              size_t rows, size_t dim, size_t shard_vocab, size_t shard_offset,
                              size_t global_vocab, const rsc_params *params, void *d_records,
                              void *stream) {
    rsc_status st = check_lmhead(s, d_hidden, d_weight_shard, rows, dim, shard_vocab);
    if (st != RSC_OK) return st;
    if (!params) return RSC_ERR_INVALID_ARGUMENT;
    if (global_vocab > kMaxVocab) return RSC_ERR_VOCAB_TOO_LARGE;
    if (shard_offset > global_vocab || shard_vocab > global_vocab - shard_offset)
        return RSC_ERR_INVALID_SHAPE;
    if (rows == 0) return RSC_OK;
    if (!d_records) return RSC_ERR_INVALID_ARGUMENT;
    // The global vocabulary decides whether top-k is on, as for the whole row.
    const rsc::CallParams cp = make_params(*params, global_vocab, nullptr, nullptr);
    if (!cp.topk_active || !cp.normal_scale ||
        params->top_k + RSC_SHARD_TIE_CAP > rsc::kLmheadRowCap)
        return RSC_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(s->device);
    st = ensure_lm_records(s);
    if (st != RSC_OK) return st;
    const uint32_t v = static_cast<uint32_t>(shard_vocab);
    const uint32_t parts = rsc::lmhead_parts(rows, v, s->num_sms);
    const size_t rec_bytes = rsc::shard_record_bytes(params->top_k);
    cudaStream_t strm = static_cast<cudaStream_t>(stream);
    cudaError_t e = rsc::launch_lmhead(d_hidden, d_weight_shard, rows, static_cast<uint32_t>(dim), v,
                                       cp, nullptr, s->lm_records, rec_bytes, parts, s->lm_error,
                                       strm, static_cast<uint32_t>(shard_offset));
    ++s->launches;
    if (e != cudaSuccess) return RSC_ERR_CUDA;
    // The shard's parts reduced to one record per row.
    e = rsc::launch_shard_reduce_block(s->lm_records, parts, rows, rec_bytes, cp, d_records, strm);
    ++s->launches;
    return cuda_status(e);
}

rsc_status rsc_expf(const float *d_x, float *d_y, size_t n, void *stream) {
    if (n == 0) return RSC_OK;
    if (!d_x || !d_y) return RSC_ERR_INVALID_ARGUMENT;
    return cuda_status(rsc::launch_expf(d_x, d_y, n, static_cast<cudaStream_t>(stream)));
}

rsc_status rsc_shard_merge_peers(rsc_sampler *s, const rsc_peer_exchange *x, uint32_t step,
                                 size_t n_shards, size_t my_shard, size_t rows,
                                 size_t global_vocab, const rsc_params *params,
                                 const float *d_uniforms, uint64_t *d_rng_states, void *stream) {
    if (!s || !s->alive) return RSC_ERR_NOT_INITIALIZED;
    if (!params || !x || n_shards == 0 || my_shard >= n_shards) return RSC_ERR_INVALID_ARGUMENT;
    if (global_vocab > kMaxVocab) return RSC_ERR_VOCAB_TOO_LARGE;
    if (rows > s->max_rows) return RSC_ERR_CAPACITY;
    if (rows > 0 && (!x->d_peer_records || !x->d_ready_records || !x->d_peer_ids ||
                     !x->d_peer_status || (x->d_ready_results_ptrs && !x->d_done_counter)))
        return RSC_ERR_INVALID_ARGUMENT;
    rsc::CallParams cp = make_params(*params, global_vocab, d_uniforms, d_rng_states);
    if (!cp.topk_active || !cp.normal_scale) return RSC_ERR_INVALID_ARGUMENT;
    // One warp merges a row: the ranks' records must fit its candidate list.
    const size_t cap = static_cast<size_t>(params->top_k) + RSC_SHARD_TIE_CAP;
    if (n_shards > 32 || n_shards * cap > rsc::kSmallCap) return RSC_ERR_CAPACITY;
    if (!cp.argmax_branch && rows > 0 && !d_uniforms && !d_rng_states) return RSC_ERR_INVALID_ARGUMENT;
    // Generator states advance on the rank that draws: every rank merges every row.
    const bool share = x->d_ready_results_ptrs != nullptr;
    if (share && d_rng_states) return RSC_ERR_INVALID_ARGUMENT;
    if (rows == 0) return RSC_OK;
    DeviceGuard guard(s->device);
    const size_t r0 = share ? rows * my_shard / n_shards : 0;
    const size_t r1 = share ? rows * (my_shard + 1) / n_shards : rows;
    rsc::PeerPointers pp{x->d_peer_records, x->d_ready_records, x->d_ready_results_ptrs,
                         x->d_done_counter, x->d_peer_ids, x->d_peer_status, x->d_peer_probs};
    cudaError_t e = rsc::launch_shard_merge_peers(pp, step, n_shards, my_shard, r0, r1,
                                                  rsc::shard_record_bytes(params->top_k), cp,
                                                  static_cast<cudaStream_t>(stream));
    ++s->launches;
    return cuda_status(e);
}

rsc_status rsc_shard_collect(const uint32_t *d_ready_results, uint32_t step, size_t n_shards,
                             size_t rows, const uint32_t *d_ids, const int32_t *d_status,
                             const float *d_probs, uint32_t *d_out_ids, int32_t *d_out_status,
                             float *d_out_probs, void *stream) {
    if (n_shards == 0 || n_shards > 32) return RSC_ERR_INVALID_ARGUMENT;
    if (rows > 0 && (!d_ready_results || !d_ids || !d_status || !d_out_ids || !d_out_status))
        return RSC_ERR_INVALID_ARGUMENT;
    return cuda_status(rsc::launch_shard_collect(d_ready_results, step, n_shards, rows, d_ids,
                                                 d_status, d_probs, d_out_ids, d_out_status,
                                                 d_out_probs, static_cast<cudaStream_t>(stream)));
}

rsc_status rsc_shard_publish(uint32_t *const *d_ready_ptrs, size_t n_shards, size_t my_shard,
                             uint32_t step, void *stream) {
    if (!d_ready_ptrs || n_shards == 0 || n_shards > 1024 || my_shard >= n_shards)
        return RSC_ERR_INVALID_ARGUMENT;
    return cuda_status(rsc::launch_shard_publish(d_ready_ptrs, n_shards,
                                                 static_cast<uint32_t>(my_shard), step,
                                                 static_cast<cudaStream_t>(stream)));
}

uint64_t rsc_launch_count(const rsc_sampler *s) { return s && s->alive ? s->launches : 0; }

rsc_status rsc_debug_hold_scratch(rsc_sampler *s, int hold, void *stream) {
    if (!s || !s->alive) return RSC_ERR_NOT_INITIALIZED;
    DeviceGuard guard(s->device);
    return cuda_status(cudaMemsetAsync(s->slot_lock, hold ? 0xff : 0,
                                       s->large_slots * sizeof(uint32_t),
                                       static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
