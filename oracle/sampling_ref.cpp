// CPU oracle for the token-sampling path: a restatement of
// crates/rusticide-sampling (platform-cortex/rusticide) in C++17.
//
// TEST INFRASTRUCTURE ONLY: the checker for the CUDA sampler and the timed CPU
// baseline. No product path links or calls it.
//
// Build (see oracle/build.py): g++ -O2 -std=c++17 -fno-fast-math
// -ffp-contract=off -fPIC -shared -pthread. Every float operation below is a
// single IEEE binary32 operation in the Rust code's order; expf is glibc's,
// the function Rust's f32::exp lowers to on x86_64-unknown-linux-gnu.
//
// Parity pins: the known-answer tests of the reference's own test files
// (tests/golden/reference_kats.json). The seeded generator is unpinned (see
// sampling_ref.h): every draw takes a caller-supplied uniform.

#include "sampling_ref.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstring>
#include <functional>
#include <limits>
#include <mutex>
#include <thread>
#include <unistd.h>
#include <utility>
#include <vector>

namespace {

const float kNegInf = -std::numeric_limits<float>::infinity();

// f32::total_cmp as an integer key: the bit pattern read as i32, with the
// magnitude bits flipped for negative values (core::f32::total_cmp).
inline int32_t total_key(float v) {
    int32_t b;
    std::memcpy(&b, &v, 4);
    b ^= static_cast<int32_t>(static_cast<uint32_t>(b >> 31) >> 1);
    return b;
}

// `if logit.is_nan() { -inf } else { logit } * scale`
// crates/rusticide-sampling/src/candidates.rs:30-37
inline float scaled(float logit, float scale) {
    float l = std::isnan(logit) ? kNegInf : logit;
    return l * scale;
}

// candidates.rs:25-29
inline float scale_of(float temperature) {
    return temperature > 0.0f ? 1.0f / temperature : 1.0f;
}

struct Entry {
    size_t index;
    float value;
};

// kth_largest, candidates.rs:93-97: select_nth_unstable_by(k - 1, desc
// total_cmp). Any exact selection yields the same value; nth_element is an
// introselect like Rust's.
float kth_largest(std::vector<float> values, size_t k) {
    auto desc = [](float a, float b) { return total_key(a) > total_key(b); };
    std::nth_element(values.begin(), values.begin() + (k - 1), values.end(),
                     desc);
    return values[k - 1];
}

// Candidates::top_k, candidates.rs:24-53
std::vector<Entry> top_k(const float *logits, size_t n, float temperature,
                         uint32_t k32) {
    float scale = scale_of(temperature);
    size_t k = k32;
    float threshold;
    if (k == 0 || k >= n) {
        threshold = kNegInf;
    } else {
        std::vector<float> s(n);
        for (size_t i = 0; i < n; ++i) s[i] = scaled(logits[i], scale);
        threshold = kth_largest(std::move(s), k);
    }
    std::vector<Entry> entries;
    for (size_t i = 0; i < n; ++i) {
        float value = scaled(logits[i], scale);
        // value != -inf && value.partial_cmp(&threshold) != Some(Less)
        if (value != kNegInf && !(value < threshold)) entries.push_back({i, value});
    }
    return entries;
}

// Candidates::top_p, candidates.rs:55-78. `before`/`after` (nullable) get
// the running sum before and after the element that crossed p (both the
// final sum when nothing crossed), for the benchmark's boundary counter.
void top_p(std::vector<Entry> &entries, float p, float *before = nullptr,
           float *after = nullptr) {
    std::sort(entries.begin(), entries.end(), [](const Entry &a, const Entry &b) {
        int32_t ka = total_key(a.value), kb = total_key(b.value);
        if (ka != kb) return ka > kb;  // b.1.total_cmp(&a.1)
        return a.index < b.index;      // .then(a.0.cmp(&b.0))
    });
    if (entries.empty()) return;
    float max = entries[0].value;
    std::vector<float> exp_vals(entries.size());
    for (size_t i = 0; i < entries.size(); ++i)
        exp_vals[i] = expf(entries[i].value - max);
    float exp_sum = 0.0f;  // fold(0.0, |sum, &value| sum + value)
    for (float v : exp_vals) exp_sum = exp_sum + v;
    float cumsum = 0.0f, prev = 0.0f;
    size_t cutoff = exp_vals.size();
    for (size_t i = 0; i < exp_vals.size(); ++i) {
        prev = cumsum;
        cumsum += exp_vals[i] / exp_sum;
        if (cumsum > p) {
            cutoff = i + 1;
            break;
        }
    }
    if (before) *before = cutoff == exp_vals.size() && !(cumsum > p) ? cumsum : prev;
    if (after) *after = cumsum;
    entries.resize(cutoff);
    std::sort(entries.begin(), entries.end(),
              [](const Entry &a, const Entry &b) { return a.index < b.index; });
}

// Candidates::filter, candidates.rs:16-22
std::vector<Entry> filter(const float *logits, size_t n, const rso_params &p) {
    std::vector<Entry> c = top_k(logits, n, p.temperature, p.top_k);
    if (p.top_p < 1.0f) top_p(c, p.top_p);
    return c;
}

// softmax, crates/rusticide-sampling/src/filters.rs:5-15
std::vector<float> softmax(const float *values, size_t n) {
    float max = kNegInf;
    for (size_t i = 0; i < n; ++i) max = std::fmax(max, values[i]);  // f32::max
    std::vector<float> probs(n);
    for (size_t i = 0; i < n; ++i) probs[i] = expf(values[i] - max);
    float sum = -0.0f;  // <f32 as Sum>::sum folds from -0.0
    for (float v : probs) sum = sum + v;
    if (std::isfinite(sum) && sum > 0.0f)
        for (float &v : probs) v /= sum;
    return probs;
}

// valid_probabilities, src/sampler.rs:133-139: false means NoValidTokens.
bool all_invalid(const std::vector<float> &probs) {
    for (float v : probs)
        if (!(std::isnan(v) || v <= 0.0f)) return false;
    return true;
}

// argmax, filters.rs:37-43: Iterator::max_by keeps the last of equal maxima.
size_t argmax(const float *values, size_t n) {
    if (n == 0) return static_cast<size_t>(-1);
    size_t best = 0;
    for (size_t i = 1; i < n; ++i)
        if (total_key(values[i]) >= total_key(values[best])) best = i;
    return best;
}

// Sampler::sample_multinomial, src/sampler.rs:111-121
size_t multinomial(const std::vector<float> &probs, float r, float *lo,
                   float *hi) {
    float cumsum = 0.0f;
    for (size_t i = 0; i < probs.size(); ++i) {
        float before = cumsum;
        cumsum += probs[i];
        if (r < cumsum) {
            *lo = before;
            *hi = cumsum;
            return i;
        }
    }
    *lo = cumsum;
    *hi = cumsum;
    return probs.size() - 1;
}

// logits.rs:25-27
void set_token(rso_result *out, size_t index) {
    if (index > 0xFFFFFFFFull) {
        out->status = RSO_VOCAB_OVERFLOW;
        out->token = 0;
    } else {
        out->status = RSO_OK;
        out->token = static_cast<uint32_t>(index);
    }
}

void reset(rso_result *out) {
    out->status = RSO_NO_VALID_TOKENS;
    out->token = 0;
    out->consumed_draw = 0;
    out->position = 0;
    out->prob = std::numeric_limits<float>::quiet_NaN();
    out->n_survivors = 0;
    out->cdf_lo = std::numeric_limits<float>::quiet_NaN();
    out->cdf_hi = std::numeric_limits<float>::quiet_NaN();
}

// A persistent pool of worker threads for the batched helpers: threads are
// created on the first call that asks for them (or for a different count)
// and then reused, so that timing a batch does not time thread creation.
// Rows are handed out one at a time from a shared counter. One batch runs at
// a time (calls are serialised by `call_mu`).
class RowPool {
  public:
    static RowPool &get() {
        static RowPool pool;
        return pool;
    }

    void run(size_t rows, size_t threads, const std::function<void(size_t)> &f) {
        std::lock_guard<std::mutex> call_lock(call_mu_);
        if (owner_ != getpid()) {
            // A forked child inherits the pool's bookkeeping but not its
            // threads: forget them (never join) and start afresh.
            for (auto *t : workers_) (void)t;  // leaked on purpose
            workers_.clear();
            owner_ = getpid();
        }
        resize(threads);
        {
            std::lock_guard<std::mutex> lk(mu_);
            job_ = &f;
            rows_ = rows;
            next_.store(0);
            pending_ = workers_.size();
            ++generation_;
        }
        cv_.notify_all();
        std::unique_lock<std::mutex> lk(mu_);
        done_cv_.wait(lk, [this] { return pending_ == 0; });
        job_ = nullptr;
    }

    ~RowPool() {
        if (owner_ == getpid()) resize(0);
    }

  private:
    void resize(size_t n) {
        if (n == workers_.size()) return;
        {
            std::lock_guard<std::mutex> lk(mu_);
            stop_ = true;
            ++generation_;
        }
        cv_.notify_all();
        for (auto *t : workers_) {
            t->join();
            delete t;
        }
        workers_.clear();
        uint64_t gen0;
        {
            std::lock_guard<std::mutex> lk(mu_);
            stop_ = false;
            gen0 = generation_;
        }
        // A worker starts from the generation current at its creation, so a
        // batch posted before the thread first runs is still seen as new.
        for (size_t w = 0; w < n; ++w) workers_.push_back(new std::thread([this, gen0] { loop(gen0); }));
    }

    void loop(uint64_t seen) {
        while (true) {
            const std::function<void(size_t)> *job;
            size_t rows;
            {
                std::unique_lock<std::mutex> lk(mu_);
                cv_.wait(lk, [&] { return stop_ || generation_ != seen; });
                if (stop_) return;
                seen = generation_;
                job = job_;
                rows = rows_;
            }
            for (size_t r = next_.fetch_add(1); r < rows; r = next_.fetch_add(1)) (*job)(r);
            std::lock_guard<std::mutex> lk(mu_);
            if (--pending_ == 0) done_cv_.notify_all();
        }
    }

    std::mutex call_mu_, mu_;
    std::condition_variable cv_, done_cv_;
    std::vector<std::thread *> workers_;
    pid_t owner_ = getpid();
    const std::function<void(size_t)> *job_ = nullptr;
    size_t rows_ = 0, pending_ = 0;
    std::atomic<size_t> next_{0};
    uint64_t generation_ = 0;
    bool stop_ = false;
};

template <typename F>
void parallel_rows(size_t rows, int threads, F f) {
    if (threads <= 1 || rows < 2) {
        for (size_t r = 0; r < rows; ++r) f(r);
        return;
    }
    const std::function<void(size_t)> job = f;
    RowPool::get().run(rows, static_cast<size_t>(threads), job);
}

}  // namespace

extern "C" {

// Sampler::sample_logits, src/sampler.rs:44-54
void rso_sample_logits(const float *logits, size_t n, const rso_params *params,
                       float u, rso_result *out) {
    reset(out);
    std::vector<Entry> c = filter(logits, n, *params);
    out->n_survivors = static_cast<uint32_t>(c.size());
    std::vector<float> values(c.size());
    for (size_t i = 0; i < c.size(); ++i) values[i] = c[i].value;
    std::vector<float> probs = softmax(values.data(), values.size());
    if (all_invalid(probs)) return;  // NoValidTokens, no draw consumed
    size_t position;
    if (params->temperature == 0.0f || params->top_k == 1) {
        position = argmax(values.data(), values.size());
    } else {
        out->consumed_draw = 1;
        position = multinomial(probs, u, &out->cdf_lo, &out->cdf_hi);
    }
    out->position = static_cast<uint32_t>(position);
    out->prob = probs[position];
    set_token(out, c[position].index);
}

// Sampler::greedy_logits, src/sampler.rs:75-88
void rso_greedy_logits(const float *logits, size_t n, rso_result *out) {
    reset(out);
    std::vector<float> cleaned(n);
    bool any_finite = false;
    for (size_t i = 0; i < n; ++i) {
        cleaned[i] = std::isnan(logits[i]) ? kNegInf : logits[i];
        any_finite = any_finite || std::isfinite(logits[i]);
    }
    size_t idx = argmax(cleaned.data(), n);
    if (idx == static_cast<size_t>(-1) || !any_finite) return;
    out->position = static_cast<uint32_t>(idx);
    set_token(out, idx);
}

// Sampler::sample_with_temp, src/sampler.rs:97-105 (after extract_logits,
// logits.rs:9-23, which maps NaN to -inf)
void rso_sample_with_temp(const float *logits, size_t n, float temperature,
                          float u, rso_result *out) {
    if (temperature == 0.0f) {
        rso_greedy_logits(logits, n, out);
        return;
    }
    reset(out);
    std::vector<float> x(n);
    for (size_t i = 0; i < n; ++i) x[i] = std::isnan(logits[i]) ? kNegInf : logits[i];
    float inv_temp = 1.0f / temperature;  // apply_temperature, filters.rs:17-22
    for (float &v : x) v *= inv_temp;
    std::vector<float> probs = softmax(x.data(), n);
    out->n_survivors = static_cast<uint32_t>(n);
    if (all_invalid(probs)) return;
    out->consumed_draw = 1;
    size_t position = multinomial(probs, u, &out->cdf_lo, &out->cdf_hi);
    out->position = static_cast<uint32_t>(position);
    out->prob = probs[position];
    set_token(out, position);
}

// pick, crates/rusticide-model/src/generate.rs:117-124
void rso_pick(const float *logits, size_t n, const rso_params *params, float u,
              rso_result *out) {
    if (params->temperature == 0.0f)
        rso_greedy_logits(logits, n, out);
    else
        rso_sample_logits(logits, n, params, u, out);
}

size_t rso_filter(const float *logits, size_t n, const rso_params *params,
                  uint32_t *out_index, float *out_value) {
    std::vector<Entry> c = filter(logits, n, *params);
    for (size_t i = 0; i < c.size(); ++i) {
        if (out_index) out_index[i] = static_cast<uint32_t>(c[i].index);
        if (out_value) out_value[i] = c[i].value;
    }
    return c.size();
}

size_t rso_topp_edge(const float *logits, size_t n, const rso_params *params,
                     float *before, float *after) {
    std::vector<Entry> c = top_k(logits, n, params->temperature, params->top_k);
    *before = *after = std::numeric_limits<float>::quiet_NaN();
    if (!(params->top_p < 1.0f)) return c.size();
    top_p(c, params->top_p, before, after);
    return c.size();
}

float rso_topk_threshold(const float *logits, size_t n, float temperature,
                         uint32_t k32) {
    size_t k = k32;
    if (k == 0 || k >= n) return kNegInf;
    float scale = scale_of(temperature);
    std::vector<float> s(n);
    for (size_t i = 0; i < n; ++i) s[i] = scaled(logits[i], scale);
    return kth_largest(std::move(s), k);
}

void rso_softmax(const float *values, size_t n, float *probs) {
    std::vector<float> p = softmax(values, n);
    for (size_t i = 0; i < n; ++i) probs[i] = p[i];
}

size_t rso_argmax(const float *values, size_t n) { return argmax(values, n); }

// apply_repetition_penalty, filters.rs:24-35
void rso_apply_repetition_penalty(float *logits, size_t n,
                                  const uint32_t *tokens, size_t n_tokens,
                                  float penalty) {
    for (size_t t = 0; t < n_tokens; ++t) {
        size_t idx = tokens[t];
        if (idx < n) {
            if (logits[idx] > 0.0f)
                logits[idx] /= penalty;
            else
                logits[idx] *= penalty;
        }
    }
}

void rso_sample_rows(const float *logits, size_t rows, size_t n,
                     size_t row_stride, const rso_params *params,
                     const float *u, rso_result *out, int threads) {
    parallel_rows(rows, threads, [&](size_t r) {
        rso_sample_logits(logits + r * row_stride, n, params, u ? u[r] : 0.0f,
                          out + r);
    });
}

void rso_greedy_rows(const float *logits, size_t rows, size_t n,
                     size_t row_stride, rso_result *out, int threads) {
    parallel_rows(rows, threads, [&](size_t r) {
        rso_greedy_logits(logits + r * row_stride, n, out + r);
    });
}

void rso_sample_with_temp_rows(const float *logits, size_t rows, size_t n,
                               size_t row_stride, float temperature,
                               const float *u, rso_result *out, int threads) {
    parallel_rows(rows, threads, [&](size_t r) {
        rso_sample_with_temp(logits + r * row_stride, n, temperature,
                             u ? u[r] : 0.0f, out + r);
    });
}

// fastrand::Rng::gen_u64 (fastrand 2.5.0, Cargo.lock:191-195; called through
// Rng::f32 at src/sampler.rs:112): wyrand with the final wyhash v4.2
// constants, as fastrand's lib.rs has them since its 2.1 release. The state
// advances by 0x2d358dccaa6c78a5; the output is the xor of the two halves of
// the 128-bit product state * (state ^ 0x8bb84b93962eacc9). Restated from the
// crate's published source, not checked against the crate's own output.
uint64_t rso_rng_next_u64(uint64_t *state) {
    uint64_t s = *state + 0x2d358dccaa6c78a5ULL;
    *state = s;
    unsigned __int128 t = static_cast<unsigned __int128>(s) *
                          static_cast<unsigned __int128>(s ^ 0x8bb84b93962eacc9ULL);
    return static_cast<uint64_t>(t) ^ static_cast<uint64_t>(t >> 64);
}

// fastrand::Rng::f32: gen_u32 is the low 32 bits of gen_u64; its top 23 bits
// fill the mantissa of a float in [1, 2) (bits (1 << 30) - (1 << 23) +
// (x >> 9)), and 1.0 is subtracted.
float rso_rng_f32(uint64_t *state) {
    uint32_t x = static_cast<uint32_t>(rso_rng_next_u64(state));
    uint32_t bits = 0x3F800000u | (x >> 9);
    float f;
    std::memcpy(&f, &bits, 4);
    return f - 1.0f;
}

void rso_expf_many(const float *x, size_t n, float *y) {
    for (size_t i = 0; i < n; ++i) y[i] = expf(x[i]);
}

}  // extern "C"
