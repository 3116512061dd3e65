// Log-probability outputs of rsc_sample_ex: each row's log-sum-exp over the
// whole vocabulary of the scaled logits the reference's Candidates hold
// (v = x * scale with NaN read as -inf, crates/rusticide-sampling/src/
// candidates.rs:25-37), the chosen token's log-probability v_token - lse and
// the listed survivors' v_i - lse. The reference itself returns none of
// these: its softmax (src/filters.rs:5-15) normalises over the survivors
// only; the log-sum-exp is what that normalisation generalises to over the
// full row.
//
// The sums use the fast binary32 exp (__expf): a log-probability is
// reported to within about 1e-6 of its value, not bit for bit.
//
// Partial log-sum-exps come from the streaming kernel's consumers (one per
// row part) or, for rows sampled by other kernels, from lse_rows_kernel (one
// per row); lse_finish_kernel combines a row's parts and writes the outputs.
#include "rsc_kernels.h"

namespace rsc {

namespace {

constexpr int kLseThreads = 256;

// One block per row: the row's (maximum, sum of exp(v - maximum)) into
// parts[row * stride].
__global__ void __launch_bounds__(kLseThreads)
lse_rows_kernel(const float *__restrict__ logits, size_t rows, uint32_t vocab, size_t row_stride,
                float scale, uint2 *__restrict__ parts, uint32_t stride) {
    __shared__ float red_m[kLseThreads / 32], red_s[kLseThreads / 32];
    const size_t row = blockIdx.x;
    if (row >= rows) return;
    const float *p = logits + row * row_stride;
    float m = kNegInf, s = 0.0f;
    const uint32_t mis = static_cast<uint32_t>((reinterpret_cast<uintptr_t>(p) >> 2) & 3u);
    const uint32_t head = mis ? min(vocab, 4u - mis) : 0u;
    const uint32_t n4 = (vocab - head) / 4u;
    const uint32_t tail0 = head + 4u * n4;
    if (threadIdx.x < head) lse_add(m, s, scale_logit(p[threadIdx.x], scale));
    if (threadIdx.x >= 32 && threadIdx.x - 32 < vocab - tail0)
        lse_add(m, s, scale_logit(p[tail0 + threadIdx.x - 32], scale));
    const float4 *p4 = reinterpret_cast<const float4 *>(p + head);
    constexpr int kB = 4;
    for (uint32_t q0 = 0; q0 < n4; q0 += kLseThreads * kB) {
        float4 x[kB];
#pragma unroll
        for (int b = 0; b < kB; ++b) {
            const uint32_t q = q0 + b * kLseThreads + threadIdx.x;
            x[b] = q < n4 ? p4[q] : make_float4(kNegInf, kNegInf, kNegInf, kNegInf);
        }
#pragma unroll
        for (int b = 0; b < kB; ++b) {
            lse_add(m, s, scale_logit(x[b].x, scale));
            lse_add(m, s, scale_logit(x[b].y, scale));
            lse_add(m, s, scale_logit(x[b].z, scale));
            lse_add(m, s, scale_logit(x[b].w, scale));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
        lse_combine(m, s, m2, s2);
    }
    if ((threadIdx.x & 31) == 0) {
        red_m[threadIdx.x >> 5] = m;
        red_s[threadIdx.x >> 5] = s;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float mm = kNegInf, ss = 0.0f;
        for (int w = 0; w < kLseThreads / 32; ++w) lse_combine(mm, ss, red_m[w], red_s[w]);
        parts[row * stride] = make_uint2(total_key(mm), __float_as_uint(ss));
    }
}

// One warp per row: combines the row's parts (a slot never written holds key
// 0, below every float's key) and writes the outputs.
__global__ void __launch_bounds__(128)
lse_finish_kernel(const float *__restrict__ logits, size_t rows, size_t row_stride, float scale,
                  const uint2 *__restrict__ parts, uint32_t stride,
                  const uint32_t *__restrict__ ids, const int32_t *__restrict__ status,
                  const uint32_t *__restrict__ n_surv, const uint32_t *__restrict__ surv,
                  uint32_t cap, float *__restrict__ out_lse, float *__restrict__ out_logprob,
                  float *__restrict__ out_surv_logp) {
    const size_t row = static_cast<size_t>(blockIdx.x) * 4 + (threadIdx.x >> 5);
    const uint32_t lane = threadIdx.x & 31u;
    if (row >= rows) return;
    float m = kNegInf, s = 0.0f;
    for (uint32_t q = lane; q < stride; q += 32) {
        const uint2 e = parts[row * stride + q];
        if (e.x != 0u) lse_combine(m, s, key_to_float(e.x), __uint_as_float(e.y));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
        lse_combine(m, s, m2, s2);
    }
    // A row with no finite scaled logit has no probability mass: -inf.
    const float lse = (m == kNegInf || !(fabsf(m) < kPosInf)) ? m : __fadd_rn(m, logf(s));
    const float *p = logits + row * row_stride;
    if (lane == 0) {
        if (out_lse) out_lse[row] = lse;
        if (out_logprob) {
            const bool ok = (status[row] & 0xff) == RSC_ROW_OK;
            out_logprob[row] =
                ok ? __fsub_rn(scale_logit(p[ids[row]], scale), lse) : __uint_as_float(0x7fc00000u);
        }
    }
    if (out_surv_logp && surv) {
        const uint32_t n = min(n_surv ? n_surv[row] : cap, cap);
        for (uint32_t i = lane; i < n; i += 32) {
            const uint32_t id = surv[row * cap + i];
            out_surv_logp[row * cap + i] = __fsub_rn(scale_logit(p[id], scale), lse);
        }
    }
}

}  // namespace

cudaError_t launch_lse_rows(const float *logits, size_t rows, uint32_t vocab, size_t row_stride,
                            float scale, uint2 *parts, uint32_t stride, cudaStream_t stream) {
    if (rows == 0) return cudaSuccess;
    lse_rows_kernel<<<static_cast<unsigned>(rows), kLseThreads, 0, stream>>>(
        logits, rows, vocab, row_stride, scale, parts, stride);
    return cudaGetLastError();
}

cudaError_t launch_lse_finish(const float *logits, size_t rows, size_t row_stride, float scale,
                              const uint2 *parts, uint32_t stride, const uint32_t *ids,
                              const int32_t *status, const uint32_t *n_surv, const uint32_t *surv,
                              uint32_t cap, float *out_lse, float *out_logprob,
                              float *out_surv_logp, cudaStream_t stream) {
    if (rows == 0) return cudaSuccess;
    lse_finish_kernel<<<static_cast<unsigned>((rows + 3) / 4), 128, 0, stream>>>(
        logits, rows, row_stride, scale, parts, stride, ids, status, n_surv, surv, cap, out_lse,
        out_logprob, out_surv_logp);
    return cudaGetLastError();
}

}  // namespace rsc
