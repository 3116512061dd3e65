// Small row-wise kernels: the repetition penalty and generator seeding.
#include "rsc_kernels.h"

namespace rsc {

namespace {

// apply_repetition_penalty, crates/rusticide-sampling/src/filters.rs:24-35:
// tokens are applied in list order, so a repeated token is penalised twice.
// One thread per row walks the list.
__global__ void penalize_kernel(float *logits, size_t rows, uint32_t vocab, size_t row_stride,
                                const uint32_t *__restrict__ tokens, size_t n_tokens,
                                float penalty) {
    size_t row = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (row >= rows) return;
    float *p = logits + row * row_stride;
    for (size_t t = 0; t < n_tokens; ++t) {
        uint32_t idx = tokens[t];
        if (idx < vocab) {
            float x = p[idx];
            p[idx] = x > 0.0f ? __fdiv_rn(x, penalty) : __fmul_rn(x, penalty);
        }
    }
}

// fastrand::Rng::with_seed(seed) starts the stream at state = seed.
__global__ void rng_seed_kernel(const uint64_t *seeds, uint64_t *states, size_t rows) {
    size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < rows) states[i] = seeds[i];
}

__global__ void expf_kernel(const float *__restrict__ x, float *__restrict__ y, size_t n) {
    __shared__ double tab[32];
    load_exp_table(tab);
    __syncthreads();
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        y[i] = expf_ref(x[i], tab);
}

}  // namespace

cudaError_t launch_expf(const float *x, float *y, size_t n, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    size_t blocks = (n + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    expf_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(x, y, n);
    return cudaGetLastError();
}

cudaError_t launch_penalize(float *logits, size_t rows, uint32_t vocab, size_t row_stride,
                            const uint32_t *tokens, size_t n_tokens, float penalty,
                            cudaStream_t stream) {
    unsigned blocks = static_cast<unsigned>((rows + 127) / 128);
    penalize_kernel<<<blocks, 128, 0, stream>>>(logits, rows, vocab, row_stride, tokens, n_tokens,
                                                penalty);
    return cudaGetLastError();
}

cudaError_t launch_rng_seed(const uint64_t *seeds, uint64_t *states, size_t rows,
                            cudaStream_t stream) {
    unsigned blocks = static_cast<unsigned>((rows + 255) / 256);
    rng_seed_kernel<<<blocks, 256, 0, stream>>>(seeds, states, rows);
    return cudaGetLastError();
}

}  // namespace rsc
