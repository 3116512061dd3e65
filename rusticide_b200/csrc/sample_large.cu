// Large-survivor kernel: one block of kThreads per row, over all rows of a
// call that the streaming kernel does not take (the per-row algorithm is in
// rsc_large.cuh).
#include "rsc_large.cuh"

namespace rsc {

namespace {

using namespace large;

constexpr int kThreads = 512;

__global__ void __launch_bounds__(kThreads, kLargeCtasPerSm)
large_kernel(const float *__restrict__ logits, size_t rows, uint32_t vocab, size_t row_stride,
             CallParams cp, uint32_t *__restrict__ out_ids, int32_t *__restrict__ out_status,
             float *__restrict__ out_probs, uint32_t *__restrict__ scratch) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    LargeSmem<kThreads> &sm = *reinterpret_cast<LargeSmem<kThreads> *>(smem_raw);
    load_exp_table(sm.exp_tab);
    __syncthreads();
    uint32_t *my_scratch = scratch + static_cast<size_t>(blockIdx.x) * 4u * vocab;
    for (size_t row = blockIdx.x; row < rows; row += gridDim.x)
        sample_row<kThreads>(cp, logits + row * row_stride, vocab, row, my_scratch, out_ids,
                             out_status, out_probs, sm);
}

}  // namespace

cudaError_t launch_large(const float *logits, size_t rows, uint32_t vocab, size_t row_stride,
                         const CallParams &p, uint32_t *out_ids, int32_t *out_status,
                         float *out_probs, uint32_t *scratch, uint32_t slots, cudaStream_t stream) {
    if (rows == 0 || slots == 0) return cudaSuccess;
    const size_t smem = sizeof(LargeSmem<kThreads>);
    cudaError_t e = cudaFuncSetAttribute(large_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    size_t grid = slots;
    if (grid > rows) grid = rows;
    large_kernel<<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(
        logits, rows, vocab, row_stride, p, out_ids, out_status, out_probs, scratch);
    return cudaGetLastError();
}

}  // namespace rsc
