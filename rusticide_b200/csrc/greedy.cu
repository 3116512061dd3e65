// Batched Sampler::greedy_logits (crates/rusticide-sampling/src/sampler.rs:75-88):
// per row, the index of the largest logit with NaN read as -inf, the last one
// among equal maxima under f32::total_cmp (src/filters.rs:37-43), and
// NoValidTokens when no logit is finite.
//
// One HBM pass. A row is split over a thread-block cluster of `parts` CTAs;
// each CTA streams its segment with 128-bit loads and reduces a 64-bit
// (total-order key << 32 | index) maximum, which selects the largest key and,
// among equal keys, the largest index. The CTAs of a cluster then merge their
// partials through distributed shared memory; no global scratch and no second
// launch.
#include <cooperative_groups.h>

#include "rsc_common.cuh"
#include "rsc_kernels.h"

namespace cg = cooperative_groups;

namespace rsc {

namespace {

constexpr int kGreedyThreads = 256;

struct GreedyPartial {
    unsigned long long best;
    unsigned int any_finite;
};

__device__ __forceinline__ void greedy_visit(float x, uint32_t i, unsigned long long &best,
                                             unsigned int &finite) {
    float c = (x != x) ? kNegInf : x;
    unsigned long long cand = pack_key_index(total_key(c), i);
    best = cand > best ? cand : best;
    finite |= (fabsf(x) < kPosInf) ? 1u : 0u;
}

__global__ void __launch_bounds__(kGreedyThreads)
greedy_kernel(const float *__restrict__ logits, uint32_t vocab, size_t row_stride,
              uint32_t parts, uint32_t *__restrict__ out_ids, int32_t *__restrict__ out_status) {
    __shared__ GreedyPartial warp_part[kGreedyThreads / 32];
    __shared__ GreedyPartial cta_part;

    const uint32_t part = blockIdx.x;
    const size_t row = blockIdx.y;
    const float *p = logits + row * row_stride;
    // The next launch on the stream may start as this grid's CTAs retire; it
    // writes nothing before this grid completes (griddepcontrol.wait below).
    if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;");

    // Segment [lo, hi) of this CTA, cut at multiples of 4 elements.
    uint32_t seg = (vocab + parts - 1) / parts;
    seg = (seg + 3u) & ~3u;
    uint32_t lo = min(vocab, part * seg);
    uint32_t hi = min(vocab, lo + seg);

    unsigned long long best = 0;  // below every real (key, index) pair of a non-empty row
    unsigned int finite = 0;

    // Scalar head up to the first 16-byte aligned element, vector body, scalar tail.
    uint32_t mis = static_cast<uint32_t>((reinterpret_cast<uintptr_t>(p + lo) >> 2) & 3u);
    uint32_t head = mis ? min(hi - lo, 4u - mis) : 0u;
    uint32_t body_lo = lo + head;
    uint32_t nvec = (hi - body_lo) / 4u;
    uint32_t body_hi = body_lo + nvec * 4u;
    for (uint32_t i = lo + threadIdx.x; i < body_lo; i += blockDim.x) greedy_visit(__ldg(p + i), i, best, finite);
    for (uint32_t i = body_hi + threadIdx.x; i < hi; i += blockDim.x) greedy_visit(__ldg(p + i), i, best, finite);

    const float4 *v4 = reinterpret_cast<const float4 *>(p + body_lo);
    constexpr int kUnroll = 8;
    uint32_t j = threadIdx.x;
    for (; j + (kUnroll - 1) * kGreedyThreads < nvec; j += kUnroll * kGreedyThreads) {
        float4 f[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) f[u] = __ldcs(v4 + j + u * kGreedyThreads);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            uint32_t i = body_lo + 4u * (j + u * kGreedyThreads);
            greedy_visit(f[u].x, i, best, finite);
            greedy_visit(f[u].y, i + 1, best, finite);
            greedy_visit(f[u].z, i + 2, best, finite);
            greedy_visit(f[u].w, i + 3, best, finite);
        }
    }
    for (; j < nvec; j += kGreedyThreads) {
        float4 f = __ldcs(v4 + j);
        uint32_t i = body_lo + 4u * j;
        greedy_visit(f.x, i, best, finite);
        greedy_visit(f.y, i + 1, best, finite);
        greedy_visit(f.z, i + 2, best, finite);
        greedy_visit(f.w, i + 3, best, finite);
    }

    best = warp_max(best);
    finite = __reduce_or_sync(0xffffffffu, finite);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) warp_part[warp] = GreedyPartial{best, finite};
    __syncthreads();
    if (warp == 0) {
        GreedyPartial w = lane < kGreedyThreads / 32 ? warp_part[lane] : GreedyPartial{0ull, 0u};
        unsigned long long b = warp_max(w.best);
        unsigned int f = __reduce_or_sync(0xffffffffu, w.any_finite);
        if (lane == 0) cta_part = GreedyPartial{b, f};
    }

    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (cluster.block_rank() == 0 && threadIdx.x < 32) {
        GreedyPartial w{0ull, 0u};
        if (threadIdx.x < parts) w = *cluster.map_shared_rank(&cta_part, threadIdx.x);
        unsigned long long b = warp_max(w.best);
        unsigned int f = __reduce_or_sync(0xffffffffu, w.any_finite);
        if (threadIdx.x == 0) {
            asm volatile("griddepcontrol.wait;" ::: "memory");
            if (vocab == 0 || !f) {
                out_ids[row] = 0;
                out_status[row] = RSC_ROW_NO_VALID_TOKENS;
            } else {
                out_ids[row] = static_cast<uint32_t>(b & 0xffffffffull);
                out_status[row] = RSC_ROW_OK;
            }
        }
    }
    // Keep every CTA's shared memory alive until rank 0 has read it.
    cluster.sync();
}

}  // namespace

cudaError_t launch_greedy(const float *logits, size_t rows, uint32_t vocab, size_t row_stride,
                          uint32_t *out_ids, int32_t *out_status, int num_sms,
                          cudaStream_t stream) {
    if (rows == 0) return cudaSuccess;
    // Split rows over up to 8 CTAs so that small batches still fill the GPU,
    // keeping at least 4096 logits per CTA.
    uint32_t parts = 1;
    size_t want = static_cast<size_t>(num_sms) * 8;
    while (parts < 8 && rows * parts < want && vocab / (parts * 2) >= 4096) parts *= 2;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(parts, static_cast<unsigned>(rows), 1);
    cfg.blockDim = dim3(kGreedyThreads, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = parts;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    // Programmatic dependent launch: overlaps the previous launch's tail.
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, greedy_kernel, logits, vocab, row_stride, parts, out_ids,
                              out_status);
}

}  // namespace rsc
