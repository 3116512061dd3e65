// Sampling fused into the LM-head GEMM. The logits of a decode step are
// H · Wᵀ (H: rows x dim hidden states, W: vocab x dim weights, both bf16,
// products accumulated in f32 on the tcgen05 tensor cores); the reference
// computes them in crates/rusticide-transformer/src/decoder.rs:104-105
// (output.matvec) and then samples them (crates/rusticide-sampling/src/
// sampler.rs:44-54). Here the logits never reach HBM: each CTA's epilogue
// reads its accumulator tile from tensor memory and keeps, per row, the
// candidates that can survive top-k, and writes one record per (part, row)
// in the vocab-sharded record format; the shard merge then finishes every
// row exactly as the streaming sampler would on the same logits. A second
// mode of the same kernel writes the logits instead, so the fused result can
// be checked against rsc_sample on identical values.
//
// One CTA per (128-row tile, vocab part), 192 threads:
//  warp 0, one lane: TMA producer (2-D tiled loads of H and W tiles, 128-byte
//    swizzle, no multicast) into a 3-stage ring;
//  warp 1, one lane: MMA issuer, tcgen05.mma.cta_group::1.kind::f16
//    (M 128, N 256, K 16) from shared-memory descriptors into one of two
//    tensor-memory accumulators (256 columns each); tcgen05.commit frees the
//    stage and publishes a finished accumulator;
//  warps 2-5: epilogue, one thread per row of the tile (tcgen05.ld 32x32b).
// All waits are bounded; a timeout sets the CTA's error flag, every role
// stops, and tensor memory is freed before the CTA exits.
#include <cuda.h>
#include <cuda_bf16.h>

#include "rsc_common.cuh"
#include "rsc_kernels.h"

namespace rsc {

namespace {

constexpr int kBM = 128;        // rows of a tile (tensor-memory lanes)
constexpr int kBN = 256;        // vocab columns of a tile
constexpr int kBK = 64;         // k per stage: 128 bytes of bf16, one swizzle span
constexpr int kUK = 16;         // k per tcgen05.mma (kind::f16)
constexpr int kGStages = 3;
constexpr int kGThreads = 192;
constexpr int kEpiWarp0 = 2;
constexpr int kRowCap = kLmheadRowCap;  // candidates a row keeps in shared memory
constexpr uint32_t kTmemCols = 2 * kBN;

struct LmSmem {
    __nv_bfloat16 a[kGStages][kBM * kBK];  // 16 KiB per stage
    __nv_bfloat16 b[kGStages][kBN * kBK];  // 32 KiB per stage
    uint32_t ckey[kRowCap][kBM];           // per-row candidate lists, row fastest
    uint32_t cidx[kRowCap][kBM];
    uint64_t full[kGStages];
    uint64_t empty[kGStages];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint32_t tmem_base;
    uint32_t error;
};
static_assert(sizeof(__nv_bfloat16) * kBM * kBK % 1024 == 0, "stages stay 1024-byte aligned");
constexpr size_t kLmSmemBytes = sizeof(LmSmem) + 1024;  // + alignment slack

// Instruction descriptor of tcgen05.mma kind::f16: f32 accumulator, bf16 A
// and B, both K-major, N = 256, M = 128 (field layout of the PTX ISA).
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) |
                            (static_cast<uint32_t>(kBN >> 3) << 17) |
                            (static_cast<uint32_t>(kBM >> 4) << 24);

// Shared-memory matrix descriptor of a K-major tile written by a 128-byte
// swizzled TMA load: rows of 128 bytes, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr) {
    return static_cast<uint64_t>((saddr & 0x3ffffu) >> 4) | (1ull << 16) | (64ull << 32) |
           (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(kIdesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive accumulator columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
        "%29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// The k-th largest key among a row's n list entries (n >= k), by a bitwise
// search over the key space (one thread).
__device__ uint32_t row_kth_key(const LmSmem &sm, uint32_t r, uint32_t n, uint32_t k) {
    uint32_t res = 0;
    for (int bit = 31; bit >= 0; --bit) {
        const uint32_t cand = res | (1u << bit);
        uint32_t c = 0;
        for (uint32_t i = 0; i < n; ++i) c += sm.ckey[i][r] >= cand ? 1u : 0u;
        if (c >= k) res = cand;
    }
    return res;
}

// Keeps a row's entries at or above floor_key; returns their number.
__device__ uint32_t row_compact(LmSmem &sm, uint32_t r, uint32_t n, uint32_t floor_key) {
    uint32_t m = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const uint32_t key = sm.ckey[i][r];
        if (key >= floor_key) {
            sm.ckey[m][r] = key;
            sm.cidx[m][r] = sm.cidx[i][r];
            ++m;
        }
    }
    return m;
}

template <bool kFused>
__global__ void __launch_bounds__(kGThreads, 1)
lmhead_kernel(const __grid_constant__ CUtensorMap map_h, const __grid_constant__ CUtensorMap map_w,
              uint32_t rows, uint32_t dim, uint32_t vocab, uint32_t n_tiles, CallParams cp,
              float *__restrict__ logits, unsigned char *__restrict__ records, size_t rec_bytes,
              uint32_t *__restrict__ error_out) {
    extern __shared__ unsigned char smem_raw[];
    LmSmem &sm = *reinterpret_cast<LmSmem *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~static_cast<uintptr_t>(1023u));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t part = blockIdx.x, parts = gridDim.x;
    const uint32_t m0 = blockIdx.y * kBM;
    const uint32_t t0 = static_cast<uint32_t>((static_cast<unsigned long long>(n_tiles) * part) / parts);
    const uint32_t t1 = static_cast<uint32_t>((static_cast<unsigned long long>(n_tiles) * (part + 1)) / parts);
    const uint32_t kblocks = (dim + kBK - 1) / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kGStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&sm.acc_full[b], 1);
            mbar_init(&sm.acc_empty[b], kBM / 32);
        }
        sm.error = 0;
        fence_barrier_init();
    }
    if (warp == 0) {  // the allocating warp also frees
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_addr(&sm.tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    volatile uint32_t *err = &sm.error;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (uint32_t t = t0; t < t1 && ok; ++t) {
                for (uint32_t kb = 0; kb < kblocks; ++kb, ++it) {
                    const uint32_t s = it % kGStages;
                    if (it >= kGStages && !mbar_wait(&sm.empty[s], ((it / kGStages) - 1u) & 1u)) {
                        *err = 1u;
                        ok = false;
                        break;
                    }
                    if (*err) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&sm.full[s],
                                          static_cast<uint32_t>(sizeof(sm.a[0]) + sizeof(sm.b[0])));
                    tma_load_2d(sm.a[s], &map_h, &sm.full[s], static_cast<int32_t>(kb * kBK),
                                static_cast<int32_t>(m0));
                    tma_load_2d(sm.b[s], &map_w, &sm.full[s], static_cast<int32_t>(kb * kBK),
                                static_cast<int32_t>(t * kBN));
                }
            }
            // Every copy issued has landed before the CTA moves on (bounded).
            const uint32_t first = it > kGStages ? it - kGStages : 0u;
            for (uint32_t i = first; i < it; ++i) mbar_wait(&sm.full[i % kGStages], (i / kGStages) & 1u);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (uint32_t t = t0, j = 0; t < t1 && ok; ++t, ++j) {
                const uint32_t buf = j & 1u;
                if (j >= 2 && !mbar_wait(&sm.acc_empty[buf], ((j >> 1) - 1u) & 1u)) {
                    *err = 1u;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + buf * kBN;
                for (uint32_t kb = 0; kb < kblocks; ++kb, ++it) {
                    const uint32_t s = it % kGStages;
                    if (!mbar_wait(&sm.full[s], (it / kGStages) & 1u) || *err) {
                        *err = 1u;
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_addr(sm.a[s]), sb = smem_addr(sm.b[s]);
#pragma unroll
                    for (int kk = 0; kk < kBK / kUK; ++kk) {
                        const uint32_t off = static_cast<uint32_t>(kk * kUK * sizeof(__nv_bfloat16));
                        mma_bf16(d, smem_desc(sa + off), smem_desc(sb + off), (kb | kk) ? 1u : 0u);
                    }
                    mma_commit(&sm.empty[s]);  // the stage is free once these MMAs have read it
                }
                if (ok) mma_commit(&sm.acc_full[buf]);
            }
            // The last commits must have landed before tensor memory is freed:
            // wait (bounded) for the final stage release.
            if (it > 0) mbar_wait(&sm.empty[(it - 1) % kGStages], ((it - 1) / kGStages) & 1u);
        }
    } else {
        // Epilogue: thread (warp, lane) owns row r of the tile; its warp reads
        // tensor-memory lanes 32 * (warp % 4) ...
        const uint32_t lane_base = 32u * (static_cast<uint32_t>(warp) & 3u);
        const uint32_t r = lane_base + lane;
        const uint32_t grow = m0 + r;
        const float scale = cp.scale;
        uint32_t count = 0;
        float tau = -3.402823466e38f;
        float vmax = kNegInf;
        bool overflow = false;
        const uint32_t k = cp.top_k;
        for (uint32_t t = t0, j = 0; t < t1; ++t, ++j) {
            const uint32_t buf = j & 1u;
            bool got = mbar_wait(&sm.acc_full[buf], (j >> 1) & 1u);
            if (__any_sync(0xffffffffu, !got) || *err) {
                if (lane == 0) *err = 1u;
                break;
            }
            tc_fence_after();
            for (uint32_t c = 0; c < kBN; c += 32) {
                uint32_t v[32];
                tmem_ld32(tmem + buf * kBN + c + (lane_base << 16), v);
                const uint32_t col0 = t * kBN + c;
                if (!kFused) {
                    if (grow < rows) {
#pragma unroll
                        for (int q = 0; q < 32; ++q)
                            if (col0 + q < vocab)
                                logits[static_cast<size_t>(grow) * vocab + col0 + q] = __uint_as_float(v[q]);
                    }
                    continue;
                }
                if (grow >= rows || overflow) continue;
#pragma unroll
                for (int q = 0; q < 32; ++q) {
                    const float x = scale_logit(__uint_as_float(v[q]), scale);
                    const bool in = col0 + q < vocab;
                    vmax = in ? fmaxf(vmax, x) : vmax;
                    if (in && x >= tau) {
                        if (count == static_cast<uint32_t>(kRowCap)) {
                            // Full: tau rises to the list's k-th largest value.
                            uint32_t kth = row_kth_key(sm, r, count, k);
                            const uint32_t floor_key = kth == kKeyPosZero ? kKeyNegZero : kth;
                            tau = key_to_float(floor_key);
                            count = row_compact(sm, r, count, floor_key);
                            if (count == static_cast<uint32_t>(kRowCap)) {
                                overflow = true;  // more than kRowCap - k ties
                                break;
                            }
                            if (!(x >= tau)) continue;
                        }
                        sm.ckey[count][r] = total_key(x);
                        sm.cidx[count][r] = col0 + q;
                        ++count;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
        }
        if (kFused && grow < rows) {
            // The record of (part, row): the part's entries at or above its own
            // k-th largest value (ties included, at most k + RSC_SHARD_TIE_CAP),
            // so that the merge's union over many parts stays small.
            const uint32_t cap = k + RSC_SHARD_TIE_CAP;
            if (!overflow && count >= k) {
                const uint32_t kth = row_kth_key(sm, r, count, k);
                const uint32_t floor_key = kth == kKeyPosZero ? kKeyNegZero : kth;
                tau = key_to_float(floor_key);
                count = row_compact(sm, r, count, floor_key);
                if (count > cap) overflow = true;
            }
            unsigned char *rec = records + (static_cast<size_t>(part) * rows + grow) * rec_bytes;
            ShardRecordHeader *h = reinterpret_cast<ShardRecordHeader *>(rec);
            uint32_t *rkey = reinterpret_cast<uint32_t *>(rec + sizeof(ShardRecordHeader));
            uint32_t *ridx = rkey + cap;
            const uint32_t n = overflow ? 0u : count;
            for (uint32_t i = 0; i < n; ++i) {
                rkey[i] = sm.ckey[i][r];
                ridx[i] = sm.cidx[i][r];
            }
            h->max_scaled = vmax;
            h->sum_exp = 0.0f;
            h->n_finite = 0;
            h->n_cand = n;
            h->n_dropped = 0;
            h->last_key = 0;
            h->flags = (overflow || *err) ? 1u : 0u;
            h->tau = tau;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols)
                     : "memory");
    }
    if (threadIdx.x == 0 && sm.error) atomicExch(error_out, 1u);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// dependency on the driver library).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// A row-major bf16 matrix [outer x dim] as 2-D tiles of box_outer x 64.
bool make_map(CUtensorMap *map, const void *base, uint64_t outer, uint64_t dim, uint32_t box_outer) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {dim, outer};
    const cuuint64_t strides[1] = {dim * sizeof(__nv_bfloat16)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

uint32_t lmhead_parts(size_t rows, uint32_t vocab, int num_sms) {
    const size_t mtiles = (rows + kBM - 1) / kBM;
    const uint32_t ntiles = (vocab + kBN - 1) / kBN;
    size_t p = mtiles ? static_cast<size_t>(num_sms) / mtiles : 1;
    if (p < 1) p = 1;
    if (p > kLmheadMaxParts) p = kLmheadMaxParts;
    if (p > ntiles) p = ntiles;
    return static_cast<uint32_t>(p);
}

cudaError_t launch_lmhead(const void *hidden, const void *weight, size_t rows, uint32_t dim,
                          uint32_t vocab, const CallParams &p, float *logits, void *records,
                          size_t rec_bytes, uint32_t parts, uint32_t *error_flag,
                          cudaStream_t stream) {
    if (rows == 0) return cudaSuccess;
    CUtensorMap mh, mw;
    if (!make_map(&mh, hidden, rows, dim, kBM) || !make_map(&mw, weight, vocab, dim, kBN))
        return cudaErrorInvalidValue;
    const uint32_t ntiles = (vocab + kBN - 1) / kBN;
    const dim3 grid(parts, static_cast<unsigned>((rows + kBM - 1) / kBM), 1);
    if (logits) {
        cudaError_t e = cudaFuncSetAttribute(lmhead_kernel<false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kLmSmemBytes));
        if (e != cudaSuccess) return e;
        lmhead_kernel<false><<<grid, kGThreads, kLmSmemBytes, stream>>>(
            mh, mw, static_cast<uint32_t>(rows), dim, vocab, ntiles, p, logits, nullptr, 0,
            error_flag);
    } else {
        cudaError_t e = cudaFuncSetAttribute(lmhead_kernel<true>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kLmSmemBytes));
        if (e != cudaSuccess) return e;
        lmhead_kernel<true><<<grid, kGThreads, kLmSmemBytes, stream>>>(
            mh, mw, static_cast<uint32_t>(rows), dim, vocab, ntiles, p, nullptr,
            static_cast<unsigned char *>(records), rec_bytes, error_flag);
    }
    return cudaGetLastError();
}

}  // namespace rsc
