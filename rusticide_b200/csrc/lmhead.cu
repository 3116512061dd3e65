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
constexpr int kBN = 256;        // vocab columns of a full tile
constexpr int kBK = 64;         // k per stage: 128 bytes of bf16, one swizzle span
constexpr int kUK = 16;         // k per tcgen05.mma (kind::f16)
constexpr int kUnit = 16;       // column granularity of parts and tiles (smallest MMA N at M 128)
constexpr int kGStages = 3;
constexpr int kGThreads = 192;
constexpr uint32_t kListCap = 96;        // candidates a row holds in shared memory per part
constexpr uint32_t kChunkCols = 16;      // accumulator columns per epilogue step
constexpr uint32_t kKeyStride = kBM + 1; // list slot stride of the keys (words)
constexpr uint32_t kIdxStride = kBM + 2; // list slot stride of the indices (halfwords)
constexpr uint32_t kTmemCols = 2 * kBN;
constexpr uint32_t kFloorSlack = 8;      // a list cut may keep up to k + 8 entries
static_assert(kLmheadRowCap <= kListCap - kChunkCols, "a record's candidates fit a list");

struct LmSmem {
    __nv_bfloat16 a[kGStages][kBM * kBK];  // 16 KiB per stage
    __nv_bfloat16 b[kGStages][kBN * kBK];  // 32 KiB per stage
    // Per-row candidate lists, slot-major (slot s of row r at s * stride + r):
    // the owning thread appends to its own row, a warp reads one row's slots
    // without bank conflicts. Indices are relative to the part's first column.
    uint32_t lkey[kListCap * kKeyStride];
    uint16_t lidx[kListCap * kIdxStride];
    uint64_t full[kGStages];
    uint64_t empty[kGStages];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint32_t tmem_base;
    uint32_t error;
};
static_assert(sizeof(__nv_bfloat16) * kBM * kBK % 1024 == 0, "stages stay 1024-byte aligned");
constexpr size_t kLmSmemBytes = sizeof(LmSmem) + 1024;  // + alignment slack
static_assert(kLmSmemBytes <= 232448, "fits the 227 KiB of shared memory a CTA may use");

// Instruction descriptor of tcgen05.mma kind::f16: f32 accumulator, bf16 A
// and B, both K-major, M = 128, N = n (field layout of the PTX ISA).
__host__ __device__ constexpr uint32_t idesc_for(uint32_t n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) |
           (static_cast<uint32_t>(kBM >> 4) << 24);
}

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

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                         uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(acc)
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

// 16 consecutive accumulator columns of this thread's lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
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

// The columns of a vocabulary part: kUnit-column units split evenly over the
// parts, so that parts differ by at most one unit; tiles of kBN columns from
// the part's start, the last one narrower.
struct PartSpan {
    uint32_t c0, cend, ntiles;
};
__host__ __device__ inline PartSpan part_span(uint32_t vocab, uint32_t part, uint32_t parts) {
    const uint64_t nunits = (vocab + kUnit - 1) / kUnit;
    const uint32_t u0 = static_cast<uint32_t>(nunits * part / parts);
    const uint32_t u1 = static_cast<uint32_t>(nunits * (part + 1) / parts);
    PartSpan s;
    s.c0 = u0 * kUnit;
    s.cend = u1 * kUnit;
    s.ntiles = (s.cend - s.c0 + kBN - 1) / kBN;
    return s;
}

// One warp cuts row rr's list to the entries whose key is at least a floor
// with at least k entries at or above it (so the floor is at most the list's
// k-th largest key). The bitwise search over the key stops as soon as the
// count at the floor is within k + slack. Returns the floor; n becomes the
// number of entries kept, in place and in list order.
__device__ __forceinline__ uint32_t warp_cut_row(uint32_t *lkey, uint16_t *lidx, uint32_t rr,
                                                 uint32_t &n, uint32_t k, uint32_t slack,
                                                 uint32_t KS = kKeyStride, uint32_t IS = kIdxStride) {
    const uint32_t lane = threadIdx.x & 31u;
    uint32_t key[3];
    uint16_t idx[3];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        const uint32_t e = lane + 32u * i;
        // Key 0 is a negative NaN pattern: never a candidate, never counted.
        key[i] = e < n ? lkey[e * KS + rr] : 0u;
        idx[i] = e < n ? lidx[e * IS + rr] : static_cast<uint16_t>(0);
    }
    uint32_t floor_key = 0;
    for (int bit = 31; bit >= 0; --bit) {
        const uint32_t cand = floor_key | (1u << bit);
        const uint32_t c = __reduce_add_sync(0xffffffffu, (key[0] >= cand ? 1u : 0u) +
                                                              (key[1] >= cand ? 1u : 0u) +
                                                              (key[2] >= cand ? 1u : 0u));
        if (c >= k) {
            floor_key = cand;
            if (c <= k + slack) break;
        }
    }
    // +0 as the floor would cut -0, which IEEE >= keeps beside +0.
    if (floor_key == kKeyPosZero) floor_key = kKeyNegZero;
    const uint32_t lt = (1u << lane) - 1u;
    uint32_t base = 0;
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        const bool keep = key[i] >= floor_key && key[i] != 0u;
        const uint32_t ball = __ballot_sync(0xffffffffu, keep);
        if (keep) {
            const uint32_t pos = base + __popc(ball & lt);
            lkey[pos * KS + rr] = key[i];
            lidx[pos * IS + rr] = idx[i];
        }
        base += __popc(ball);
    }
    __syncwarp();
    n = base;
    return floor_key;
}

template <bool kFused>
__global__ void __launch_bounds__(kGThreads, 1)
lmhead_kernel(const __grid_constant__ CUtensorMap map_h, const __grid_constant__ CUtensorMap map_w,
              const __grid_constant__ CUtensorMap map_w16, uint32_t rows, uint32_t dim,
              uint32_t vocab, CallParams cp, float *__restrict__ logits, bool vec_out,
              unsigned char *__restrict__ records, size_t rec_bytes, uint32_t index_offset,
              uint32_t *__restrict__ error_out) {
    extern __shared__ unsigned char smem_raw[];
    LmSmem &sm = *reinterpret_cast<LmSmem *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~static_cast<uintptr_t>(1023u));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t part = blockIdx.x, parts = gridDim.x;
    const uint32_t m0 = blockIdx.y * kBM;
    const PartSpan span = part_span(vocab, part, parts);
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
            for (uint32_t t = 0; t < span.ntiles && ok; ++t) {
                const uint32_t c = span.c0 + t * kBN;
                const uint32_t w = min(static_cast<uint32_t>(kBN), span.cend - c);
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
                    // Full boxes count their out-of-range (zero-filled) elements.
                    mbar_arrive_expect_tx(&sm.full[s], static_cast<uint32_t>(sizeof(sm.a[0])) +
                                                           w * kBK * static_cast<uint32_t>(sizeof(__nv_bfloat16)));
                    const int32_t x = static_cast<int32_t>(kb * kBK);
                    tma_load_2d(sm.a[s], &map_h, &sm.full[s], x, static_cast<int32_t>(m0));
                    if (w == static_cast<uint32_t>(kBN)) {
                        tma_load_2d(sm.b[s], &map_w, &sm.full[s], x, static_cast<int32_t>(c));
                    } else {
                        // A narrow tile: 16-row boxes stacked at 2 KiB steps keep
                        // the 128-byte swizzle phase of a full box.
                        for (uint32_t i = 0; i < w / kUnit; ++i)
                            tma_load_2d(sm.b[s] + i * kUnit * kBK, &map_w16, &sm.full[s], x,
                                        static_cast<int32_t>(c + i * kUnit));
                    }
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
            for (uint32_t t = 0; t < span.ntiles && ok; ++t) {
                const uint32_t buf = t & 1u;
                const uint32_t w = min(static_cast<uint32_t>(kBN), span.cend - (span.c0 + t * kBN));
                const uint32_t idesc = idesc_for(w);
                if (t >= 2 && !mbar_wait(&sm.acc_empty[buf], ((t >> 1) - 1u) & 1u)) {
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
                        mma_bf16(d, smem_desc(sa + off), smem_desc(sb + off), idesc, (kb | kk) ? 1u : 0u);
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
        const bool row_ok = grow < rows;
        const float scale = cp.scale;
        const uint32_t k = cp.top_k;
        // Row state, in the owning thread's registers: the part's maximum, the
        // number of listed candidates, and the admission bound (NaN admits
        // nothing: padding rows and rows whose ties overflowed the list).
        float vmax = kNegInf;
        uint32_t cnt = 0;
        bool ovf = false;
        float tau = row_ok ? -3.402823466e38f : __int_as_float(0x7fffffff);
        for (uint32_t t = 0; t < span.ntiles; ++t) {
            const uint32_t buf = t & 1u;
            const uint32_t c = span.c0 + t * kBN;
            const uint32_t w = min(static_cast<uint32_t>(kBN), span.cend - c);
            bool got = mbar_wait(&sm.acc_full[buf], (t >> 1) & 1u);
            if (__any_sync(0xffffffffu, !got) || *err) {
                if (lane == 0) *err = 1u;
                break;
            }
            tc_fence_after();
            if (!kFused) {
                for (uint32_t cc = 0; cc < w; cc += 32) {
                    uint32_t v[32];
                    tmem_ld32(tmem + buf * kBN + cc + (lane_base << 16), v);
                    if (row_ok) {
                        const uint32_t col0 = c + cc;
                        const uint32_t lim = min(min(32u, w - cc), vocab - min(vocab, col0));
                        float *dst = logits + static_cast<size_t>(grow) * vocab + col0;
                        if (vec_out && lim == 32u) {
#pragma unroll
                            for (int q = 0; q < 32; q += 4)
                                *reinterpret_cast<float4 *>(dst + q) =
                                    make_float4(__uint_as_float(v[q]), __uint_as_float(v[q + 1]),
                                                __uint_as_float(v[q + 2]), __uint_as_float(v[q + 3]));
                        } else {
#pragma unroll
                            for (int q = 0; q < 32; ++q)
                                if (static_cast<uint32_t>(q) < lim) dst[q] = __uint_as_float(v[q]);
                        }
                    }
                }
            } else {
                if (t == 0) {
                    // First tile of the part: a starting bound for each row.
                    // Its columns fall into 48 disjoint groups (column within a
                    // 16-column step, step mod 3); the smallest of the 48 group
                    // maxima has 48 distinct values at or above it, so it is at
                    // most the part's k-th largest value (k <= 48). An empty
                    // group leaves the bound at -inf.
                    float gm[3][kChunkCols];
#pragma unroll
                    for (int g = 0; g < 3; ++g)
#pragma unroll
                        for (int q = 0; q < static_cast<int>(kChunkCols); ++q) gm[g][q] = kNegInf;
                    for (uint32_t cc = 0, step = 0; cc < w; cc += kChunkCols, ++step) {
                        uint32_t v[kChunkCols];
                        tmem_ld16(tmem + buf * kBN + cc + (lane_base << 16), v);
                        const uint32_t g = step % 3u;
#pragma unroll
                        for (int q = 0; q < static_cast<int>(kChunkCols); ++q) {
                            const float x = c + cc + q < vocab ? scale_logit(__uint_as_float(v[q]), scale)
                                                               : kNegInf;
                            if (g == 0) gm[0][q] = fmaxf(gm[0][q], x);
                            else if (g == 1) gm[1][q] = fmaxf(gm[1][q], x);
                            else gm[2][q] = fmaxf(gm[2][q], x);
                        }
                    }
                    float b = kPosInf;
#pragma unroll
                    for (int g = 0; g < 3; ++g)
#pragma unroll
                        for (int q = 0; q < static_cast<int>(kChunkCols); ++q) b = fminf(b, gm[g][q]);
                    if (k <= 3u * kChunkCols && b > tau) tau = b;
                }
                for (uint32_t cc = 0; cc < w; cc += kChunkCols) {
                    // Room for a whole chunk: rows near the cap are cut first,
                    // one at a time by the whole warp.
                    uint32_t need = __ballot_sync(0xffffffffu, !ovf && cnt > kListCap - kChunkCols);
                    while (need) {
                        const int i = __ffs(need) - 1;
                        need &= need - 1u;
                        uint32_t n = __shfl_sync(0xffffffffu, cnt, i);
                        const uint32_t fk = warp_cut_row(sm.lkey, sm.lidx, lane_base + i, n, k, kFloorSlack);
                        if (lane == i) {
                            cnt = n;
                            const float f = key_to_float(fk);
                            if (f > tau) tau = f;
                            if (cnt > kListCap - kChunkCols) {
                                // More ties at the k-th value than the list
                                // holds: the row is reported, not sampled.
                                ovf = true;
                                tau = __int_as_float(0x7fffffff);
                            }
                        }
                    }
                    uint32_t v[kChunkCols];
                    tmem_ld16(tmem + buf * kBN + cc + (lane_base << 16), v);
                    const uint32_t col0 = c + cc;
                    float x[kChunkCols];
                    bool any = false;
#pragma unroll
                    for (int q = 0; q < static_cast<int>(kChunkCols); ++q) {
                        x[q] = scale_logit(__uint_as_float(v[q]), scale);
                        if (col0 + q < vocab) {
                            vmax = fmaxf(vmax, x[q]);
                            any |= x[q] >= tau;
                        }
                    }
                    if (any) {
#pragma unroll
                        for (int q = 0; q < static_cast<int>(kChunkCols); ++q) {
                            if (col0 + q < vocab && x[q] >= tau) {
                                sm.lkey[cnt * kKeyStride + r] = total_key(x[q]);
                                sm.lidx[cnt * kIdxStride + r] = static_cast<uint16_t>(col0 + q - span.c0);
                                ++cnt;
                            }
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
        }
        if (kFused) {
            // The record of each (part, row) of the warp: the part's entries at
            // or above a floor no higher than its own k-th largest value (ties
            // included, at most k + RSC_SHARD_TIE_CAP), so that merges over
            // many parts stay small.
            const uint32_t cap = k + RSC_SHARD_TIE_CAP;
            __syncwarp();
            for (uint32_t i = 0; i < 32u; ++i) {
                const uint32_t rr = lane_base + i;
                const uint32_t gr = m0 + rr;
                if (gr >= rows) break;
                uint32_t n = __shfl_sync(0xffffffffu, cnt, static_cast<int>(i));
                bool o = __shfl_sync(0xffffffffu, ovf ? 1u : 0u, static_cast<int>(i)) != 0u;
                float rt = __shfl_sync(0xffffffffu, tau, static_cast<int>(i));
                const float rmax = __shfl_sync(0xffffffffu, vmax, static_cast<int>(i));
                if (!o && n > cap) {
                    const uint32_t fk = warp_cut_row(sm.lkey, sm.lidx, rr, n, k, kFloorSlack);
                    const float f = key_to_float(fk);
                    if (f > rt) rt = f;
                    if (n > cap) o = true;
                }
                unsigned char *rec = records + (static_cast<size_t>(part) * rows + gr) * rec_bytes;
                ShardRecordHeader *h = reinterpret_cast<ShardRecordHeader *>(rec);
                uint32_t *rkey = reinterpret_cast<uint32_t *>(rec + sizeof(ShardRecordHeader));
                uint32_t *ridx = rkey + cap;
                const uint32_t nw = o ? 0u : n;
                for (uint32_t e = lane; e < nw; e += 32u) {
                    rkey[e] = sm.lkey[e * kKeyStride + rr];
                    ridx[e] = index_offset + span.c0 + sm.lidx[e * kIdxStride + rr];
                }
                if (lane == 0) {
                    h->max_scaled = rmax;
                    h->sum_exp = 0.0f;
                    h->n_finite = 0;
                    h->n_cand = nw;
                    h->n_dropped = 0;
                    h->last_key = 0;
                    h->flags = (o || *err) ? 1u : 0u;
                    h->tau = o ? -3.402823466e38f : rt;
                }
                __syncwarp();
            }
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

// --- decode-sized batches: operands swapped --------------------------------
//
// For rows <= kSN the tensor cores compute the transposed product: A is a
// tile of up to 128 vocabulary rows of W, B the whole batch of hidden states
// (N = rows rounded up to 16), so that an accumulator holds 128 vocabulary
// entries (lanes) by the batch (columns). A stage then carries 16 KiB of W
// and at most 8 KiB of H, and 6 (64 rows) to 11 (16 rows) stages stream the
// weights. The epilogue
// transposes each tile through shared memory, and warp e of the epilogue
// owns the batch rows b = e (mod 4): it filters the tile's 128 values of its
// rows (4 per lane, ballot appends) into the rows' lists, with the same cuts
// and records as the row-tile kernel.
constexpr int kSN = 64;                       // batch rows of the swapped path (MMA N <= 64)
constexpr uint32_t kSMaxStages = 16;
constexpr uint32_t kSTmemCols = 2 * kSN;
constexpr uint32_t kSWStage = kBM * kBK * sizeof(__nv_bfloat16);  // 16 KiB of W per stage
constexpr uint32_t kMaxDynSmem = 232448;                           // 227 KiB per CTA
constexpr uint32_t kSAtoms = 2;                                    // 64-column k atoms per stage

// Row state and barriers, after the ring and the buffers.
struct SmallHead {
    float rtau[kSN];  // per batch row: bound, count, overflow, max key
    uint32_t rcnt[kSN];
    uint32_t rovf[kSN];
    uint32_t rmaxkey[kSN];
    uint64_t full[kSMaxStages];
    uint64_t empty[kSMaxStages];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint32_t tmem_base;
    uint32_t error;
};

// Shared memory of the swapped path, sized for the batch (n_pad rows): nst
// ring stages of W (16 KiB) and H (n_pad x 128 B), the tile transpose
// [n_pad][128] f32, the lists with slot strides n_pad + 1 (keys) and
// n_pad + 2 (indices: odd word strides keep a row's slots in distinct banks),
// then the head. Everything a batch does not use goes to more stages: the
// weights in flight per SM bound this kernel.
struct SmallLayout {
    uint32_t nst, apb, wb, hb, ks, is;
    uint32_t off_h, off_tb, off_key, off_idx, off_head, bytes;
};
// apb: 64-column k atoms per stage, so that a stage reads apb * 128
// contiguous bytes of each weight row.
__host__ __device__ inline SmallLayout small_layout(uint32_t n_pad, uint32_t nst, uint32_t apb) {
    SmallLayout L;
    L.nst = nst;
    L.apb = apb;
    L.wb = apb * kSWStage;
    L.hb = apb * n_pad * kBK * static_cast<uint32_t>(sizeof(__nv_bfloat16));
    L.ks = n_pad + 1;
    L.is = n_pad + 2;
    L.off_h = nst * L.wb;
    L.off_tb = L.off_h + nst * L.hb;
    L.off_key = L.off_tb + n_pad * kBM * 4u;
    L.off_idx = L.off_key + kListCap * L.ks * 4u;
    L.off_head = (L.off_idx + kListCap * L.is * 2u + 15u) & ~15u;
    L.bytes = L.off_head + static_cast<uint32_t>(sizeof(SmallHead)) + 1024u;  // + alignment slack
    return L;
}
// The most stages that fit (at least 2).
inline uint32_t small_stages(uint32_t n_pad, uint32_t apb) {
    uint32_t nst = kSMaxStages;
    while (nst > 2 && small_layout(n_pad, nst, apb).bytes > kMaxDynSmem) --nst;
    return nst;
}

// Tile t of a part's span in the swapped path: full 128-column tiles from
// the part's start, the last one narrower. (Splitting a part evenly into
// tiles of 112 and 128 columns made most tiles narrow; a narrow tile's
// 16-row boxes stream at two thirds of the rate of full boxes.)
__device__ __forceinline__ void small_tile(const PartSpan &sp, uint32_t t, uint32_t &c, uint32_t &w) {
    c = sp.c0 + t * kBM;
    w = min(static_cast<uint32_t>(kBM), sp.cend - c);
}
__host__ __device__ inline uint32_t small_tiles(const PartSpan &sp) {
    const uint32_t units = (sp.cend - sp.c0) / kUnit;
    return (units + kBM / kUnit - 1) / (kBM / kUnit);
}

// Named barrier 1 over the 128 epilogue threads, plain and with an OR vote.
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
__device__ __forceinline__ bool epi_bar_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, 1, 128, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"(v ? 1u : 0u)
        : "memory");
    return r != 0u;
}

template <bool kFused>
__global__ void __launch_bounds__(kGThreads, 1)
lmhead_small_kernel(const __grid_constant__ CUtensorMap map_h, const __grid_constant__ CUtensorMap map_w,
                    const __grid_constant__ CUtensorMap map_w16, uint32_t rows, uint32_t n_pad,
                    uint32_t nst, uint32_t apb, uint32_t dim, uint32_t vocab, CallParams cp,
                    float *__restrict__ logits, unsigned char *__restrict__ records,
                    size_t rec_bytes, uint32_t index_offset, uint32_t *__restrict__ error_out) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char *base = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~static_cast<uintptr_t>(1023u));
    const SmallLayout lay = small_layout(n_pad, nst, apb);
    SmallHead &sm = *reinterpret_cast<SmallHead *>(base + lay.off_head);
    float *tb = reinterpret_cast<float *>(base + lay.off_tb);
    uint32_t *lkey = reinterpret_cast<uint32_t *>(base + lay.off_key);
    uint16_t *lidx = reinterpret_cast<uint16_t *>(base + lay.off_idx);
    const uint32_t ks = lay.ks, is = lay.is;
    auto wst = [&](uint32_t s) { return reinterpret_cast<__nv_bfloat16 *>(base + s * lay.wb); };
    auto hst = [&](uint32_t s) { return reinterpret_cast<__nv_bfloat16 *>(base + lay.off_h + s * lay.hb); };
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t part = blockIdx.x, parts = gridDim.x;
    PartSpan span = part_span(vocab, part, parts);
    span.ntiles = small_tiles(span);
    const uint32_t kblocks = (dim + kBK * apb - 1) / (kBK * apb);

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < nst; ++s) {
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
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_addr(&sm.tmem_base)),
                     "r"(kSTmemCols)
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
            const uint32_t hbytes = n_pad * kBK * static_cast<uint32_t>(sizeof(__nv_bfloat16));
            for (uint32_t t = 0; t < span.ntiles && ok; ++t) {
                uint32_t c, w;
                small_tile(span, t, c, w);
                for (uint32_t kb = 0; kb < kblocks; ++kb, ++it) {
                    const uint32_t s = it % nst;
                    if (it >= nst && !mbar_wait(&sm.empty[s], ((it / nst) - 1u) & 1u)) {
                        *err = 1u;
                        ok = false;
                        break;
                    }
                    if (*err) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&sm.full[s], apb * (hbytes + w * kBK * static_cast<uint32_t>(
                                                                                  sizeof(__nv_bfloat16))));
                    for (uint32_t a = 0; a < apb; ++a) {
                        // Atoms past dim read zeros (out-of-range boxes).
                        const int32_t x = static_cast<int32_t>((kb * apb + a) * kBK);
                        __nv_bfloat16 *wa = wst(s) + a * kBM * kBK;
                        tma_load_2d(hst(s) + a * n_pad * kBK, &map_h, &sm.full[s], x, 0);
                        if (w == static_cast<uint32_t>(kBM)) {
                            tma_load_2d(wa, &map_w, &sm.full[s], x, static_cast<int32_t>(c));
                        } else {
                            for (uint32_t i = 0; i < w / kUnit; ++i)
                                tma_load_2d(wa + i * kUnit * kBK, &map_w16, &sm.full[s], x,
                                            static_cast<int32_t>(c + i * kUnit));
                        }
                    }
                }
            }
            const uint32_t first = it > nst ? it - nst : 0u;
            for (uint32_t i = first; i < it; ++i) mbar_wait(&sm.full[i % nst], (i / nst) & 1u);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            const uint32_t idesc = idesc_for(n_pad);
            for (uint32_t t = 0; t < span.ntiles && ok; ++t) {
                const uint32_t buf = t & 1u;
                if (t >= 2 && !mbar_wait(&sm.acc_empty[buf], ((t >> 1) - 1u) & 1u)) {
                    *err = 1u;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + buf * kSN;
                for (uint32_t kb = 0; kb < kblocks; ++kb, ++it) {
                    const uint32_t s = it % nst;
                    if (!mbar_wait(&sm.full[s], (it / nst) & 1u) || *err) {
                        *err = 1u;
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    for (uint32_t a = 0; a < apb; ++a) {
                        const uint32_t sa = smem_addr(wst(s) + a * kBM * kBK);
                        const uint32_t sb = smem_addr(hst(s) + a * n_pad * kBK);
#pragma unroll
                        for (int kk = 0; kk < kBK / kUK; ++kk) {
                            const uint32_t off = static_cast<uint32_t>(kk * kUK * sizeof(__nv_bfloat16));
                            mma_bf16(d, smem_desc(sa + off), smem_desc(sb + off), idesc,
                                     (kb | a | static_cast<uint32_t>(kk)) ? 1u : 0u);
                        }
                    }
                    mma_commit(&sm.empty[s]);
                }
                if (ok) mma_commit(&sm.acc_full[buf]);
            }
            if (it > 0) mbar_wait(&sm.empty[(it - 1) % nst], ((it - 1) / nst) & 1u);
        }
    } else {
        // Epilogue: thread (warp, lane) reads tensor-memory lane 32 * (warp % 4)
        // + lane, vocabulary row v of the tile, for every batch row.
        const uint32_t q = static_cast<uint32_t>(warp) & 3u;
        const uint32_t ew = static_cast<uint32_t>(warp) - 2u;  // owns batch rows ew + 4j
        const uint32_t v = 32u * q + lane;
        const float scale = cp.scale;
        const uint32_t k = cp.top_k;
        if (kFused) {
            for (uint32_t b = ew; b < static_cast<uint32_t>(kSN); b += 4u) {
                if (lane == 0) {
                    sm.rtau[b] = -3.402823466e38f;
                    sm.rcnt[b] = 0;
                    sm.rovf[b] = 0;
                    sm.rmaxkey[b] = total_key(kNegInf);
                }
            }
            __syncwarp();
        }
        for (uint32_t t = 0; t < span.ntiles; ++t) {
            const uint32_t buf = t & 1u;
            uint32_t c, w;
            small_tile(span, t, c, w);
            const uint32_t col = c + v;
            const bool valid = v < w && col < vocab;
            const bool got = mbar_wait(&sm.acc_full[buf], (t >> 1) & 1u);
            // The fused epilogue's warps meet at named barriers, so they give
            // up together (a vote) or not at all.
            const bool bad = kFused ? epi_bar_or(!got || *err != 0u)
                                    : __any_sync(0xffffffffu, !got) || *err != 0u;
            if (bad) {
                if (lane == 0) *err = 1u;
                break;
            }
            tc_fence_after();
            if (!kFused) {
                for (uint32_t cb = 0; cb < n_pad; cb += 16) {
                    uint32_t r16[16];
                    tmem_ld16(tmem + buf * kSN + cb + ((32u * q) << 16), r16);
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const uint32_t b = cb + j;
                        if (valid && b < rows) logits[static_cast<size_t>(b) * vocab + col] = __uint_as_float(r16[j]);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
            } else {
            for (uint32_t cb = 0; cb < n_pad; cb += 16) {
                uint32_t r16[16];
                tmem_ld16(tmem + buf * kSN + cb + ((32u * q) << 16), r16);
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    tb[(cb + j) * kBM + v] = valid ? scale_logit(__uint_as_float(r16[j]), scale) : kNegInf;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
            epi_bar();  // the tile's values are in tb
            const uint32_t steps = (w + 31u) / 32u;
            for (uint32_t b = ew; b < rows; b += 4u) {
                if (sm.rovf[b]) continue;
                float tau = sm.rtau[b];
                uint32_t cnt = sm.rcnt[b];
                bool ovf = false;
                float lmax = kNegInf;
                for (uint32_t i = 0; i < steps; ++i) {
                    if (cnt > kListCap - 32u) {
                        uint32_t n = cnt;
                        const uint32_t fk = warp_cut_row(lkey, lidx, b, n, k, kFloorSlack, ks, is);
                        cnt = n;
                        const float f = key_to_float(fk);
                        if (f > tau) tau = f;
                        if (cnt > kListCap - 32u) {
                            // More ties at the k-th value than the list holds.
                            ovf = true;
                            break;
                        }
                    }
                    const uint32_t vi = lane + 32u * i;
                    const float x = tb[b * kBM + vi];
                    lmax = fmaxf(lmax, x);
                    const bool take = x >= tau;
                    const uint32_t ball = __ballot_sync(0xffffffffu, take);
                    if (take) {
                        const uint32_t pos = cnt + __popc(ball & ((1u << lane) - 1u));
                        lkey[pos * ks + b] = total_key(x);
                        lidx[pos * is + b] = static_cast<uint16_t>(c + vi - span.c0);
                    }
                    cnt += __popc(ball);
                    __syncwarp();
                }
                const uint32_t mk = __reduce_max_sync(0xffffffffu, total_key(lmax));
                if (lane == 0) {
                    sm.rtau[b] = tau;
                    sm.rcnt[b] = cnt;
                    sm.rovf[b] = ovf ? 1u : 0u;
                    if (mk > sm.rmaxkey[b]) sm.rmaxkey[b] = mk;
                }
                __syncwarp();
            }
            epi_bar();  // tb is free for the next tile
            }
        }
        if (kFused) {
            const uint32_t cap = k + RSC_SHARD_TIE_CAP;
            for (uint32_t b = ew; b < rows; b += 4u) {
                uint32_t n = sm.rcnt[b];
                bool o = sm.rovf[b] != 0u;
                float rt = sm.rtau[b];
                if (!o && n > cap) {
                    const uint32_t fk = warp_cut_row(lkey, lidx, b, n, k, kFloorSlack, ks, is);
                    const float f = key_to_float(fk);
                    if (f > rt) rt = f;
                    if (n > cap) o = true;
                }
                unsigned char *rec = records + (static_cast<size_t>(part) * rows + b) * rec_bytes;
                ShardRecordHeader *h = reinterpret_cast<ShardRecordHeader *>(rec);
                uint32_t *rkey = reinterpret_cast<uint32_t *>(rec + sizeof(ShardRecordHeader));
                uint32_t *ridx = rkey + cap;
                const uint32_t nw = o ? 0u : n;
                for (uint32_t e = lane; e < nw; e += 32u) {
                    rkey[e] = lkey[e * ks + b];
                    ridx[e] = index_offset + span.c0 + lidx[e * is + b];
                }
                if (lane == 0) {
                    h->max_scaled = key_to_float(sm.rmaxkey[b]);
                    h->sum_exp = 0.0f;
                    h->n_finite = 0;
                    h->n_cand = nw;
                    h->n_dropped = 0;
                    h->last_key = 0;
                    h->flags = (o || *err) ? 1u : 0u;
                    h->tau = o ? -3.402823466e38f : rt;
                }
                __syncwarp();
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kSTmemCols)
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
    // Swapped operands (rows <= kSN): one part per SM, tiles of 128 columns;
    // row tiles otherwise: the SMs shared among the row tiles.
    const uint32_t ntiles = rows <= static_cast<size_t>(kSN) ? (vocab + kBM - 1) / kBM
                                                              : (vocab + kBN - 1) / kBN;
    size_t p = rows <= static_cast<size_t>(kSN) ? static_cast<size_t>(num_sms)
               : mtiles                         ? static_cast<size_t>(num_sms) / mtiles
                                                : 1;
    if (p < 1) p = 1;
    if (p > ntiles) p = ntiles;
    // Candidate indices are kept relative to the part's first column in 16
    // bits: no part spans more than 65536 columns.
    const size_t nunits = (vocab + kUnit - 1) / kUnit;
    const size_t min_parts = (nunits + 4095) / 4096;
    if (p < min_parts) p = min_parts;
    if (p > kLmheadMaxParts) p = kLmheadMaxParts;
    return static_cast<uint32_t>(p);
}

cudaError_t launch_lmhead(const void *hidden, const void *weight, size_t rows, uint32_t dim,
                          uint32_t vocab, const CallParams &p, float *logits, void *records,
                          size_t rec_bytes, uint32_t parts, uint32_t *error_flag,
                          cudaStream_t stream, uint32_t index_offset) {
    if (rows == 0) return cudaSuccess;
    if ((static_cast<uint64_t>(vocab) + kUnit - 1) / kUnit > static_cast<uint64_t>(parts) * 4096u)
        return cudaErrorInvalidValue;  // a part would span more than 65536 columns
    CUtensorMap mh, mw, mw16;
    if (rows <= static_cast<size_t>(kSN)) {
        const uint32_t n_pad = static_cast<uint32_t>((rows + 15) / 16 * 16);
        // Two k atoms per stage: 256 contiguous bytes of each weight row. One
        // atom streamed the weights at 4.7 TB/s, two at 6.1 TB/s (1 row);
        // four fit only 2 stages and gained nothing.
        const uint32_t apb = kSAtoms;
        if (small_layout(n_pad, 2, apb).bytes > kMaxDynSmem) return cudaErrorInvalidValue;
        const uint32_t nst = small_stages(n_pad, apb);
        const uint32_t smem = small_layout(n_pad, nst, apb).bytes;
        if (!make_map(&mh, hidden, rows, dim, n_pad) || !make_map(&mw, weight, vocab, dim, kBM) ||
            !make_map(&mw16, weight, vocab, dim, kUnit))
            return cudaErrorInvalidValue;
        const dim3 grid(parts, 1, 1);
        if (logits) {
            cudaError_t e = cudaFuncSetAttribute(lmhead_small_kernel<false>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(kMaxDynSmem));
            if (e != cudaSuccess) return e;
            lmhead_small_kernel<false><<<grid, kGThreads, smem, stream>>>(
                mh, mw, mw16, static_cast<uint32_t>(rows), n_pad, nst, apb, dim, vocab, p, logits, nullptr,
                0, index_offset, error_flag);
        } else {
            cudaError_t e = cudaFuncSetAttribute(lmhead_small_kernel<true>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(kMaxDynSmem));
            if (e != cudaSuccess) return e;
            lmhead_small_kernel<true><<<grid, kGThreads, smem, stream>>>(
                mh, mw, mw16, static_cast<uint32_t>(rows), n_pad, nst, apb, dim, vocab, p, nullptr,
                static_cast<unsigned char *>(records), rec_bytes, index_offset, error_flag);
        }
        return cudaGetLastError();
    }
    if (!make_map(&mh, hidden, rows, dim, kBM) || !make_map(&mw, weight, vocab, dim, kBN) ||
        !make_map(&mw16, weight, vocab, dim, kUnit))
        return cudaErrorInvalidValue;
    const dim3 grid(parts, static_cast<unsigned>((rows + kBM - 1) / kBM), 1);
    if (logits) {
        cudaError_t e = cudaFuncSetAttribute(lmhead_kernel<false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kLmSmemBytes));
        if (e != cudaSuccess) return e;
        const bool vec = vocab % 4 == 0 && (reinterpret_cast<uintptr_t>(logits) & 15u) == 0;
        lmhead_kernel<false><<<grid, kGThreads, kLmSmemBytes, stream>>>(
            mh, mw, mw16, static_cast<uint32_t>(rows), dim, vocab, p, logits, vec, nullptr, 0,
            index_offset, error_flag);
    } else {
        cudaError_t e = cudaFuncSetAttribute(lmhead_kernel<true>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kLmSmemBytes));
        if (e != cudaSuccess) return e;
        lmhead_kernel<true><<<grid, kGThreads, kLmSmemBytes, stream>>>(
            mh, mw, mw16, static_cast<uint32_t>(rows), dim, vocab, p, nullptr, false,
            static_cast<unsigned char *>(records), rec_bytes, index_offset, error_flag);
    }
    return cudaGetLastError();
}

}  // namespace rsc
