// Large-survivor sampler: Sampler::sample_logits
// (crates/rusticide-sampling/src/sampler.rs:44-54) for rows whose surviving
// set is too large for shared memory (top-k disabled on a wide row, or a
// threshold tied by thousands of logits), every row of a call whose scale can
// create NaN (T = +inf, or T so small that 1/T overflows), and
// Sampler::sample_with_temp (sampler.rs:97-105).
//
// One CTA per row. The row stays in global memory (L2-resident while the CTA
// works on it) and is re-read per pass:
//  1. top-k threshold: radix select of the k-th largest total-order key over
//     the whole row (candidates.rs:38-43, 93-97);
//  2. top-p: the survivors are compacted in index order into scratch and
//     stably radix-sorted by descending key, which is the reference's
//     (value desc, index asc) order; exp_sum and the cut-off running sum are
//     replayed exactly over that order (candidates.rs:55-78). The kept set is
//     "key above the last kept key, or equal to it with index up to its index";
//  3. softmax: the maximum, then the exact index-order sum of exp(v - max)
//     (filters.rs:5-15), non-survivors adding +0;
//  4. argmax (last maximum) or the draw: the exact index-order running sum of
//     the probabilities, stopping at the first r < cumsum
//     (sampler.rs:111-121), falling back to the last survivor.
// The sums use block_replay, which reproduces the sequential binary32 loop
// bit for bit.
#include "rsc_block.cuh"
#include "rsc_kernels.h"

namespace rsc {

namespace {

constexpr int kThreads = 512;
constexpr int kItems = 4;
constexpr int kWarps = kThreads / 32;

struct LargeSmem {
    double exp_tab[32];
    uint32_t hist[256];
    uint32_t sel[2];
    uint32_t red32[32];
    unsigned long long red64[32];
    float redf[32];
    ReplaySmem rs;
    uint32_t wcount[kWarps][256];
    uint32_t base[256];
    uint32_t tile_total[256];
    uint32_t bcast[4];
};

struct RowView {
    const float *p;
    uint32_t n;
    float scale;
    bool with_temp;  // sample_with_temp: every position takes part, no filters

    __device__ __forceinline__ float value(uint32_t i) const {
        if (with_temp) {
            // extract_logits (logits.rs:14-18) then apply_temperature
            // (filters.rs:17-22): NaN -> -inf, then x * (1/T) for any T.
            float x = p[i];
            float l = (x != x) ? kNegInf : x;
            float v = __fmul_rn(l, scale);
            if (v != v) v = __uint_as_float(kX86DefaultNaN);
            return v;
        }
        return scale_logit(p[i], scale);
    }
};

// Stable LSD radix sort (4 passes of 8 bits) of n (key, idx) pairs by key
// ascending, ping-ponging between (ka, ia) and (kb, ib); the result ends in
// (ka, ia). Within a tile, warp w owns 32 * kItems consecutive items in
// striped order, so processing j-major keeps the input order per digit.
__device__ void block_radix_sort(uint32_t *ka, uint32_t *ia, uint32_t *kb, uint32_t *ib,
                                 uint32_t n, LargeSmem &sm) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr uint32_t kTile = kThreads * kItems;
    const uint32_t lt_mask = (1u << lane) - 1u;
    uint32_t *kin = ka, *iin = ia, *kout = kb, *iout = ib;
    for (int shift = 0; shift < 32; shift += 8) {
        for (int b = threadIdx.x; b < 256; b += kThreads) sm.hist[b] = 0;
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < n; i += kThreads)
            atomicAdd(&sm.hist[(kin[i] >> shift) & 255u], 1u);
        __syncthreads();
        if (threadIdx.x < 32) {
            uint32_t c[8], tot = 0;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                c[q] = sm.hist[8 * lane + q];
                tot += c[q];
            }
            uint32_t incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            uint32_t run = incl - tot;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                sm.base[8 * lane + q] = run;
                run += c[q];
            }
        }
        __syncthreads();
        for (uint32_t t0 = 0; t0 < n; t0 += kTile) {
            for (int b = lane; b < 256; b += 32) sm.wcount[warp][b] = 0;
            __syncwarp();
            const uint32_t wbase = t0 + static_cast<uint32_t>(warp) * 32u * kItems;
            uint32_t kk[kItems], ii[kItems], dg[kItems];
#pragma unroll
            for (int j = 0; j < kItems; ++j) {
                uint32_t i = wbase + static_cast<uint32_t>(j) * 32u + lane;
                bool in = i < n;
                kk[j] = in ? kin[i] : 0u;
                ii[j] = in ? iin[i] : 0u;
                dg[j] = in ? ((kk[j] >> shift) & 255u) : 256u;
                uint32_t peers = __match_any_sync(0xffffffffu, dg[j]);
                if (in && lane == __ffs(peers) - 1) sm.wcount[warp][dg[j]] += __popc(peers);
                __syncwarp();
            }
            __syncthreads();
            // Exclusive prefix of the per-warp counts for each digit.
            for (int b = threadIdx.x; b < 256; b += kThreads) {
                uint32_t run = 0;
#pragma unroll
                for (int w = 0; w < kWarps; ++w) {
                    uint32_t c = sm.wcount[w][b];
                    sm.wcount[w][b] = run;
                    run += c;
                }
                sm.tile_total[b] = run;
            }
            __syncthreads();
#pragma unroll
            for (int j = 0; j < kItems; ++j) {
                uint32_t peers = __match_any_sync(0xffffffffu, dg[j]);
                if (dg[j] < 256u) {
                    uint32_t pos = sm.base[dg[j]] + sm.wcount[warp][dg[j]] + __popc(peers & lt_mask);
                    kout[pos] = kk[j];
                    iout[pos] = ii[j];
                }
                __syncwarp();
                if (dg[j] < 256u && lane == __ffs(peers) - 1) sm.wcount[warp][dg[j]] += __popc(peers);
                __syncwarp();
            }
            __syncthreads();
            for (int b = threadIdx.x; b < 256; b += kThreads) sm.base[b] += sm.tile_total[b];
            __syncthreads();
        }
        uint32_t *t = kin;
        kin = kout;
        kout = t;
        t = iin;
        iin = iout;
        iout = t;
    }
    // Four passes: the result is back in (ka, ia).
}

__device__ void large_row(const CallParams &cp, const RowView &rv, size_t row, uint32_t *scratch,
                          uint32_t *out_ids, int32_t *out_status, float *out_probs,
                          LargeSmem &sm) {
    const uint32_t n = rv.n;
    const bool with_temp = rv.with_temp;

    // --- top-k threshold (candidates.rs:38-43) --------------------------------
    float thr = kNegInf;
    if (!with_temp && cp.topk_active) {
        uint32_t kth = block_select_kth_largest<kThreads>(
            n, cp.top_k, [&](uint32_t i) { return total_key(rv.value(i)); }, sm.hist, sm.sel);
        thr = key_to_float(kth);
    }
    auto in_topk = [&](uint32_t i, float v) { return with_temp || survives(v, thr); };

    // --- top-p (candidates.rs:55-78) --------------------------------------------
    bool cut = false;
    uint32_t cut_key = 0, cut_idx = 0;
    if (!with_temp && cp.topp_active) {
        uint32_t *ka = scratch, *ia = scratch + n, *kb = scratch + 2 * static_cast<size_t>(n),
                 *ib = scratch + 3 * static_cast<size_t>(n);
        // Order-preserving compaction of the top-k survivors as (~key, idx).
        uint32_t written = 0;
        constexpr uint32_t kTile = kThreads * kItems;
        for (uint32_t t0 = 0; t0 < n; t0 += kTile) {
            uint32_t kk[kItems], cnt = 0;
            bool keep[kItems];
#pragma unroll
            for (int q = 0; q < kItems; ++q) {
                uint32_t i = t0 + threadIdx.x * kItems + q;
                keep[q] = false;
                if (i < n) {
                    float v = rv.value(i);
                    keep[q] = in_topk(i, v);
                    kk[q] = ~total_key(v);
                }
                cnt += keep[q] ? 1u : 0u;
            }
            uint32_t total;
            uint32_t off = block_exclusive_add<kThreads>(cnt, sm.red32, &total);
#pragma unroll
            for (int q = 0; q < kItems; ++q) {
                if (keep[q]) {
                    ka[written + off] = kk[q];
                    ia[written + off] = t0 + threadIdx.x * kItems + q;
                    ++off;
                }
            }
            written += total;
        }
        __syncthreads();
        const uint32_t ns = written;
        if (ns > 0) {
            block_radix_sort(ka, ia, kb, ib, ns, sm);
            __syncthreads();
            const float maxv = key_to_float(~ka[0]);
            const double *tab = sm.exp_tab;
            auto ev = [&](uint32_t j) { return expf_ref(__fsub_rn(key_to_float(~ka[j]), maxv), tab); };
            ReplayResult es = block_replay<kThreads, kItems>(
                ns, ev, [](float) { return false; }, sm.rs);
            const float exp_sum = es.sum;
            const float p = cp.top_p;
            ReplayResult cs = block_replay<kThreads, kItems>(
                ns, [&](uint32_t j) { return __fdiv_rn(ev(j), exp_sum); },
                [p](float s) { return s > p; }, sm.rs);
            if (cs.stop >= 0 && static_cast<uint32_t>(cs.stop) + 1 < ns) {
                cut = true;
                cut_key = ~ka[cs.stop];
                cut_idx = ia[cs.stop];
            }
        }
        __syncthreads();
    }
    auto survivor = [&](uint32_t i, float v) {
        if (!in_topk(i, v)) return false;
        if (!cut) return true;
        uint32_t k = total_key(v);
        return k > cut_key || (k == cut_key && i <= cut_idx);
    };

    // --- softmax maximum, argmax and the last survivor -------------------------
    float mx = kNegInf;
    unsigned long long amax = 0;
    uint32_t last = 0, any = 0;
    for (uint32_t i = threadIdx.x; i < n; i += kThreads) {
        float v = rv.value(i);
        if (survivor(i, v)) {
            mx = fmaxf(mx, v);
            unsigned long long c = pack_key_index(total_key(v), i);
            amax = c > amax ? c : amax;
            last = max(last, i);
            any = 1;
        }
    }
    mx = block_reduce<kThreads>(mx, sm.redf, OpFMax());
    amax = block_reduce<kThreads>(amax, sm.red64, OpMaxU64());
    last = block_reduce<kThreads>(last, sm.red32, OpMaxU32());
    any = block_reduce<kThreads>(any, sm.red32, OpOrU32());

    // Optional survivor outputs (count, and the first surv_cap ids in order).
    if (cp.out_nsurv || cp.out_surv) {
        uint32_t written = 0;
        constexpr uint32_t kTile = kThreads * kItems;
        for (uint32_t t0 = 0; t0 < n; t0 += kTile) {
            uint32_t cnt = 0;
            bool keep[kItems];
#pragma unroll
            for (int q = 0; q < kItems; ++q) {
                uint32_t i = t0 + threadIdx.x * kItems + q;
                keep[q] = i < n && survivor(i, rv.value(i));
                cnt += keep[q] ? 1u : 0u;
            }
            uint32_t total;
            uint32_t off = block_exclusive_add<kThreads>(cnt, sm.red32, &total);
            if (cp.out_surv) {
#pragma unroll
                for (int q = 0; q < kItems; ++q) {
                    if (keep[q]) {
                        if (written + off < cp.surv_cap)
                            cp.out_surv[row * cp.surv_cap + written + off] = t0 + threadIdx.x * kItems + q;
                        ++off;
                    }
                }
            }
            written += total;
        }
        if (cp.out_nsurv && threadIdx.x == 0) cp.out_nsurv[row] = written;
        __syncthreads();
    }

    // --- softmax sum (filters.rs:7-8) -----------------------------------------------
    const double *tab = sm.exp_tab;
    auto e_of = [&](uint32_t i) -> float {
        float v = rv.value(i);
        if (!survivor(i, v)) return 0.0f;
        return expf_ref(__fsub_rn(v, mx), tab);
    };
    float sum = -0.0f;
    if (any) sum = block_replay<kThreads, kItems>(n, e_of, [](float) { return false; }, sm.rs).sum;
    const bool norm = (fabsf(sum) < kPosInf) && sum > 0.0f;

    // valid_probabilities (sampler.rs:133-139): some survivor has p > 0.
    uint32_t valid = 0;
    for (uint32_t i = threadIdx.x; i < n; i += kThreads) {
        float v = rv.value(i);
        if (survivor(i, v)) {
            float pi = expf_ref(__fsub_rn(v, mx), tab);
            if (norm) pi = __fdiv_rn(pi, sum);
            if (!(pi != pi || pi <= 0.0f)) valid = 1;
        }
    }
    valid = block_reduce<kThreads>(valid, sm.red32, OpOrU32());

    int32_t status = RSC_ROW_NO_VALID_TOKENS | RSC_ROW_FLAG_LARGE_PATH;
    uint32_t token = 0;
    float prob = __uint_as_float(0x7fc00000u);
    if (valid) {
        uint32_t pos;
        int32_t flags = RSC_ROW_FLAG_LARGE_PATH;
        if (!with_temp && cp.argmax_branch) {
            pos = static_cast<uint32_t>(amax);
        } else {
            if (threadIdx.x == 0) sm.bcast[0] = __float_as_uint(row_uniform(cp, row));
            __syncthreads();
            const float r = __uint_as_float(sm.bcast[0]);
            __syncthreads();
            auto p_of = [&](uint32_t i) -> float {
                float e = e_of(i);
                return norm ? __fdiv_rn(e, sum) : e;
            };
            ReplayResult dr = block_replay<kThreads, kItems>(
                n, p_of, [r](float c) { return r < c; }, sm.rs);
            float lo, hi;
            if (dr.stop >= 0) {
                pos = static_cast<uint32_t>(dr.stop);
                lo = dr.before;
                hi = dr.after;
            } else {
                // sample_multinomial's fallback, the last survivor; for
                // sample_with_temp every position is one.
                pos = with_temp ? n - 1 : last;
                lo = hi = dr.sum;
            }
            if (fabsf(r - hi) < 1e-6f || fabsf(r - lo) < 1e-6f) flags |= RSC_ROW_FLAG_DRAW_NEAR_BOUNDARY;
        }
        token = pos;
        {
            float v = rv.value(pos);
            float e = expf_ref(__fsub_rn(v, mx), tab);
            prob = norm ? __fdiv_rn(e, sum) : e;
        }
        status = RSC_ROW_OK | flags;
    }
    if (threadIdx.x == 0) {
        out_ids[row] = token;
        out_status[row] = status;
        if (out_probs) out_probs[row] = prob;
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kThreads)
large_kernel(const float *__restrict__ logits, size_t rows, uint32_t vocab, size_t row_stride,
             CallParams cp, uint32_t *__restrict__ out_ids, int32_t *__restrict__ out_status,
             float *__restrict__ out_probs, const uint32_t *__restrict__ large_rows,
             uint32_t *large_count, uint32_t *__restrict__ scratch) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    LargeSmem &sm = *reinterpret_cast<LargeSmem *>(smem_raw);
    load_exp_table(sm.exp_tab);
    __syncthreads();
    // In list mode this grid is launched as a programmatic dependent of the
    // streaming kernel: wait until that grid has completed and its writes
    // (the list of overflowing rows) are visible.
    if (large_rows) asm volatile("griddepcontrol.wait;" ::: "memory");
    const size_t count = large_rows ? static_cast<size_t>(large_count[0]) : rows;
    uint32_t *my_scratch = scratch + static_cast<size_t>(blockIdx.x) * 4u * vocab;
    for (size_t w = blockIdx.x; w < count; w += gridDim.x) {
        const size_t row = large_rows ? large_rows[w] : w;
        RowView rv{logits + row * row_stride, vocab, cp.scale, cp.mode == kModeSampleWithTemp};
        large_row(cp, rv, row, my_scratch, out_ids, out_status, out_probs, sm);
    }
    if (large_rows) {
        // The last CTA to leave resets the list counter (word 0) and the exit
        // counter (word 1) for the next call; every CTA read word 0 before
        // counting itself out.
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            if (atomicAdd(&large_count[1], 1u) == gridDim.x - 1) {
                large_count[0] = 0;
                large_count[1] = 0;
                __threadfence();
            }
        }
    }
}

}  // namespace

cudaError_t launch_large(const float *logits, size_t rows, uint32_t vocab, size_t row_stride,
                         const CallParams &p, uint32_t *out_ids, int32_t *out_status,
                         float *out_probs, const uint32_t *large_rows,
                         uint32_t *large_count, uint32_t *scratch, uint32_t slots,
                         cudaStream_t stream) {
    if (rows == 0 || slots == 0) return cudaSuccess;
    const size_t smem = sizeof(LargeSmem);
    cudaError_t e = cudaFuncSetAttribute(large_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    size_t grid = slots;
    if (grid > rows) grid = rows;
    if (!large_rows) {
        large_kernel<<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(
            logits, rows, vocab, row_stride, p, out_ids, out_status, out_probs, large_rows,
            large_count, scratch);
        return cudaGetLastError();
    }
    // List mode: a programmatic dependent launch, so that this grid's launch
    // overlaps the tail of the streaming kernel that fills the list.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, large_kernel, logits, rows, vocab, row_stride, p, out_ids,
                              out_status, out_probs, large_rows, large_count, scratch);
}

}  // namespace rsc
