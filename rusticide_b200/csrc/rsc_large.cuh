// The large-row sampling code shared by the large-survivor kernel and the
// streaming kernel's overflow epilogue, for a block of T threads:
// Sampler::sample_logits (crates/rusticide-sampling/src/sampler.rs:44-54) on
// rows whose surviving set is too large for shared memory (top-k disabled on
// a wide row, or a threshold tied by thousands of logits), rows whose scale
// can create NaN (T = +inf, or T so small that 1/T overflows), and
// Sampler::sample_with_temp (sampler.rs:97-105).
//
// One block per row. The row stays in global memory (L2-resident while the
// block works on it) and is re-read per pass:
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
// bit for bit. Rows without any filter take plain_row, which needs no
// threshold, sort or scratch.
#pragma once

#include "rsc_block.cuh"
#include "rsc_kernels.h"

namespace rsc {
namespace large {

constexpr int kItems = 4;
constexpr int kBatch = 8;  // loads in flight per thread in the row passes

// Shared memory of the large-row code for a block of T threads.
template <int T>
struct LargeSmem {
    double exp_tab[32];
    ReplaySmem rs;
    uint32_t hist[256];
    uint32_t sel[2];
    uint32_t red32[32];
    unsigned long long red64[32];
    float redf[32];
    uint32_t wcount[T / 32][256];
    uint32_t base[256];
    uint32_t tile_total[256];
    uint32_t bcast[4];
};

struct RowView {
    const float *p;
    uint32_t n;
    float scale;
    bool with_temp;  // sample_with_temp: every position takes part, no filters

    // extract_logits (logits.rs:14-18) then the temperature
    // (candidates.rs:25-37, filters.rs:17-22): NaN -> -inf, then x * scale.
    __device__ __forceinline__ float scaled(float x) const { return scale_logit(x, scale); }
    __device__ __forceinline__ float value(uint32_t i) const { return scaled(p[i]); }
};

// Terms exp(v - mx) (or fl(exp(v - mx) / div)) of the replays. load(j) only
// reads position j's value (the replay issues all of a thread's loads before
// it uses any); eval(j, v) applies the filter and the exp. prepare(tmin) sets
// a bound below which a value's term is certainly under tmin, so its exp is
// skipped: v - mx < ln(tmin * div) - 1/16 gives a term below 0.94 * tmin (exp
// and the division are correctly rounded to within an ulp; tmin >= 2^-100
// keeps every bound clear of subnormal rounding).
template <typename Load, typename Keep>
struct ExpTerm {
    Load load_at;  // j -> the scaled logit at position j
    Keep keep;     // (j, v) -> whether position j takes part
    float mx;
    float div;
    bool divide;
    const double *tab;
    float vthr;

    __device__ void prepare(float tmin) {
        const bool ok = tmin >= 0x1p-100f && fabsf(mx) < kPosInf &&
                        (!divide || (div > 0.0f && div < kPosInf));
        vthr = ok ? mx + logf(tmin) + (divide ? logf(div) : 0.0f) - 0.0625f : kNegInf;
    }
    __device__ float load(uint32_t j) const { return load_at(j); }
    __device__ float eval(uint32_t j, float v) const {
        if (!keep(j, v)) return 0.0f;
        if (v < vthr) return 0.0f;
        const float e = expf_ref(__fsub_rn(v, mx), tab);
        return divide ? __fdiv_rn(e, div) : e;
    }
};

template <typename Load, typename Keep>
__device__ __forceinline__ ExpTerm<Load, Keep> exp_term(Load load, Keep keep, float mx, float div,
                                                        bool divide, const double *tab) {
    return ExpTerm<Load, Keep>{load, keep, mx, div, divide, tab, kNegInf};
}

constexpr int kReplayItems = 8;

// Stable LSD radix sort (4 passes of 8 bits) of n (key, idx) pairs by key
// ascending, ping-ponging between (ka, ia) and (kb, ib); the result ends in
// (ka, ia). Within a tile, warp w owns 32 * kItems consecutive items in
// striped order, so processing j-major keeps the input order per digit.
template <int T>
__device__ void block_radix_sort(uint32_t *ka, uint32_t *ia, uint32_t *kb, uint32_t *ib,
                                 uint32_t n, LargeSmem<T> &sm) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr uint32_t kTile = T * kItems;
    const uint32_t lt_mask = (1u << lane) - 1u;
    uint32_t *kin = ka, *iin = ia, *kout = kb, *iout = ib;
    for (int shift = 0; shift < 32; shift += 8) {
        for (int b = threadIdx.x; b < 256; b += T) sm.hist[b] = 0;
        __syncthreads();
        for (uint32_t i0 = 0; i0 < n; i0 += T * kBatch) {
            uint32_t kb[kBatch];
#pragma unroll
            for (int q = 0; q < kBatch; ++q) {  // loads first, all in flight together
                const uint32_t i = i0 + q * T + threadIdx.x;
                kb[q] = i < n ? kin[i] : 0u;
            }
#pragma unroll
            for (int q = 0; q < kBatch; ++q)
                if (i0 + q * T + threadIdx.x < n) atomicAdd(&sm.hist[(kb[q] >> shift) & 255u], 1u);
        }
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
            for (int j = 0; j < kItems; ++j) {  // loads first, all in flight together
                const uint32_t i = wbase + static_cast<uint32_t>(j) * 32u + lane;
                kk[j] = i < n ? kin[i] : 0u;
                ii[j] = i < n ? iin[i] : 0u;
            }
#pragma unroll
            for (int j = 0; j < kItems; ++j) {
                uint32_t i = wbase + static_cast<uint32_t>(j) * 32u + lane;
                bool in = i < n;
                dg[j] = in ? ((kk[j] >> shift) & 255u) : 256u;
                uint32_t peers = __match_any_sync(0xffffffffu, dg[j]);
                if (in && lane == __ffs(peers) - 1) sm.wcount[warp][dg[j]] += __popc(peers);
                __syncwarp();
            }
            __syncthreads();
            // Exclusive prefix of the per-warp counts for each digit.
            for (int b = threadIdx.x; b < 256; b += T) {
                uint32_t run = 0;
#pragma unroll
                for (int w = 0; w < (T / 32); ++w) {
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
            for (int b = threadIdx.x; b < 256; b += T) sm.base[b] += sm.tile_total[b];
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

// Rows with no filter: sample_logits with top_k = 0 and top_p >= 1 at a
// normal scale, and sample_with_temp. Every logit that is not -inf survives
// (sample_with_temp keeps -inf too, whose term is +0 all the same), so the row
// needs no threshold, no sort and no survivor test beyond v != -inf:
//  1. one pass for the maximum, the last survivor and (argmax branch) the
//     last maximum, with 128-bit loads;
//  2. the exact index-order sum of exp(v - max) (filters.rs:5-15);
//  3. the draw: the exact running sum of the probabilities up to the first
//     r < cumsum (sampler.rs:111-121).
template <int T>
__device__ void plain_row(const CallParams &cp, const RowView &rv, size_t row, uint32_t *out_ids,
                          int32_t *out_status, float *out_probs, LargeSmem<T> &sm) {
    const uint32_t n = rv.n;
    const bool with_temp = rv.with_temp;
    const bool want_amax = !with_temp && cp.argmax_branch;
    float mx = kNegInf;
    uint32_t last = 0;
    unsigned long long amax = 0;
    auto visit = [&](float x, uint32_t i) {
        const float v = rv.scaled(x);
        mx = fmaxf(mx, v);
        last = (v != kNegInf && i > last) ? i : last;
        if (want_amax && v != kNegInf) {
            const unsigned long long c = pack_key_index(total_key(v), i);
            amax = c > amax ? c : amax;
        }
    };
    // Scalar head up to a 16-byte boundary, float4 body, scalar tail.
    const uint32_t mis = static_cast<uint32_t>((reinterpret_cast<uintptr_t>(rv.p) >> 2) & 3u);
    const uint32_t head = mis ? min(n, 4u - mis) : 0u;
    const uint32_t n4 = (n - head) / 4u;
    const uint32_t tail0 = head + 4u * n4;
    if (threadIdx.x < head) visit(rv.p[threadIdx.x], threadIdx.x);
    if (threadIdx.x >= 32 && threadIdx.x - 32 < n - tail0)
        visit(rv.p[tail0 + threadIdx.x - 32], tail0 + threadIdx.x - 32);
    const float4 *p4 = reinterpret_cast<const float4 *>(rv.p + head);
    for (uint32_t q0 = 0; q0 < n4; q0 += T * kBatch) {
        float4 f[kBatch];
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {  // loads first, all in flight together
            const uint32_t q = q0 + b * T + threadIdx.x;
            f[b] = q < n4 ? p4[q] : make_float4(kNegInf, kNegInf, kNegInf, kNegInf);
        }
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
            const uint32_t q = q0 + b * T + threadIdx.x;
            if (q < n4) {
                const uint32_t i = head + 4u * q;
                visit(f[b].x, i);
                visit(f[b].y, i + 1);
                visit(f[b].z, i + 2);
                visit(f[b].w, i + 3);
            }
        }
    }
    mx = block_reduce<T>(mx, sm.redf, OpFMax());
    last = block_reduce<T>(last, sm.red32, OpMaxU32());
    if (want_amax) amax = block_reduce<T>(amax, sm.red64, OpMaxU64());
    // Some survivor exists when the maximum is above -inf (a normal scale
    // makes no NaN) or, for sample_with_temp, when the row is not empty;
    // valid_probabilities (sampler.rs:133-139) then holds exactly when the
    // maximum is finite (its own p is 1 or 1 / sum > 0; with +inf every p is
    // NaN or 0).
    const bool any = with_temp ? n > 0 : mx != kNegInf;
    const bool valid = any && fabsf(mx) < kPosInf;
    if (with_temp) last = n ? n - 1 : 0;

    int32_t status = RSC_ROW_NO_VALID_TOKENS | RSC_ROW_FLAG_LARGE_PATH;
    uint32_t token = 0;
    float prob = __uint_as_float(0x7fc00000u);
    const double *tab = sm.exp_tab;
    auto row_value = [&](uint32_t i) { return rv.value(i); };
    auto not_neg_inf = [](uint32_t, float v) { return v != kNegInf; };
    if (valid) {
        // softmax sum (filters.rs:7-8), from -0.0 (the row is not empty).
        auto s_term = exp_term(row_value, not_neg_inf, mx, 1.0f, false, tab);
        const float sum = block_replay<T, kReplayItems>(n, s_term, [](float) { return false; },
                                                               sm.rs).sum;
        const bool norm = (fabsf(sum) < kPosInf) && sum > 0.0f;
        uint32_t pos;
        int32_t flags = RSC_ROW_FLAG_LARGE_PATH;
        if (want_amax) {
            pos = static_cast<uint32_t>(amax);
        } else {
            if (threadIdx.x == 0) sm.bcast[0] = __float_as_uint(row_uniform(cp, row));
            __syncthreads();
            const float r = __uint_as_float(sm.bcast[0]);
            __syncthreads();
            auto p_term = exp_term(row_value, not_neg_inf, mx, sum, norm, tab);
            ReplayResult dr = block_replay<T, kReplayItems>(
                n, p_term, [r](float c) { return r < c; }, sm.rs);
            float lo, hi;
            if (dr.stop >= 0) {
                pos = static_cast<uint32_t>(dr.stop);
                lo = dr.before;
                hi = dr.after;
            } else {
                pos = last;  // sample_multinomial's fallback, the last survivor
                lo = hi = dr.sum;
            }
            if (fabsf(r - hi) < 1e-6f || fabsf(r - lo) < 1e-6f) flags |= RSC_ROW_FLAG_DRAW_NEAR_BOUNDARY;
        }
        token = pos;
        const float e = expf_ref(__fsub_rn(rv.value(pos), mx), tab);
        prob = norm ? __fdiv_rn(e, sum) : e;
        status = RSC_ROW_OK | flags;
    }
    if (threadIdx.x == 0) {
        out_ids[row] = token;
        out_status[row] = status;
        if (out_probs) out_probs[row] = prob;
    }
    __syncthreads();
}

template <int T>
__device__ void large_row(const CallParams &cp, const RowView &rv, size_t row, uint32_t *scratch,
                          uint32_t *out_ids, int32_t *out_status, float *out_probs,
                          LargeSmem<T> &sm) {
    const uint32_t n = rv.n;
    const bool with_temp = rv.with_temp;

    // --- top-k threshold (candidates.rs:38-43) --------------------------------
    float thr = kNegInf;
    if (!with_temp && cp.topk_active) {
        uint32_t kth = block_select_kth_largest<T>(
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
        constexpr uint32_t kTile = T * kItems;
        for (uint32_t t0 = 0; t0 < n; t0 += kTile) {
            uint32_t kk[kItems], cnt = 0;
            bool keep[kItems];
            float v[kItems];
#pragma unroll
            for (int q = 0; q < kItems; ++q) {  // loads first, all in flight together
                const uint32_t i = t0 + threadIdx.x * kItems + q;
                v[q] = i < n ? rv.value(i) : kNegInf;
            }
#pragma unroll
            for (int q = 0; q < kItems; ++q) {
                const uint32_t i = t0 + threadIdx.x * kItems + q;
                keep[q] = i < n && in_topk(i, v[q]);
                kk[q] = ~total_key(v[q]);
                cnt += keep[q] ? 1u : 0u;
            }
            uint32_t total;
            uint32_t off = block_exclusive_add<T>(cnt, sm.red32, &total);
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
            block_radix_sort<T>(ka, ia, kb, ib, ns, sm);
            __syncthreads();
            const float maxv = key_to_float(~ka[0]);
            const double *tab = sm.exp_tab;
            auto sorted_value = [&](uint32_t j) { return key_to_float(~ka[j]); };
            auto all = [](uint32_t, float) { return true; };
            auto es_term = exp_term(sorted_value, all, maxv, 1.0f, false, tab);
            ReplayResult es = block_replay<T, kReplayItems>(
                ns, es_term, [](float) { return false; }, sm.rs);
            const float exp_sum = es.sum;
            const float p = cp.top_p;
            auto cs_term = exp_term(sorted_value, all, maxv, exp_sum, true, tab);
            ReplayResult cs = block_replay<T, kReplayItems>(
                ns, cs_term, [p](float s) { return s > p; }, sm.rs);
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
    for (uint32_t i0 = 0; i0 < n; i0 += T * kBatch) {
        float v[kBatch];
#pragma unroll
        for (int q = 0; q < kBatch; ++q) {  // loads first, all in flight together
            const uint32_t i = i0 + q * T + threadIdx.x;
            v[q] = i < n ? rv.value(i) : kNegInf;
        }
#pragma unroll
        for (int q = 0; q < kBatch; ++q) {
            const uint32_t i = i0 + q * T + threadIdx.x;
            if (i < n && survivor(i, v[q])) {
                mx = fmaxf(mx, v[q]);
                const unsigned long long c = pack_key_index(total_key(v[q]), i);
                amax = c > amax ? c : amax;
                last = max(last, i);
                any = 1;
            }
        }
    }
    mx = block_reduce<T>(mx, sm.redf, OpFMax());
    amax = block_reduce<T>(amax, sm.red64, OpMaxU64());
    last = block_reduce<T>(last, sm.red32, OpMaxU32());
    any = block_reduce<T>(any, sm.red32, OpOrU32());

    // --- softmax sum (filters.rs:7-8) -----------------------------------------------
    const double *tab = sm.exp_tab;
    auto row_value = [&](uint32_t i) { return rv.value(i); };
    float sum = -0.0f;
    if (any) {
        auto s_term = exp_term(row_value, survivor, mx, 1.0f, false, tab);
        sum = block_replay<T, kReplayItems>(n, s_term, [](float) { return false; }, sm.rs).sum;
    }
    const bool norm = (fabsf(sum) < kPosInf) && sum > 0.0f;

    // Optional survivor outputs: the count, and the first surv_cap ids in
    // index order with their probabilities (the softmax vector of
    // filters.rs:5-15: exp(v - max), divided by the sum when it is finite
    // and positive).
    if (cp.out_nsurv || cp.out_surv || cp.out_survp) {
        uint32_t written = 0;
        constexpr uint32_t kTile = T * kItems;
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
            uint32_t off = block_exclusive_add<T>(cnt, sm.red32, &total);
            if (cp.out_surv || cp.out_survp) {
#pragma unroll
                for (int q = 0; q < kItems; ++q) {
                    if (keep[q]) {
                        const uint32_t i = t0 + threadIdx.x * kItems + q;
                        if (written + off < cp.surv_cap) {
                            const size_t at = row * cp.surv_cap + written + off;
                            if (cp.out_surv) cp.out_surv[at] = i;
                            if (cp.out_survp) {
                                const float e = expf_ref(__fsub_rn(rv.value(i), mx), tab);
                                cp.out_survp[at] = norm ? __fdiv_rn(e, sum) : e;
                            }
                        }
                        ++off;
                    }
                }
            }
            written += total;
        }
        if (cp.out_nsurv && threadIdx.x == 0) cp.out_nsurv[row] = written;
        __syncthreads();
    }

    // valid_probabilities (sampler.rs:133-139): some survivor has p > 0 and
    // is not NaN. exp and the division are monotone, so with a finite
    // maximum its own p (exp(0) = 1, or 1 / sum > 0 for a finite sum) is
    // positive; with mx = +inf every survivor's p is NaN or 0; with no
    // survivor there is none.
    const uint32_t valid = (any && fabsf(mx) < kPosInf) ? 1u : 0u;

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
            auto p_term = exp_term(row_value, survivor, mx, sum, norm, tab);
            ReplayResult dr = block_replay<T, kReplayItems>(
                n, p_term, [r](float c) { return r < c; }, sm.rs);
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

// One row: plain_row when it has no filter (and no survivor outputs are
// requested), large_row otherwise. `scratch` holds 4 * vocab uint32.
template <int T>
__device__ void sample_row(const CallParams &cp, const float *p, uint32_t vocab, size_t row,
                           uint32_t *scratch, uint32_t *out_ids, int32_t *out_status,
                           float *out_probs, LargeSmem<T> &sm) {
    RowView rv{p, vocab, cp.scale, cp.mode == kModeSampleWithTemp};
    const bool plain = !cp.out_nsurv && !cp.out_surv && !cp.out_survp &&
                       (rv.with_temp || (cp.normal_scale && !cp.topk_active && !cp.topp_active));
    if (plain) plain_row<T>(cp, rv, row, out_ids, out_status, out_probs, sm);
    else large_row<T>(cp, rv, row, scratch, out_ids, out_status, out_probs, sm);
}

}  // namespace large
}  // namespace rsc
