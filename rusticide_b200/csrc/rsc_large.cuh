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
// The sums use block_replay2, which reproduces the sequential binary32 loop
// bit for bit. Rows without any filter take plain_row, which needs no
// threshold, sort or scratch.
#pragma once

#include <type_traits>

#include "rsc_block.cuh"
#include "rsc_kernels.h"

namespace rsc {
namespace large {

constexpr int kItems = 4;
constexpr int kBatch = 8;  // loads in flight per thread in the row passes

// Shared memory of the large-row code for a block of T threads.
#ifndef RSC_REPLAY_ITEMS
#define RSC_REPLAY_ITEMS 8
#endif
constexpr int kReplayItems = RSC_REPLAY_ITEMS;
constexpr int kReplayRaw = 8;  // positions per thread per round of the compacting replay

template <int T>
struct LargeSmem {
    double exp_tab[32];
    uint32_t hist[256];
    uint32_t sel[2];
    uint32_t red32[32];
    unsigned long long red64[32];
    float redf[32];
    uint32_t bcast[4];
    union {
        struct {  // the radix sort's per-warp digit counts
            uint32_t wcount[T / 32][256];
            uint32_t base[256];
            uint32_t tile_total[256];
        };
        // The replays (never live with the sorts): the compacting form for
        // the large kernel's blocks, the plain form in the streaming
        // kernel's smaller epilogue workspace.
        typename std::conditional<(T >= 512), Replay3Smem<T, kReplayItems, kReplayRaw>,
                                  Replay2Smem<T, kReplayItems>>::type rs;
        uint32_t dbucket[T >= 512 ? 8192 : 4096];  // the distance sort's buckets
        Replay2Smem<T, kReplayItems> rs2;           // replays over a relevant-term list
        struct {
            uint32_t cmax[1024];  // plain rows: chunk maxima (total keys), then bounds
            // A round of the list, staged for coalesced stores (large blocks
            // only: the streaming kernel's epilogue workspace is smaller).
            float stage_t[T >= 512 ? T * 16 : 1];
            uint32_t stage_i[T >= 512 ? T * 16 : 1];
        };
    };
};

// Buckets of the distance sort for a block of T threads, and the largest
// bucket it sorts (a row with a larger one takes the radix sort).
template <int T>
constexpr uint32_t kDBuckets = T >= 512 ? 8192u : 4096u;
constexpr uint32_t kDMaxBucket = 512;

// The exact replay of a large-row block of T threads.
template <int T, typename Term, typename Pred>
__device__ __forceinline__ ReplayResult row_replay(uint32_t n, Term &term, Pred pred,
                                                   LargeSmem<T> &sm) {
    if constexpr (T >= 512)
        return block_replay3<T, kReplayItems, kReplayRaw>(n, term, pred, sm.rs);
    else
        return block_replay2<T, kReplayItems>(n, term, pred, sm.rs);
}

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
    const float *raw;  // load_at(j) reads raw[j] (for L2 prefetch), or null

    __device__ const float *raw_ptr() const { return raw; }

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
                                                        bool divide, const double *tab,
                                                        const float *raw = nullptr) {
    return ExpTerm<Load, Keep>{load, keep, mx, div, divide, tab, kNegInf, raw};
}

// Terms read from an array of precomputed exp values (+0 or a negative value
// marks a position that takes no part): t[j], or fl(t[j] / div). prepare
// drops terms certainly below tmin: t < tmin, or t < tmin * div * (1 - 2^-20)
// for the quotient (within an ulp of t / div).
template <typename Keep>
struct ArrayTerm {
    const float *t;
    Keep keep;  // (j, t) -> whether position j takes part (t >= 0 already checked)
    float div;
    bool divide;
    float thr;

    __device__ const float *raw_ptr() const { return t; }
    __device__ void prepare(float tmin) {
        thr = divide ? (div > 0.0f && div < kPosInf ? tmin * div * (1.0f - 0x1p-20f) : 0.0f) : tmin;
    }
    __device__ float load(uint32_t j) const { return t[j]; }
    __device__ float eval(uint32_t j, float v) const {
        if (!(v >= 0.0f) || v < thr || !keep(j, v)) return 0.0f;
        return divide ? __fdiv_rn(v, div) : v;
    }
};

template <typename Keep>
__device__ __forceinline__ ArrayTerm<Keep> array_term(const float *t, Keep keep, float div,
                                                      bool divide) {
    return ArrayTerm<Keep>{t, keep, div, divide, 0.0f};
}

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
// needs no threshold and no sort:
//  1. one pass (128-bit loads) for the maximum, the last survivor, the
//     argmax branch's last maximum, and the maximum of each chunk of the row;
//  2. one pass that lists, in order, the positions whose term can change a
//     running sum, with their terms exp(v - max). The running sum before
//     position j is at least the largest term before it, which is at least
//     the largest term of the chunks before j's chunk, T_c; a term at most
//     T_c * 2^-27 is below half a spacing of the softmax sum there, and of
//     the draw's running sum of probabilities (each divided by the sum), so
//     it rounds away in both and is left out: v_j < max(chunks before) -
//     18.75 (27 ln 2 = 18.715, plus the rounding of the exps and of v - max);
//  3. the exact index-order sum of the listed terms (filters.rs:5-15);
//  4. the draw: the exact running sum of the listed probabilities up to the
//     first r < cumsum (sampler.rs:111-121), else the last survivor.
// Scratch: the list, 2 * n words.
template <int T>
__device__ __noinline__ void plain_row(const CallParams &cp, const RowView &rv, size_t row, uint32_t *scratch,
                          uint32_t *out_ids, int32_t *out_status, float *out_probs,
                          LargeSmem<T> &sm) {
    constexpr uint32_t kMaxChunks = 1024;
    const uint32_t n = rv.n;
    const bool with_temp = rv.with_temp;
    const bool want_amax = !with_temp && cp.argmax_branch;
    // Chunks of whole rounds of the first pass (T * kBatch float4) past the
    // scalar head; at most kMaxChunks of them.
    constexpr uint32_t kRound = T * kBatch * 4u;
    const uint32_t chunk = max(1u, (n + kMaxChunks * kRound - 1) / (kMaxChunks * kRound)) * kRound;
    for (uint32_t c = threadIdx.x; c < kMaxChunks; c += T) sm.cmax[c] = kKeyNegInf;
    __syncthreads();
    float mx = kNegInf;
    uint32_t last = 0;
    unsigned long long amax = 0;
    const uint32_t mis = static_cast<uint32_t>((reinterpret_cast<uintptr_t>(rv.p) >> 2) & 3u);
    const uint32_t head = mis ? min(n, 4u - mis) : 0u;
    const uint32_t n4 = (n - head) / 4u;
    const uint32_t tail0 = head + 4u * n4;
    auto chunk_of = [&](uint32_t i) { return i < head ? 0u : min((i - head) / chunk, kMaxChunks - 1); };
    auto visit = [&](float v, uint32_t i) {
        mx = fmaxf(mx, v);
        last = (v != kNegInf && i > last) ? i : last;
        if (want_amax && v != kNegInf) {
            const unsigned long long c = pack_key_index(total_key(v), i);
            amax = c > amax ? c : amax;
        }
    };
    // Scalar head up to a 16-byte boundary, float4 body, scalar tail.
    if (threadIdx.x < head) {
        const float v = rv.value(threadIdx.x);
        visit(v, threadIdx.x);
        atomicMax(&sm.cmax[0], total_key(v));
    }
    if (threadIdx.x >= 32 && threadIdx.x - 32 < n - tail0) {
        const uint32_t i = tail0 + threadIdx.x - 32;
        const float v = rv.value(i);
        visit(v, i);
        atomicMax(&sm.cmax[chunk_of(i)], total_key(v));
    }
    const float4 *p4 = reinterpret_cast<const float4 *>(rv.p + head);
    const uint32_t lane = threadIdx.x & 31u;
    for (uint32_t q0 = 0; q0 < n4; q0 += T * kBatch) {
        float4 f[kBatch];
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {  // loads first, all in flight together
            const uint32_t q = q0 + b * T + threadIdx.x;
            f[b] = q < n4 ? p4[q] : make_float4(kNegInf, kNegInf, kNegInf, kNegInf);
        }
        float gm = kNegInf;
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
            const uint32_t q = q0 + b * T + threadIdx.x;
            if (q < n4) {
                const uint32_t i = head + 4u * q;
                const float v0 = rv.scaled(f[b].x), v1 = rv.scaled(f[b].y);
                const float v2 = rv.scaled(f[b].z), v3 = rv.scaled(f[b].w);
                visit(v0, i);
                visit(v1, i + 1);
                visit(v2, i + 2);
                visit(v3, i + 3);
                gm = fmaxf(gm, fmaxf(fmaxf(v0, v1), fmaxf(v2, v3)));
            }
        }
        // A round lies in one chunk (chunk is a whole number of rounds).
        gm = warp_max(gm);
        if (lane == 0) atomicMax(&sm.cmax[(4u * q0) / chunk], total_key(gm));
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
    if (valid) {
        // Exclusive prefix maximum of the chunk maxima, as the leave-out
        // bound of each chunk: v < bound is left out.
        if (threadIdx.x < 32) {
            constexpr uint32_t kPer = kMaxChunks / 32;
            uint32_t m = kKeyNegInf;
            for (uint32_t e = 0; e < kPer; ++e) m = max(m, sm.cmax[lane * kPer + e]);
            uint32_t incl = m;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= static_cast<uint32_t>(o)) incl = max(incl, v);
            }
            uint32_t run = __shfl_up_sync(0xffffffffu, incl, 1);
            if (lane == 0) run = kKeyNegInf;
            __syncwarp();
            for (uint32_t e = 0; e < kPer; ++e) {
                const uint32_t ce = sm.cmax[lane * kPer + e];
                const float pm = key_to_float(run);
                // No chunk before: every logit is listed.
                sm.cmax[lane * kPer + e] =
                    __float_as_uint(pm == kNegInf ? kNegInf : __fsub_rn(pm, 18.75f));
                run = max(run, ce);
            }
        }
        __syncthreads();
        // The list of terms that can matter, in index order.
        float *lt = reinterpret_cast<float *>(scratch);
        uint32_t *li = scratch + n;
        uint32_t cnt = 0;
        auto listed = [&](float v, uint32_t i) {
            return v != kNegInf && !(v < __uint_as_float(sm.cmax[chunk_of(i)]));
        };
        if (head > 0) {
            // The head, in order, by the first lanes.
            const float v = threadIdx.x < head ? rv.value(threadIdx.x) : kNegInf;
            const bool k = threadIdx.x < head && listed(v, threadIdx.x);
            const uint32_t bal = __ballot_sync(0xffffffffu, k);
            if (threadIdx.x < 32 && k) {
                const uint32_t at = __popc(bal & ((1u << lane) - 1u));
                lt[at] = expf_ref(__fsub_rn(v, mx), tab);
                li[at] = threadIdx.x;
            }
            if (threadIdx.x < 32) sm.bcast[1] = __popc(bal);
            __syncthreads();
            cnt = sm.bcast[1];
            __syncthreads();
        }
        // The body, each thread a run of kListBatch consecutive float4 (one
        // chunk: a chunk is a multiple of the run).
        constexpr int kListBatch = 4;
        for (uint32_t q0 = 0; q0 < n4; q0 += T * kListBatch) {
            float4 f[kListBatch];
            const uint32_t qt = q0 + threadIdx.x * kListBatch;
#pragma unroll
            for (int b = 0; b < kListBatch; ++b)
                f[b] = qt + b < n4 ? p4[qt + b] : make_float4(kNegInf, kNegInf, kNegInf, kNegInf);
            const float bound = __uint_as_float(sm.cmax[min((4u * qt) / chunk, kMaxChunks - 1)]);
            uint32_t mine = 0;
#pragma unroll
            for (int b = 0; b < kListBatch; ++b) {
                f[b] = make_float4(rv.scaled(f[b].x), rv.scaled(f[b].y), rv.scaled(f[b].z),
                                   rv.scaled(f[b].w));
                mine += (f[b].x != kNegInf && !(f[b].x < bound)) ? 1u : 0u;
                mine += (f[b].y != kNegInf && !(f[b].y < bound)) ? 1u : 0u;
                mine += (f[b].z != kNegInf && !(f[b].z < bound)) ? 1u : 0u;
                mine += (f[b].w != kNegInf && !(f[b].w < bound)) ? 1u : 0u;
            }
            // The next round into L2 meanwhile: one 128-byte line per thread.
            if (q0 + T * kListBatch + 8u * threadIdx.x < n4)
                prefetch_l2(p4 + q0 + T * kListBatch + 8u * threadIdx.x);
            uint32_t total;
            uint32_t at = block_exclusive_add<T>(mine, sm.red32, &total);
            constexpr bool kStage = T >= 512;
            if (!kStage) at += cnt;
            if (mine) {
                // Staged in shared memory, then stored in order, coalesced.
#pragma unroll
                for (int b = 0; b < kListBatch; ++b) {
                    const uint32_t i = head + 4u * (qt + b);
                    const float v[4] = {f[b].x, f[b].y, f[b].z, f[b].w};
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        if (v[c] != kNegInf && !(v[c] < bound)) {
                            const float t = expf_ref(__fsub_rn(v[c], mx), tab);
                            if (kStage) {
                                sm.stage_t[at] = t;
                                sm.stage_i[at] = i + c;
                            } else {
                                lt[at] = t;
                                li[at] = i + c;
                            }
                            ++at;
                        }
                    }
                }
            }
            if (kStage) {
                __syncthreads();
                for (uint32_t e = threadIdx.x; e < total; e += T) {
                    lt[cnt + e] = sm.stage_t[e];
                    li[cnt + e] = sm.stage_i[e];
                }
                __syncthreads();
            }
            cnt += total;
        }
        if (tail0 < n) {
            const uint32_t i = tail0 + threadIdx.x;
            const float v = threadIdx.x < n - tail0 ? rv.value(i) : kNegInf;
            const bool k = threadIdx.x < n - tail0 && listed(v, i);
            const uint32_t bal = __ballot_sync(0xffffffffu, k);
            if (threadIdx.x < 32 && k) {
                const uint32_t at = cnt + __popc(bal & ((1u << lane) - 1u));
                lt[at] = expf_ref(__fsub_rn(v, mx), tab);
                li[at] = i;
            }
            if (threadIdx.x < 32) sm.bcast[1] = __popc(bal);
            __syncthreads();
            cnt += sm.bcast[1];
            __syncthreads();
        }
        __syncthreads();
        auto all = [](uint32_t, float) { return true; };
        // softmax sum (filters.rs:7-8), from -0.0 (the row is not empty).
        auto s_term = array_term(lt, all, 1.0f, false);
        const float sum =
            block_replay2<T, kReplayItems>(cnt, s_term, [](float) { return false; }, sm.rs2).sum;
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
            auto p_term = array_term(lt, all, sum, norm);
            ReplayResult dr = block_replay2<T, kReplayItems>(
                cnt, p_term, [r](float c) { return r < c; }, sm.rs2);
            float lo, hi;
            if (dr.stop >= 0) {
                pos = li[dr.stop];
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

// The distance sort of the top-p step. The reference sorts the survivors by
// value, descending, with ties by index (candidates.rs:56-57), and its sums
// then add exp(v - max) in that order (candidates.rs:62-75). Here the sort
// key is the distance d = fl(max - v) >= 0 instead:
//  - d is non-increasing in v, and elements with equal d have equal terms
//    exp(-d) = exp(fl(v - max)), so the running sums over d ascending equal
//    the reference's sums over value descending;
//  - which elements a cut-off keeps is decided on d, and only inside the
//    group of elements that share the cut-off's d (contiguous in the
//    reference's order) does the reference's (value, index) order matter.
// The sort itself: a histogram of d over kDBuckets linear buckets (d >= 104,
// whose term is +0, all in the last bucket), a scatter into the buckets, and
// within each bucket a rank count (the last bucket keeps any order: its
// terms are all +0, and a cut-off never falls on a +0 term).
__device__ __forceinline__ uint32_t dist_bucket(float d, float inv, uint32_t nb) {
    if (!(d < 104.0f)) return nb - 1u;
    return min(__float2uint_rz(__fmul_rn(d, inv)), nb - 2u);
}

// Calls f(v, i) for every position i of the row, v its scaled logit, in no
// particular order: a scalar head up to a 16-byte boundary, a float4 body with
// kB loads per thread in flight, a scalar tail.
template <int T, int kB = 4, typename F>
__device__ __forceinline__ void for_each_scaled(const RowView &rv, F f) {
    const uint32_t n = rv.n;
    const uint32_t mis = static_cast<uint32_t>((reinterpret_cast<uintptr_t>(rv.p) >> 2) & 3u);
    const uint32_t head = mis ? min(n, 4u - mis) : 0u;
    const uint32_t n4 = (n - head) / 4u;
    const uint32_t tail0 = head + 4u * n4;
    if (threadIdx.x < head) f(rv.value(threadIdx.x), threadIdx.x);
    if (threadIdx.x >= 32 && threadIdx.x - 32 < n - tail0)
        f(rv.value(tail0 + threadIdx.x - 32), tail0 + threadIdx.x - 32);
    const float4 *p4 = reinterpret_cast<const float4 *>(rv.p + head);
    for (uint32_t q0 = 0; q0 < n4; q0 += T * kB) {
        float4 x[kB];
#pragma unroll
        for (int b = 0; b < kB; ++b) {  // loads first, all in flight together
            const uint32_t q = q0 + b * T + threadIdx.x;
            if (q < n4) x[b] = p4[q];
        }
#pragma unroll
        for (int b = 0; b < kB; ++b) {
            const uint32_t q = q0 + b * T + threadIdx.x;
            if (q < n4) {
                const uint32_t i = head + 4u * q;
                f(rv.scaled(x[b].x), i);
                f(rv.scaled(x[b].y), i + 1);
                f(rv.scaled(x[b].z), i + 2);
                f(rv.scaled(x[b].w), i + 3);
            }
        }
    }
}

// Sampler::sample_logits on a row with top-p on and a finite surviving set
// (src/sampler.rs:44-54; Candidates::filter, candidates.rs:16-78; softmax,
// filters.rs:5-15; the draw, sampler.rs:111-121), through the distance sort
// above. Scratch: S1, S2 and SB (n words each) for the sort, and E (n floats):
// E[i] = exp(fl(v_i - max)) for a survivor of top-k, -1 otherwise. Each
// term is computed once: the sorted sums read S2 (the same values in the
// reference's order), the index-order sums read E.
// Returns false, having written no output, when the row does not qualify
// (a NaN or infinite survivor, no survivor, or a bucket above kDMaxBucket);
// the caller then samples it with large_row's radix sort.
template <int T>
__device__ __noinline__ bool topp_dist_row(const CallParams &cp, const RowView &rv, size_t row, float thr,
                              uint32_t *scratch, uint32_t *out_ids, int32_t *out_status,
                              float *out_probs, LargeSmem<T> &sm) {
    const uint32_t n = rv.n;
    uint32_t *S1 = scratch, *S2 = scratch + n;
    float *E = reinterpret_cast<float *>(scratch + 2 * static_cast<size_t>(n));
    uint32_t *SB = scratch + 3 * static_cast<size_t>(n);  // bucket of each S1 entry
    const double *tab = sm.exp_tab;
    constexpr uint32_t NB = kDBuckets<T>;

    // A: the survivors' maximum, minimum and count, and whether any is NaN
    // or infinite.
    float smax = kNegInf, smin = kPosInf;
    uint32_t nsurv = 0, odd = 0;
    for_each_scaled<T>(rv, [&](float v, uint32_t) {
        if (survives(v, thr)) {
            ++nsurv;
            if (!(fabsf(v) < kPosInf)) odd = 1;
            smax = fmaxf(smax, v);
            smin = fminf(smin, v);
        }
    });
    smax = block_reduce<T>(smax, sm.redf, OpFMax());
    smin = -block_reduce<T>(-smin, sm.redf, OpFMax());
    nsurv = block_reduce<T>(nsurv, sm.red32, OpAddU32());
    odd = block_reduce<T>(odd, sm.red32, OpOrU32());
    if (nsurv == 0 || odd) return false;
    const float span = fminf(__fsub_rn(smax, smin), 104.0f);
    const float inv = span > 0.0f ? __fdiv_rn(static_cast<float>(NB - 1), span) : 0.0f;

    // B: histogram of the buckets of d = fl(max - v).
    for (uint32_t b = threadIdx.x; b < NB; b += T) sm.dbucket[b] = 0;
    __syncthreads();
    for_each_scaled<T>(rv, [&](float v, uint32_t) {
        if (survives(v, thr)) atomicAdd(&sm.dbucket[dist_bucket(__fsub_rn(smax, v), inv, NB)], 1u);
    });
    __syncthreads();
    // The largest sorted bucket decides; then the exclusive prefix. Thread t
    // owns buckets [t * kPer, (t + 1) * kPer) (T need not divide NB).
    constexpr uint32_t kPer = (NB + T - 1) / T;
    uint32_t tot = 0, big = 0;
    for (uint32_t e = 0; e < kPer; ++e) {
        const uint32_t b = threadIdx.x * kPer + e;
        if (b >= NB) break;
        const uint32_t c = sm.dbucket[b];
        tot += c;
        if (b < NB - 1) big = max(big, c);
    }
    big = block_reduce<T>(big, sm.red32, OpMaxU32());
    if (big > kDMaxBucket) return false;
    {
        uint32_t all;
        uint32_t run = block_exclusive_add<T>(tot, sm.red32, &all);
        for (uint32_t e = 0; e < kPer; ++e) {
            const uint32_t b = threadIdx.x * kPer + e;
            if (b >= NB) break;
            const uint32_t c = sm.dbucket[b];
            sm.dbucket[b] = run;
            run += c;
        }
    }
    __syncthreads();

    // C: the terms, once: E in index order, and S1 in bucket order (the
    // order inside a bucket is the scatter's). After it, dbucket[b] is the
    // end of bucket b.
    for_each_scaled<T>(rv, [&](float v, uint32_t i) {
        float t = -1.0f;
        if (survives(v, thr)) {
            const float d = __fsub_rn(smax, v);
            // exp(v - max) of the reference: fl(v - max) = -d exactly.
            t = expf_ref(-d, tab);
            const uint32_t b = dist_bucket(d, inv, NB);
            const uint32_t pos = atomicAdd(&sm.dbucket[b], 1u);
            S1[pos] = __float_as_uint(t);
            SB[pos] = b;
        }
        E[i] = t;
    });
    __syncthreads();

    // D: each bucket in order of its terms, descending (t >= 0: the bit
    // patterns order like the values; equal terms keep the scatter order,
    // and any order of equal terms gives the reference's sums). A bucket
    // holds an interval of d, so the whole array is in the reference's order
    // of terms. The last bucket (d >= 104, every term +0) keeps any order.
    for (uint32_t q0 = 0; q0 < nsurv; q0 += T) {
        const uint32_t q = q0 + threadIdx.x;
        if (q < nsurv) {
            const uint32_t tb = S1[q];
            const uint32_t b = SB[q];
            const uint32_t st = b ? sm.dbucket[b - 1] : 0u, en = sm.dbucket[b];
            uint32_t rank = q - st;
            if (b < NB - 1) {
                rank = 0;
                for (uint32_t r = st; r < en; ++r) {
                    const uint32_t o = S1[r];
                    rank += (o > tb || (o == tb && r < q)) ? 1u : 0u;
                }
            }
            S2[st + rank] = tb;
        }
    }
    __syncthreads();

    // E, F: exp_sum and the cut-off over the sorted terms (candidates.rs:62-75).
    const float *sorted = reinterpret_cast<const float *>(S2);
    auto all = [](uint32_t, float) { return true; };
    auto es_term = array_term(sorted, all, 1.0f, false);
    const float exp_sum = row_replay<T>(nsurv, es_term, [](float) { return false; }, sm).sum;
    const float p = cp.top_p;
    auto cs_term = array_term(sorted, all, exp_sum, true);
    const ReplayResult cs = row_replay<T>(nsurv, cs_term, [p](float x) { return x > p; }, sm);
    bool cut = false, gsplit = false;
    float tc = 0.0f;
    uint32_t cut_key = 0, cut_idx = 0;
    if (cs.stop >= 0 && static_cast<uint32_t>(cs.stop) + 1 < nsurv) {
        cut = true;
        const uint32_t c = static_cast<uint32_t>(cs.stop);
        tc = sorted[c];
        // The group of terms equal to the cut-off's: how many of it precede
        // the cut-off, and its size. Only inside it does the reference's
        // (value desc, index asc) order decide who is kept.
        uint32_t above = 0, eq = 0;
        for (uint32_t q0 = 0; q0 < nsurv; q0 += T) {
            const uint32_t q = q0 + threadIdx.x;
            if (q < nsurv) {
                const float o = sorted[q];
                above += o > tc ? 1u : 0u;
                eq += o == tc ? 1u : 0u;
            }
        }
        above = block_reduce<T>(above, sm.red32, OpAddU32());
        eq = block_reduce<T>(eq, sm.red32, OpAddU32());
        const uint32_t m = c - above + 1u;
        if (m < eq) {
            // The group's first m in the reference's order: gather it (S1 and
            // S2 are free now), rank it, and take the m-th.
            gsplit = true;
            if (threadIdx.x == 0) sm.bcast[1] = 0;
            __syncthreads();
            uint32_t *gk = S1, *gi = S2;
            for (uint32_t i0 = 0; i0 < n; i0 += T) {
                const uint32_t i = i0 + threadIdx.x;
                if (i < n && E[i] == tc) {
                    const uint32_t at = atomicAdd(&sm.bcast[1], 1u);
                    gk[at] = total_key(rv.value(i));
                    gi[at] = i;
                }
            }
            __syncthreads();
            const uint32_t gn = sm.bcast[1];
            for (uint32_t a = threadIdx.x; a < gn; a += T) {
                uint32_t rank = 0;
                for (uint32_t b = 0; b < gn; ++b)
                    rank += (gk[b] > gk[a] || (gk[b] == gk[a] && gi[b] < gi[a])) ? 1u : 0u;
                if (rank + 1u == m) {
                    sm.bcast[2] = gk[a];
                    sm.bcast[3] = gi[a];
                }
            }
            __syncthreads();
            cut_key = sm.bcast[2];
            cut_idx = sm.bcast[3];
            __syncthreads();
        }
    }
    // Kept after top-p: E[i] >= 0 (a top-k survivor) and at or before the
    // cut-off in the reference's order.
    auto kept = [&](uint32_t i, float e) {
        if (!(e >= 0.0f)) return false;
        if (!cut || e > tc) return true;
        if (e < tc) return false;
        if (!gsplit) return true;
        const uint32_t k = total_key(rv.value(i));
        return k > cut_key || (k == cut_key && i <= cut_idx);
    };

    // G: the last kept position (sample_multinomial's fallback).
    uint32_t last = 0;
    for (uint32_t i0 = 0; i0 < n; i0 += T * kBatch) {
        float e[kBatch];
#pragma unroll
        for (int q = 0; q < kBatch; ++q) {
            const uint32_t i = i0 + q * T + threadIdx.x;
            e[q] = i < n ? E[i] : -1.0f;
        }
#pragma unroll
        for (int q = 0; q < kBatch; ++q) {
            const uint32_t i = i0 + q * T + threadIdx.x;
            if (kept(i, e[q])) last = max(last, i);
        }
    }
    last = block_reduce<T>(last, sm.red32, OpMaxU32());

    // H: the softmax sum in index order (filters.rs:7-8); its maximum is the
    // row's (the largest survivor is always kept), so its terms are E.
    auto s_term = array_term(E, kept, 1.0f, false);
    const float sum = row_replay<T>(n, s_term, [](float) { return false; }, sm).sum;
    // sum >= 1 (the maximum's own term), finite: normalise.

    // Optional survivor outputs (as large_row).
    if (cp.out_nsurv || cp.out_surv || cp.out_survp) {
        uint32_t written = 0;
        constexpr uint32_t kTile = T * kItems;
        for (uint32_t t0 = 0; t0 < n; t0 += kTile) {
            uint32_t cnt = 0;
            bool keep[kItems];
#pragma unroll
            for (int q = 0; q < kItems; ++q) {
                const uint32_t i = t0 + threadIdx.x * kItems + q;
                keep[q] = i < n && kept(i, E[i]);
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
                            if (cp.out_survp) cp.out_survp[at] = __fdiv_rn(E[i], sum);
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

    // I: the draw (sampler.rs:111-121).
    if (threadIdx.x == 0) sm.bcast[0] = __float_as_uint(row_uniform(cp, row));
    __syncthreads();
    const float r = __uint_as_float(sm.bcast[0]);
    __syncthreads();
    auto p_term = array_term(E, kept, sum, true);
    const ReplayResult dr = row_replay<T>(n, p_term, [r](float x) { return r < x; }, sm);
    uint32_t pos;
    float lo, hi;
    if (dr.stop >= 0) {
        pos = static_cast<uint32_t>(dr.stop);
        lo = dr.before;
        hi = dr.after;
    } else {
        pos = last;
        lo = hi = dr.sum;
    }
    int32_t status = RSC_ROW_OK | RSC_ROW_FLAG_LARGE_PATH;
    if (fabsf(r - hi) < 1e-6f || fabsf(r - lo) < 1e-6f) status |= RSC_ROW_FLAG_DRAW_NEAR_BOUNDARY;
    if (threadIdx.x == 0) {
        out_ids[row] = pos;
        out_status[row] = status;
        if (out_probs) out_probs[row] = __fdiv_rn(E[pos], sum);
    }
    __syncthreads();
    return true;
}

template <int T>
__device__ __noinline__ void large_row(const CallParams &cp, const RowView &rv, size_t row, uint32_t *scratch,
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
    if (!with_temp && cp.topp_active && !cp.argmax_branch &&
        topp_dist_row<T>(cp, rv, row, thr, scratch, out_ids, out_status, out_probs, sm))
        return;

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
            ReplayResult es = row_replay<T>(ns, es_term, [](float) { return false; }, sm);
            const float exp_sum = es.sum;
            const float p = cp.top_p;
            auto cs_term = exp_term(sorted_value, all, maxv, exp_sum, true, tab);
            ReplayResult cs = row_replay<T>(ns, cs_term, [p](float x) { return x > p; }, sm);
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
        sum = row_replay<T>(n, s_term, [](float) { return false; }, sm).sum;
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
            ReplayResult dr = row_replay<T>(
                n, p_term, [r](float c) { return r < c; }, sm);
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
    if (plain) plain_row<T>(cp, rv, row, scratch, out_ids, out_status, out_probs, sm);
    else large_row<T>(cp, rv, row, scratch, out_ids, out_status, out_probs, sm);
}

}  // namespace large
}  // namespace rsc
