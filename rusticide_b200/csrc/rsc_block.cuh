// Block-level building blocks of the sampling kernels: reductions, scans,
// an in-shared-memory bitonic sort, a radix select of the k-th largest key, and
// the exact parallel replay of a sequential binary32 sum.
#pragma once

#include "rsc_common.cuh"

namespace rsc {

// ---------------------------------------------------------------------------
// Reductions and scans over a whole block. `red` is shared scratch of at least
// THREADS/32 elements of the reduced type; every call ends with the result
// visible to all threads and `red` free for reuse.
// ---------------------------------------------------------------------------
template <int THREADS, typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, T *red, Op op) {
    constexpr int W = THREADS / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    T r = red[0];
#pragma unroll
    for (int w = 1; w < W; ++w) r = op(r, red[w]);
    return r;
}

struct OpMaxU64 {
    __device__ unsigned long long operator()(unsigned long long a, unsigned long long b) const {
        return a > b ? a : b;
    }
};
struct OpMinU32 {
    __device__ uint32_t operator()(uint32_t a, uint32_t b) const { return a < b ? a : b; }
};
struct OpMaxU32 {
    __device__ uint32_t operator()(uint32_t a, uint32_t b) const { return a > b ? a : b; }
};
struct OpOrU32 {
    __device__ uint32_t operator()(uint32_t a, uint32_t b) const { return a | b; }
};
struct OpAddU32 {
    __device__ uint32_t operator()(uint32_t a, uint32_t b) const { return a + b; }
};
// f32::max as the reference's softmax folds it (src/filters.rs:6): a NaN
// operand yields the other one.
struct OpFMax {
    __device__ float operator()(float a, float b) const { return fmaxf(a, b); }
};

// Saturating add used by the replay: the operands never exceed kSat, so the
// sum never wraps.
constexpr uint32_t kSat = 1u << 26;
__device__ __forceinline__ uint32_t sat_add(uint32_t a, uint32_t b) {
    uint32_t s = a + b;
    return s > kSat ? kSat : s;
}

// Plain (non-saturating) exclusive block scan of counts.
template <int THREADS>
__device__ __forceinline__ uint32_t block_exclusive_add(uint32_t v, uint32_t *red, uint32_t *total) {
    constexpr int W = THREADS / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    __syncthreads();
    if (lane == 31) red[warp] = incl;
    __syncthreads();
    uint32_t before = 0, all = 0;
#pragma unroll
    for (int w = 0; w < W; ++w) {
        uint32_t x = red[w];
        if (w < warp) before += x;
        all += x;
    }
    *total = all;
    return before + incl - v;
}

// ---------------------------------------------------------------------------
// Synchronisation of a group of threads that runs a collective routine: the
// whole block, the first NT threads through named barrier BAR, or one warp.
// A group's threads are threadIdx.x % THREADS = 0 .. THREADS-1 of warps that
// all belong to it.
// ---------------------------------------------------------------------------
struct SyncBlock {
    __device__ __forceinline__ static void sync() { __syncthreads(); }
};
struct SyncWarp {
    __device__ __forceinline__ static void sync() { __syncwarp(); }
};
template <int BAR, int NT>
struct SyncNamed {
    __device__ __forceinline__ static void sync() {
        asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(NT) : "memory");
    }
};

// ---------------------------------------------------------------------------
// Bitonic sort, ascending, of n64 (a power of two) 64-bit items in shared
// memory by a group of THREADS threads.
// ---------------------------------------------------------------------------
template <int THREADS, typename Sync = SyncBlock>
__device__ void group_bitonic_sort(unsigned long long *a, uint32_t n64) {
    const uint32_t tid = threadIdx.x % THREADS;
    for (uint32_t k = 2; k <= n64; k <<= 1) {
        for (uint32_t j = k >> 1; j > 0; j >>= 1) {
            Sync::sync();
            for (uint32_t t = tid; t < n64 / 2; t += THREADS) {
                uint32_t i = 2 * t - (t & (j - 1));  // lower element of the pair
                uint32_t l = i + j;
                bool up = (i & k) == 0;
                unsigned long long x = a[i], y = a[l];
                if ((x > y) == up) {
                    a[i] = y;
                    a[l] = x;
                }
            }
        }
    }
    Sync::sync();
}

template <int THREADS>
__device__ void block_bitonic_sort(unsigned long long *a, uint32_t n64) {
    group_bitonic_sort<THREADS, SyncBlock>(a, n64);
}

// ---------------------------------------------------------------------------
// Radix select of the k-th largest 32-bit key (1 <= k <= count) among
// `count` keys produced by get(i). 8-bit digits from the top; `hist` is 256
// shared counters, `sel` two shared words. Every thread of the group returns
// the key.
// ---------------------------------------------------------------------------
template <int THREADS, typename Sync, typename Get>
__device__ uint32_t group_select_kth_largest(uint32_t count, uint32_t k, Get get, uint32_t *hist,
                                             uint32_t *sel) {
    const uint32_t tid = threadIdx.x % THREADS;
    uint32_t prefix = 0, mask = 0;
    uint32_t kk = k;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (uint32_t b = tid; b < 256; b += THREADS) hist[b] = 0;
        Sync::sync();
        // Lanes of a warp that share a digit add once, through their leader:
        // keys of one row crowd into few top digits, and same-address shared
        // atomics would serialise.
        const uint32_t rounds = (count + THREADS - 1) / THREADS;
        for (uint32_t r = 0; r < rounds; ++r) {
            const uint32_t i = r * THREADS + tid;
            uint32_t digit = 256u;
            if (i < count) {
                const uint32_t key = get(i);
                if ((key & mask) == prefix) digit = (key >> shift) & 255u;
            }
            const uint32_t peers = __match_any_sync(0xffffffffu, digit);
            if (digit < 256u && (threadIdx.x & 31) == static_cast<uint32_t>(__ffs(peers) - 1))
                atomicAdd(&hist[digit], static_cast<uint32_t>(__popc(peers)));
        }
        Sync::sync();
        if (tid < 32) {
            const int lane = static_cast<int>(tid);
            // Lane l owns digits 255-8l .. 248-8l (descending).
            uint32_t c[8], tot = 0;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                c[q] = hist[255 - 8 * lane - q];
                tot += c[q];
            }
            uint32_t incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                uint32_t n = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += n;
            }
            uint32_t excl = incl - tot;
            bool mine = excl < kk && kk <= incl;
            if (mine) {
                uint32_t run = excl;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    if (run < kk && kk <= run + c[q]) {
                        sel[0] = static_cast<uint32_t>(255 - 8 * lane - q);
                        sel[1] = kk - run;
                    }
                    run += c[q];
                }
            }
        }
        Sync::sync();
        prefix |= sel[0] << shift;
        mask |= 255u << shift;
        kk = sel[1];
        Sync::sync();
    }
    return prefix;
}

template <int THREADS, typename Get>
__device__ uint32_t block_select_kth_largest(uint32_t count, uint32_t k, Get get, uint32_t *hist,
                                             uint32_t *sel) {
    return group_select_kth_largest<THREADS, SyncBlock>(count, k, get, hist, sel);
}

// ---------------------------------------------------------------------------
// Exact parallel replay of a sequential binary32 sum s <- fl(s + t_j), j in
// order, over non-negative terms (NaN allowed), as the reference's fold and
// running sums compute them (src/candidates.rs:66-75, src/filters.rs:8,
// src/sampler.rs:113-119).
// ---------------------------------------------------------------------------
struct ReplayResult {
    float sum;     // full sum (stop < 0), else undefined
    long long stop;  // first j with pred(s_{j+1}), or -1
    float before;  // running sum before t_stop
    float after;   // running sum after t_stop
};

constexpr uint32_t kNoPos = 0xffffffffu;

// The float S * u of binade Ef (S up to 2^24, which is 2^(E+1)).
__device__ __forceinline__ float replay_make(uint32_t S, uint32_t Ef) {
    return __uint_as_float(((Ef - 1u) << 23) + S);
}

// The model: while s stays inside one binade [2^E, 2^(E+1)) (E >= -126; the
// subnormal range counts as one binade with the same spacing), every
// representable s is S * u with u = 2^(E-23), S < 2^24, and a term t with
// t/u = q + f adds q, plus 1 when f > 1/2. Two further facts make it parallel:
//  - A tie (t/u = q + 1/2) is no barrier. Round-half-to-even makes the step
//    S -> S + q + ((S + q) & 1): its increment depends only on the parity of
//    S. So a run of steps maps S to S + delta[S & 1], a pair of increments
//    for even and odd S, and pairs compose associatively; a block scan of
//    pairs replays ties exactly, in order.
//  - The running sum never decreases (terms >= +0), so a tile whose total
//    stays inside the binade and does not satisfy the (monotone) stop
//    predicate needs no per-element search; only the rare tile with an event
//    (binade exit, term of the next binade or above, NaN, or the stop) is
//    searched, and the event step is done as one real binary32 add.
// Terms come from a functor with prepare(tmin), called once per tile with
// tmin = u/2 of the tile's starting binade (any term below it rounds away
// for the rest of the tile, since u only grows), load(j) (a plain read) and
// eval(j, loaded) (the term).
// ---------------------------------------------------------------------------
struct ReplayPair {
    uint32_t d0, d1;  // increment of S for even S, for odd S
};

// `a` then `b`.
__device__ __forceinline__ ReplayPair rp_compose(ReplayPair a, ReplayPair b) {
    ReplayPair r;
    r.d0 = sat_add(a.d0, (a.d0 & 1u) ? b.d1 : b.d0);
    r.d1 = sat_add(a.d1, (a.d1 & 1u) ? b.d0 : b.d1);
    return r;
}

// The step of term t in the binade with exponent field Ef (>= 1). NaN, and
// terms of binade Ef + 1 or above, saturate (always an event).
__device__ __forceinline__ ReplayPair rp_term(float tv, uint32_t Ef) {
    const uint32_t tb = __float_as_uint(tv);
    if ((tv != tv) || (tb >> 31)) return ReplayPair{kSat, kSat};
    const uint32_t tf = tb >> 23;
    const uint32_t mt = tf ? ((tb & 0x7fffffu) | 0x800000u) : (tb & 0x7fffffu);
    const int shift = static_cast<int>(Ef) - static_cast<int>(max(tf, 1u));
    if (shift < 0) return ReplayPair{kSat, kSat};
    if (shift == 0) return ReplayPair{mt, mt};
    if (shift >= 25) return ReplayPair{0u, 0u};
    const uint32_t q = mt >> shift;
    const uint32_t rem = mt & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half) return ReplayPair{q + 1u, q + 1u};
    if (rem < half) return ReplayPair{q, q};
    return ReplayPair{q + (q & 1u), q + 1u - (q & 1u)};
}

__device__ __forceinline__ uint32_t rp_apply(ReplayPair p, uint32_t S) {
    return sat_add(S, (S & 1u) ? p.d1 : p.d0);
}

struct ReplaySmem {
    ReplayPair wsm[33];
    uint32_t red[32];
    float s_before;
    float s_new;
    int stop_flag;
};

// Exclusive block scan of pairs (in thread order); *total gets the whole
// block's composition. Ends with wsm free for reuse.
template <int THREADS>
__device__ __forceinline__ ReplayPair block_exclusive_pairs(ReplayPair v, ReplaySmem &sm,
                                                            ReplayPair *total) {
    constexpr int W = THREADS / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    ReplayPair inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        ReplayPair up{__shfl_up_sync(0xffffffffu, inc.d0, o), __shfl_up_sync(0xffffffffu, inc.d1, o)};
        if (lane >= o) inc = rp_compose(up, inc);
    }
    ReplayPair ex{__shfl_up_sync(0xffffffffu, inc.d0, 1), __shfl_up_sync(0xffffffffu, inc.d1, 1)};
    if (lane == 0) ex = ReplayPair{0u, 0u};
    if (lane == 31) sm.wsm[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        ReplayPair w = lane < W ? sm.wsm[lane] : ReplayPair{0u, 0u};
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            ReplayPair up{__shfl_up_sync(0xffffffffu, w.d0, o), __shfl_up_sync(0xffffffffu, w.d1, o)};
            if (lane >= o) w = rp_compose(up, w);
        }
        ReplayPair wex{__shfl_up_sync(0xffffffffu, w.d0, 1), __shfl_up_sync(0xffffffffu, w.d1, 1)};
        if (lane == 0) wex = ReplayPair{0u, 0u};
        __syncwarp();
        if (lane < W) sm.wsm[lane] = wex;
        if (lane == W - 1) sm.wsm[32] = w;
    }
    __syncthreads();
    const ReplayPair r = rp_compose(sm.wsm[warp], ex);
    *total = sm.wsm[32];
    __syncthreads();
    return r;
}

template <int THREADS, int ITEMS, typename Term, typename Pred>
__device__ ReplayResult block_replay(uint32_t n, Term &term, Pred pred, ReplaySmem &sm) {
    constexpr uint32_t CH = THREADS * ITEMS;
    constexpr uint32_t kTop = 1u << 24;
    const uint32_t tid = threadIdx.x;
    float s = 0.0f;
    for (uint32_t base = 0; base < n; base += CH) {
        if (s != s) return ReplayResult{s, -1, s, s};  // NaN stays NaN; no predicate fires
        {
            const uint32_t Ef0 = max(__float_as_uint(s) >> 23, 1u);
            // u/2 = 2^(Ef - 151); below 2^-149 nothing rounds away.
            term.prepare(__uint_as_float(Ef0 << 23) * 0x1p-24f);
        }
        float t[ITEMS];
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {  // loads first, all in flight together
            const uint32_t j = base + tid * ITEMS + i;
            t[i] = j < n ? term.load(j) : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
            const uint32_t j = base + tid * ITEMS + i;
            t[i] = j < n ? term.eval(j, t[i]) : 0.0f;
        }
        uint32_t start = 0;
        while (true) {
            if (s != s) return ReplayResult{s, -1, s, s};
            const uint32_t sb = __float_as_uint(s);
            const uint32_t Ef = max(sb >> 23, 1u);
            const uint32_t S0 = (sb >> 23) ? ((sb & 0x7fffffu) | 0x800000u) : (sb & 0x7fffffu);
            ReplayPair pr[ITEMS];
            ReplayPair acc{0u, 0u};
#pragma unroll
            for (int i = 0; i < ITEMS; ++i) {
                const uint32_t pos = tid * ITEMS + i;
                pr[i] = ReplayPair{0u, 0u};
                // +0 terms (skipped or filtered positions) leave S unchanged.
                if (pos >= start && base + pos < n && __float_as_uint(t[i]) != 0u) {
                    pr[i] = rp_term(t[i], Ef);
                    acc = rp_compose(acc, pr[i]);
                }
            }
            ReplayPair total;
            const ReplayPair ex = block_exclusive_pairs<THREADS>(acc, sm, &total);
            const uint32_t S_end = rp_apply(total, S0);
            if (S_end < kTop && !pred(replay_make(S_end, Ef))) {
                s = replay_make(S_end, Ef);
                break;
            }
            // The first event of the tile: a step leaving the binade (or a
            // saturated one), or the first sum satisfying the predicate.
            uint32_t S = rp_apply(ex, S0);
            uint32_t ev_local = kNoPos;
#pragma unroll
            for (int i = 0; i < ITEMS; ++i) {
                const uint32_t pos = tid * ITEMS + i;
                if (ev_local == kNoPos && pos >= start && base + pos < n) {
                    const uint32_t after = rp_apply(pr[i], S);
                    if (after >= kTop || pred(replay_make(after, Ef))) ev_local = pos;
                    S = after;
                }
            }
            const uint32_t ev = block_reduce<THREADS>(ev_local, sm.red, OpMinU32());
            if (ev == kNoPos) {  // not reached: the total saw an event
                s = replay_make(min(S_end, kTop), Ef);
                break;
            }
            if (ev_local == ev) {
                // Its owner redoes the walk up to the event.
                uint32_t Sb = rp_apply(ex, S0);
#pragma unroll
                for (int i = 0; i < ITEMS; ++i) {
                    const uint32_t pos = tid * ITEMS + i;
                    if (pos >= start && pos < ev) Sb = rp_apply(pr[i], Sb);
                    if (pos == ev) {
                        const float before = replay_make(Sb, Ef);
                        const uint32_t Sa = rp_apply(pr[i], Sb);
                        float after;
                        if (Sa >= kTop) after = __fadd_rn(before, t[i]);  // the real step
                        else after = replay_make(Sa, Ef);
                        sm.s_before = before;
                        sm.s_new = after;
                        sm.stop_flag = pred(after) ? 1 : 0;
                    }
                }
            }
            __syncthreads();
            const float s_new = sm.s_new, s_before = sm.s_before;
            const int stop = sm.stop_flag;
            __syncthreads();
            if (stop) return ReplayResult{0.0f, static_cast<long long>(base + ev), s_before, s_new};
            s = s_new;
            start = ev + 1;
            if (start >= CH || base + start >= n) break;
        }
    }
    return ReplayResult{s, -1, s, s};
}


// ---------------------------------------------------------------------------
// Exact replay, second form: the same sequential binary32 sum with the
// per-element work done by real binary32 adds.
//
// Within one run of equally spaced floats (a binade [2^E, 2^(E+1)), or the
// subnormals together with the lowest normal binade, both of spacing
// 2^-149), a float s is its bit pattern b, the spacing is one unit of b, and
// fl(s + t) for t >= 0 that stays in the run adds to b an amount that
// depends only on t and on the parity of b (the tie case of round to
// nearest even). A run of adds is therefore the pair of increments (d0, d1)
// for even and odd b, the map of the ReplayPair model above. Here a thread
// measures its pair directly: it adds its terms, in order, to two starting
// values of the predicted run, one even and one odd, and reads the two
// increments off the bit patterns. That costs two adds per term.
//
// The predicted run of a thread comes from an approximate prefix sum (binary32
// adds in any order): the sequential sum before the thread lies within a
// relative 2^-24 per term of it, so the prediction is wrong only when that
// sum sits next to a power of two. Every prediction is checked against the
// exact value: one warp walks the tile's threads in order with the exact
// running sum, applying each thread's pair when the sum lies in the thread's
// run and the result stays in it (per warp of 32 threads at once when the
// whole warp agrees), and doing the thread's adds one by one otherwise: at a
// binade crossing, a wrong prediction, a NaN or infinity, or where the
// monotone stop predicate first holds.
//
// A tile is THREADS * ITEMS terms; thread k holds the ITEMS consecutive
// terms from k * ITEMS. Terms are staged in shared memory in rows of
// ITEMS + 1 words (a lane reads its own row without bank conflicts), where
// the walking warp reads them for its one-by-one adds.
// ---------------------------------------------------------------------------
template <int THREADS>
struct ReplayTileSmem {
    static constexpr int W = THREADS / 32;
    uint32_t d0[THREADS], d1[THREADS], top[THREADS];  // top 0: no usable pair
    uint32_t wd0[W], wd1[W], wtop[W];
    float wsum[W];
    uint32_t wcnt[W];
    float s_out, before, after;
    uint32_t stop_at;
    int stop_flag;
};

template <int THREADS, int ITEMS>
struct Replay2Smem {
    float terms[THREADS * (ITEMS + 1)];
    ReplayTileSmem<THREADS> tile;
};

// The run of equally spaced floats that bit pattern b (a finite s >= +0)
// lies in, as the pattern just above its last float.
__device__ __forceinline__ uint32_t run_top(uint32_t b) {
    const uint32_t ef = b >> 23;
    return ((ef > 1u ? ef : 1u) + 1u) << 23;
}

// b after the adds of a pair (d0 for even b, d1 for odd b).
__device__ __forceinline__ uint32_t pair_apply(uint32_t b, uint32_t d0, uint32_t d1) {
    return b + ((b & 1u) ? d1 : d0);
}

// One warp resolves a sequence of pair records [i0, i1) against the exact
// running sum *sb (a bit pattern): lane l takes record i0 + l, and the warp
// applies at once the longest prefix of records that are usable (same run as
// *sb, result still below the run's top, predicate not yet true at their
// end). Returns the number of records applied (up to 32 or i1 - i0); the
// record after them, if any, needs the adds one by one.
template <typename Pred>
__device__ __forceinline__ uint32_t warp_apply_pairs(uint32_t *sb, const uint32_t *d0,
                                                     const uint32_t *d1, const uint32_t *top,
                                                     uint32_t i0, uint32_t i1, Pred &pred) {
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t b = *sb;
    const uint32_t i = i0 + lane;
    const bool in = i < i1;
    const uint32_t rt = (b >> 23) < 255u ? run_top(b) : 1u;  // 1 matches no record
    const uint32_t t = in ? top[i] : 0u;
    uint32_t c0 = in ? d0[i] : 0u, c1 = in ? d1[i] : 0u;
    // Inclusive composition of the pairs of lanes 0..l.
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t p0 = __shfl_up_sync(0xffffffffu, c0, o);
        const uint32_t p1 = __shfl_up_sync(0xffffffffu, c1, o);
        if (lane >= static_cast<uint32_t>(o)) {
            // (p0, p1) then (c0, c1)
            const uint32_t n0 = sat_add(p0, (p0 & 1u) ? c1 : c0);
            const uint32_t n1 = sat_add(p1, (p1 & 1u) ? c0 : c1);
            c0 = n0;
            c1 = n1;
        }
    }
    const uint32_t ok_mask = __ballot_sync(0xffffffffu, in && t != 0u && t == rt);
    const uint32_t upto = (lane == 31u) ? 0xffffffffu : ((2u << lane) - 1u);
    const bool prefix_ok = (ok_mask & upto) == upto;
    const uint32_t nb = pair_apply(b, c0, c1);
    const bool good = prefix_ok && nb < rt && !pred(__uint_as_float(nb));
    const uint32_t bad = __ballot_sync(0xffffffffu, !good);
    const uint32_t napplied = bad ? static_cast<uint32_t>(__ffs(bad) - 1) : 32u;
    if (napplied > 0) *sb = __shfl_sync(0xffffffffu, nb, napplied - 1);
    return napplied;
}

// One tile of an exact replay. Thread k holds tile positions [k * ITEMS,
// (k + 1) * ITEMS) in t; terms_at(k) points at the same ITEMS terms in shared
// memory; index_of(p) is the element index of tile position p; tile_n
// positions are real (the rest hold +0). s is the exact sum before the tile
// (the same on every thread) and is the exact sum after it on return.
// Returns true when the predicate first held inside the tile; then sm holds
// the element index and the sums before and after its add.
template <int THREADS, int ITEMS, typename Pred, typename TermsAt, typename IndexOf>
__device__ __forceinline__ bool replay_tile(float &s, const float (&t)[ITEMS], uint32_t tile_n,
                                            Pred &pred, TermsAt terms_at, IndexOf index_of,
                                            ReplayTileSmem<THREADS> &sm) {
    constexpr int W = THREADS / 32;
    const uint32_t tid = threadIdx.x % THREADS;
    const int lane = tid & 31, warp = tid >> 5;
    float a = 0.0f;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) a += t[i];
    // Approximate prefix: the warp's inclusive scan of the lane sums, then
    // the sums of the warps before.
    float incl = a;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) sm.wsum[warp] = incl;
    __syncthreads();
    float ws = lane < W ? sm.wsum[lane] : 0.0f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float v = __shfl_up_sync(0xffffffffu, ws, o);
        if (lane >= o) ws += v;
    }
    const float before_w = warp ? __shfl_sync(0xffffffffu, ws, warp - 1) : 0.0f;
    const float g = s + (before_w + (incl - a));
    // The thread's pair in the run predicted for it.
    const uint32_t gb = __float_as_uint(g);
    uint32_t top = (gb >> 23) < 255u ? run_top(gb) : 0u;
    const uint32_t b0 = gb & ~1u;
    float r0 = __uint_as_float(b0), r1 = __uint_as_float(b0 + 1u);
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        r0 = __fadd_rn(r0, t[i]);
        r1 = __fadd_rn(r1, t[i]);
    }
    // r0 <= r1, and a NaN (either sign) has a pattern above every top.
    if (!(__float_as_uint(r1) < top)) top = 0u;
    uint32_t d0 = __float_as_uint(r0) - b0, d1 = __float_as_uint(r1) - (b0 + 1u);
    sm.d0[tid] = d0;
    sm.d1[tid] = d1;
    sm.top[tid] = top;
    // The warp's composed pair, valid when all its lanes share one run.
    const uint32_t top0 = __shfl_sync(0xffffffffu, top, 0);
    const bool wvalid = __all_sync(0xffffffffu, top != 0u && top == top0);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t e0 = __shfl_down_sync(0xffffffffu, d0, o);
        const uint32_t e1 = __shfl_down_sync(0xffffffffu, d1, o);
        if ((lane & (2 * o - 1)) == 0) {
            // (d0, d1) then (e0, e1); saturates harmlessly in a warp that
            // is not used as a whole.
            const uint32_t n0 = sat_add(d0, (d0 & 1u) ? e1 : e0);
            const uint32_t n1 = sat_add(d1, (d1 & 1u) ? e0 : e1);
            d0 = n0;
            d1 = n1;
        }
    }
    if (lane == 0) {
        sm.wd0[warp] = d0;
        sm.wd1[warp] = d1;
        sm.wtop[warp] = wvalid ? top0 : 0u;
    }
    __syncthreads();
    if (warp == 0) {
        // The walk, with the exact running sum, by warp 0: whole warps'
        // pairs where they apply, else the warp's threads' pairs, else one
        // thread's adds one by one.
        uint32_t sb = __float_as_uint(s);
        bool stop = false;
        uint32_t stop_at = 0;
        float bef = 0.0f, aft = 0.0f;
        const uint32_t nthreads = (tile_n + ITEMS - 1) / ITEMS;
        const uint32_t nwarps = (nthreads + 31) / 32;
        uint32_t w = 0;
        while (w < nwarps && !stop) {
            w += warp_apply_pairs(&sb, sm.wd0, sm.wd1, sm.wtop, w, nwarps, pred);
            if (w >= nwarps) break;
            // Warp w does not apply as a whole: its threads.
            const uint32_t k1 = min((w + 1) * 32, nthreads);
            uint32_t k = w * 32;
            while (k < k1 && !stop) {
                k += warp_apply_pairs(&sb, sm.d0, sm.d1, sm.top, k, k1, pred);
                if (k >= k1) break;
                // Thread k: one add at a time, as the reference adds.
                if (lane == 0) {
                    const float *kterms = terms_at(k);
                    const uint32_t i1 = min(static_cast<uint32_t>(ITEMS), tile_n - k * ITEMS);
                    float tk[ITEMS];
#pragma unroll
                    for (int i = 0; i < ITEMS; ++i) tk[i] = kterms[i];
                    float sv = __uint_as_float(sb);
#pragma unroll
                    for (int i = 0; i < ITEMS; ++i) {
                        if (static_cast<uint32_t>(i) < i1 && !stop) {
                            const float prev = sv;
                            sv = __fadd_rn(sv, tk[i]);
                            if (pred(sv)) {
                                stop = true;
                                stop_at = index_of(k * ITEMS + i);
                                bef = prev;
                                aft = sv;
                            }
                        }
                    }
                    sb = __float_as_uint(sv);
                }
                sb = __shfl_sync(0xffffffffu, sb, 0);
                stop = __shfl_sync(0xffffffffu, stop, 0);
                ++k;
            }
            ++w;
        }
        if (lane == 0) {
            sm.s_out = __uint_as_float(sb);
            sm.stop_flag = stop ? 1 : 0;
            sm.stop_at = stop_at;
            sm.before = bef;
            sm.after = aft;
        }
    }
    __syncthreads();
    s = sm.s_out;
    return sm.stop_flag != 0;
}

// The replay over positions [0, n) of `term` (load(j), then eval(j, loaded);
// prepare(tmin) before each tile), in tiles of THREADS * ITEMS.
template <int THREADS, int ITEMS, typename Term, typename Pred>
__device__ ReplayResult block_replay2(uint32_t n, Term &term, Pred pred,
                                      Replay2Smem<THREADS, ITEMS> &sm) {
    constexpr uint32_t CH = THREADS * ITEMS;
    constexpr uint32_t kWarpSpan = 32 * ITEMS;
    const uint32_t tid = threadIdx.x % THREADS;
    const int lane = tid & 31, warp = tid >> 5;
    float s = 0.0f;
    // Raw loads run one tile ahead: the next tile's values are in flight
    // while this tile is summed.
    float nxt[ITEMS];
    auto issue = [&](uint32_t base) {
        const uint32_t wbase = base + static_cast<uint32_t>(warp) * kWarpSpan;
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
            const uint32_t j = wbase + static_cast<uint32_t>(i) * 32u + lane;
            nxt[i] = j < n ? term.load(j) : 0.0f;
        }
    };
    if (n > 0) issue(0);
    for (uint32_t base = 0; base < n; base += CH) {
        if (s != s) return ReplayResult{s, -1, s, s};  // NaN stays NaN; no predicate fires
        {
            const uint32_t Ef0 = max(__float_as_uint(s) >> 23, 1u);
            // u/2 = 2^(Ef - 151); below 2^-149 nothing rounds away.
            term.prepare(__uint_as_float(Ef0 << 23) * 0x1p-24f);
        }
        // The warp's span of the tile, read in coalesced order and staged so
        // that each lane then holds ITEMS consecutive terms.
        const uint32_t wbase = base + static_cast<uint32_t>(warp) * kWarpSpan;
        float t[ITEMS];
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) t[i] = nxt[i];
        if (base + CH < n) issue(base + CH);
        float *wterms = sm.terms + warp * 32 * (ITEMS + 1);
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
            const uint32_t e = static_cast<uint32_t>(i) * 32u + lane;  // position in the span
            const uint32_t j = wbase + e;
            wterms[(e / ITEMS) * (ITEMS + 1) + e % ITEMS] = j < n ? term.eval(j, t[i]) : 0.0f;
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) t[i] = wterms[lane * (ITEMS + 1) + i];
        const bool stopped = replay_tile<THREADS, ITEMS>(
            s, t, min(CH, n - base), pred,
            [&](uint32_t k) { return sm.terms + k * (ITEMS + 1); },
            [&](uint32_t p) { return base + p; }, sm.tile);
        if (stopped) {
            const ReplayResult r{0.0f, static_cast<long long>(sm.tile.stop_at), sm.tile.before,
                                 sm.tile.after};
            __syncthreads();
            return r;
        }
    }
    return ReplayResult{s, -1, s, s};
}

// ---------------------------------------------------------------------------
// Exact replay, third form: block_replay2 with the terms that cannot change
// the sum dropped first. A term below half a spacing of the running sum
// rounds away (fl(s + t) = s), and a +0 term changes nothing, so the replay
// streams the positions in rounds of THREADS * RAW, evaluates them against
// the exact sum known so far (a lower bound of the running sum at every later
// position, so every term it drops would round away), keeps the non-zero
// terms in order in a shared buffer with their positions, and replays the
// buffer a full tile at a time. On rows where most terms fall under the
// running sum's rounding, this replays only the few that matter.
// ---------------------------------------------------------------------------
template <int THREADS, int ITEMS, int RAW>
struct Replay3Smem {
    static constexpr int W = THREADS / 32;
    static constexpr uint32_t CH = THREADS * ITEMS;
    static constexpr uint32_t CAP = CH + THREADS * RAW;  // a ring of CAP positions
    static constexpr uint32_t PADDED = CAP + CAP / ITEMS;
    float term[PADDED];  // buffered terms, ring position q at q + q / ITEMS
    uint32_t idx[PADDED];
    uint32_t keep[W][RAW];  // a round's ballots of non-zero terms, per warp
    ReplayTileSmem<THREADS> tile;
};

template <int THREADS, int ITEMS, int RAW, typename Term, typename Pred>
__device__ ReplayResult block_replay3(uint32_t n, Term &term, Pred pred,
                                      Replay3Smem<THREADS, ITEMS, RAW> &sm) {
    using S = Replay3Smem<THREADS, ITEMS, RAW>;
    constexpr int W = THREADS / 32;
    constexpr uint32_t CH = THREADS * ITEMS;
    constexpr uint32_t CAP = S::CAP;
    constexpr uint32_t kRound = THREADS * RAW;
    constexpr uint32_t kWarpSpan = 32 * RAW;
    static_assert(CAP % ITEMS == 0, "tile rows must not wrap around the ring");
    const uint32_t tid = threadIdx.x % THREADS;
    const uint32_t lane = tid & 31u, warp = tid >> 5;
    // Ring position q (q < 2 * CAP) in the padded arrays.
    auto at = [](uint32_t q) {
        const uint32_t r = q >= CAP ? q - CAP : q;
        return r + r / ITEMS;
    };
    float s = 0.0f;
    uint32_t head = 0;  // ring position of the first buffered term
    uint32_t cnt = 0;   // buffered terms (the same on every thread)
    float nxt[RAW];
    const float *raw = term.raw_ptr();
    auto issue = [&](uint32_t base) {
        const uint32_t wbase = base + warp * kWarpSpan;
#pragma unroll
        for (int i = 0; i < RAW; ++i) {
            const uint32_t j = wbase + static_cast<uint32_t>(i) * 32u + lane;
            nxt[i] = j < n ? term.load(j) : 0.0f;
        }
        // The round after next into L2: one 128-byte line per thread.
        const uint32_t pf = base + 2 * kRound + tid * 32u;
        if (raw && tid < kRound / 32u && pf < n) prefetch_l2(raw + pf);
    };
    // Replays the first `len` buffered terms (len <= CH). Returns true when
    // the predicate held.
    auto flush = [&](uint32_t len) -> bool {
        float t[ITEMS];
        const uint32_t row0 = head + tid * ITEMS;  // a tile row never wraps
#pragma unroll
        for (int i = 0; i < ITEMS; ++i)
            t[i] = tid * ITEMS + i < len ? sm.term[at(row0 + i)] : 0.0f;
        const uint32_t h = head;
        const bool stopped = replay_tile<THREADS, ITEMS>(
            s, t, len, pred, [&](uint32_t k) { return sm.term + at(h + k * ITEMS); },
            [&](uint32_t p) { return sm.idx[at(h + p)]; }, sm.tile);
        head = head + len >= CAP ? head + len - CAP : head + len;
        cnt -= len;
        return stopped;
    };
    auto stopped_result = [&]() {
        const ReplayResult r{0.0f, static_cast<long long>(sm.tile.stop_at), sm.tile.before,
                             sm.tile.after};
        __syncthreads();
        return r;
    };
    if (n > 0) issue(0);
    for (uint32_t base = 0; base < n; base += kRound) {
        if (s != s) return ReplayResult{s, -1, s, s};  // NaN stays NaN; no predicate fires
        {
            const uint32_t Ef0 = max(__float_as_uint(s) >> 23, 1u);
            term.prepare(__uint_as_float(Ef0 << 23) * 0x1p-24f);
        }
        float t[RAW];
#pragma unroll
        for (int i = 0; i < RAW; ++i) t[i] = nxt[i];
        if (base + kRound < n) issue(base + kRound);
        // Evaluate, and count the non-zero terms: the warp's span is
        // (i, lane)-major, so the ballots of i = 0, 1, ... give the order.
        const uint32_t wbase = base + warp * kWarpSpan;
        uint32_t wtotal = 0;
#pragma unroll
        for (int i = 0; i < RAW; ++i) {
            const uint32_t j = wbase + static_cast<uint32_t>(i) * 32u + lane;
            t[i] = j < n ? term.eval(j, t[i]) : 0.0f;
            const uint32_t kb = __ballot_sync(0xffffffffu, __float_as_uint(t[i]) != 0u);
            if (lane == 0) sm.keep[warp][i] = kb;
            wtotal += __popc(kb);
        }
        if (lane == 0) sm.tile.wcnt[warp] = wtotal;
        __syncthreads();
        uint32_t wbefore = 0, total = 0;
#pragma unroll
        for (int w = 0; w < W; ++w) {
            const uint32_t c = sm.tile.wcnt[w];
            wbefore += static_cast<uint32_t>(w) < warp ? c : 0u;
            total += c;
        }
        uint32_t q = head + cnt + wbefore;
        const uint32_t below = (1u << lane) - 1u;
#pragma unroll
        for (int i = 0; i < RAW; ++i) {
            const uint32_t kb = sm.keep[warp][i];
            if ((kb >> lane) & 1u) {
                const uint32_t qq = q + __popc(kb & below);
                sm.term[at(qq)] = t[i];
                sm.idx[at(qq)] = wbase + static_cast<uint32_t>(i) * 32u + lane;
            }
            q += __popc(kb);
        }
        cnt += total;
        __syncthreads();
        while (cnt >= CH) {
            if (flush(CH)) return stopped_result();
            if (s != s) return ReplayResult{s, -1, s, s};
        }
    }
    if (cnt > 0 && s == s) {
        if (flush(cnt)) return stopped_result();
    }
    return ReplayResult{s, -1, s, s};
}

}  // namespace rsc
