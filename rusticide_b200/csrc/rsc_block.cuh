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

}  // namespace rsc
