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

// Exclusive block scan of saturating sums; returns the thread's exclusive
// prefix and writes the block total to *total.
template <int THREADS>
__device__ __forceinline__ uint32_t block_exclusive_sat(uint32_t v, uint32_t *red, uint32_t *total) {
    constexpr int W = THREADS / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl = sat_add(incl, n);
    }
    __syncthreads();
    if (lane == 31) red[warp] = incl;
    __syncthreads();
    uint32_t before = 0, all = 0;
#pragma unroll
    for (int w = 0; w < W; ++w) {
        uint32_t x = red[w];
        if (w < warp) before = sat_add(before, x);
        all = sat_add(all, x);
    }
    *total = all;
    uint32_t excl_in_warp = __shfl_up_sync(0xffffffffu, incl, 1);
    if (lane == 0) excl_in_warp = 0;
    return sat_add(before, excl_in_warp);
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
// running sums compute it (src/candidates.rs:66-75, src/filters.rs:8,
// src/sampler.rs:113-119).
//
// While s stays inside one binade [2^E, 2^(E+1)) (E >= -126; the subnormal
// range counts as one binade with the same spacing), every representable s is
// an integer multiple S of u = 2^(E-23), S < 2^24, and fl(s + t) is S + q + up
// where t/u = q + f, up = (f > 1/2): an integer sum, which a block scan adds
// up exactly. The model breaks at a "barrier": a term whose rounding is a tie
// (f = 1/2, where the result depends on the parity of the running S), a term
// of at least 2^(E+1), a NaN, or the first step whose exact sum leaves the
// binade (S + P_j + q_j >= 2^24). At a barrier the step is done as one real
// binary32 add, the binade is re-derived, and the scan restarts after it.
// Results are bit-identical to the sequential loop.
//
// Terms come from term(j) for j in [0, n). pred(s_after) is a stop
// predicate: the replay returns the first j whose running sum after adding
// t_j satisfies it (or stop = -1 and the full sum).
// ---------------------------------------------------------------------------
struct ReplayResult {
    float sum;     // full sum (stop < 0), else undefined
    long long stop;  // first j with pred(s_{j+1}), or -1
    float before;  // running sum before t_stop
    float after;   // running sum after t_stop
};

struct ReplaySmem {
    uint32_t red[32];
    uint32_t total;
    uint32_t ev;
    uint32_t pr;
    float s_new;
    float s_before;
    float s_after;
    int stop_flag;
};

constexpr uint32_t kNoPos = 0xffffffffu;

__device__ __forceinline__ float replay_make(uint32_t S, uint32_t Ef) {
    return __uint_as_float(((Ef - 1u) << 23) + S);
}

template <int THREADS, int ITEMS, typename Term, typename Pred>
__device__ ReplayResult block_replay(uint32_t n, Term term, Pred pred, ReplaySmem &sm) {
    constexpr uint32_t CH = THREADS * ITEMS;
    const uint32_t tid = threadIdx.x;
    float s = 0.0f;
    for (uint32_t base = 0; base < n; base += CH) {
        float t[ITEMS];
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
            uint32_t j = base + tid * ITEMS + i;
            t[i] = j < n ? term(j) : 0.0f;
        }
        uint32_t start = 0;
        while (true) {
            if (s != s) return ReplayResult{s, -1, s, s};  // NaN stays NaN; no predicate fires
            const uint32_t sb = __float_as_uint(s);
            const uint32_t Ef = max(sb >> 23, 1u);
            const uint32_t S = (sb >> 23) ? ((sb & 0x7fffffu) | 0x800000u) : (sb & 0x7fffffu);
            uint32_t d[ITEMS], q[ITEMS];
            uint32_t ev_local = kNoPos;
            uint32_t acc = 0;
#pragma unroll
            for (int i = 0; i < ITEMS; ++i) {
                const uint32_t pos = tid * ITEMS + i;
                d[i] = 0;
                q[i] = 0;
                if (pos >= start) {
                    const float tv = t[i];
                    const uint32_t tb = __float_as_uint(tv);
                    const uint32_t tf = tb >> 23;  // terms are >= +0 or NaN (sign 0 or NaN)
                    bool barrier = (tv != tv) || (tb >> 31);
                    const uint32_t mt = tf ? ((tb & 0x7fffffu) | 0x800000u) : (tb & 0x7fffffu);
                    const int shift = static_cast<int>(Ef) - static_cast<int>(max(tf, 1u));
                    if (shift < 0) {
                        barrier = true;
                    } else if (shift == 0) {
                        q[i] = mt;
                    } else if (shift < 25) {
                        const uint32_t qq = mt >> shift;
                        const uint32_t rem = mt & ((1u << shift) - 1u);
                        const uint32_t half = 1u << (shift - 1);
                        q[i] = qq;
                        d[i] = (rem > half) ? 1u : 0u;
                        if (rem == half) barrier = true;
                    }
                    d[i] += q[i];
                    if (barrier) {
                        ev_local = min(ev_local, pos);
                        d[i] = 0;
                        q[i] = 0;
                    }
                }
                acc = sat_add(acc, d[i]);
            }
            uint32_t total;
            const uint32_t excl = block_exclusive_sat<THREADS>(acc, sm.red, &total);
            // First step whose exact sum leaves the binade: S + P_j + q_j >= 2^24.
            uint32_t run = excl;
#pragma unroll
            for (int i = 0; i < ITEMS; ++i) {
                const uint32_t pos = tid * ITEMS + i;
                if (pos >= start && S + run + q[i] >= (1u << 24)) ev_local = min(ev_local, pos);
                run = sat_add(run, d[i]);
            }
            const uint32_t ev = block_reduce<THREADS>(ev_local, sm.red, OpMinU32());
            // Predicate on the modelled steps before the event.
            uint32_t pr_local = kNoPos;
            run = excl;
#pragma unroll
            for (int i = 0; i < ITEMS; ++i) {
                const uint32_t pos = tid * ITEMS + i;
                const uint32_t after = sat_add(run, d[i]);
                if (pos >= start && pos < ev && base + pos < n && pr_local == kNoPos &&
                    pred(replay_make(S + after, Ef)))
                    pr_local = pos;
                run = after;
            }
            const uint32_t pr = block_reduce<THREADS>(pr_local, sm.red, OpMinU32());
            if (pr != kNoPos) {
                run = excl;
#pragma unroll
                for (int i = 0; i < ITEMS; ++i) {
                    const uint32_t pos = tid * ITEMS + i;
                    if (pos == pr) {
                        sm.s_before = replay_make(S + run, Ef);
                        sm.s_after = replay_make(S + run + d[i], Ef);
                    }
                    run = sat_add(run, d[i]);
                }
                __syncthreads();
                ReplayResult r{0.0f, static_cast<long long>(base + pr), sm.s_before, sm.s_after};
                __syncthreads();
                return r;
            }
            if (ev == kNoPos) {
                s = replay_make(S + total, Ef);
                break;
            }
            // The event step, done as one binary32 add by its owner.
            run = excl;
#pragma unroll
            for (int i = 0; i < ITEMS; ++i) {
                const uint32_t pos = tid * ITEMS + i;
                if (pos == ev) {
                    const float before = replay_make(S + run, Ef);
                    const float after = __fadd_rn(before, t[i]);
                    sm.s_before = before;
                    sm.s_new = after;
                    sm.stop_flag = (base + pos < n && pred(after)) ? 1 : 0;
                }
                run = sat_add(run, d[i]);
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
