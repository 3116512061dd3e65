// Exact replay of a sequential binary32 sum over tiles of runs, for one block
// of T threads (the whole-row kernel, sample_whole.cu).
//
// The sum s <- fl(s + t_j) over non-negative finite terms, in order, as the
// reference's folds and running sums compute it (crates/rusticide-sampling/
// src/candidates.rs:66-75, src/filters.rs:8, src/sampler.rs:113-119).
//
// Model (the pair model of rsc_block.cuh): inside one run of equally spaced
// floats (a binade, or the subnormals with the lowest normal binade) a float
// is its bit pattern b, and adding t >= 0 without leaving the run adds to b an
// amount that depends only on t and on the parity of b. A run of adds is the
// pair (d0, d1) of increments for an even and an odd start, and pairs compose
// associatively.
//
// A tile is T runs of R consecutive terms; thread k owns run k. Per tile:
//  - workers (every thread): the run's terms, an approximate prefix sum (any
//    order of binary32 adds), which predicts the run of floats the exact sum
//    is in at the start of each run; the run's pair measured by real adds from
//    the bottom of that predicted run, from an even and an odd start (a run
//    that leaves it from there has no pair: "bad"); and, per warp, the
//    segmented inclusive composition of its runs' pairs, segments breaking
//    after a bad run and where the predicted run changes. A warp whose runs
//    all share one predicted run gives a warp record: its composed pair.
//  - the walker (warp 0) then applies the records to the exact sum. At the
//    start of a segment it knows the exact sum b, so lane j checks record j
//    of the segment in one step: b lies in the record's run, b plus the
//    composed pair up to j stays below the run's top, and the stop
//    predicate does not yet hold there; one ballot gives how many records
//    apply. A record that does not (a bad run, a mispredicted run, or the
//    stop) is opened one level down (warp record -> its runs), and a run
//    that does not apply is added term by term, as the reference adds.
// Binade crossings and the stop cost a descent each; everything else is
// checked 32 records at a time without a serial chain.
#pragma once

#include "rsc_block.cuh"

namespace rsc {
namespace walk {

constexpr uint32_t kFull = 0xffffffffu;

template <int T>
struct WalkSmem {
    static constexpr int W = T / 32;
    uint32_t l0[T], l1[T], ltop[T];  // run records: pair and run top (0: bad)
    uint32_t p0[T], p1[T];           // segmented inclusive composition within the warp
    uint32_t lhead[T];               // 1 where a run starts a segment
    uint32_t w0[W], w1[W], wtop[W];  // warp records (wtop 0: not one run)
    float wsum[W];
    float s_out, before, after;
    uint32_t stop_at;
    int stop_flag;
};

// The run of floats just below pattern `top` starts at this pattern (the
// subnormals belong to the lowest normal binade's run).
__device__ __forceinline__ uint32_t run_bottom(uint32_t top) {
    const uint32_t ef = (top >> 23) - 1u;
    return ef > 1u ? (ef << 23) : 0u;
}

// (a0, a1) then (q0, q1), into (q0, q1); saturating (an oversized composition
// can never validate, and never wraps).
__device__ __forceinline__ void pair_then(uint32_t a0, uint32_t a1, uint32_t &q0, uint32_t &q1) {
    const uint32_t n0 = sat_add(a0, (a0 & 1u) ? q1 : q0);
    const uint32_t n1 = sat_add(a1, (a1 & 1u) ? q0 : q1);
    q0 = n0;
    q1 = n1;
}

// Segmented inclusive scan of pairs across a warp; `head` marks segment starts.
__device__ __forceinline__ void seg_scan(uint32_t &q0, uint32_t &q1, bool head, uint32_t lane) {
    uint32_t f = head ? 1u : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t x0 = __shfl_up_sync(kFull, q0, o);
        const uint32_t x1 = __shfl_up_sync(kFull, q1, o);
        const uint32_t xf = __shfl_up_sync(kFull, f, o);
        if (lane >= static_cast<uint32_t>(o) && !f) {
            pair_then(x0, x1, q0, q1);
            f = xf;
        }
    }
}

// The lane of the last segment start at or before each lane.
__device__ __forceinline__ uint32_t seg_start(bool head, uint32_t lane) {
    uint32_t s = head ? lane : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t x = __shfl_up_sync(kFull, s, o);
        if (lane >= static_cast<uint32_t>(o)) s = max(s, x);
    }
    return s;
}

// The walker at a segment start i (i < n <= 32): lane j in the segment holds
// the composition (q0, q1) of records i..j; applies the longest prefix of
// them that holds against the exact sum b (same run `top_i`, end below its
// top, predicate false at the end). Returns the number applied.
template <typename Pred>
__device__ __forceinline__ uint32_t validate_from(uint32_t &b, uint32_t i, uint32_t n,
                                                  uint32_t top_i, uint32_t q0, uint32_t q1,
                                                  uint32_t seg, uint32_t lane, Pred &pred) {
    const uint32_t e = b + ((b & 1u) ? q1 : q0);
    const bool same_run = (b >> 23) < 255u && run_top(b) == top_i;
    const bool ok = lane >= i && lane < n && seg == i && same_run && e < top_i &&
                    !pred(__uint_as_float(e));
    const uint32_t okm = __ballot_sync(kFull, ok);
    const uint32_t bad = ~okm & (kFull << i);
    const uint32_t stop = bad ? static_cast<uint32_t>(__ffs(bad) - 1) : 32u;
    const uint32_t napp = stop - i;
    const uint32_t eb = __shfl_sync(kFull, e, (stop - 1u) & 31u);
    if (napp) b = eb;
    return napp;
}

// Run k of the tile, term by term from the exact sum b, as the reference adds.
// Every lane of the walker computes the same chain (lanes 0..R-1 first read
// and transform one term each); sets stop, and the stop's tile position, the
// sums before and after that add, when the predicate first holds.
template <int R, typename Xf, typename Pred>
__device__ __forceinline__ void serial_run(uint32_t &b, const float *runs, uint32_t k,
                                           uint32_t tile_n, Xf &xf, Pred &pred, bool &stop,
                                           uint32_t &stop_pos, float &bef, float &aft) {
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t p0 = k * R;
    const float mine =
        lane < static_cast<uint32_t>(R) && p0 + lane < tile_n ? xf(runs[k * (R + 1) + lane]) : 0.0f;
    float tk[R];
#pragma unroll
    for (int i = 0; i < R; ++i) tk[i] = __shfl_sync(kFull, mine, i);
    // The adds form the only dependent chain; terms past tile_n are +0.
    float sv = __uint_as_float(b);
    bool hit = false;
    uint32_t at = 0;
    float bf = 0.0f, af = 0.0f;
#pragma unroll
    for (int i = 0; i < R; ++i) {
        const float prev = sv;
        sv = __fadd_rn(sv, tk[i]);
        const bool h = !hit && p0 + i < tile_n && pred(sv);
        at = h ? p0 + i : at;
        bf = h ? prev : bf;
        af = h ? sv : af;
        hit = hit || h;
    }
    if (hit) {
        stop = true;
        stop_pos = at;
        bef = bf;
        aft = af;
    }
    b = __float_as_uint(sv);
}

// The walker's pass over the runs of warp record w.
template <int T, int R, typename Xf, typename Pred>
__device__ void walk_runs(uint32_t &b, uint32_t w, uint32_t nruns, const float *runs,
                          uint32_t tile_n, Xf &xf, Pred &pred, WalkSmem<T> &sm, bool &stop,
                          uint32_t &stop_pos, float &bef, float &aft) {
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t k0 = w * 32u;
    const uint32_t nl = min(32u, nruns - k0);
    const uint32_t lt = lane < nl ? sm.ltop[k0 + lane] : 0u;
    const uint32_t q0 = sm.p0[k0 + lane], q1 = sm.p1[k0 + lane];
    const bool lh = sm.lhead[k0 + lane] != 0u;
    const uint32_t seg = seg_start(lh, lane);
    uint32_t l = 0;
    bool failed = false;
    while (l < nl && !stop) {
        const uint32_t tl = __shfl_sync(kFull, lt, l);
        const bool hl = __shfl_sync(kFull, lh ? 1u : 0u, l) != 0u;
        if (tl != 0u && !failed) {
            const uint32_t napp =
                hl ? validate_from(b, l, nl, tl, q0, q1, seg, lane, pred)
                   : warp_apply_pairs(&b, sm.l0 + k0, sm.l1 + k0, sm.ltop + k0, l, nl, pred);
            l += napp;
            if (l >= nl) break;
            const bool next_head = __shfl_sync(kFull, lh ? 1u : 0u, l) != 0u &&
                                   __shfl_sync(kFull, lt, l) != 0u;
            failed = !(napp > 0 && next_head);
            continue;
        }
        serial_run<R>(b, runs, k0 + l, tile_n, xf, pred, stop, stop_pos, bef, aft);
        ++l;
        failed = false;
    }
}

// One tile. `runs` is shared memory holding the tile's terms (before xf) with
// thread k's run at runs[k * (R + 1) + i]; tile_n terms are real. s is the
// exact sum before the tile and after it on return. Returns true when the
// predicate first held; sm.stop_at is then the tile position of that term and
// sm.before / sm.after the sums around its add. Ends with a block barrier.
template <int T, int R, typename Xf, typename Pred>
__device__ bool walk_tile(float &s, const float *runs, uint32_t tile_n, Xf xf, Pred &pred,
                          WalkSmem<T> &sm) {
    constexpr int W = T / 32;
    const uint32_t tid = threadIdx.x;
    const uint32_t lane = tid & 31u, warp = tid >> 5;
    const uint32_t nruns = (tile_n + R - 1) / R;

    // The run's terms and their approximate sum.
    float t[R];
    const float *my = runs + tid * (R + 1);
#pragma unroll
    for (int i = 0; i < R; ++i) t[i] = tid * R + i < tile_n ? xf(my[i]) : 0.0f;
    float a = 0.0f;
#pragma unroll
    for (int i = 0; i < R; ++i) a = __fadd_rn(a, t[i]);
    // Approximate exclusive prefix over the tile, plus the exact start.
    float incl = a;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float v = __shfl_up_sync(kFull, incl, o);
        if (lane >= static_cast<uint32_t>(o)) incl = __fadd_rn(incl, v);
    }
    if (lane == 31) sm.wsum[warp] = incl;
    __syncthreads();
    float ws = lane < static_cast<uint32_t>(W) ? sm.wsum[lane] : 0.0f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float v = __shfl_up_sync(kFull, ws, o);
        if (lane >= static_cast<uint32_t>(o)) ws = __fadd_rn(ws, v);
    }
    const float before_w = warp ? __shfl_sync(kFull, ws, (warp - 1u) & 31u) : 0.0f;
    const float g = __fadd_rn(s, __fadd_rn(before_w, __fsub_rn(incl, a)));

    // The run's pair, measured from the bottom of its predicted run of floats.
    const uint32_t gb = __float_as_uint(g);
    uint32_t top = (gb >> 23) < 255u ? run_top(gb) : 0u;
    const uint32_t b0 = top ? run_bottom(top) : 0u;
    float r0 = __uint_as_float(b0), r1 = __uint_as_float(b0 + 1u);
#pragma unroll
    for (int i = 0; i < R; ++i) {
        r0 = __fadd_rn(r0, t[i]);
        r1 = __fadd_rn(r1, t[i]);
    }
    if (!(__float_as_uint(r1) < top)) top = 0u;
    const uint32_t d0 = __float_as_uint(r0) - b0, d1 = __float_as_uint(r1) - (b0 + 1u);
    // Segments of the warp's runs, and their inclusive compositions.
    const uint32_t ptop = __shfl_up_sync(kFull, top, 1);
    const bool head = lane == 0 || top == 0u || ptop == 0u || ptop != top;
    uint32_t q0 = d0, q1 = d1;
    seg_scan(q0, q1, head, lane);
    sm.l0[tid] = d0;
    sm.l1[tid] = d1;
    sm.ltop[tid] = top;
    sm.p0[tid] = q0;
    sm.p1[tid] = q1;
    sm.lhead[tid] = head ? 1u : 0u;
    const uint32_t top0 = __shfl_sync(kFull, top, 0);
    const bool one_run = __all_sync(kFull, top != 0u && top == top0);
    if (lane == 31) {
        sm.w0[warp] = q0;
        sm.w1[warp] = q1;
        sm.wtop[warp] = one_run ? top0 : 0u;
    }
    __syncthreads();

    if (warp == 0) {
        uint32_t b = __float_as_uint(s);
        bool stop = false;
        uint32_t stop_pos = 0;
        float bef = 0.0f, aft = 0.0f;
        const uint32_t nw = (nruns + 31) / 32;
        const uint32_t wt = lane < nw ? sm.wtop[lane] : 0u;
        uint32_t c0 = lane < static_cast<uint32_t>(W) ? sm.w0[lane] : 0u;
        uint32_t c1 = lane < static_cast<uint32_t>(W) ? sm.w1[lane] : 0u;
        const uint32_t pwt = __shfl_up_sync(kFull, wt, 1);
        const bool wh = lane == 0 || wt == 0u || pwt == 0u || pwt != wt;
        seg_scan(c0, c1, wh, lane);
        const uint32_t seg = seg_start(wh, lane);
        uint32_t w = 0;
        bool failed = false;
        while (w < nw && !stop) {
            const uint32_t tw = __shfl_sync(kFull, wt, w);
            const bool hw = __shfl_sync(kFull, wh ? 1u : 0u, w) != 0u;
            if (tw != 0u && !failed) {
                const uint32_t napp =
                    hw ? validate_from(b, w, nw, tw, c0, c1, seg, lane, pred)
                       : warp_apply_pairs(&b, sm.w0, sm.w1, sm.wtop, w, nw, pred);
                w += napp;
                if (w >= nw) break;
                const bool next_head = __shfl_sync(kFull, wh ? 1u : 0u, w) != 0u &&
                                       __shfl_sync(kFull, wt, w) != 0u;
                failed = !(napp > 0 && next_head);
                continue;
            }
            walk_runs<T, R>(b, w, nruns, runs, tile_n, xf, pred, sm, stop, stop_pos, bef, aft);
            ++w;
            failed = false;
        }
        if (lane == 0) {
            sm.s_out = __uint_as_float(b);
            sm.stop_flag = stop ? 1 : 0;
            sm.stop_at = stop_pos;
            sm.before = bef;
            sm.after = aft;
        }
    }
    __syncthreads();
    s = sm.s_out;
    return sm.stop_flag != 0;
}

// Position p of a padded array of runs of R (p at p + p / R).
template <int R>
__device__ __forceinline__ uint32_t padded(uint32_t p) {
    return p + p / R;
}

struct Identity {
    __device__ float operator()(float x) const { return x; }
};

// The replay over n terms held in shared memory in padded order (term p at
// arr[padded<R>(p)]), each read through xf. The stop's index is its position.
template <int T, int R, typename Xf, typename Pred>
__device__ ReplayResult replay_array(const float *arr, uint32_t n, Xf xf, Pred pred,
                                     WalkSmem<T> &sm) {
    constexpr uint32_t kTile = T * R;
    float s = 0.0f;
    for (uint32_t base = 0; base < n; base += kTile) {
        const uint32_t tn = min(kTile, n - base);
        if (walk_tile<T, R>(s, arr + padded<R>(base), tn, xf, pred, sm)) {
            const ReplayResult r{0.0f, static_cast<long long>(base + sm.stop_at), sm.before,
                                 sm.after};
            __syncthreads();
            return r;
        }
    }
    return ReplayResult{s, -1, s, s};
}

// The replay over positions [0, n) whose terms fill(base, tn, s, buf) writes
// tile by tile into buf (T * (R + 1) floats, thread k's run at k * (R + 1)),
// given the exact sum s before the tile. The stop's index is its position.
template <int T, int R, typename Fill, typename Pred>
__device__ ReplayResult replay_fill(uint32_t n, Fill &fill, Pred pred, float *buf,
                                    WalkSmem<T> &sm) {
    constexpr uint32_t kTile = T * R;
    float s = 0.0f;
    for (uint32_t base = 0; base < n; base += kTile) {
        const uint32_t tn = min(kTile, n - base);
        fill(base, tn, s, buf);
        if (walk_tile<T, R>(s, buf, tn, Identity(), pred, sm)) {
            const ReplayResult r{0.0f, static_cast<long long>(base + sm.stop_at), sm.before,
                                 sm.after};
            __syncthreads();
            return r;
        }
    }
    return ReplayResult{s, -1, s, s};
}

// Where a warp's coalesced item i (lane l) of a tile lands in the run layout:
// the warp's span is 32 * R consecutive positions, e = i * 32 + l within it,
// which is item e % R of the warp's run e / R.
template <int R>
__device__ __forceinline__ uint32_t fill_slot(uint32_t warp, uint32_t e) {
    return (warp * 32u + e / R) * (R + 1) + e % R;
}

}  // namespace walk
}  // namespace rsc
