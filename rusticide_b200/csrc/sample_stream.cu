// Streaming top-k sampler: Sampler::sample_logits
// (crates/rusticide-sampling/src/sampler.rs:44-54) for rows whose surviving
// candidate set is small, which is every row once top-k is on.
//
// One HBM pass per row, three CTAs per SM, each with three warp roles:
//
//  producer (1 warp, one lane): keeps a ring of kStages shared-memory stages
//    filled with 1-D TMA bulk copies (no multicast) of kChunk logits, running
//    ahead across rows; a stage is refilled as soon as the consumers release it.
//  consumers (8 warps): scale every logit (candidates.rs:30-37) with one
//    multiply and compare it with a running lower bound `tau` of the row's
//    k-th largest scaled value; the few logits at or above it are appended to
//    the row's candidate list. tau comes from per-lane running maxima: each
//    warp's t-th largest lane maximum (t = ceil(k/8)) stands for t distinct
//    logits at or above it, so the minimum over the 8 warps is at most the
//    k-th largest of the row. Every logit that can survive top-k is therefore
//    in the list. The list is double-buffered per row.
//  finisher (1 warp): takes a finished list and applies the reference's exact
//    arithmetic while the consumers stream the next row: the k-th largest key
//    (candidates.rs:38-43, 93-97), the keep test (:44-51), top-p over the
//    (value desc, index asc) order with its sequential sums (:55-78), softmax
//    in index order (filters.rs:5-15), and the argmax or the inverse-CDF draw
//    (sampler.rs:48-52, 111-121). Sets are small; the sequential sums run on
//    one lane in the reference's order, so every result is bit-identical.
//
// Rows whose list overflows kCap (thousands of logits tied with the k-th) are
// kept in a per-CTA list and sampled at the end of the CTA by all its threads
// with the large-row code (rsc_large.cuh), so a call is one launch.
//
// All waits are bounded (mbar_wait); the consumer warps decide together
// through barrier reductions, so a timeout can never leave some of them at a
// barrier the others have left.
#include "rsc_large.cuh"

namespace rsc {

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kFinisherWarp = kConsumerWarps + 1;
constexpr int kThreads = (kConsumerWarps + 2) * 32;
constexpr uint32_t kChunk = 4096;     // logits per stage (16 KiB)
constexpr uint32_t kStages = 3;       // 48 KiB in flight per CTA
constexpr int kCtasPerSm = 3;         // three row pipelines per SM: 144 KiB in flight
constexpr uint32_t kCap = kSmallCap;  // candidate list capacity
constexpr uint32_t kCompactAt = kCap / 2;
constexpr int kBarConsumers = 1;      // named barrier of the consumer warps
constexpr uint32_t kMaxSplits = kStreamMaxSplits;
constexpr uint32_t kOvfCap = kStreamOvfCap;  // overflowing rows a CTA can defer
static_assert(kSmallTopK <= 8 * 32, "tau uses the t-th of 32 lane maxima per warp, t = ceil(k/8)");
static_assert(kSmallTopK <= kCompactAt / 2, "the list must hold k plus a chunk's new candidates");

using ConsumerSync = SyncNamed<kBarConsumers, kConsumers>;

struct CandList {
    uint32_t key[kCap];
    uint32_t idx[kCap];
};

// Lists up to this size are ordered by ranks (each lane counts, for its few
// entries, the entries that precede them) instead of radix select and sorts.
constexpr uint32_t kRankMax = 128;
// No list to finish (a finisher piece that only publishes or defers).
constexpr uint32_t kNoList = 0xffffffffu;
// Shortest row part the balanced schedule makes for batches of at most one
// row per CTA.
constexpr uint32_t kMinPartChunks = 16;
// Chunks past a piece's first whose lane maxima join its first bound (the
// ring holds them all: the first chunk and kPeekChunks more).
constexpr uint32_t kPeekChunks = 2;
static_assert(kPeekChunks < kStages, "the peeked chunks and the first fit the ring");

// Workspace of one finishing warp.
struct FinishWork {
    static constexpr uint32_t kCapacity = kCap;  // survivors it can finish
    unsigned long long items[kCap];   // (~key, idx): value desc, index asc
    unsigned long long items2[kCap];  // (idx, key): index asc
    float vals[kCap];
    uint32_t hist[256];
    uint32_t sel[2];
};

// The vocab-sharded merge's workspace of one warp: room for kMergeCap
// survivors of the keep test (k plus ties), in 2.5 KB instead of 11 KB, so
// that more merging warps fit an SM. The radix select's histogram shares
// items2's space: finish_list is done with it before items2 is written. A row
// with more survivors (more than kMergeCap - k values tied with the k-th) is
// finished again with a FinishWork.
constexpr uint32_t kMergeCap = 128;
struct MergeWork {
    static constexpr uint32_t kCapacity = kMergeCap;
    unsigned long long items[kMergeCap];
    union {
        unsigned long long items2[kMergeCap];
        uint32_t hist[256];
    };
    float vals[kMergeCap];
    uint32_t sel[2];
};
static_assert(sizeof(unsigned long long) * kMergeCap == sizeof(uint32_t) * 256,
              "the histogram fills items2's space exactly");

struct StreamSmem {
    alignas(128) float ring[kStages][kChunk];
    CandList list[2];
    FinishWork fw;
    double exp_tab[32];
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t list_full[2];
    uint64_t list_empty[2];
    uint32_t count[2];
    uint32_t overflow[2];
    float tau_final[2];  // the consumers' last bound of the row (<= its k-th largest value)
    float warp_tau[2][kConsumerWarps];
    float st_max[2][kConsumerWarps];
    float lse_m[2][kConsumerWarps];  // per consumer warp: partial log-sum-exp of the piece
    float lse_s[2][kConsumerWarps];
    uint32_t chist[256];
    uint32_t csel[2];
    uint32_t error;
    uint32_t issued;
    uint32_t ovf_count;  // rows deferred to the epilogue (finisher only)
    uint32_t ovf_rows[kOvfCap];
    uint32_t slot;
};
static_assert(sizeof(large::LargeSmem<kThreads>) <= sizeof(float) * kStages * kChunk,
              "the epilogue's large-row workspace lives in the idle ring");
// The epilogue's top-k histogram (4096 bins) sits in the idle ring after the
// large-row workspace. Its gather serves k up to kTwoPassMaxK (the list keeps
// room for ties).
constexpr uint32_t kTopkBins = 4096;
constexpr uint32_t kTwoPassMaxK = kCap - RSC_SHARD_TIE_CAP;
static_assert(kTwoPassMaxK == kTwoPassTopK, "the host routes exactly the k the epilogue serves");
constexpr size_t kTopkHistOffset = (sizeof(large::LargeSmem<kThreads>) + 255) & ~static_cast<size_t>(255);
static_assert(kTopkHistOffset + kTopkBins * sizeof(uint32_t) <= sizeof(float) * kStages * kChunk,
              "the top-k histogram fits the idle ring beside the large-row workspace");

// Geometry of one row: a scalar head up to 16-byte alignment, a body of
// `nbody` logits copied by TMA in chunks, a scalar tail.
struct RowGeom {
    const float *p;
    uint32_t head;    // logits [0, head) read directly
    uint32_t nbody;   // logits [head, head + nbody) by TMA, a multiple of 4
    uint32_t nchunks;
};

__device__ __forceinline__ RowGeom row_geom(const float *logits, size_t row, size_t stride,
                                            uint32_t vocab) {
    RowGeom g;
    g.p = logits + row * stride;
    uint32_t mis = static_cast<uint32_t>((reinterpret_cast<uintptr_t>(g.p) >> 2) & 3u);
    g.head = mis ? min(vocab, 4u - mis) : 0u;
    g.nbody = ((vocab - g.head) / 4u) * 4u;
    g.nchunks = (g.nbody + kChunk - 1) / kChunk;
    return g;
}

// Barrier of the consumer warps that also ORs a predicate across them: every
// consumer thread gets the same answer.
__device__ __forceinline__ bool consumers_any(bool p) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\t"
        "setp.ne.u32 pi, %1, 0;\n\t"
        "bar.red.or.pred po, %2, %3, pi;\n\t"
        "selp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(r)
        : "r"(p ? 1u : 0u), "n"(kBarConsumers), "n"(kConsumers)
        : "memory");
    return r != 0;
}

// Appends the logits whose bit is set in `m` (bit 4*jj + e: element e of
// float4 jj, global index i0 + 4*kConsumers*jj + e) with one shared atomic.
// Returns true if the list grew past `mark`.
template <int N>
__device__ __forceinline__ bool append_mask(CandList &L, uint32_t *count, uint32_t *overflow,
                                            uint32_t m, const float (&v)[N], uint32_t i0,
                                            uint32_t mark) {
    uint32_t pos = atomicAdd(count, static_cast<uint32_t>(__popc(m)));
#pragma unroll
    for (int e = 0; e < N; ++e) {  // unrolled: v stays in registers
        if ((m >> e) & 1u) {
            if (pos < kCap) {
                L.key[pos] = total_key(v[e]);
                L.idx[pos] = i0 + static_cast<uint32_t>(e >> 2) * (4 * kConsumers) + (e & 3);
            } else {
                *overflow = 1;
            }
            ++pos;
        }
    }
    return pos > mark;
}

// Warp-aggregated append of (key, idx) when `take`. Returns true if this
// warp's append reached position `mark` or beyond.
__device__ __forceinline__ bool append_candidate(CandList &L, uint32_t *count, uint32_t *overflow,
                                                 bool take, uint32_t key, uint32_t idx,
                                                 uint32_t mark) {
    const uint32_t ballot = __ballot_sync(0xffffffffu, take);
    if (!ballot) return false;
    const int lane = threadIdx.x & 31;
    const int leader = __ffs(ballot) - 1;
    uint32_t base = 0;
    if (lane == leader) base = atomicAdd(count, static_cast<uint32_t>(__popc(ballot)));
    base = __shfl_sync(0xffffffffu, base, leader);
    if (take) {
        uint32_t pos = base + __popc(ballot & ((1u << lane) - 1u));
        if (pos < kCap) {
            L.key[pos] = key;
            L.idx[pos] = idx;
        } else {
            *overflow = 1;
        }
    }
    return base + __popc(ballot) > mark;
}

// Each warp's t-th largest lane maximum, written for the consumers' next
// barrier (double-buffered by `par`).
__device__ __forceinline__ void post_warp_bound(StreamSmem &sm, float lmax, uint32_t t, int cw,
                                                uint32_t par) {
    const int lane = threadIdx.x & 31;
    if (t <= 8) {
        // Small t: t-1 rounds of "remove one lane holding the maximum", then
        // the maximum of the rest, with hardware warp max reductions on
        // total-order keys (-inf maps above 0, the removed value).
        uint32_t key = total_key(lmax);
        for (uint32_t i = 1; i < t; ++i) {
            const uint32_t m = __reduce_max_sync(0xffffffffu, key);
            const uint32_t b = __ballot_sync(0xffffffffu, key == m);
            if (lane == __ffs(b) - 1) key = 0u;
        }
        const uint32_t m = __reduce_max_sync(0xffffffffu, key);
        if (lane == 0) sm.warp_tau[par][cw] = key_to_float(m);
        return;
    }
    float m = lmax;
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const float o = __shfl_xor_sync(0xffffffffu, m, j);
            const bool ascending = (lane & k) == 0;
            const bool lower = (lane & j) == 0;
            m = (lower == ascending) ? fminf(m, o) : fmaxf(m, o);
        }
    }
    // Ascending across lanes: lane 32 - t holds the t-th largest.
    const float bound = __shfl_sync(0xffffffffu, m, 32 - static_cast<int>(t));
    if (lane == 0) sm.warp_tau[par][cw] = bound;
}

__device__ __forceinline__ float read_bound(const StreamSmem &sm, uint32_t par) {
    float b = sm.warp_tau[par][0];
#pragma unroll
    for (int w = 1; w < kConsumerWarps; ++w) b = fminf(b, sm.warp_tau[par][w]);
    return b;
}

// --- finisher (one warp) ------------------------------------------------------

// s <- fl(s + v[i]) over i in order (one lane; loads batched ahead of the adds).
__device__ __forceinline__ float chain_sum(const float *v, uint32_t n, float s) {
    uint32_t i = 0;
    for (; i + 8 <= n; i += 8) {
        float t[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) t[q] = v[i + q];
#pragma unroll
        for (int q = 0; q < 8; ++q) s = __fadd_rn(s, t[q]);
    }
    for (; i < n; ++i) s = __fadd_rn(s, v[i]);
    return s;
}

// First i whose running sum (from +0) after v[i] exceeds p (candidates.rs:67-75); n if none.
__device__ __forceinline__ uint32_t chain_cut_above(const float *v, uint32_t n, float p) {
    float s = 0.0f;
    uint32_t i = 0;
    for (; i + 8 <= n; i += 8) {
        float t[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) t[q] = v[i + q];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            s = __fadd_rn(s, t[q]);
            if (s > p) return i + q;
        }
    }
    for (; i < n; ++i) {
        s = __fadd_rn(s, v[i]);
        if (s > p) return i;
    }
    return n;
}

// sample_multinomial's loop (sampler.rs:111-121): first i with r < cumsum.
__device__ __forceinline__ uint32_t chain_draw(const float *v, uint32_t n, float r, float *lo,
                                               float *hi) {
    float s = 0.0f;
    uint32_t i = 0;
    for (; i + 8 <= n; i += 8) {
        float t[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) t[q] = v[i + q];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float b = s;
            s = __fadd_rn(s, t[q]);
            if (r < s) {
                *lo = b;
                *hi = s;
                return i + q;
            }
        }
    }
    for (; i < n; ++i) {
        const float b = s;
        s = __fadd_rn(s, v[i]);
        if (r < s) {
            *lo = b;
            *hi = s;
            return i;
        }
    }
    *lo = s;
    *hi = s;
    return n;
}

__device__ __forceinline__ uint32_t pow2_at_least(uint32_t n) {
    uint32_t p = 32;
    while (p < n) p <<= 1;
    return p;
}

// Survivors of the keep test against `thr` packed into fw.items (warp ballot
// compaction); returns their number.
template <typename FW, typename Pack>
__device__ __forceinline__ uint32_t gather_survivors(FW &fw, const uint32_t *ckey,
                                                     const uint32_t *cidx, uint32_t count,
                                                     Pack pack) {
    const int lane = threadIdx.x & 31;
    uint32_t n = 0;
    for (uint32_t base = 0; base < count; base += 32) {
        const uint32_t i = base + lane;
        bool keep = false;
        unsigned long long it = 0;
        if (i < count) keep = pack(ckey[i], cidx[i], &it);
        const uint32_t ballot = __ballot_sync(0xffffffffu, keep);
        if (keep) fw.items[n + __popc(ballot & ((1u << lane) - 1u))] = it;
        n += __popc(ballot);
    }
    return n;
}

// Drops, in place, the candidates below `tau` (one warp). tau is at most the
// row's k-th largest value, so nothing dropped could survive top-k; an IEEE
// compare keeps -0.0 against +0.0 as the keep test does.
__device__ __forceinline__ uint32_t precut_list(CandList &L, uint32_t count, float tau) {
    const int lane = threadIdx.x & 31;
    uint32_t n = 0;
    for (uint32_t base = 0; base < count; base += 32) {
        const uint32_t i = base + lane;
        uint32_t key = 0, idx = 0;
        bool keep = false;
        if (i < count) {
            key = L.key[i];
            idx = L.idx[i];
            keep = key_to_float(key) >= tau;
        }
        const uint32_t ballot = __ballot_sync(0xffffffffu, keep);
        if (keep) {
            const uint32_t pos = n + __popc(ballot & ((1u << lane) - 1u));
            L.key[pos] = key;
            L.idx[pos] = idx;
        }
        n += __popc(ballot);
        __syncwarp();
    }
    return n;
}

// Finishes a row from its candidate list (one warp). Writes the row's outputs
// and returns true; with a workspace smaller than the list (MergeWork) it
// returns false, having written nothing, when more candidates survive the
// keep test than the workspace holds.
template <typename FW>
__device__ bool finish_list(FW &fw, const double *tab, const uint32_t *ckey,
                            const uint32_t *cidx, uint32_t count, const CallParams &cp, size_t row,
                            uint32_t *out_ids, int32_t *out_status, float *out_probs) {
    const int lane = threadIdx.x & 31;
    const bool topp = cp.topp_active;
    // Exact top-k threshold (candidates.rs:38-43) and the survivors of the
    // keep test (:44-51) in (value desc, index asc) order. With fewer than k
    // candidates every candidate survives (the k-th largest is then -inf or
    // below, which keeps every value that is not -inf). The survivors are a
    // prefix of that order: the keys at or above the threshold's, then -0.0
    // after a +0.0 threshold (IEEE -0.0 < +0.0 is false).
    float thr = kNegInf;
    uint32_t n;
    if (count <= kRankMax) {
        // (key, ~idx) as one 64-bit word: entry j precedes entry i in the
        // (value desc, index asc) order exactly when its word is larger, so a
        // rank is a count of larger words (branch-free compares).
        constexpr int kPer = kRankMax / 32;
        for (uint32_t i = lane; i < count; i += 32) fw.items2[i] = pack_key_index(ckey[i], ~cidx[i]);
        __syncwarp();
        unsigned long long mine[kPer];
        uint32_t rank[kPer];
#pragma unroll
        for (int q = 0; q < kPer; ++q) {
            const uint32_t i = lane + 32 * q;
            mine[q] = i < count ? fw.items2[i] : ~0ull;
            rank[q] = 0;
        }
        uint32_t j = 0;
        for (; j + 4 <= count; j += 4) {
            unsigned long long w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) w[e] = fw.items2[j + e];
#pragma unroll
            for (int e = 0; e < 4; ++e)
#pragma unroll
                for (int q = 0; q < kPer; ++q) rank[q] += w[e] > mine[q] ? 1u : 0u;
        }
        for (; j < count; ++j) {
            const unsigned long long w = fw.items2[j];
#pragma unroll
            for (int q = 0; q < kPer; ++q) rank[q] += w > mine[q] ? 1u : 0u;
        }
#pragma unroll
        for (int q = 0; q < kPer; ++q) {
            if (lane + 32 * q < count) {
                const uint32_t key = static_cast<uint32_t>(mine[q] >> 32);
                const uint32_t idx = ~static_cast<uint32_t>(mine[q]);
                fw.items[rank[q]] = pack_key_index(~key, idx);
            }
        }
        __syncwarp();
        uint32_t mk[kPer];
#pragma unroll
        for (int q = 0; q < kPer; ++q) mk[q] = static_cast<uint32_t>(mine[q] >> 32);
        if (cp.topk_active && count >= cp.top_k)
            thr = key_to_float(~static_cast<uint32_t>(fw.items[cp.top_k - 1] >> 32));
        uint32_t s = 0;
#pragma unroll
        for (int q = 0; q < kPer; ++q)
            s += (lane + 32 * q < count && survives(key_to_float(mk[q]), thr)) ? 1u : 0u;
        n = __reduce_add_sync(0xffffffffu, s);
    } else {
        if (cp.topk_active && count >= cp.top_k) {
            const uint32_t kth = group_select_kth_largest<32, SyncWarp>(
                count, cp.top_k, [&](uint32_t i) { return ckey[i]; }, fw.hist, fw.sel);
            thr = key_to_float(kth);
        }
        if constexpr (FW::kCapacity < kCap) {
            uint32_t ns = 0;
            for (uint32_t base = 0; base < count; base += 32) {
                const uint32_t i = base + lane;
                ns += __popc(__ballot_sync(0xffffffffu, i < count && survives(key_to_float(ckey[i]), thr)));
            }
            if (ns > FW::kCapacity) return false;
        }
        n = gather_survivors(fw, ckey, cidx, count,
                             [&](uint32_t key, uint32_t idx, unsigned long long *it) {
                                 *it = pack_key_index(~key, idx);
                                 return survives(key_to_float(key), thr);
                             });
        const uint32_t n64 = pow2_at_least(n);
        for (uint32_t i = n + lane; i < n64; i += 32) fw.items[i] = ~0ull;
        group_bitonic_sort<32, SyncWarp>(fw.items, n64);
    }

    if (topp && n > 0) {
        // Candidates::top_p (candidates.rs:55-78): items are (~key, idx)
        // ascending = value descending, index ascending.
        const float maxv = key_to_float(~static_cast<uint32_t>(fw.items[0] >> 32));
        for (uint32_t i = lane; i < n; i += 32)
            fw.vals[i] = expf_ref(__fsub_rn(key_to_float(~static_cast<uint32_t>(fw.items[i] >> 32)), maxv), tab);
        __syncwarp();
        float exp_sum = 0.0f;
        if (lane == 0) exp_sum = chain_sum(fw.vals, n, 0.0f);  // fold(0.0, +)
        exp_sum = __shfl_sync(0xffffffffu, exp_sum, 0);
        for (uint32_t i = lane; i < n; i += 32) fw.vals[i] = __fdiv_rn(fw.vals[i], exp_sum);
        __syncwarp();
        uint32_t cut = 0;
        if (lane == 0) {
            const uint32_t at = chain_cut_above(fw.vals, n, cp.top_p);
            cut = at < n ? at + 1 : n;
        }
        n = __shfl_sync(0xffffffffu, cut, 0);
    }

    // The kept set back in index order (Candidates::top_p re-sorts by index,
    // candidates.rs:77), as (idx, key) in fw.items2.
    if (n <= kRankMax) {
        constexpr int kPer = kRankMax / 32;
        uint32_t mi[kPer], mk[kPer], rank[kPer];
#pragma unroll
        for (int q = 0; q < kPer; ++q) {
            const uint32_t i = lane + 32 * q;
            const unsigned long long x = i < n ? fw.items[i] : ~0ull;
            mi[q] = static_cast<uint32_t>(x);
            mk[q] = ~static_cast<uint32_t>(x >> 32);
            rank[q] = 0;
        }
        uint32_t j = 0;
        for (; j + 4 <= n; j += 4) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) w[e] = static_cast<uint32_t>(fw.items[j + e]);
#pragma unroll
            for (int e = 0; e < 4; ++e)
#pragma unroll
                for (int q = 0; q < kPer; ++q) rank[q] += w[e] < mi[q] ? 1u : 0u;
        }
        for (; j < n; ++j) {
            const uint32_t ij = static_cast<uint32_t>(fw.items[j]);
#pragma unroll
            for (int q = 0; q < kPer; ++q) rank[q] += ij < mi[q] ? 1u : 0u;
        }
#pragma unroll
        for (int q = 0; q < kPer; ++q)
            if (lane + 32 * q < n) fw.items2[rank[q]] = pack_key_index(mi[q], mk[q]);
        __syncwarp();
    } else {
        const uint32_t n64 = pow2_at_least(n);
        for (uint32_t i = lane; i < n64; i += 32) {
            const unsigned long long x = fw.items[i];
            fw.items2[i] = i < n ? pack_key_index(static_cast<uint32_t>(x), ~static_cast<uint32_t>(x >> 32))
                                 : ~0ull;
        }
        group_bitonic_sort<32, SyncWarp>(fw.items2, n64);
    }

    if (cp.out_nsurv && lane == 0) cp.out_nsurv[row] = n;
    if (cp.out_surv) {
        const uint32_t m = min(n, cp.surv_cap);
        for (uint32_t i = lane; i < m; i += 32)
            cp.out_surv[row * cp.surv_cap + i] = static_cast<uint32_t>(fw.items2[i] >> 32);
    }

    // softmax (filters.rs:5-15) over the survivors in index order.
    float mx = kNegInf;
    unsigned long long amax = 0;
    for (uint32_t i = lane; i < n; i += 32) {
        const uint32_t key = static_cast<uint32_t>(fw.items2[i]);
        mx = fmaxf(mx, key_to_float(key));
        const unsigned long long c = pack_key_index(key, i);
        amax = c > amax ? c : amax;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const unsigned long long a = __shfl_xor_sync(0xffffffffu, amax, o);
        amax = a > amax ? a : amax;
    }
    for (uint32_t i = lane; i < n; i += 32)
        fw.vals[i] = expf_ref(__fsub_rn(key_to_float(static_cast<uint32_t>(fw.items2[i])), mx), tab);
    __syncwarp();
    float sum = 0.0f;
    if (lane == 0) sum = chain_sum(fw.vals, n, -0.0f);  // <f32 as Sum>::sum folds from -0.0
    sum = __shfl_sync(0xffffffffu, sum, 0);
    const bool norm = (fabsf(sum) < kPosInf) && sum > 0.0f;
    bool valid = false;
    for (uint32_t i = lane; i < n; i += 32) {
        float pi = fw.vals[i];
        if (norm) pi = __fdiv_rn(pi, sum);
        fw.vals[i] = pi;
        if (!(pi != pi || pi <= 0.0f)) valid = true;
    }
    valid = __any_sync(0xffffffffu, valid);
    __syncwarp();
    if (cp.out_survp) {
        const uint32_t m = min(n, cp.surv_cap);
        for (uint32_t i = lane; i < m; i += 32) cp.out_survp[row * cp.surv_cap + i] = fw.vals[i];
    }
    if (lane == 0) {
        int32_t status = RSC_ROW_NO_VALID_TOKENS;
        uint32_t token = 0;
        float prob = __uint_as_float(0x7fc00000u);
        if (valid) {
            uint32_t pos;
            status = RSC_ROW_OK;
            if (cp.argmax_branch) {
                pos = static_cast<uint32_t>(amax);
            } else {
                const float r = row_uniform(cp, row);
                float lo, hi;
                pos = chain_draw(fw.vals, n, r, &lo, &hi);
                if (pos >= n) pos = n - 1;
                if (fabsf(r - hi) < 1e-6f || fabsf(r - lo) < 1e-6f)
                    status |= RSC_ROW_FLAG_DRAW_NEAR_BOUNDARY;
            }
            token = static_cast<uint32_t>(fw.items2[pos] >> 32);
            prob = fw.vals[pos];
        }
        out_ids[row] = token;
        out_status[row] = status;
        if (out_probs) out_probs[row] = prob;
    }
    __syncwarp();
    return true;
}

// Record of one part of a row (a vocab shard, or a segment of a split row),
// written by one warp: the part's candidates that can reach the row's k-th
// largest value, at most `cap_entries` of them, and the part's row statistics.
// If the pre-cut list fits, it is written as it is (every entry is at or above
// `tau`, a lower bound of the part's k-th largest value). Otherwise only the
// entries at or above the part's own k-th largest key are kept, sorted (key
// desc, index asc) and capped, and the number dropped is recorded.
__device__ void record_list(FinishWork &fw, const uint32_t *ckey, const uint32_t *cidx,
                            uint32_t count, const CallParams &cp, float M, float S, uint32_t nfin,
                            unsigned char *rec, uint32_t cap_entries, float tau) {
    const int lane = threadIdx.x & 31;
    ShardRecordHeader *h = reinterpret_cast<ShardRecordHeader *>(rec);
    uint32_t *rkey = reinterpret_cast<uint32_t *>(rec + sizeof(ShardRecordHeader));
    uint32_t *ridx = rkey + cap_entries;
    if (count <= cap_entries) {
        for (uint32_t i = lane; i < count; i += 32) {
            rkey[i] = ckey[i];
            ridx[i] = cidx[i];
        }
        if (lane == 0) {
            h->max_scaled = M;
            h->sum_exp = S;
            h->n_finite = nfin;
            h->n_cand = count;
            h->n_dropped = 0;
            h->last_key = 0;
            h->flags = 0;
            h->tau = tau;
        }
        __syncwarp();
        return;
    }
    uint32_t floor_key = kKeyNegInf + 1u;
    if (count >= cp.top_k) {
        const uint32_t kth = group_select_kth_largest<32, SyncWarp>(
            count, cp.top_k, [&](uint32_t i) { return ckey[i]; }, fw.hist, fw.sel);
        // A +0.0 threshold also keeps -0.0 (IEEE -0.0 < +0.0 is false).
        floor_key = kth == kKeyPosZero ? kKeyNegZero : kth;
    }
    // The entries above the floor (fewer than k of them), then entries at the
    // floor while room remains: whatever is dropped is tied with last_key,
    // the smallest key kept. No order is needed: the merge reads the set.
    uint32_t n_above = 0, n_at = 0, nc = 0;
    for (int pass = 0; pass < 2; ++pass) {
        for (uint32_t base = 0; base < count; base += 32) {
            const uint32_t i = base + lane;
            uint32_t key = 0, idx = 0;
            bool take = false;
            if (i < count) {
                key = ckey[i];
                idx = cidx[i];
                take = pass == 0 ? key > floor_key : key == floor_key;
            }
            const uint32_t ballot = __ballot_sync(0xffffffffu, take);
            const uint32_t pos = nc + __popc(ballot & ((1u << lane) - 1u));
            if (take && pos < cap_entries) {
                rkey[pos] = key;
                ridx[pos] = idx;
            }
            const uint32_t got = __popc(ballot);
            if (pass == 0) n_above += got;
            else n_at += got;
            nc = min(nc + got, cap_entries);
        }
    }
    if (lane == 0) {
        const uint32_t n = n_above + n_at;
        h->max_scaled = M;
        h->sum_exp = S;
        h->n_finite = nfin;
        h->n_cand = nc;
        h->n_dropped = n - nc;
        h->last_key = n_at ? floor_key : 0u;
        h->flags = 0;
        h->tau = key_to_float(floor_key);
    }
    __syncwarp();
}

// Gathers one row's records from `n` parts (vocab shards or row segments)
// into the candidate list L (one warp) and returns their number. The entries
// below the largest of the parts' bounds are dropped on the way: each bound is
// at most its part's k-th largest value, hence at most the row's. *ok becomes
// false when the union cannot be trusted: a part overflowed, the union exceeds
// kCap, or a part dropped tied entries that could reach the row's k-th
// largest value. Records may come from other CTAs of the same grid, so they
// are read past L1 (ld.global.cg).
template <typename RecAt>
__device__ uint32_t merge_records(CandList &L, FinishWork &fw, RecAt rec_at, uint32_t n,
                                  uint32_t cap_entries, const CallParams &cp, bool *ok,
                                  float *tau_out = nullptr) {
    const int lane = threadIdx.x & 31;
    // Headers: lane s reads part s (n <= 32), all at once.
    uint32_t flags = 0, ndrop = 0, ncand = 0;
    float tau_s = -3.402823466e38f;
    if (static_cast<uint32_t>(lane) < n) {
        const uint32_t *h = reinterpret_cast<const uint32_t *>(rec_at(lane));
        ncand = min(__ldcg(h + 3), cap_entries);
        ndrop = __ldcg(h + 4);
        flags = __ldcg(h + 6);
        tau_s = __uint_as_float(__ldcg(h + 7));
    }
    bool good = !__any_sync(0xffffffffu, flags != 0u);
    float tau = tau_s;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tau = fmaxf(tau, __shfl_xor_sync(0xffffffffu, tau, o));
    if (tau_out) *tau_out = tau;
    const bool any_dropped = __any_sync(0xffffffffu, ndrop > 0u);
    uint32_t count = 0;
    for (uint32_t s = 0; s < n && good; ++s) {
        const uint32_t nc = __shfl_sync(0xffffffffu, ncand, static_cast<int>(s));
        const uint32_t *rkey = reinterpret_cast<const uint32_t *>(rec_at(s)) + 8;
        const uint32_t *ridx = rkey + cap_entries;
        constexpr int kBatchLoads = 4;  // loads in flight per lane
        for (uint32_t base = 0; base < nc; base += 32 * kBatchLoads) {
            uint32_t kk[kBatchLoads], ii[kBatchLoads];
#pragma unroll
            for (int q = 0; q < kBatchLoads; ++q) {
                const uint32_t i = base + q * 32 + lane;
                kk[q] = i < nc ? __ldcg(rkey + i) : 0u;
                ii[q] = i < nc ? __ldcg(ridx + i) : 0u;
            }
#pragma unroll
            for (int q = 0; q < kBatchLoads; ++q) {
                const uint32_t i = base + q * 32 + lane;
                const bool keep = i < nc && key_to_float(kk[q]) >= tau;
                const uint32_t ballot = __ballot_sync(0xffffffffu, keep);
                const uint32_t pos = count + __popc(ballot & ((1u << lane) - 1u));
                if (keep && pos < kCap) {
                    L.key[pos] = kk[q];
                    L.idx[pos] = ii[q];
                }
                count += __popc(ballot);
            }
        }
    }
    if (count > kCap) good = false;
    __syncwarp();
    if (good && any_dropped) {
        uint32_t floor_key = 0u;
        const bool have_kth = cp.topk_active && count >= cp.top_k;
        if (have_kth) {
            const uint32_t kth = group_select_kth_largest<32, SyncWarp>(
                count, cp.top_k, [&](uint32_t i) { return L.key[i]; }, fw.hist, fw.sel);
            floor_key = kth == kKeyPosZero ? kKeyNegZero : kth;
        }
        for (uint32_t s = 0; s < n; ++s) {
            const uint32_t *h = reinterpret_cast<const uint32_t *>(rec_at(s));
            if (__ldcg(h + 4) > 0 && (!have_kth || __ldcg(h + 5) >= floor_key)) good = false;
        }
    }
    *ok = good;
    return min(count, kCap);
}

// merge_records for the vocab-sharded merge, with every part's entries in
// flight at once: lane l serves part l / (32 / n) and reads every (32 / n)-th
// of its entries, so a row costs one or two L2 round trips instead of one per
// part. The union is the same set of entries (in another order, which the
// finisher's ranks do not see), cut by the same bound and checked the same way.
template <typename FW, typename RecAt>
__device__ uint32_t merge_parts_batched(CandList &L, FW &fw, RecAt rec_at, uint32_t n,
                                        uint32_t cap_entries, const CallParams &cp, bool *ok) {
    const uint32_t lane = threadIdx.x & 31u;
    uint32_t flags = 0, ndrop = 0, ncand = 0;
    float tau_s = -3.402823466e38f;
    if (lane < n) {
        const uint32_t *h = reinterpret_cast<const uint32_t *>(rec_at(lane));
        ncand = min(__ldcg(h + 3), cap_entries);
        ndrop = __ldcg(h + 4);
        flags = __ldcg(h + 6);
        tau_s = __uint_as_float(__ldcg(h + 7));
    }
    bool good = !__any_sync(0xffffffffu, flags != 0u);
    float tau = tau_s;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tau = fmaxf(tau, __shfl_xor_sync(0xffffffffu, tau, o));
    const bool any_dropped = __any_sync(0xffffffffu, ndrop > 0u);
    const uint32_t lps = 32u / n;  // lanes per part (n <= 32)
    const uint32_t part = lane / lps, sub = lane % lps;
    const uint32_t nc = __shfl_sync(0xffffffffu, ncand, part < n ? part : 0u);
    const bool mine = part < n;
    const uint32_t *rkey =
        mine ? reinterpret_cast<const uint32_t *>(rec_at(part)) + 8 : nullptr;
    const uint32_t *ridx = mine ? rkey + cap_entries : nullptr;
    const uint32_t most = (cap_entries + lps - 1) / lps;  // entries a lane may hold
    const uint32_t below = (1u << lane) - 1u;
    uint32_t count = 0;
    constexpr uint32_t kBatchLoads = 8;
    for (uint32_t q0 = 0; q0 < most && good; q0 += kBatchLoads) {
        uint32_t kk[kBatchLoads], ii[kBatchLoads];
#pragma unroll
        for (uint32_t q = 0; q < kBatchLoads; ++q) {
            const uint32_t j = sub + (q0 + q) * lps;
            const bool in = mine && j < nc;
            kk[q] = in ? __ldcg(rkey + j) : 0u;
            ii[q] = in ? __ldcg(ridx + j) : 0u;
        }
#pragma unroll
        for (uint32_t q = 0; q < kBatchLoads; ++q) {
            const uint32_t j = sub + (q0 + q) * lps;
            const bool keep = mine && j < nc && key_to_float(kk[q]) >= tau;
            const uint32_t ballot = __ballot_sync(0xffffffffu, keep);
            const uint32_t pos = count + __popc(ballot & below);
            if (keep && pos < kCap) {
                L.key[pos] = kk[q];
                L.idx[pos] = ii[q];
            }
            count += __popc(ballot);
        }
    }
    if (count > kCap) good = false;
    __syncwarp();
    if (good && any_dropped) {
        uint32_t floor_key = 0u;
        const bool have_kth = cp.topk_active && count >= cp.top_k;
        if (have_kth) {
            const uint32_t kth = group_select_kth_largest<32, SyncWarp>(
                count, cp.top_k, [&](uint32_t i) { return L.key[i]; }, fw.hist, fw.sel);
            floor_key = kth == kKeyPosZero ? kKeyNegZero : kth;
        }
        for (uint32_t s = 0; s < n; ++s) {
            const uint32_t *h = reinterpret_cast<const uint32_t *>(rec_at(s));
            if (__ldcg(h + 4) > 0 && (!have_kth || __ldcg(h + 5) >= floor_key)) good = false;
        }
    }
    *ok = good;
    return min(count, kCap);
}

// --- work schedule -------------------------------------------------------------
//
// The batch is rows x nch chunks (nch = ceil(vocab / kChunk), the same for
// every row; chunks past a row's own body are empty). Two schedules:
//  - whole rows, round-robin over the CTAs (streamk = 0);
//  - balanced ranges (streamk = 1): CTA b takes the chunks
//    [b*T/G, (b+1)*T/G) of the batch in row-major order, T = rows * nch,
//    G = gridDim.x. A row whose chunks fall to several CTAs is finished by
//    the last of its parts to arrive, from the parts' records. Every CTA
//    streams the same number of chunks (+-1), so no SM idles while another
//    finishes a last row.
struct Piece {
    size_t row;
    uint32_t c0, c1;  // chunks [c0, c1) of the row
    uint32_t part;    // this CTA's part of the row, 0 .. nparts-1
    uint32_t nparts;
};

// The CTA that owns global chunk x under the balanced schedule: the largest
// b with floor(b*T/G) <= x.
__device__ __forceinline__ uint32_t chunk_owner(unsigned long long x, unsigned long long T,
                                                uint32_t G) {
    return static_cast<uint32_t>(((x + 1ull) * G - 1ull) / T);
}

// The u-th piece of this CTA; false past the last. Under the balanced
// schedule a CTA takes its last piece (in row order) first: that piece is
// the head of a row whose tail the next CTA also streams first, so both parts
// of every split row arrive early and the row's merge overlaps streaming. The
// CTA then ends on one of its whole rows, which needs no merge.
__device__ __forceinline__ bool get_piece(size_t rows, uint32_t nch, uint32_t streamk, uint32_t u,
                                          Piece &pc) {
    if (!streamk) {
        const size_t row = blockIdx.x + static_cast<size_t>(u) * gridDim.x;
        if (row >= rows) return false;
        pc.row = row;
        pc.c0 = 0;
        pc.c1 = nch;
        pc.part = 0;
        pc.nparts = 1;
        return true;
    }
    const unsigned long long T = static_cast<unsigned long long>(rows) * nch;
    const unsigned long long G = gridDim.x;
    const unsigned long long begin = T * blockIdx.x / G;
    const unsigned long long end = T * (blockIdx.x + 1ull) / G;
    // Pieces: the rows r >= begin / nch that start before `end` (an empty
    // range inside a row still makes one empty piece of it).
    const size_t first_row = static_cast<size_t>(begin / nch);
    const unsigned long long frs = static_cast<unsigned long long>(first_row) * nch;
    const uint32_t npieces =
        frs < end ? static_cast<uint32_t>((end + nch - 1ull) / nch - first_row) : 0u;
    if (u >= npieces) return false;
    const size_t row = first_row + (u == 0 ? npieces - 1u : u - 1u);
    const unsigned long long rs = static_cast<unsigned long long>(row) * nch;
    pc.row = row;
    pc.c0 = static_cast<uint32_t>((begin > rs ? begin : rs) - rs);
    pc.c1 = static_cast<uint32_t>((end < rs + nch ? end : rs + nch) - rs);
    const uint32_t first = chunk_owner(rs, T, gridDim.x);
    const uint32_t last = chunk_owner(rs + nch - 1ull, T, gridDim.x);
    pc.part = blockIdx.x - first;
    pc.nparts = last - first + 1u;
    return true;
}

// A row whose candidates overflowed joins the CTA's epilogue list (one lane
// of the finisher). The host bounds the rows per CTA below kOvfCap; a full
// list would report the row as not sampled.
__device__ __forceinline__ void defer_row(StreamSmem &sm, size_t row, uint32_t *out_ids,
                                          int32_t *out_status) {
    if (sm.ovf_count < kOvfCap) {
        sm.ovf_rows[sm.ovf_count++] = static_cast<uint32_t>(row);
    } else {
        out_ids[row] = 0;
        out_status[row] = RSC_ROW_INTERNAL;
    }
}

// Whether the streaming filter serves a row with parameters r (the host's
// routing rule for a whole call, applied to one row).
__device__ __forceinline__ bool streams_row(const CallParams &r, uint32_t vocab) {
    return r.mode == kModeSampleLogits && r.normal_scale &&
           ((r.topk_active && r.top_k <= kSmallTopK) || (!r.topk_active && vocab <= kSmallCap));
}

// A deferred row with top-k on (its list overflowed, so its bound admitted
// more than the list holds), by the whole CTA in two passes over the row:
// a histogram of the top 12 bits of the candidates' keys finds the bin that
// holds the k-th largest value; a second pass gathers every candidate at or
// above that bin's smallest value into the finisher's list, which
// finish_list completes exactly as for a streamed row (its list is any
// superset of the survivors, all candidates at or above a bound no higher
// than the k-th value). Returns false, with nothing written, when the row's
// parameters are not the streaming filter's (top-k on, k <= kSmallTopK, a
// normal scale) or the gather would exceed the list (heavy ties); the row
// then takes the large-row code.
// With `rec` (a vocab shard's partial pass) the gathered list becomes the
// shard's record instead (indices offset by index_offset), cut exactly as a
// streamed row's record.
__device__ __noinline__ bool epilogue_topk_row(const CallParams &call, const float *p, uint32_t vocab,
                                               size_t row, StreamSmem &sm, uint32_t *hist,
                                               uint32_t *out_ids, int32_t *out_status,
                                               float *out_probs, unsigned char *rec,
                                               uint32_t index_offset) {
    const CallParams cp = for_row(call, row, vocab);
    if (cp.mode != kModeSampleLogits || !cp.normal_scale || !cp.topk_active || cp.top_k > kTwoPassMaxK)
        return false;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float scale = cp.scale;
    // Every pass visits the row's scaled values with one call of fn(v, i)
    // per value and the same number of calls in every thread (fn may use
    // warp-collective operations; values past the row come as -inf): a scalar
    // head up to 16-byte alignment and a scalar tail (a single call each),
    // and the body in float4 loads, kGather4 of them in flight per thread.
    constexpr uint32_t kGather4 = 8;
    const uint32_t mis = static_cast<uint32_t>((reinterpret_cast<uintptr_t>(p) >> 2) & 3u);
    const uint32_t head = mis ? min(vocab, 4u - mis) : 0u;
    const uint32_t n4 = (vocab - head) / 4u;
    const uint32_t tail0 = head + 4u * n4;
    const float4 *p4 = reinterpret_cast<const float4 *>(p + head);
    auto visit = [&](auto &&fn) {
        {
            uint32_t i = ~0u;
            if (threadIdx.x < head) i = threadIdx.x;
            else if (threadIdx.x >= 32 && threadIdx.x - 32 < vocab - tail0) i = tail0 + threadIdx.x - 32;
            fn(i != ~0u ? scale_logit(p[i], scale) : kNegInf, i);
        }
        for (uint32_t base = 0; base < n4; base += kThreads * kGather4) {
            float4 f[kGather4];
#pragma unroll
            for (uint32_t q = 0; q < kGather4; ++q) {
                const uint32_t j = base + q * kThreads + threadIdx.x;
                f[q] = j < n4 ? p4[j] : make_float4(kNegInf, kNegInf, kNegInf, kNegInf);
            }
#pragma unroll
            for (uint32_t q = 0; q < kGather4; ++q) {
                const uint32_t i = head + 4u * (base + q * kThreads + threadIdx.x);
                fn(scale_logit(f[q].x, scale), i);
                fn(scale_logit(f[q].y, scale), i + 1u);
                fn(scale_logit(f[q].z, scale), i + 2u);
                fn(scale_logit(f[q].w, scale), i + 3u);
            }
        }
    };
    // Pass 0: each thread's two largest candidates (every scaled value but
    // -inf; NaN reads as -inf). The k-th largest of these 2 x kThreads values
    // has k distinct values at or above it, so it bounds the row's k-th value
    // from below: the histogram then counts only the values at or above it,
    // and its few hot bins see few atomics.
    float m1 = kNegInf, m2 = kNegInf;
    visit([&](float v, uint32_t) {
        if (v > m1) {
            m2 = m1;
            m1 = v;
        } else if (v > m2) {
            m2 = v;
        }
    });
    // Key 0 (a NaN pattern) stands for "no candidate".
    hist[threadIdx.x] = m1 != kNegInf ? total_key(m1) : 0u;
    hist[kThreads + threadIdx.x] = m2 != kNegInf ? total_key(m2) : 0u;
    const uint32_t kmax = __reduce_max_sync(0xffffffffu, hist[threadIdx.x]);
    if (threadIdx.x == 0) {
        sm.count[0] = 0;
        sm.csel[0] = 0;  // the row's largest key
    }
    __syncthreads();
    if (lane == 0 && kmax) atomicMax(&sm.csel[0], kmax);
    float bound = -3.402823466e38f;
    if (cp.top_k <= 2u * kThreads) {
        const uint32_t bkey = group_select_kth_largest<kThreads, SyncBlock>(
            2u * kThreads, cp.top_k, [&](uint32_t i) { return hist[i]; }, hist + 1024, hist + 1280);
        if (bkey) bound = key_to_float(bkey);
    }
    __syncthreads();
    for (uint32_t b = threadIdx.x; b < kTopkBins; b += kThreads) hist[b] = 0;
    __syncthreads();
    // Pass 1: the histogram of the top 12 key bits of the values at or above
    // the bound. Lanes of a warp that share a bin add once, through their
    // leader.
    visit([&](float v, uint32_t) {
        const bool counted = v != kNegInf && v >= bound;
        if (!__any_sync(0xffffffffu, counted)) return;  // most warps, with a tight bound
        const uint32_t bin = counted ? total_key(v) >> 20 : kTopkBins;
        const uint32_t peers = __match_any_sync(0xffffffffu, bin);
        if (counted && lane == __ffs(peers) - 1)
            atomicAdd(&hist[bin], static_cast<uint32_t>(__popc(peers)));
    });
    __syncthreads();
    // Warp 0: the bin of the k-th largest value, scanning from the top (lane l
    // owns bins 4095 - 128 l down to 3968 - 128 l). chist[0..2] get the bin,
    // the candidates above it and the bin's own population.
    if (warp == 0) {
        constexpr uint32_t kPer = kTopkBins / 32;
        uint32_t tot = 0;
        for (uint32_t q = 0; q < kPer; ++q) tot += hist[kTopkBins - 1 - lane * kPer - q];
        uint32_t incl = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t n = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += n;
        }
        const uint32_t all = __shfl_sync(0xffffffffu, incl, 31);
        const uint32_t k = cp.top_k;
        if (incl - tot < k && k <= incl) {
            uint32_t run = incl - tot;
            for (uint32_t q = 0; q < kPer; ++q) {
                const uint32_t b = kTopkBins - 1 - lane * kPer - q;
                if (run + hist[b] >= k) {
                    sm.chist[0] = b;
                    sm.chist[1] = run;
                    sm.chist[2] = hist[b];
                    break;
                }
                run += hist[b];
            }
        }
        if (lane == 0 && all < k) {
            // Fewer than k candidates: every candidate survives the cut.
            sm.chist[0] = 0xffffffffu;
            sm.tau_final[0] = -3.402823466e38f;
        }
    }
    __syncthreads();
    const uint32_t kbin = sm.chist[0];
    if (kbin != 0xffffffffu) {
        uint32_t floor_key = kbin << 20;
        if (sm.chist[1] + sm.chist[2] > kCap) {
            // The k-th value's bin holds more candidates than the list: one
            // more histogram, of the next 12 key bits inside that bin.
            const uint32_t above = sm.chist[1];
            __syncthreads();
            for (uint32_t b = threadIdx.x; b < kTopkBins; b += kThreads) hist[b] = 0;
            __syncthreads();
            visit([&](float v, uint32_t) {
                const uint32_t key = total_key(v);
                const bool counted = v != kNegInf && v >= bound && (key >> 20) == kbin;
                if (!__any_sync(0xffffffffu, counted)) return;
                const uint32_t sub = counted ? (key >> 8) & 0xfffu : kTopkBins;
                const uint32_t peers = __match_any_sync(0xffffffffu, sub);
                if (counted && lane == __ffs(peers) - 1)
                    atomicAdd(&hist[sub], static_cast<uint32_t>(__popc(peers)));
            });
            __syncthreads();
            if (warp == 0) {
                constexpr uint32_t kPer = kTopkBins / 32;
                uint32_t tot = 0;
                for (uint32_t q = 0; q < kPer; ++q) tot += hist[kTopkBins - 1 - lane * kPer - q];
                uint32_t incl = tot;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t n = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += n;
                }
                const uint32_t k = cp.top_k - above;  // still to find inside the bin
                if (incl - tot < k && k <= incl) {
                    uint32_t run = incl - tot;
                    for (uint32_t q = 0; q < kPer; ++q) {
                        const uint32_t b = kTopkBins - 1 - lane * kPer - q;
                        if (run + hist[b] >= k) {
                            sm.chist[3] = b;
                            break;
                        }
                        run += hist[b];
                    }
                }
            }
            __syncthreads();
            floor_key |= sm.chist[3] << 8;
        }
        // Both the bin floor and the pass-0 bound are at most the k-th value.
        if (threadIdx.x == 0) sm.tau_final[0] = fmaxf(key_to_float(floor_key), bound);
    }
    __syncthreads();
    // The bin's smallest value as an IEEE bound: a +0 floor also gathers -0.
    const float floor_v = sm.tau_final[0];
    CandList &L = sm.list[0];
    visit([&](float v, uint32_t i) {
        const bool take = v != kNegInf && v >= floor_v;
        const uint32_t ballot = __ballot_sync(0xffffffffu, take);
        if (ballot == 0u) return;
        uint32_t at = 0;
        if (lane == 0) at = atomicAdd(&sm.count[0], static_cast<uint32_t>(__popc(ballot)));
        at = __shfl_sync(0xffffffffu, at, 0);
        if (take) {
            const uint32_t pos = at + __popc(ballot & ((1u << lane) - 1u));
            if (pos < kCap) {
                L.key[pos] = total_key(v);
                L.idx[pos] = i + index_offset;
            }
        }
    });
    __syncthreads();
    const uint32_t count = sm.count[0];
    if (count > kCap) return false;
    if (warp == 0) {
        if (rec) {
            const float M = sm.csel[0] ? key_to_float(sm.csel[0]) : kNegInf;
            record_list(sm.fw, L.key, L.idx, count, cp, M, 0.0f, 0u, rec,
                        cp.top_k + RSC_SHARD_TIE_CAP, floor_v);
        } else {
            finish_list(sm.fw, sm.exp_tab, L.key, L.idx, count, cp, row, out_ids, out_status,
                        out_probs);
        }
    }
    __syncthreads();
    return true;
}

// The epilogue's per-row work, kept out of line so that the large-row code's
// register pressure stays out of the streaming loops.
__device__ __noinline__ void epilogue_row(const CallParams &cp, const float *p, uint32_t vocab,
                                          size_t row, uint32_t *scratch, uint32_t *out_ids,
                                          int32_t *out_status, float *out_probs,
                                          large::LargeSmem<kThreads> &ls) {
    large::sample_row<kThreads>(for_row(cp, row, vocab), p, vocab, row, scratch, out_ids, out_status,
                                out_probs, ls);
}

// --- the streaming kernel -------------------------------------------------------

// kRows: one parameter set per row (cp.row_params); a separate instance, so
// that calls with one set for every row pay nothing for the lookups.
// kLse: the consumers also accumulate each row part's log-sum-exp of its
// scaled logits (cp.lse_parts), for the log-probability outputs.
// cp is a grid constant: the out-of-line epilogue functions take it by
// reference, and the address of a grid constant points into the parameter
// space, where a plain parameter would be copied to every thread's stack (96
// bytes of local-memory stores per thread and launch, 13.5 MB per 512-row
// call, most of the kernel's DRAM writes).
template <bool kRecord, bool kRows = false, bool kLse = false>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
stream_topk_kernel(const float *__restrict__ logits, size_t rows, uint32_t vocab,
                   size_t row_stride, const __grid_constant__ CallParams cp,
                   uint32_t *__restrict__ out_ids,
                   int32_t *__restrict__ out_status, float *__restrict__ out_probs,
                   uint32_t *__restrict__ scratch, uint32_t slots, uint32_t *__restrict__ slot_lock,
                   uint32_t index_offset, unsigned char *__restrict__ records, size_t rec_bytes,
                   uint32_t nch, uint32_t streamk, uint32_t max_parts,
                   unsigned char *__restrict__ seg_records, uint32_t *__restrict__ row_arrivals) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    StreamSmem &sm = *reinterpret_cast<StreamSmem *>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Pieces of rows (get_piece): a piece is a run of whole chunks of one row;
    // the piece that starts at chunk 0 also takes the row's scalar head, the
    // one that ends at chunk nch the scalar tail. A row cut into several
    // pieces keeps one record per part (kCap / max_parts entries each).
    const uint32_t seg_cap = kCap / max_parts;

    load_exp_table(sm.exp_tab);
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < kStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], kConsumerWarps);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&sm.list_full[b], 1);
            mbar_init(&sm.list_empty[b], 1);
        }
        sm.error = 0;
        sm.issued = 0;
        sm.ovf_count = 0;
        fence_barrier_init();
    }
    __syncthreads();  // the roles split here and meet again in the epilogue
    // A programmatic dependent launch of the next call may start now: its
    // CTAs stream logits (read only) as this grid's CTAs retire, and wait for
    // this grid's completion before they write anything to global memory.
    if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;");

    // Consumers: warps 0 .. kConsumerWarps-1 (a consumer that leaves early
    // does not wait for the others: the finisher's and producer's bounded
    // waits end their roles, and every role meets in the epilogue).
    auto consume = [&]() {
        const int cw = warp;
        uint32_t consumed = 0, par = 0;
        Piece pc;
        for (uint32_t j = 0; get_piece(rows, nch, streamk, j, pc); ++j) {
            const size_t row = pc.row;
            const uint32_t b = j & 1u;
            // The row's parameters. A row with its own parameter set that the
            // streaming filter cannot serve (no top-k over a long row, k above
            // kSmallTopK, T = inf) is marked overflowing from the start: its
            // chunks pass through unfiltered and the epilogue samples it.
            const CallParams rp = kRows ? for_row(cp, row, vocab) : cp;
            const bool live = !kRows || streams_row(rp, vocab);
            const float scale = rp.scale;
            const uint32_t top_k = rp.top_k;
            const uint32_t t_bound =
                live && rp.topk_active ? (top_k + kConsumerWarps - 1) / kConsumerWarps : 0u;
            bool bad = false;
            if (threadIdx.x == 0) {
                if (j >= 2 && !mbar_wait(&sm.list_empty[b], ((j >> 1) - 1u) & 1u)) bad = true;
                sm.count[b] = 0;
                sm.overflow[b] = live ? 0u : 1u;
            }
            if (consumers_any(bad || *static_cast<volatile uint32_t *>(&sm.error) != 0)) break;
            CandList &L = sm.list[b];
            uint32_t *count = &sm.count[b];
            uint32_t *ovf = &sm.overflow[b];
            const RowGeom g = row_geom(logits, row, row_stride, vocab);
            const uint32_t c0 = pc.c0;
            const uint32_t c1 = live ? min(pc.c1, g.nchunks) : c0;  // the producer skips it
            // Candidates satisfy v >= tau. -FLT_MAX admits everything but -inf and
            // NaN (NaN reads as -inf in the reference, and -inf never survives);
            // an IEEE compare also admits -0.0 against +0.0, as the keep test does.
            // NaN admits nothing (a row left to the epilogue).
            float tau = live ? -3.402823466e38f : __int_as_float(0x7fffffff);
            float lmax = kNegInf;  // this lane's largest scaled logit of the piece
            float lse_m = kNegInf, lse_s = 0.0f;  // kLse: this lane's partial log-sum-exp
            // Scalar head and tail (at most 3 logits each).
            {
                const uint32_t ntail = vocab - g.head - g.nbody;
                const uint32_t i = threadIdx.x;
                uint32_t idx = ~0u;
                if (pc.c0 == 0 && i < g.head) idx = i;
                else if (pc.c1 == nch && i >= 4 && i - 4 < ntail) idx = g.head + g.nbody + (i - 4);
                float v = kNegInf;
                if (idx != ~0u) {
                    v = __fmul_rn(g.p[idx], scale);
                    lmax = fmaxf(lmax, v);
                    if constexpr (kLse) lse_add(lse_m, lse_s, scale_logit(g.p[idx], scale));
                }
                append_candidate(L, count, ovf, v >= tau, total_key(v), idx + index_offset, kCap);
            }
            bool stop = false;
            bool got = true, mark = false;
            for (uint32_t c = c0; c < c1; ++c) {
                const uint32_t s = consumed % kStages;
                got &= mbar_wait(&sm.full[s], (consumed / kStages) & 1u);
                const uint32_t len = min(kChunk, g.nbody - c * kChunk);
                const float4 *r4 = reinterpret_cast<const float4 *>(sm.ring[s]);
                const uint32_t base_idx = g.head + c * kChunk + index_offset;
                if (c == c0 && t_bound) {
                    // First chunk: lane maxima before filtering, so that tau is
                    // already high for this chunk's own logits.
                    float cmr = kNegInf;
#pragma unroll
                    for (uint32_t jj = 0; jj < kChunk / 4 / kConsumers; ++jj) {
                        const uint32_t q = threadIdx.x + jj * kConsumers;
                        if (4 * q < len) {
                            const float4 f = r4[q];
                            cmr = fmaxf(fmaxf(cmr, fmaxf(f.x, f.y)), fmaxf(f.z, f.w));
                        }
                    }
                    lmax = fmaxf(lmax, __fmul_rn(cmr, scale));
                    // A bound from one chunk admits about 1% of each chunk
                    // until the first refresh; with the lane maxima of the
                    // next kPeekChunks chunks too (their stages are peeked,
                    // not consumed: the producer is at most kStages ahead)
                    // the first chunks admit about a third of that. This
                    // matters most on a vocab shard's rows, a few chunks long.
#pragma unroll
                    for (uint32_t e = 1; e <= kPeekChunks; ++e) {
                        if (c + e < c1) {
                            const uint32_t s2 = (consumed + e) % kStages;
                            got &= mbar_wait(&sm.full[s2], ((consumed + e) / kStages) & 1u);
                            const uint32_t len2 = min(kChunk, g.nbody - (c + e) * kChunk);
                            const float4 *r42 = reinterpret_cast<const float4 *>(sm.ring[s2]);
                            float cm2 = kNegInf;
#pragma unroll
                            for (uint32_t jj = 0; jj < kChunk / 4 / kConsumers; ++jj) {
                                const uint32_t q = threadIdx.x + jj * kConsumers;
                                if (4 * q < len2) {
                                    const float4 f = r42[q];
                                    cm2 = fmaxf(fmaxf(cm2, fmaxf(f.x, f.y)), fmaxf(f.z, f.w));
                                }
                            }
                            lmax = fmaxf(lmax, __fmul_rn(cm2, scale));
                        }
                    }
                    post_warp_bound(sm, lmax, t_bound, cw, par);
                    if (consumers_any(!got)) {
                        stop = true;
                        break;
                    }
                    tau = fmaxf(tau, read_bound(sm, par));
                    par ^= 1u;
                    if (len < kChunk && len >= top_k) {
                        // A partial first chunk (a row's tail part, or a short
                        // row) spreads too thin over the lanes for their maxima
                        // to bound the k-th largest value: take the chunk's own
                        // exact k-th largest instead (the stage is still held).
                        const float *ring = sm.ring[s];
                        const uint32_t kth = group_select_kth_largest<kConsumers, ConsumerSync>(
                            len, top_k,
                            [&](uint32_t i) { return total_key(scale_logit(ring[i], scale)); },
                            sm.chist, sm.csel);
                        tau = fmaxf(tau, key_to_float(kth));
                    }
                }
                constexpr uint32_t kPerThread = kChunk / 4 / kConsumers;
                float4 f[kPerThread];
                if (len == kChunk) {  // every chunk but a row's last
#pragma unroll
                    for (uint32_t jj = 0; jj < kPerThread; ++jj) f[jj] = r4[threadIdx.x + jj * kConsumers];
                } else {
#pragma unroll
                    for (uint32_t jj = 0; jj < kPerThread; ++jj) {
                        const uint32_t q = threadIdx.x + jj * kConsumers;
                        f[jj] = (4 * q < len) ? r4[q] : make_float4(kNegInf, kNegInf, kNegInf, kNegInf);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.empty[s]);  // stage s released by this warp
                ++consumed;
                // x -> fl(x * scale) is non-decreasing for a finite scale > 0, so
                // the largest scaled value of a group of logits is the scaled
                // largest raw value: one max per logit decides whether this
                // thread's slice holds a candidate at all, and one max per float4
                // which of its float4s do (fmaxf skips NaN, which reads as -inf).
                float m4[kPerThread];
#pragma unroll
                for (uint32_t jj = 0; jj < kPerThread; ++jj)
                    m4[jj] = fmaxf(fmaxf(f[jj].x, f[jj].y), fmaxf(f[jj].z, f[jj].w));
                float cmr = m4[0];
#pragma unroll
                for (uint32_t jj = 1; jj < kPerThread; ++jj) cmr = fmaxf(cmr, m4[jj]);
                const float cm = __fmul_rn(cmr, scale);
                lmax = fmaxf(lmax, cm);
                if constexpr (kLse) {
                    // The slice's scaled maximum first, then its terms (NaN
                    // reads as -inf, whose term is 0).
                    if (cm > lse_m) {
                        lse_s = lse_m == kNegInf ? 0.0f : lse_s * __expf(lse_m - cm);
                        lse_m = cm;
                    }
                    if (lse_m != kNegInf) {
#pragma unroll
                        for (uint32_t jj = 0; jj < kPerThread; ++jj) {
                            lse_s += __expf(scale_logit(f[jj].x, scale) - lse_m);
                            lse_s += __expf(scale_logit(f[jj].y, scale) - lse_m);
                            lse_s += __expf(scale_logit(f[jj].z, scale) - lse_m);
                            lse_s += __expf(scale_logit(f[jj].w, scale) - lse_m);
                        }
                    }
                }
                if (cm >= tau) {
#pragma unroll
                    for (uint32_t jj = 0; jj < kPerThread; ++jj) {
                        if (__fmul_rn(m4[jj], scale) >= tau) {
                            const float v[4] = {__fmul_rn(f[jj].x, scale), __fmul_rn(f[jj].y, scale),
                                                __fmul_rn(f[jj].z, scale), __fmul_rn(f[jj].w, scale)};
                            const uint32_t m = (v[0] >= tau ? 1u : 0u) | (v[1] >= tau ? 2u : 0u) |
                                               (v[2] >= tau ? 4u : 0u) | (v[3] >= tau ? 8u : 0u);
                            mark |= append_mask(L, count, ovf, m, v,
                                                base_idx + 4 * (threadIdx.x + jj * kConsumers), kCompactAt);
                        }
                    }
                }
                const bool last = c + 1 == c1;
                // Bounds refresh after chunks 4 and 8, then every 8, and at the
                // end. (After chunks 1 to kPeekChunks + 1 a refresh would add
                // nothing: the first bound already holds their lane maxima.)
                const uint32_t done = c + 1 - c0;
                const bool refresh =
                    last || (done < 8 ? (done & (done - 1)) == 0 && done > kPeekChunks + 1 : done % 8 == 0);
                if (!refresh) continue;
                if (t_bound) post_warp_bound(sm, lmax, t_bound, cw, par);
                // One barrier per refresh: settles the list, publishes
                // the bounds, and raises the rare events (a failed wait, a long
                // list).
                const bool want_compact = mark && rp.topk_active && !last;
                mark = false;
                if (consumers_any(!got || want_compact)) {
                    if (consumers_any(!got)) {
                        stop = true;
                        break;
                    }
                    // Compaction: tau rises to the list's own k-th largest value.
                    const uint32_t cnt = min(*count, kCap);
                    if (cnt >= top_k) {
                        const uint32_t kth = group_select_kth_largest<kConsumers, ConsumerSync>(
                            cnt, top_k, [&](uint32_t i) { return L.key[i]; }, sm.chist, sm.csel);
                        tau = fmaxf(tau, key_to_float(kth));
                        constexpr int kPer = kCap / kConsumers;
                        uint32_t kk[kPer], ii[kPer];
#pragma unroll
                        for (int e = 0; e < kPer; ++e) {
                            const uint32_t i = threadIdx.x + e * kConsumers;
                            kk[e] = i < cnt ? L.key[i] : 0u;
                            ii[e] = i < cnt ? L.idx[i] : 0u;
                        }
                        ConsumerSync::sync();
                        if (threadIdx.x == 0) *count = 0;
                        ConsumerSync::sync();
#pragma unroll
                        for (int e = 0; e < kPer; ++e) {
                            const uint32_t i = threadIdx.x + e * kConsumers;
                            append_candidate(L, count, ovf, i < cnt && key_to_float(kk[e]) >= tau, kk[e],
                                             ii[e], kCap);
                        }
                        ConsumerSync::sync();
                        if (*count > kCompactAt && threadIdx.x == 0) *ovf = 1;
                    }
                }
                if (t_bound) {
                    tau = fmaxf(tau, read_bound(sm, par));
                    par ^= 1u;
                }
            }
            if (stop) break;
            if (kRecord) {
                const float wm = warp_max(lmax);
                if (lane == 0) sm.st_max[b][cw] = wm;
            }
            if constexpr (kLse) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float m2 = __shfl_xor_sync(0xffffffffu, lse_m, o);
                    const float s2 = __shfl_xor_sync(0xffffffffu, lse_s, o);
                    lse_combine(lse_m, lse_s, m2, s2);
                }
                if (lane == 0) {
                    sm.lse_m[b][cw] = lse_m;
                    sm.lse_s[b][cw] = lse_s;
                }
            }
            if (threadIdx.x == 0) sm.tau_final[b] = tau;
            ConsumerSync::sync();  // the row's list is complete
            if (threadIdx.x == 0) mbar_arrive(&sm.list_full[b]);
        }
    };

    if (warp == kProducerWarp) {
      if (lane == 0) {
        uint32_t q = 0;
        bool ok = true;
        Piece pc;
        for (uint32_t u = 0; ok && get_piece(rows, nch, streamk, u, pc); ++u) {
            // A row the filter cannot serve is not streamed: its consumers
            // hand over an overflowed list and the epilogue samples it.
            if (kRows && !streams_row(for_row(cp, pc.row, vocab), vocab)) continue;
            const RowGeom g = row_geom(logits, pc.row, row_stride, vocab);
            const uint32_t c1 = min(pc.c1, g.nchunks);
            for (uint32_t c = pc.c0; c < c1; ++c) {
                const uint32_t s = q % kStages;
                if (q >= kStages && !mbar_wait(&sm.empty[s], ((q / kStages) - 1u) & 1u)) {
                    atomicExch(&sm.error, 1u);
                    ok = false;
                    break;
                }
                if (*static_cast<volatile uint32_t *>(&sm.error)) {
                    ok = false;
                    break;
                }
                const uint32_t len = min(kChunk, g.nbody - c * kChunk);
                mbar_arrive_expect_tx(&sm.full[s], len * 4u);
                tma_load_1d(sm.ring[s], g.p + g.head + c * kChunk, len * 4u, &sm.full[s]);
                ++q;
            }
        }
        // Before the ring is reused, every copy this thread issued has landed
        // (bounded): the last phase of each stage.
        const uint32_t first = q > kStages ? q - kStages : 0u;
        for (uint32_t i = first; i < q; ++i) mbar_wait(&sm.full[i % kStages], (i / kStages) & 1u);
      }
    } else if (warp == kFinisherWarp) {
        // Global writes wait for the previous grid of the stream (a no-op
        // unless this grid was launched as its programmatic dependent).
        asm volatile("griddepcontrol.wait;" ::: "memory");
        uint32_t u = 0;
        Piece pc;
        for (; get_piece(rows, nch, streamk, u, pc); ++u) {
            const size_t row = pc.row;
            const CallParams rp = kRows ? for_row(cp, row, vocab) : cp;
            const uint32_t j = u;
            const uint32_t b = j & 1u;
            const bool got = mbar_wait(&sm.list_full[b], (j >> 1) & 1u);
            if (__any_sync(0xffffffffu, !got)) {
                if (lane == 0) atomicExch(&sm.error, 1u);
                break;
            }
            if constexpr (kLse) {
                if (lane == 0 && cp.lse_parts) {
                    float m = kNegInf, sum = 0.0f;
                    for (int w = 0; w < kConsumerWarps; ++w) lse_combine(m, sum, sm.lse_m[b][w], sm.lse_s[b][w]);
                    cp.lse_parts[row * cp.lse_stride + pc.part] =
                        make_uint2(total_key(m), __float_as_uint(sum));
                }
            }
            uint32_t cnt = sm.count[b];
            const bool ov = sm.overflow[b] != 0 || cnt > kCap;
            if (!ov && rp.topk_active) cnt = precut_list(sm.list[b], cnt, sm.tau_final[b]);
            uint32_t fin_count = kNoList;  // the list to finish, if any
            if (kRecord) {
                unsigned char *rec = records + row * rec_bytes;
                if (ov) {
                    // Rescued in the epilogue while the deferral list has room;
                    // otherwise the record says so and the merge reports the row.
                    if (lane == 0) {
                        if (sm.ovf_count < kOvfCap) {
                            sm.ovf_rows[sm.ovf_count++] = static_cast<uint32_t>(row);
                        } else {
                            ShardRecordHeader *h = reinterpret_cast<ShardRecordHeader *>(rec);
                            h->flags = 1;
                            h->n_cand = 0;
                            h->n_dropped = 0;
                        }
                    }
                } else {
                    float M = kNegInf;
                    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sm.st_max[b][w]);
                    record_list(sm.fw, sm.list[b].key, sm.list[b].idx, cnt, cp, M, 0.0f, 0u, rec,
                                cp.top_k + RSC_SHARD_TIE_CAP, sm.tau_final[b]);
                }
            } else if (pc.nparts == 1) {
                if (ov) {
                    if (lane == 0) defer_row(sm, row, out_ids, out_status);
                } else {
                    fin_count = cnt;
                }
            } else {
                // One part of a split row: publish its record, and the part
                // that completes the row merges all of them.
                unsigned char *rec = seg_records + (row * max_parts + pc.part) * rec_bytes;
                if (ov) {
                    if (lane == 0) {
                        ShardRecordHeader *h = reinterpret_cast<ShardRecordHeader *>(rec);
                        h->n_cand = 0;
                        h->n_dropped = 0;
                        h->flags = 1;
                    }
                } else {
                    record_list(sm.fw, sm.list[b].key, sm.list[b].idx, cnt, rp, 0.0f, 0.0f, 0u, rec,
                                seg_cap, sm.tau_final[b]);
                }
                __threadfence();
                __syncwarp();
                uint32_t arrived = 0;
                if (lane == 0) arrived = atomicAdd(&row_arrivals[row], 1u);
                arrived = __shfl_sync(0xffffffffu, arrived, 0);
                if (arrived == pc.nparts - 1) {
                    __threadfence();
                    bool ok = true;
                    const uint32_t n = merge_records(
                        sm.list[b], sm.fw,
                        [&](uint32_t part) { return seg_records + (row * max_parts + part) * rec_bytes; },
                        pc.nparts, seg_cap, rp, &ok);
                    if (!ok) {
                        if (lane == 0) defer_row(sm, row, out_ids, out_status);
                    } else {
                        fin_count = n;
                    }
                    // Ready for the next call, whose finisher writes only after
                    // this grid completes (griddepcontrol.wait).
                    if (lane == 0) row_arrivals[row] = 0;
                }
            }
            // One call site for whole rows and merged split rows: the final
            // whole row then runs code the CTA's earlier merges have fetched.
            if (fin_count != kNoList)
                finish_list(sm.fw, sm.exp_tab, sm.list[b].key, sm.list[b].idx, fin_count, rp, row,
                            out_ids, out_status, out_probs);
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.list_empty[b]);
        }
        // Pieces this warp could not finish because a wait gave up: their
        // rows report RSC_ROW_INTERNAL. A part of a split row still publishes
        // a (failed) record and arrives, so that the row is completed.
        for (; get_piece(rows, nch, streamk, u, pc); ++u) {
            const size_t row = pc.row;
            if (kRecord) {
                if (lane == 0) reinterpret_cast<ShardRecordHeader *>(records + row * rec_bytes)->flags = 2;
            } else if (pc.nparts == 1) {
                if (lane == 0) {
                    out_ids[row] = 0;
                    out_status[row] = RSC_ROW_INTERNAL;
                }
            } else if (lane == 0) {
                ShardRecordHeader *h = reinterpret_cast<ShardRecordHeader *>(
                    seg_records + (row * max_parts + pc.part) * rec_bytes);
                h->n_cand = 0;
                h->n_dropped = 0;
                h->flags = 2;
                __threadfence();
                if (atomicAdd(&row_arrivals[row], 1u) == pc.nparts - 1) {
                    out_ids[row] = 0;
                    out_status[row] = RSC_ROW_INTERNAL;
                    row_arrivals[row] = 0;
                }
            }
            __syncwarp();
        }
    } else {
        consume();
    }

    // --- epilogue: the rows this CTA deferred ---------------------------------
    // Every role is done and every copy into the ring has landed, so the ring
    // holds the large-row workspace. The CTA takes a scratch slot (a bounded
    // spin on a lock; holders never wait on anyone) and samples the rows one
    // by one with all its threads.
    __syncthreads();
    if (kRecord && sm.ovf_count > 0) {
        // A shard's overflowing rows: the two-pass top-k into their records.
        uint32_t *hist = reinterpret_cast<uint32_t *>(reinterpret_cast<unsigned char *>(&sm.ring[0][0]) +
                                                      kTopkHistOffset);
        for (uint32_t k = 0; k < sm.ovf_count; ++k) {
            const size_t row = sm.ovf_rows[k];
            unsigned char *rec = records + row * rec_bytes;
            if (!epilogue_topk_row(cp, logits + row * row_stride, vocab, row, sm, hist, nullptr, nullptr,
                                   nullptr, rec, index_offset)) {
                if (threadIdx.x == 0) {
                    ShardRecordHeader *h = reinterpret_cast<ShardRecordHeader *>(rec);
                    h->flags = 1;
                    h->n_cand = 0;
                    h->n_dropped = 0;
                }
                __syncthreads();
            }
        }
    }
    if (!kRecord && sm.ovf_count > 0) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        large::LargeSmem<kThreads> &ls = *reinterpret_cast<large::LargeSmem<kThreads> *>(&sm.ring[0][0]);
        load_exp_table(ls.exp_tab);
        uint32_t *hist = reinterpret_cast<uint32_t *>(reinterpret_cast<unsigned char *>(&sm.ring[0][0]) +
                                                      kTopkHistOffset);
        // A scratch slot is taken only for a row that needs the large-row code
        // (a bounded spin on a lock; holders never wait on anyone).
        uint32_t slot = ~0u;
        bool tried = false;
        for (uint32_t k = 0; k < sm.ovf_count; ++k) {
            const size_t row = sm.ovf_rows[k];
            if (epilogue_topk_row(cp, logits + row * row_stride, vocab, row, sm, hist, out_ids,
                                  out_status, out_probs, nullptr, 0u))
                continue;
            if (!tried) {
                tried = true;
                if (threadIdx.x == 0) {
                    uint32_t got = ~0u;
                    const unsigned long long t0 = global_ns();
                    for (uint32_t i = 0; got == ~0u; ++i) {
                        const uint32_t s = (blockIdx.x + i) % slots;
                        if (atomicCAS(&slot_lock[s], 0u, 1u) == 0u) {
                            got = s;
                            break;
                        }
                        if (global_ns() - t0 > kWaitLimitNs) break;
                        __nanosleep(1000);
                    }
                    __threadfence();
                    sm.slot = got;
                }
                __syncthreads();
                slot = sm.slot;
            }
            if (slot == ~0u) {
                if (threadIdx.x == 0) {
                    out_ids[row] = 0;
                    out_status[row] = RSC_ROW_INTERNAL;
                }
                continue;
            }
            epilogue_row(cp, logits + row * row_stride, vocab, row,
                         scratch + static_cast<size_t>(slot) * 4u * vocab, out_ids, out_status,
                         out_probs, ls);
        }
        __syncthreads();
        if (threadIdx.x == 0 && slot != ~0u) {
            __threadfence();
            atomicExch(&slot_lock[slot], 0u);
        }
    }
}

// Vocab-sharded merge: each warp gathers the shards' records of one row into
// its candidate list and finishes the row exactly as the streaming kernel does.
// Two warps per CTA: 31 KB of shared memory a CTA, so 7 CTAs (14 warps) share
// an SM, against 12 warps with four-warp CTAs.
constexpr int kMergeWarps = 4;
// Most ranks the peer-memory merge reads (records in flight per warp).
constexpr uint32_t kMergeMaxPeers = 32;

// Shared memory of a merge CTA. Each warp merges one row with a MergeWork
// (about 6.5 KB a warp with its list, so eight CTAs, 32 warps, fit an SM).
// The rare row whose survivors overflow a MergeWork (heavy ties at the k-th
// value) is merged again after the CTA's rows, by warp 0, with a CandList
// and a FinishWork laid over the warps' space.
struct MergeLanes {
    CandList list[kMergeWarps];
    MergeWork fw[kMergeWarps];
};
struct MergeRetry {
    CandList list;
    FinishWork fw;
};
struct MergeSmem {
    double exp_tab[32];
    uint32_t retry;  // bit w: warp w's row is to be merged again
    union {
        MergeLanes lanes;
        MergeRetry full;
    };
};
static_assert(sizeof(MergeRetry) <= sizeof(MergeLanes), "the retry workspace fits the warps' space");

// Merges one row (one warp): the union of the parts' records, cut by their
// bounds, finished exactly. Returns false when the workspace is too small
// for the row's survivors (nothing written then); a union that cannot be
// trusted is reported as RSC_ROW_INTERNAL.
template <typename FW, typename RecAt>
__device__ __forceinline__ bool merge_row(CandList &L, FW &fw, const double *tab, RecAt rec_at,
                                          uint32_t n_parts, const CallParams &cp, size_t row,
                                          uint32_t *out_ids, int32_t *out_status,
                                          float *out_probs) {
    bool ok = true;
    const uint32_t count =
        merge_parts_batched(L, fw, rec_at, n_parts, cp.top_k + RSC_SHARD_TIE_CAP, cp, &ok);
    if (!ok) {
        if ((threadIdx.x & 31) == 0) {
            out_ids[row] = 0;
            out_status[row] = RSC_ROW_INTERNAL;
            if (out_probs) out_probs[row] = __uint_as_float(0x7fc00000u);
        }
        __syncwarp();
        return true;
    }
    return finish_list(fw, tab, L.key, L.idx, count, cp, row, out_ids, out_status, out_probs);
}

// The rows [r0, r0 + kMergeWarps) of a merge CTA, one per warp (rows past
// `end` are skipped), then the retries on the full workspace. `done(row)`
// runs on each warp after its row's outputs are written. Every thread of the
// CTA calls this.
template <typename RecAt, typename Done>
__device__ __forceinline__ void merge_cta_rows(MergeSmem &sm, size_t r0, size_t end,
                                               RecAt rec_at_row, uint32_t n_parts,
                                               const CallParams &cp, uint32_t *out_ids,
                                               int32_t *out_status, float *out_probs, Done done) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) sm.retry = 0;
    __syncthreads();
    const size_t row = r0 + warp;
    if (row < end) {
        auto rec_at = [&](uint32_t part) { return rec_at_row(part, row); };
        if (merge_row(sm.lanes.list[warp], sm.lanes.fw[warp], sm.exp_tab, rec_at, n_parts, cp, row,
                      out_ids, out_status, out_probs)) {
            done(row);
        } else if (lane == 0) {
            atomicOr(&sm.retry, 1u << warp);
        }
    }
    __syncthreads();
    const uint32_t retry = sm.retry;
    if (retry != 0u && warp == 0) {
        for (int w = 0; w < kMergeWarps; ++w) {
            if (!(retry & (1u << w))) continue;
            const size_t rr = r0 + w;
            auto rec_at = [&](uint32_t part) { return rec_at_row(part, rr); };
            merge_row(sm.full.list, sm.full.fw, sm.exp_tab, rec_at, n_parts, cp, rr, out_ids,
                      out_status, out_probs);
            done(rr);
        }
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kMergeWarps * 32)
shard_merge_kernel(const unsigned char *__restrict__ records, size_t n_shards, size_t rows,
                   size_t rec_bytes, CallParams cp, uint32_t *__restrict__ out_ids,
                   int32_t *__restrict__ out_status, float *__restrict__ out_probs) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    MergeSmem &sm = *reinterpret_cast<MergeSmem *>(smem_raw);
    load_exp_table(sm.exp_tab);
    for (size_t r0 = static_cast<size_t>(blockIdx.x) * kMergeWarps; r0 < rows;
         r0 += static_cast<size_t>(gridDim.x) * kMergeWarps) {
        merge_cta_rows(
            sm, r0, rows,
            [&](uint32_t part, size_t row) { return records + (part * rows + row) * rec_bytes; },
            static_cast<uint32_t>(n_shards), cp, out_ids, out_status, out_probs, [](size_t) {});
    }
}

// The vocab-sharded merge reading every rank's records in place over NVLink
// (peer memory), instead of from an all-gathered copy. x.records[p] is rank
// p's record array ([rows] records in rank p's memory, mapped here);
// x.ready_records[p], a word of this GPU, is the step rank p has published.
// Before reading, each CTA waits (bounded) until every ready word has reached
// `step`; a wait that runs out marks the CTA's rows RSC_ROW_INTERNAL and reads
// nothing. Rows [row_begin, row_end) are merged exactly as in
// shard_merge_kernel, their results written to this rank's output arrays
// (x.ids[my_shard], ...) and, when results are shared, to every other rank's
// too; the last CTA to finish then stores `step` into word my_shard of every
// rank's results-ready array (x.ready_results_ptrs[p]).
struct PeerArgs {
    const unsigned char *const *records;
    const uint32_t *ready_records;
    uint32_t *const *ready_results_ptrs;  // null: results are not shared
    uint32_t *done_counter;
    uint32_t *const *ids;
    int32_t *const *status;
    float *const *probs;  // null: no probabilities
};

__device__ __forceinline__ bool wait_ready(const uint32_t *ready, uint32_t n, uint32_t step) {
    const unsigned long long t0 = global_ns();
    for (uint32_t p = 0; p < n; ++p) {
        while (true) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(ready + p) : "memory");
            if (static_cast<int32_t>(v - step) >= 0) break;
            if (global_ns() - t0 > kWaitLimitNs) return false;
            __nanosleep(200);
        }
    }
    return true;
}

__device__ __forceinline__ void store_release_sys(uint32_t *dst, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(dst), "r"(v) : "memory");
}

__global__ void __launch_bounds__(kMergeWarps * 32)
shard_merge_peers_kernel(const __grid_constant__ PeerArgs x, uint32_t step, uint32_t n_shards,
                         uint32_t my_shard, size_t row_begin, size_t row_end, size_t rec_bytes,
                         const __grid_constant__ CallParams cp) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    MergeSmem &sm = *reinterpret_cast<MergeSmem *>(smem_raw);
    __shared__ uint32_t all_ready;
    __shared__ const unsigned char *base[kMergeMaxPeers];
    load_exp_table(sm.exp_tab);
    if (threadIdx.x < n_shards) base[threadIdx.x] = x.records[threadIdx.x];
    if (threadIdx.x == 0) all_ready = wait_ready(x.ready_records, n_shards, step) ? 1u : 0u;
    __syncthreads();
    uint32_t *const ids = x.ids[my_shard];
    int32_t *const status = x.status[my_shard];
    float *const probs = x.probs ? x.probs[my_shard] : nullptr;
    const bool share = x.ready_results_ptrs != nullptr;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // This row's results to every other rank (NVLink stores), by lane 0 of
    // the warp that wrote them.
    auto share_row = [&](size_t row) {
        if (share && lane == 0) {
            const uint32_t id = ids[row];
            const int32_t st = status[row];
            const float pb = probs ? probs[row] : 0.0f;
            for (uint32_t p = 0; p < n_shards; ++p) {
                if (p == my_shard) continue;
                x.ids[p][row] = id;
                x.status[p][row] = st;
                if (probs) x.probs[p][row] = pb;
            }
        }
        __syncwarp();
    };
    for (size_t r0 = row_begin + static_cast<size_t>(blockIdx.x) * kMergeWarps; r0 < row_end;
         r0 += static_cast<size_t>(gridDim.x) * kMergeWarps) {
        if (all_ready != 0u) {
            merge_cta_rows(
                sm, r0, row_end,
                [&](uint32_t part, size_t row) { return base[part] + row * rec_bytes; }, n_shards,
                cp, ids, status, probs, share_row);
        } else {
            const size_t row = r0 + warp;
            if (row < row_end) {
                if (lane == 0) {
                    ids[row] = 0;
                    status[row] = RSC_ROW_INTERNAL;
                    if (probs) probs[row] = __uint_as_float(0x7fc00000u);
                }
                __syncwarp();
                share_row(row);
            }
        }
    }
    if (share) {
        // The last CTA to finish publishes the results (every CTA fences its
        // stores at system scope before it counts itself done).
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence_system();
            const uint32_t prev = atomicAdd(x.done_counter, 1u);
            if (prev + 1u == gridDim.x) {
                __threadfence_system();
                for (uint32_t p = 0; p < n_shards; ++p)
                    store_release_sys(x.ready_results_ptrs[p] + my_shard, step);
                *x.done_counter = 0u;
            }
        }
    }
}

// The shared results of `step`, once every rank has published them (bounded
// wait, as above), copied from this rank's result arrays to the caller's; a
// wait that runs out gives RSC_ROW_INTERNAL rows.
__global__ void shard_collect_kernel(const uint32_t *ready_results, uint32_t step, uint32_t n_shards,
                                     size_t rows, const uint32_t *__restrict__ ids,
                                     const int32_t *__restrict__ status,
                                     const float *__restrict__ probs, uint32_t *__restrict__ out_ids,
                                     int32_t *__restrict__ out_status,
                                     float *__restrict__ out_probs) {
    __shared__ uint32_t ok;
    if (threadIdx.x == 0) ok = wait_ready(ready_results, n_shards, step) ? 1u : 0u;
    __syncthreads();
    for (size_t r = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; r < rows;
         r += static_cast<size_t>(gridDim.x) * blockDim.x) {
        if (ok) {
            out_ids[r] = __ldcg(ids + r);
            out_status[r] = __ldcg(status + r);
            if (out_probs) out_probs[r] = probs ? __ldcg(probs + r) : __uint_as_float(0x7fc00000u);
        } else {
            out_ids[r] = 0;
            out_status[r] = RSC_ROW_INTERNAL;
            if (out_probs) out_probs[r] = __uint_as_float(0x7fc00000u);
        }
    }
}

// Publishes this rank's records of `step` to every rank: after the stream's
// earlier work (the partial pass) has completed, a system-wide fence makes
// its record writes visible, then thread p stores `step` into rank p's ready
// word for this rank (ready_ptrs[p] + my_shard, peer memory).
__global__ void shard_publish_kernel(uint32_t *const *__restrict__ ready_ptrs, uint32_t n_shards,
                                     uint32_t my_shard, uint32_t step) {
    __threadfence_system();
    const uint32_t p = threadIdx.x;
    if (p < n_shards) {
        uint32_t *dst = ready_ptrs[p] + my_shard;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(dst), "r"(step) : "memory");
    }
}

// One block per row: the records of up to kLmheadMaxParts parts of a row in
// one pass, for rows spread over more parts than a warp's candidate list can
// merge (the LM-head epilogue's 148 and more). Two lower bounds of the row's
// k-th largest value cut the union before it is read: the largest of the
// parts' own bounds, and the k-th largest of the parts' maxima (k distinct
// values, each the top of its part). Only parts whose maximum reaches the
// bound are read; their entries at or above it go to shared memory, where
// the block selects the row's k-th largest key (radix select), keeps the
// entries at or above it (ties included) and finishes the row with one warp
// exactly as the streaming kernel does: the result of the warp merge
// (shard_merge_kernel) over the same records, for any number of parts.
constexpr int kBlockMergeThreads = 512;

struct BlockMergeSmem {
    CandList list;
    FinishWork fw;
    double exp_tab[32];
    uint32_t hist[256];
    uint32_t sel[2];
    float redf[kBlockMergeThreads / 32];
    uint32_t red32[kBlockMergeThreads / 32];
    uint32_t count, kept, nsel;
    float bound;
    uint32_t ncand[kLmheadMaxParts];  // entries of each part
    float pmax[kLmheadMaxParts];      // each part's largest scaled logit
    uint32_t psel[kLmheadMaxParts];   // the parts that can hold candidates
    // then uint32 key[entries], uint32 idx[entries]
};

// kEmit: instead of sampling the row, write its record (the parts reduced to
// one part) to out_records.
template <bool kEmit>
__global__ void __launch_bounds__(kBlockMergeThreads)
shard_merge_block_kernel(const unsigned char *__restrict__ records, uint32_t n_parts, size_t rows,
                         size_t rec_bytes, uint32_t cap_entries, CallParams cp,
                         uint32_t *__restrict__ out_ids, int32_t *__restrict__ out_status,
                         float *__restrict__ out_probs, unsigned char *__restrict__ out_records) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    BlockMergeSmem &sm = *reinterpret_cast<BlockMergeSmem *>(smem_raw);
    const uint32_t entries = n_parts * cap_entries;
    uint32_t *bkey = reinterpret_cast<uint32_t *>(smem_raw + sizeof(BlockMergeSmem));
    uint32_t *bidx = bkey + entries;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t row = blockIdx.x;
    auto rec_at = [&](uint32_t part) { return records + (static_cast<size_t>(part) * rows + row) * rec_bytes; };
    load_exp_table(sm.exp_tab);
    if (threadIdx.x == 0) {
        sm.count = 0;
        sm.kept = 0;
        sm.nsel = 0;
        sm.bound = kNegInf;
    }
    // Headers: the parts' flags and bounds.
    uint32_t bad = 0, dropped = 0;
    float tau = -3.402823466e38f;
    for (uint32_t p = threadIdx.x; p < n_parts; p += kBlockMergeThreads) {
        const uint32_t *h = reinterpret_cast<const uint32_t *>(rec_at(p));
        if (__ldcg(h + 6) != 0u) bad = 1u;
        if (__ldcg(h + 4) != 0u) dropped = 1u;
        tau = fmaxf(tau, __uint_as_float(__ldcg(h + 7)));
        sm.ncand[p] = min(__ldcg(h + 3), cap_entries);
        sm.pmax[p] = __uint_as_float(__ldcg(h + 0));
    }
    tau = block_reduce<kBlockMergeThreads>(tau, sm.redf, OpFMax());
    float rmax = kNegInf;  // the row's largest scaled logit over the parts
    for (uint32_t p = threadIdx.x; p < n_parts; p += kBlockMergeThreads) rmax = fmaxf(rmax, sm.pmax[p]);
    rmax = block_reduce<kBlockMergeThreads>(rmax, sm.redf, OpFMax());
    bad = block_reduce<kBlockMergeThreads>(bad, sm.red32, OpOrU32());
    dropped = block_reduce<kBlockMergeThreads>(dropped, sm.red32, OpOrU32());
    // The k-th largest part maximum (by value, then part): the part whose
    // maximum has exactly k - 1 parts before it.
    if (cp.topk_active && n_parts >= cp.top_k) {
        for (uint32_t p = threadIdx.x; p < n_parts; p += kBlockMergeThreads) {
            const float m = sm.pmax[p];
            uint32_t rank = 0;
            for (uint32_t q = 0; q < n_parts; ++q) {
                const float o = sm.pmax[q];
                rank += (o > m || (o == m && q < p)) ? 1u : 0u;
            }
            if (rank == cp.top_k - 1u) sm.bound = m;
        }
    }
    __syncthreads();
    tau = fmaxf(tau, sm.bound);
    // The parts whose maximum reaches the bound.
    for (uint32_t p = threadIdx.x; p < n_parts; p += kBlockMergeThreads)
        if (sm.pmax[p] >= tau) sm.psel[atomicAdd(&sm.nsel, 1u)] = p;
    __syncthreads();
    const uint32_t slots = sm.nsel * cap_entries;
    // Entries at or above the bound. Entry e of selected part j is flat slot
    // j * cap + e; each thread loads kGather slots at once, so that the loads
    // overlap.
    constexpr uint32_t kGather = 8;
    if (!bad) {
        for (uint32_t base = 0; base < slots; base += kBlockMergeThreads * kGather) {
            uint32_t key[kGather], idx[kGather];
#pragma unroll
            for (uint32_t q = 0; q < kGather; ++q) {
                const uint32_t f = base + q * kBlockMergeThreads + threadIdx.x;
                const uint32_t j = f / cap_entries, e = f - j * cap_entries;
                const uint32_t p = f < slots ? sm.psel[j] : 0u;
                const bool valid = f < slots && e < sm.ncand[p];
                const uint32_t *rkey = reinterpret_cast<const uint32_t *>(rec_at(p)) + 8;
                key[q] = valid ? __ldcg(rkey + e) : 0u;
                idx[q] = valid ? __ldcg(rkey + cap_entries + e) : 0u;
                if (!valid) key[q] = 0u;  // key 0 (a NaN pattern) is never kept
            }
#pragma unroll
            for (uint32_t q = 0; q < kGather; ++q) {
                const bool keep = key[q] != 0u && key_to_float(key[q]) >= tau;
                const uint32_t ballot = __ballot_sync(0xffffffffu, keep);
                uint32_t at = 0;
                if (lane == 0 && ballot) at = atomicAdd(&sm.count, static_cast<uint32_t>(__popc(ballot)));
                at = __shfl_sync(0xffffffffu, at, 0);
                if (keep) {
                    const uint32_t pos = at + __popc(ballot & ((1u << lane) - 1u));
                    bkey[pos] = key[q];
                    bidx[pos] = idx[q];
                }
            }
        }
    }
    __syncthreads();
    const uint32_t count = sm.count;  // <= entries: each part gives at most cap_entries
    uint32_t floor_key = 0u;
    const bool have_kth = !bad && cp.topk_active && count >= cp.top_k;
    if (have_kth) {
        const uint32_t kth = block_select_kth_largest<kBlockMergeThreads>(
            count, cp.top_k, [&](uint32_t i) { return bkey[i]; }, sm.hist, sm.sel);
        floor_key = kth == kKeyPosZero ? kKeyNegZero : kth;
    }
    // A part that dropped tied entries that can reach the row's k-th value
    // leaves the union incomplete.
    if (!bad && dropped) {
        uint32_t b = 0;
        for (uint32_t p = threadIdx.x; p < n_parts; p += kBlockMergeThreads) {
            const uint32_t *h = reinterpret_cast<const uint32_t *>(rec_at(p));
            if (__ldcg(h + 4) > 0 && (!have_kth || __ldcg(h + 5) >= floor_key)) b = 1u;
        }
        bad = block_reduce<kBlockMergeThreads>(b, sm.red32, OpOrU32());
    }
    // The row's candidates: the entries at or above the k-th (all of them
    // without top-k), into the finisher's list.
    if (!bad) {
        for (uint32_t i = threadIdx.x; i < count; i += kBlockMergeThreads) {
            if (bkey[i] >= floor_key) {
                const uint32_t pos = atomicAdd(&sm.kept, 1u);
                if (pos < kCap) {
                    sm.list.key[pos] = bkey[i];
                    sm.list.idx[pos] = bidx[i];
                }
            }
        }
    }
    __syncthreads();
    const uint32_t kept = sm.kept;
    if (kEmit) {
        if (warp == 0) {
            unsigned char *rec = out_records + row * rec_bytes;
            if (bad || kept > kCap) {
                if (lane == 0) {
                    ShardRecordHeader *h = reinterpret_cast<ShardRecordHeader *>(rec);
                    h->max_scaled = rmax;
                    h->sum_exp = 0.0f;
                    h->n_finite = 0;
                    h->n_cand = 0;
                    h->n_dropped = 0;
                    h->last_key = 0;
                    h->flags = 1;
                    h->tau = -3.402823466e38f;
                }
            } else {
                // Entries at or above the row's k-th value (or, without a
                // k-th, every candidate at or above the precut bound).
                record_list(sm.fw, sm.list.key, sm.list.idx, kept, cp, rmax, 0.0f, 0u, rec,
                            cap_entries, have_kth ? key_to_float(floor_key) : tau);
            }
        }
        return;
    }
    if (warp == 0) {
        if (bad || kept > kCap) {
            if (lane == 0) {
                out_ids[row] = 0;
                out_status[row] = RSC_ROW_INTERNAL;
                if (out_probs) out_probs[row] = __uint_as_float(0x7fc00000u);
            }
        } else {
            finish_list(sm.fw, sm.exp_tab, sm.list.key, sm.list.idx, kept, cp, row, out_ids,
                        out_status, out_probs);
        }
    }
}


template <typename K>
cudaError_t prepare(K kernel, size_t smem) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
}

}  // namespace

size_t stream_topk_smem_bytes() { return sizeof(StreamSmem); }

size_t split_record_bytes(uint32_t splits) {
    const size_t entries = kSmallCap / (splits ? splits : 1u);
    return (sizeof(ShardRecordHeader) + 8 * entries + 15) & ~static_cast<size_t>(15);
}

StreamPlan stream_plan(size_t rows, uint32_t vocab, bool topk_active, uint32_t top_k,
                       int num_sms, size_t seg_capacity_bytes) {
    const size_t ctas = static_cast<size_t>(num_sms) * kCtasPerSm;
    uint32_t nch = (vocab + kChunk - 1) / kChunk;
    if (nch == 0) nch = 1;
    StreamPlan pl;
    pl.nch = nch;
    pl.streamk = 0;
    pl.max_parts = 1;
    pl.grid = static_cast<uint32_t>(rows < ctas ? rows : ctas);
    // Balanced ranges need top-k (a part's record keeps k + ties) and rows of
    // more than one chunk; otherwise whole rows go round-robin.
    if (rows == 0 || !topk_active || nch < 2) return pl;
    uint32_t pmax = kCap / (top_k + RSC_SHARD_TIE_CAP);
    if (pmax > kMaxSplits) pmax = kMaxSplits;
    // A batch with no more rows than CTAs splits rows for parallelism only:
    // parts of at least kMinPartChunks chunks. Shorter parts cost more in
    // records, arrivals and a long merged list than they save in streaming
    // (1 x 32000: 25.7 -> 9.6 us a call; 64 x 151936: 42.5 -> 19.6 us).
    if (rows <= ctas && pmax > nch / kMinPartChunks) pmax = nch / kMinPartChunks;
    if (pmax < 2) return pl;
    const unsigned long long T = static_cast<unsigned long long>(rows) * nch;
    unsigned long long G = T < ctas ? T : ctas;
    uint32_t parts;
    if (rows <= 4096) {
        // Exact: the most CTAs any row is spread over, for this grid; fewer
        // CTAs until the rows' merged records fit one candidate list.
        auto owner = [&](unsigned long long x, unsigned long long g) {
            return ((x + 1ull) * g - 1ull) / T;
        };
        for (;; --G) {
            unsigned long long most = 1;
            for (size_t r = 0; r < rows; ++r) {
                const unsigned long long a = static_cast<unsigned long long>(r) * nch;
                const unsigned long long n = owner(a + nch - 1ull, G) - owner(a, G) + 1ull;
                if (n > most) most = n;
            }
            if (most <= pmax || G == 1) {
                parts = static_cast<uint32_t>(most);
                break;
            }
        }
    } else {
        // Every CTA's range spans at least R = floor(T / G) chunks, so a row
        // is cut by at most (nch - 2) / R + 1 range ends.
        unsigned long long R = T / G;
        if ((nch - 2ull) / R + 2ull > pmax) {
            G = T / ((nch - 2ull) / (pmax - 1ull) + 1ull);
            if (G < 1) G = 1;
            R = T / G;
        }
        parts = static_cast<uint32_t>((nch - 2ull) / R + 2ull);
        if (parts > nch) parts = nch;
    }
    if (parts > pmax) return pl;
    if (static_cast<unsigned long long>(rows) * parts * split_record_bytes(parts) > seg_capacity_bytes)
        return pl;
    pl.streamk = 1;
    pl.grid = static_cast<uint32_t>(G);
    pl.max_parts = parts;
    return pl;
}

cudaError_t launch_stream_topk(const float *logits, size_t rows, uint32_t vocab,
                               size_t row_stride, const CallParams &p, uint32_t *out_ids,
                               int32_t *out_status, float *out_probs, const StreamPlan &plan,
                               void *seg_records, uint32_t *row_arrivals, uint32_t *scratch,
                               uint32_t slots, uint32_t *slot_lock, cudaStream_t stream) {
    if (rows == 0) return cudaSuccess;
    // The per-row instance also serves calls whose k is above the streaming
    // filter's: every row goes straight to the epilogue's two passes.
    const bool rows_instance = p.row_params || (p.topk_active && p.top_k > kSmallTopK);
    auto kernel = rows_instance ? stream_topk_kernel<false, true>
                  : p.lse_parts ? stream_topk_kernel<false, false, true>
                                : stream_topk_kernel<false, false>;
    cudaError_t e = prepare(kernel, sizeof(StreamSmem));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = sizeof(StreamSmem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, logits, rows, vocab, row_stride, p,
                              out_ids, out_status, out_probs, scratch, slots, slot_lock, 0u,
                              static_cast<unsigned char *>(nullptr),
                              split_record_bytes(plan.max_parts), plan.nch, plan.streamk,
                              plan.max_parts, static_cast<unsigned char *>(seg_records),
                              row_arrivals);
}

cudaError_t launch_shard_partial(const float *logits, size_t rows, uint32_t shard_vocab,
                                 size_t row_stride, uint32_t shard_offset, const CallParams &p,
                                 void *records, size_t rec_bytes, int num_sms,
                                 cudaStream_t stream) {
    if (rows == 0) return cudaSuccess;
    cudaError_t e = prepare(stream_topk_kernel<true>, sizeof(StreamSmem));
    if (e != cudaSuccess) return e;
    const size_t ctas = static_cast<size_t>(num_sms) * kCtasPerSm;
    const size_t grid = rows < ctas ? rows : ctas;
    const uint32_t nch = shard_vocab ? (shard_vocab + kChunk - 1) / kChunk : 1u;
    stream_topk_kernel<true><<<static_cast<unsigned>(grid), kThreads, sizeof(StreamSmem), stream>>>(
        logits, rows, shard_vocab, row_stride, p, nullptr, nullptr, nullptr, nullptr, 0u, nullptr,
        shard_offset, static_cast<unsigned char *>(records), rec_bytes, nch, 0u, 1u, nullptr,
        nullptr);
    return cudaGetLastError();
}

size_t shard_merge_block_smem(uint32_t n_parts, uint32_t cap_entries) {
    return sizeof(BlockMergeSmem) + static_cast<size_t>(n_parts) * cap_entries * 8u;
}

cudaError_t launch_shard_merge_block(const void *records, size_t n_parts, size_t rows,
                                     size_t rec_bytes, const CallParams &p, uint32_t *out_ids,
                                     int32_t *out_status, float *out_probs, cudaStream_t stream) {
    if (rows == 0) return cudaSuccess;
    const uint32_t cap = p.top_k + RSC_SHARD_TIE_CAP;
    const size_t smem = shard_merge_block_smem(static_cast<uint32_t>(n_parts), cap);
    if (n_parts > kLmheadMaxParts || smem > 232448) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(shard_merge_block_kernel<false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    shard_merge_block_kernel<false><<<static_cast<unsigned>(rows), kBlockMergeThreads, smem, stream>>>(
        static_cast<const unsigned char *>(records), static_cast<uint32_t>(n_parts), rows, rec_bytes,
        cap, p, out_ids, out_status, out_probs, nullptr);
    return cudaGetLastError();
}

cudaError_t launch_shard_reduce_block(const void *records, size_t n_parts, size_t rows,
                                      size_t rec_bytes, const CallParams &p, void *out_records,
                                      cudaStream_t stream) {
    if (rows == 0) return cudaSuccess;
    const uint32_t cap = p.top_k + RSC_SHARD_TIE_CAP;
    const size_t smem = shard_merge_block_smem(static_cast<uint32_t>(n_parts), cap);
    if (n_parts > kLmheadMaxParts || smem > 232448) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(shard_merge_block_kernel<true>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    shard_merge_block_kernel<true><<<static_cast<unsigned>(rows), kBlockMergeThreads, smem, stream>>>(
        static_cast<const unsigned char *>(records), static_cast<uint32_t>(n_parts), rows, rec_bytes,
        cap, p, nullptr, nullptr, nullptr, static_cast<unsigned char *>(out_records));
    return cudaGetLastError();
}

cudaError_t launch_shard_merge(const void *records, size_t n_shards, size_t rows, size_t rec_bytes,
                               const CallParams &p, uint32_t *out_ids, int32_t *out_status,
                               float *out_probs, int num_sms, cudaStream_t stream) {
    if (rows == 0) return cudaSuccess;
    cudaError_t e = prepare(shard_merge_kernel, sizeof(MergeSmem));
    if (e != cudaSuccess) return e;
    const size_t grid = (rows + kMergeWarps - 1) / kMergeWarps;
    shard_merge_kernel<<<static_cast<unsigned>(grid), kMergeWarps * 32, sizeof(MergeSmem), stream>>>(
        static_cast<const unsigned char *>(records), n_shards, rows, rec_bytes, p, out_ids,
        out_status, out_probs);
    return cudaGetLastError();
}


cudaError_t launch_shard_merge_peers(const PeerPointers &x, uint32_t step, size_t n_shards,
                                     size_t my_shard, size_t row_begin, size_t row_end,
                                     size_t rec_bytes, const CallParams &p, cudaStream_t stream) {
    if (row_end <= row_begin) {
        // No rows to merge here; still publish this rank's (empty) share.
        if (x.ready_results_ptrs) return launch_shard_publish(x.ready_results_ptrs, n_shards,
                                                               static_cast<uint32_t>(my_shard),
                                                               step, stream);
        return cudaSuccess;
    }
    if (n_shards == 0 || n_shards > kMergeMaxPeers || my_shard >= n_shards) return cudaErrorInvalidValue;
    cudaError_t e = prepare(shard_merge_peers_kernel, sizeof(MergeSmem));
    if (e != cudaSuccess) return e;
    const size_t grid = (row_end - row_begin + kMergeWarps - 1) / kMergeWarps;
    PeerArgs a{reinterpret_cast<const unsigned char *const *>(x.records), x.ready_records,
               x.ready_results_ptrs, x.done_counter, x.ids, x.status, x.probs};
    shard_merge_peers_kernel<<<static_cast<unsigned>(grid), kMergeWarps * 32, sizeof(MergeSmem),
                               stream>>>(a, step, static_cast<uint32_t>(n_shards),
                                         static_cast<uint32_t>(my_shard), row_begin, row_end,
                                         rec_bytes, p);
    return cudaGetLastError();
}

cudaError_t launch_shard_collect(const uint32_t *ready_results, uint32_t step, size_t n_shards,
                                 size_t rows, const uint32_t *ids, const int32_t *status,
                                 const float *probs, uint32_t *out_ids, int32_t *out_status,
                                 float *out_probs, cudaStream_t stream) {
    if (rows == 0) return cudaSuccess;
    size_t grid = (rows + 255) / 256;
    if (grid > 1024) grid = 1024;
    shard_collect_kernel<<<static_cast<unsigned>(grid), 256, 0, stream>>>(
        ready_results, step, static_cast<uint32_t>(n_shards), rows, ids, status, probs, out_ids,
        out_status, out_probs);
    return cudaGetLastError();
}

cudaError_t launch_shard_publish(uint32_t *const *d_ready_ptrs, size_t n_shards, uint32_t my_shard,
                                 uint32_t step, cudaStream_t stream) {
    if (n_shards == 0 || n_shards > 1024 || my_shard >= n_shards) return cudaErrorInvalidValue;
    shard_publish_kernel<<<1, 32 * static_cast<unsigned>((n_shards + 31) / 32), 0, stream>>>(
        d_ready_ptrs, static_cast<uint32_t>(n_shards), my_shard, step);
    return cudaGetLastError();
}

}  // namespace rsc
