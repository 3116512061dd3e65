// Streaming top-k sampler: Sampler::sample_logits
// (crates/rusticide-sampling/src/sampler.rs:44-54) for rows whose surviving
// candidate set is small, which is every row once top-k is on.
//
// One HBM pass per row. A CTA owns a sequence of rows; one thread keeps a ring
// of NSTAGE shared-memory stages filled with 1-D TMA bulk copies (no
// multicast) of CHUNK logits, running ahead across row boundaries. Every
// thread scales its logits (candidates.rs:30-37), turns them into
// f32::total_cmp keys, and compares them with a running lower bound `tau` of
// the row's k-th largest key; the rare logits at or above it are appended to a
// shared candidate list. When the list fills up, a radix select of its k-th
// largest key raises tau and the list is compacted. The list always holds
// every logit that can survive top-k, so at the end of the row one more
// select gives the exact threshold of kth_largest (candidates.rs:93-97).
//
// The survivors (at most kSmallCap) are then finished in shared memory with
// the reference's exact arithmetic: top-p over the (value desc, index asc)
// order with sequential sums (candidates.rs:55-78), softmax in index order
// (filters.rs:5-15), and the argmax or the inverse-CDF draw
// (sampler.rs:48-52,111-121). The sequential sums run on one thread: the
// sets are small, and replaying the reference's order is what makes every
// result bit-identical.
#include "rsc_block.cuh"
#include "rsc_kernels.h"

namespace rsc {

namespace {

constexpr int kThreads = 256;
constexpr uint32_t kChunk = 2048;   // logits per stage (8 KiB)
constexpr uint32_t kStages = 6;
constexpr uint32_t kCap = kSmallCap;  // candidate list capacity
static_assert(kCap >= 2 * kChunk, "a chunk must fit after a compaction");

struct StreamSmem {
    alignas(128) float ring[kStages][kChunk];
    alignas(16) union {
        struct {
            uint32_t key[kCap];
            uint32_t idx[kCap];
        } cand;
        unsigned long long items[kCap];
    } u;
    alignas(16) float vals[kCap];
    double exp_tab[32];
    uint64_t full[kStages];
    uint32_t hist[256];
    uint32_t sel[2];
    uint32_t count;
    uint32_t overflow;
    uint32_t error;
    uint32_t issued;
    uint32_t n;
    uint32_t red32[kThreads / 32];
    unsigned long long red64[kThreads / 32];
    float redf[kThreads / 32];
    float bcast_f[2];
    uint32_t bcast_u[2];
};

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

// Warp-aggregated append of (key, idx) when `take`.
__device__ __forceinline__ void append_candidate(StreamSmem &sm, bool take, uint32_t key,
                                                 uint32_t idx) {
    const uint32_t ballot = __ballot_sync(0xffffffffu, take);
    if (!ballot) return;
    const int lane = threadIdx.x & 31;
    const int leader = __ffs(ballot) - 1;
    uint32_t base = 0;
    if (lane == leader) base = atomicAdd(&sm.count, static_cast<uint32_t>(__popc(ballot)));
    base = __shfl_sync(0xffffffffu, base, leader);
    if (take) {
        uint32_t pos = base + __popc(ballot & ((1u << lane) - 1u));
        if (pos < kCap) {
            sm.u.cand.key[pos] = key;
            sm.u.cand.idx[pos] = idx;
        } else {
            sm.overflow = 1;
        }
    }
}

__device__ __forceinline__ uint32_t relax_tau(uint32_t t) {
    // A threshold of +0.0 also keeps -0.0: -0.0 < +0.0 is false in IEEE.
    return t == kKeyPosZero ? kKeyNegZero : t;
}

// Raises tau to the k-th largest candidate key and drops candidates below it.
__device__ void compact(StreamSmem &sm, uint32_t k, uint32_t &tau) {
    __syncthreads();
    const uint32_t count = min(sm.count, kCap);
    if (count < k) return;  // uniform: every thread read the same count
    uint32_t kth = block_select_kth_largest<kThreads>(
        count, k, [&](uint32_t i) { return sm.u.cand.key[i]; }, sm.hist, sm.sel);
    uint32_t nt = relax_tau(kth);
    if (nt > tau) tau = nt;
    constexpr int kPer = kCap / kThreads;
    uint32_t kk[kPer], ii[kPer];
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
        uint32_t i = threadIdx.x + q * kThreads;
        kk[q] = i < count ? sm.u.cand.key[i] : 0u;
        ii[q] = i < count ? sm.u.cand.idx[i] : 0u;
    }
    __syncthreads();
    if (threadIdx.x == 0) sm.count = 0;
    __syncthreads();
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
        uint32_t i = threadIdx.x + q * kThreads;
        append_candidate(sm, i < count && kk[q] >= tau, kk[q], ii[q]);
    }
    __syncthreads();
}

// Finishes a row from its candidate list: exact threshold, survivors, top-p,
// softmax, argmax or draw. Writes the row's outputs.
__device__ void finish_row(StreamSmem &sm, const CallParams &cp, size_t row, uint32_t *out_ids,
                           int32_t *out_status, float *out_probs) {
    __syncthreads();
    const uint32_t count = min(sm.count, kCap);
    // Exact top-k threshold (candidates.rs:38-43). With fewer than k
    // candidates every candidate survives (the k-th largest is then -inf or
    // below, which keeps all values that are not -inf).
    float thr = kNegInf;
    if (cp.topk_active && count >= cp.top_k) {
        uint32_t kth = block_select_kth_largest<kThreads>(
            count, cp.top_k, [&](uint32_t i) { return sm.u.cand.key[i]; }, sm.hist, sm.sel);
        thr = key_to_float(kth);
    }
    // Survivors, packed for a (value desc, index asc) sort when top-p is on,
    // else (index asc).
    constexpr int kPer = kCap / kThreads;
    unsigned long long it[kPer];
    bool keep[kPer];
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
        uint32_t i = threadIdx.x + q * kThreads;
        keep[q] = false;
        it[q] = 0;
        if (i < count) {
            uint32_t key = sm.u.cand.key[i];
            uint32_t idx = sm.u.cand.idx[i];
            keep[q] = survives(key_to_float(key), thr);
            it[q] = cp.topp_active ? pack_key_index(~key, idx) : pack_key_index(idx, key);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) sm.n = 0;
    __syncthreads();
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
        const uint32_t ballot = __ballot_sync(0xffffffffu, keep[q]);
        if (!ballot) continue;
        const int lane = threadIdx.x & 31;
        const int leader = __ffs(ballot) - 1;
        uint32_t base = 0;
        if (lane == leader) base = atomicAdd(&sm.n, static_cast<uint32_t>(__popc(ballot)));
        base = __shfl_sync(0xffffffffu, base, leader);
        if (keep[q]) sm.u.items[base + __popc(ballot & ((1u << lane) - 1u))] = it[q];
    }
    __syncthreads();
    uint32_t n = sm.n;
    uint32_t n64 = 32;
    while (n64 < n) n64 <<= 1;
    for (uint32_t i = n + threadIdx.x; i < n64; i += kThreads) sm.u.items[i] = ~0ull;
    block_bitonic_sort<kThreads>(sm.u.items, n64);

    if (cp.topp_active && n > 0) {
        // Candidates::top_p, candidates.rs:55-78: items are (~key, idx)
        // ascending = value descending, index ascending.
        const float maxv = key_to_float(~static_cast<uint32_t>(sm.u.items[0] >> 32));
        for (uint32_t i = threadIdx.x; i < n; i += kThreads) {
            float v = key_to_float(~static_cast<uint32_t>(sm.u.items[i] >> 32));
            sm.vals[i] = expf_ref(__fsub_rn(v, maxv), sm.exp_tab);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float exp_sum = 0.0f;
            for (uint32_t i = 0; i < n; ++i) exp_sum = __fadd_rn(exp_sum, sm.vals[i]);
            float cumsum = 0.0f;
            uint32_t cutoff = n;
            for (uint32_t i = 0; i < n; ++i) {
                cumsum = __fadd_rn(cumsum, __fdiv_rn(sm.vals[i], exp_sum));
                if (cumsum > cp.top_p) {
                    cutoff = i + 1;
                    break;
                }
            }
            sm.n = cutoff;
        }
        __syncthreads();
        n = sm.n;
        // Re-key the kept prefix by index and sort it back to index order.
        for (uint32_t i = threadIdx.x; i < n64; i += kThreads) {
            unsigned long long x = sm.u.items[i];
            uint32_t key = ~static_cast<uint32_t>(x >> 32);
            uint32_t idx = static_cast<uint32_t>(x);
            sm.u.items[i] = i < n ? pack_key_index(idx, key) : ~0ull;
        }
        block_bitonic_sort<kThreads>(sm.u.items, n64);
    }

    if (cp.out_nsurv && threadIdx.x == 0) cp.out_nsurv[row] = n;
    if (cp.out_surv) {
        const uint32_t m = min(n, cp.surv_cap);
        for (uint32_t i = threadIdx.x; i < m; i += kThreads)
            cp.out_surv[row * cp.surv_cap + i] = static_cast<uint32_t>(sm.u.items[i] >> 32);
    }

    // softmax (filters.rs:5-15) over the survivors in index order.
    float mx = kNegInf;
    unsigned long long amax = 0;
    for (uint32_t i = threadIdx.x; i < n; i += kThreads) {
        uint32_t key = static_cast<uint32_t>(sm.u.items[i]);
        mx = fmaxf(mx, key_to_float(key));
        unsigned long long c = pack_key_index(key, i);
        amax = c > amax ? c : amax;
    }
    mx = block_reduce<kThreads>(mx, sm.redf, OpFMax());
    amax = block_reduce<kThreads>(amax, sm.red64, OpMaxU64());
    for (uint32_t i = threadIdx.x; i < n; i += kThreads) {
        float v = key_to_float(static_cast<uint32_t>(sm.u.items[i]));
        sm.vals[i] = expf_ref(__fsub_rn(v, mx), sm.exp_tab);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = -0.0f;  // <f32 as Sum>::sum
        for (uint32_t i = 0; i < n; ++i) s = __fadd_rn(s, sm.vals[i]);
        sm.bcast_f[0] = s;
    }
    __syncthreads();
    const float sum = sm.bcast_f[0];
    const bool norm = (fabsf(sum) < kPosInf) && sum > 0.0f;
    uint32_t valid = 0;
    for (uint32_t i = threadIdx.x; i < n; i += kThreads) {
        float pi = sm.vals[i];
        if (norm) pi = __fdiv_rn(pi, sum);
        sm.vals[i] = pi;
        if (!(pi != pi || pi <= 0.0f)) valid = 1;
    }
    valid = block_reduce<kThreads>(valid, sm.red32, OpOrU32());
    if (threadIdx.x == 0) {
        int32_t status = RSC_ROW_NO_VALID_TOKENS;
        uint32_t token = 0;
        float prob = __uint_as_float(0x7fc00000u);
        if (valid) {
            uint32_t pos;
            if (cp.argmax_branch) {
                pos = static_cast<uint32_t>(amax);
            } else {
                const float r = row_uniform(cp, row);
                float cumsum = 0.0f, before = 0.0f;
                pos = n - 1;
                bool hit = false;
                for (uint32_t i = 0; i < n; ++i) {
                    before = cumsum;
                    cumsum = __fadd_rn(cumsum, sm.vals[i]);
                    if (r < cumsum) {
                        pos = i;
                        hit = true;
                        break;
                    }
                }
                if (!hit) before = cumsum;
                status = 0;
                if (fabsf(r - cumsum) < 1e-6f || fabsf(r - before) < 1e-6f)
                    status |= RSC_ROW_FLAG_DRAW_NEAR_BOUNDARY;
            }
            token = static_cast<uint32_t>(sm.u.items[pos] >> 32);
            prob = sm.vals[pos];
            status = (status & ~0xff) | RSC_ROW_OK;
        }
        out_ids[row] = token;
        out_status[row] = status;
        if (out_probs) out_probs[row] = prob;
    }
    __syncthreads();
}

// Shard record of the vocab-sharded mode: the scaled row maximum and online
// exp-sum of the shard, and every logit of the shard at or above its local
// k-th largest key (which is at most the global one), sorted (key desc,
// index asc) and capped at k + RSC_SHARD_TIE_CAP entries.
__device__ void record_row(StreamSmem &sm, const CallParams &cp, size_t row, float mx_t,
                           float se_t, uint32_t cnt_t, unsigned char *records, size_t rec_bytes) {
    __syncthreads();
    const uint32_t count = min(sm.count, kCap);
    const uint32_t cap_entries = cp.top_k + RSC_SHARD_TIE_CAP;
    uint32_t floor_key = kKeyNegInf + 1u;
    if (count >= cp.top_k) {
        uint32_t kth = block_select_kth_largest<kThreads>(
            count, cp.top_k, [&](uint32_t i) { return sm.u.cand.key[i]; }, sm.hist, sm.sel);
        floor_key = relax_tau(kth);
    }
    constexpr int kPer = kCap / kThreads;
    unsigned long long it[kPer];
    bool keep[kPer];
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
        uint32_t i = threadIdx.x + q * kThreads;
        keep[q] = false;
        it[q] = 0;
        if (i < count) {
            uint32_t key = sm.u.cand.key[i];
            keep[q] = key >= floor_key;
            it[q] = pack_key_index(~key, sm.u.cand.idx[i]);
        }
    }
    // Row statistics: max, sum of exp(v - max) rescaled per thread, count.
    const float M = block_reduce<kThreads>(mx_t, sm.redf, OpFMax());
    float se_scaled = (se_t > 0.0f) ? se_t * __expf(mx_t - M) : 0.0f;
    se_scaled = block_reduce<kThreads>(se_scaled, sm.redf, [](float a, float b) { return a + b; });
    const uint32_t nfin = block_reduce<kThreads>(cnt_t, sm.red32, OpAddU32());
    __syncthreads();
    if (threadIdx.x == 0) sm.n = 0;
    __syncthreads();
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
        const uint32_t ballot = __ballot_sync(0xffffffffu, keep[q]);
        if (!ballot) continue;
        const int lane = threadIdx.x & 31;
        const int leader = __ffs(ballot) - 1;
        uint32_t base = 0;
        if (lane == leader) base = atomicAdd(&sm.n, static_cast<uint32_t>(__popc(ballot)));
        base = __shfl_sync(0xffffffffu, base, leader);
        if (keep[q]) sm.u.items[base + __popc(ballot & ((1u << lane) - 1u))] = it[q];
    }
    __syncthreads();
    const uint32_t n = sm.n;
    uint32_t n64 = 32;
    while (n64 < n) n64 <<= 1;
    for (uint32_t i = n + threadIdx.x; i < n64; i += kThreads) sm.u.items[i] = ~0ull;
    block_bitonic_sort<kThreads>(sm.u.items, n64);
    const uint32_t nc = min(n, cap_entries);
    unsigned char *rec = records + row * rec_bytes;
    ShardRecordHeader *h = reinterpret_cast<ShardRecordHeader *>(rec);
    uint32_t *rkey = reinterpret_cast<uint32_t *>(rec + sizeof(ShardRecordHeader));
    uint32_t *ridx = rkey + cap_entries;
    for (uint32_t i = threadIdx.x; i < nc; i += kThreads) {
        unsigned long long x = sm.u.items[i];
        rkey[i] = ~static_cast<uint32_t>(x >> 32);
        ridx[i] = static_cast<uint32_t>(x);
    }
    if (threadIdx.x == 0) {
        h->max_scaled = M;
        h->sum_exp = se_scaled;
        h->n_finite = nfin;
        h->n_cand = nc;
        h->n_dropped = n - nc;
        h->last_key = nc ? ~static_cast<uint32_t>(sm.u.items[nc - 1] >> 32) : 0u;
        h->flags = 0;
        h->reserved = 0;
    }
    __syncthreads();
}

template <bool kRecord>
__global__ void __launch_bounds__(kThreads)
stream_topk_kernel(const float *__restrict__ logits, size_t rows, uint32_t vocab,
                   size_t row_stride, CallParams cp, uint32_t *__restrict__ out_ids,
                   int32_t *__restrict__ out_status, float *__restrict__ out_probs,
                   uint32_t *__restrict__ large_rows, uint32_t *__restrict__ large_count,
                   uint32_t index_offset, unsigned char *__restrict__ records, size_t rec_bytes) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    StreamSmem &sm = *reinterpret_cast<StreamSmem *>(smem_raw);

    load_exp_table(sm.exp_tab);
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < kStages; ++s) mbar_init(&sm.full[s], 1);
        sm.error = 0;
        sm.issued = 0;
        fence_barrier_init();
    }
    __syncthreads();

    // Producer cursor over this CTA's (row, chunk) sequence; thread 0 only.
    size_t prow = blockIdx.x;
    uint32_t pchunk = 0;
    uint32_t issued = 0;
    auto produce_one = [&]() {
        while (prow < rows) {
            RowGeom g = row_geom(logits, prow, row_stride, vocab);
            if (pchunk < g.nchunks) {
                uint32_t off = g.head + pchunk * kChunk;
                uint32_t len = min(kChunk, g.nbody - pchunk * kChunk);
                uint32_t s = issued % kStages;
                mbar_arrive_expect_tx(&sm.full[s], len * 4u);
                tma_load_1d(sm.ring[s], g.p + off, len * 4u, &sm.full[s]);
                ++issued;
                ++pchunk;
                sm.issued = issued;
                return;
            }
            prow += gridDim.x;
            pchunk = 0;
        }
    };
    if (threadIdx.x == 0)
        for (uint32_t s = 0; s < kStages; ++s) produce_one();

    uint32_t consumed = 0;
    size_t row = blockIdx.x;
    for (; row < rows; row += gridDim.x) {
        const RowGeom g = row_geom(logits, row, row_stride, vocab);
        uint32_t tau = kKeyNegInf + 1u;  // excludes -inf; everything else is a candidate
        float mx_t = kNegInf, se_t = 0.0f;
        uint32_t cnt_t = 0;
        auto stats = [&](float v) {
            if (kRecord) {
                if (v != kNegInf) {
                    ++cnt_t;
                    if (v > mx_t) {
                        se_t = (mx_t == kNegInf ? 0.0f : se_t * __expf(mx_t - v)) + 1.0f;
                        mx_t = v;
                    } else {
                        se_t += __expf(v - mx_t);
                    }
                }
            }
        };
        if (threadIdx.x == 0) {
            sm.count = 0;
            sm.overflow = 0;
        }
        __syncthreads();
        // Scalar head and tail.
        {
            uint32_t ntail = vocab - g.head - g.nbody;
            uint32_t i = threadIdx.x;
            bool take = false;
            uint32_t key = 0, idx = ~0u;
            if (i < g.head) idx = i;
            else if (i >= 4 && i - 4 < ntail) idx = g.head + g.nbody + (i - 4);
            if (idx != ~0u) {
                float v = scale_logit(g.p[idx], cp.scale);
                stats(v);
                key = total_key(v);
                take = key >= tau;
            }
            append_candidate(sm, take, key, idx + index_offset);
        }
        for (uint32_t c = 0; c < g.nchunks; ++c) {
            const uint32_t s = consumed % kStages;
            const uint32_t parity = (consumed / kStages) & 1u;
            if (!mbar_wait(&sm.full[s], parity)) atomicExch(&sm.error, 1u);
            const uint32_t len = min(kChunk, g.nbody - c * kChunk);
            const uint32_t base_idx = g.head + c * kChunk + index_offset;
            const float4 *r4 = reinterpret_cast<const float4 *>(sm.ring[s]);
#pragma unroll
            for (uint32_t jj = 0; jj < kChunk / 4 / kThreads; ++jj) {
                const uint32_t j = threadIdx.x + jj * kThreads;
                float4 f = (4 * j < len) ? r4[j] : make_float4(kNegInf, kNegInf, kNegInf, kNegInf);
                const uint32_t i0 = base_idx + 4 * j;
                const float v0 = scale_logit(f.x, cp.scale), v1 = scale_logit(f.y, cp.scale);
                const float v2 = scale_logit(f.z, cp.scale), v3 = scale_logit(f.w, cp.scale);
                stats(v0);
                stats(v1);
                stats(v2);
                stats(v3);
                const uint32_t k0 = total_key(v0), k1 = total_key(v1);
                const uint32_t k2 = total_key(v2), k3 = total_key(v3);
                const bool any = (k0 >= tau) | (k1 >= tau) | (k2 >= tau) | (k3 >= tau);
                if (__any_sync(0xffffffffu, any)) {
                    append_candidate(sm, k0 >= tau, k0, i0);
                    append_candidate(sm, k1 >= tau, k1, i0 + 1);
                    append_candidate(sm, k2 >= tau, k2, i0 + 2);
                    append_candidate(sm, k3 >= tau, k3, i0 + 3);
                }
            }
            __syncthreads();  // stage s fully read; candidate count settled
            ++consumed;
            if (threadIdx.x == 0) produce_one();
            if (sm.error) break;
            if (cp.topk_active && c + 1 < g.nchunks && sm.count > kCap - kChunk) {
                compact(sm, cp.top_k, tau);
                if (sm.count > kCap - kChunk) sm.overflow = 1;  // all threads write the same value
            }
        }
        __syncthreads();
        if (sm.error) break;
        if (kRecord) {
            if (sm.overflow || sm.count > kCap) {
                if (threadIdx.x == 0) {
                    ShardRecordHeader *h = reinterpret_cast<ShardRecordHeader *>(records + row * rec_bytes);
                    h->flags = 1;
                    h->n_cand = 0;
                    h->n_dropped = 0;
                }
                __syncthreads();
                continue;
            }
            record_row(sm, cp, row, mx_t, se_t, cnt_t, records, rec_bytes);
        } else {
            if (sm.overflow || sm.count > kCap) {
                if (threadIdx.x == 0) large_rows[atomicAdd(large_count, 1u)] = static_cast<uint32_t>(row);
                __syncthreads();
                continue;
            }
            finish_row(sm, cp, row, out_ids, out_status, out_probs);
        }
    }
    if (row < rows) {
        // A wait gave up. Wait (bounded) for the copies still in flight into
        // this CTA's shared memory, then report the unfinished rows.
        if (threadIdx.x == 0) {
            const uint32_t n_issued = sm.issued;
            for (uint32_t q = consumed; q < n_issued; ++q)
                mbar_wait(&sm.full[q % kStages], (q / kStages) & 1u);
        }
        for (; row < rows; row += gridDim.x) {
            if (threadIdx.x != 0) continue;
            if (kRecord) {
                reinterpret_cast<ShardRecordHeader *>(records + row * rec_bytes)->flags = 2;
            } else {
                out_ids[row] = 0;
                out_status[row] = RSC_ROW_INTERNAL;
            }
        }
    }
}

// Vocab-sharded merge: one CTA per row gathers the shards' records into the
// candidate list and finishes the row exactly as the unsharded kernel does.
__global__ void __launch_bounds__(kThreads)
shard_merge_kernel(const unsigned char *__restrict__ records, size_t n_shards, size_t rows,
                   size_t rec_bytes, CallParams cp, uint32_t *__restrict__ out_ids,
                   int32_t *__restrict__ out_status, float *__restrict__ out_probs) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    StreamSmem &sm = *reinterpret_cast<StreamSmem *>(smem_raw);
    load_exp_table(sm.exp_tab);
    const uint32_t cap_entries = cp.top_k + RSC_SHARD_TIE_CAP;
    for (size_t row = blockIdx.x; row < rows; row += gridDim.x) {
        if (threadIdx.x == 0) {
            sm.count = 0;
            sm.overflow = 0;
        }
        __syncthreads();
        for (size_t s = 0; s < n_shards; ++s) {
            const unsigned char *rec = records + (s * rows + row) * rec_bytes;
            const ShardRecordHeader *h = reinterpret_cast<const ShardRecordHeader *>(rec);
            const uint32_t *rkey = reinterpret_cast<const uint32_t *>(rec + sizeof(ShardRecordHeader));
            const uint32_t *ridx = rkey + cap_entries;
            const uint32_t base = sm.count;
            const uint32_t nc = h->flags ? 0u : min(h->n_cand, cap_entries);
            for (uint32_t i = threadIdx.x; i < nc; i += kThreads) {
                if (base + i < kCap) {
                    sm.u.cand.key[base + i] = rkey[i];
                    sm.u.cand.idx[base + i] = ridx[i];
                }
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                sm.count = base + nc;
                if (h->flags || base + nc > kCap) sm.overflow = 1;
            }
            __syncthreads();
        }
        bool bad = sm.overflow != 0;
        if (!bad && cp.topk_active && sm.count >= cp.top_k) {
            // A shard that dropped tied entries is harmless only if everything
            // it dropped lies below the global threshold.
            uint32_t kth = block_select_kth_largest<kThreads>(
                sm.count, cp.top_k, [&](uint32_t i) { return sm.u.cand.key[i]; }, sm.hist, sm.sel);
            const uint32_t floor_key = relax_tau(kth);
            for (size_t s = 0; s < n_shards; ++s) {
                const ShardRecordHeader *h =
                    reinterpret_cast<const ShardRecordHeader *>(records + (s * rows + row) * rec_bytes);
                if (h->n_dropped > 0 && h->last_key >= floor_key) bad = true;
            }
        } else if (!bad) {
            for (size_t s = 0; s < n_shards; ++s) {
                const ShardRecordHeader *h =
                    reinterpret_cast<const ShardRecordHeader *>(records + (s * rows + row) * rec_bytes);
                if (h->n_dropped > 0) bad = true;
            }
        }
        if (bad) {
            if (threadIdx.x == 0) {
                out_ids[row] = 0;
                out_status[row] = RSC_ROW_INTERNAL;
                if (out_probs) out_probs[row] = __uint_as_float(0x7fc00000u);
            }
            __syncthreads();
            continue;
        }
        finish_row(sm, cp, row, out_ids, out_status, out_probs);
    }
}

template <typename K>
cudaError_t grid_for(K kernel, size_t rows, int num_sms, size_t *grid) {
    const size_t smem = sizeof(StreamSmem);
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    size_t g = static_cast<size_t>(num_sms) * per_sm;
    *grid = g > rows ? rows : g;
    return cudaSuccess;
}

}  // namespace

size_t stream_topk_smem_bytes() { return sizeof(StreamSmem); }

cudaError_t launch_stream_topk(const float *logits, size_t rows, uint32_t vocab,
                               size_t row_stride, const CallParams &p, uint32_t *out_ids,
                               int32_t *out_status, float *out_probs, uint32_t *large_rows,
                               uint32_t *large_count, int num_sms, cudaStream_t stream) {
    if (rows == 0) return cudaSuccess;
    size_t grid = 0;
    cudaError_t e = grid_for(stream_topk_kernel<false>, rows, num_sms, &grid);
    if (e != cudaSuccess) return e;
    stream_topk_kernel<false><<<static_cast<unsigned>(grid), kThreads, sizeof(StreamSmem), stream>>>(
        logits, rows, vocab, row_stride, p, out_ids, out_status, out_probs, large_rows,
        large_count, 0u, nullptr, 0);
    return cudaGetLastError();
}

cudaError_t launch_shard_partial(const float *logits, size_t rows, uint32_t shard_vocab,
                                 size_t row_stride, uint32_t shard_offset, const CallParams &p,
                                 void *records, size_t rec_bytes, int num_sms,
                                 cudaStream_t stream) {
    if (rows == 0) return cudaSuccess;
    size_t grid = 0;
    cudaError_t e = grid_for(stream_topk_kernel<true>, rows, num_sms, &grid);
    if (e != cudaSuccess) return e;
    stream_topk_kernel<true><<<static_cast<unsigned>(grid), kThreads, sizeof(StreamSmem), stream>>>(
        logits, rows, shard_vocab, row_stride, p, nullptr, nullptr, nullptr, nullptr, nullptr,
        shard_offset, static_cast<unsigned char *>(records), rec_bytes);
    return cudaGetLastError();
}

cudaError_t launch_shard_merge(const void *records, size_t n_shards, size_t rows, size_t rec_bytes,
                               const CallParams &p, uint32_t *out_ids, int32_t *out_status,
                               float *out_probs, int num_sms, cudaStream_t stream) {
    if (rows == 0) return cudaSuccess;
    size_t grid = 0;
    cudaError_t e = grid_for(shard_merge_kernel, rows, num_sms, &grid);
    if (e != cudaSuccess) return e;
    shard_merge_kernel<<<static_cast<unsigned>(grid), kThreads, sizeof(StreamSmem), stream>>>(
        static_cast<const unsigned char *>(records), n_shards, rows, rec_bytes, p, out_ids,
        out_status, out_probs);
    return cudaGetLastError();
}

}  // namespace rsc
