// Whole-row kernel for rows with top-p on and top-k off whose survivors fit
// in shared memory (vocab <= kWholeMaxToppVocab): Sampler::sample_logits
// (crates/rusticide-sampling/src/sampler.rs:44-54) with Candidates::filter
// at k = 0 (candidates.rs:16-78): the survivors sorted by value, exp_sum and
// the cut-off running sum in that order (candidates.rs:55-78), then the
// softmax sum (filters.rs:5-15) and the draw (sampler.rs:111-121) in index
// order. One 1024-thread block per SM, a row at a time.
//
// Each row is read from HBM once; later passes find it in L2. The four sums
// are replayed exactly by the tile walk of rsc_walk.cuh. The survivors are
// sorted in shared memory, and their terms kept in index order in the
// block's scratch slot (n floats, L2-resident):
//  - the sort key is the distance d = fl(max - v) >= 0: equal d give equal
//    terms exp(-d) = exp(fl(v - max)), and larger d smaller terms, so sums
//    in d order equal the reference's sums in value order;
//  - survivors are counted into 8192 linear buckets of d, scattered into
//    their buckets in shared memory (with their terms, not their indices),
//    and each bucket is sorted in place by term, descending;
//  - only inside the group of survivors that share the cut-off's term does
//    the reference's (value desc, index asc) order decide who is kept; that
//    group is ranked explicitly.
// A row that does not qualify (a survivor of +-inf, or a bucket above
// kMaxBucket) is sampled by the large-row code (rsc_large.cuh) in the same
// block and shared memory.
#include "rsc_large.cuh"
#include "rsc_walk.cuh"

namespace rsc {
namespace whole {

using large::dist_bucket;
using large::for_each_scaled;
using large::RowView;

constexpr int kR = 16;               // terms per run of the tile walk
constexpr uint32_t kNB = 8192;       // distance buckets of the top-p sort
constexpr uint32_t kMaxBucket = 128; // largest bucket sorted in place

template <int T>
struct WholeSmem {
    double exp_tab[32];
    uint32_t red32[32];
    unsigned long long red64[32];
    float redf[32];
    uint32_t bcast[8];
    union {
        walk::WalkSmem<T> walk;
        uint32_t boff[kNB];  // top-p sort: bucket counts, then offsets
    };
};

template <int T>
constexpr size_t big_offset() {
    return (sizeof(WholeSmem<T>) + 15) & ~static_cast<size_t>(15);
}

struct Never {
    __device__ bool operator()(float) const { return false; }
};

// Half the spacing of binary32 floats at s (the largest term that s absorbs
// is below it).
__device__ __forceinline__ float half_spacing(float s) {
    const uint32_t ef = max(__float_as_uint(s) >> 23, 1u);
    return __uint_as_float(ef << 23) * 0x1p-24f;
}

// One tile of stored terms E (index order; negative: not a survivor) into
// the run layout, keeping those `kept` accepts, optionally divided by div.
// Terms below half the spacing at s (or whose quotient certainly is) are +0.
template <int T, typename Keep>
__device__ __forceinline__ void fill_array(const float *E, uint32_t base, uint32_t tn, Keep &kept,
                                           float s, float div, bool divide, float *buf) {
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t w0 = warp * 32u * kR;
    const float tmin = half_spacing(s);
    const float thr = divide ? tmin * div * (1.0f - 0x1p-20f) : tmin;
    float ev[kR];
#pragma unroll
    for (int i = 0; i < kR; ++i) {
        const uint32_t p = w0 + static_cast<uint32_t>(i) * 32u + lane;
        ev[i] = p < tn ? E[base + p] : -1.0f;
    }
#pragma unroll
    for (int i = 0; i < kR; ++i) {
        const uint32_t e = static_cast<uint32_t>(i) * 32u + lane;
        const uint32_t p = w0 + e;
        float t = 0.0f;
        if (ev[i] >= 0.0f && !(ev[i] < thr) && kept(base + p, ev[i]))
            t = divide ? __fdiv_rn(ev[i], div) : ev[i];
        buf[walk::fill_slot<kR>(warp, e)] = t;
    }
    __syncwarp();
}

__device__ __forceinline__ void write_row(size_t row, uint32_t token, int32_t status, float prob,
                                          uint32_t *out_ids, int32_t *out_status,
                                          float *out_probs) {
    if (threadIdx.x == 0) {
        out_ids[row] = token;
        out_status[row] = status;
        if (out_probs) out_probs[row] = prob;
    }
}

// The uniform of a row that draws, read once and shared with the block.
template <int T>
__device__ __forceinline__ float block_uniform(const CallParams &cp, size_t row, WholeSmem<T> &sm) {
    if (threadIdx.x == 0) sm.bcast[0] = __float_as_uint(row_uniform(cp, row));
    __syncthreads();
    const float r = __uint_as_float(sm.bcast[0]);
    __syncthreads();
    return r;
}

// A row with top-p on and top-k off (Candidates::filter with k = 0,
// candidates.rs:16-78, then softmax and the draw): see the file comment.
// E: the block's scratch (n + 3 floats, 16-byte aligned) for the terms in
// index order; G: 2 * n words for the tie group. S: shared memory, `cap`
// floats. Returns false, having written nothing, when the row does not
// qualify.
template <int T>
__device__ __noinline__ bool topp_row(const CallParams &cp, const RowView &rv, size_t row,
                                      float *E16, uint32_t *G, uint32_t *out_ids,
                                      int32_t *out_status, float *out_probs, WholeSmem<T> &sm,
                                      float *S, uint32_t cap) {
    const uint32_t n = rv.n;
    const uint32_t tid = threadIdx.x;
    const double *tab = sm.exp_tab;

    // A: the survivors' maximum, minimum and count; whether any is infinite.
    float smax = kNegInf, smin = kPosInf;
    uint32_t nsurv = 0, odd = 0;
    for_each_scaled<T, 8>(rv, [&](float v, uint32_t) {
        if (v != kNegInf) {
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
    if (nsurv == 0 || odd || walk::padded<kR>(nsurv) + kR > cap) return false;
    const float span = fminf(__fsub_rn(smax, smin), 104.0f);
    const float inv = span > 0.0f ? __fdiv_rn(static_cast<float>(kNB - 1), span) : 0.0f;

    // B: bucket counts of d = fl(max - v), the largest (the last bucket, d >=
    // 104 with terms +0, is not sorted), then the exclusive offsets.
    for (uint32_t b = tid; b < kNB; b += T) sm.boff[b] = 0;
    __syncthreads();
    for_each_scaled<T, 8>(rv, [&](float v, uint32_t) {
        if (v != kNegInf) atomicAdd(&sm.boff[dist_bucket(__fsub_rn(smax, v), inv, kNB)], 1u);
    });
    __syncthreads();
    constexpr uint32_t kPer = kNB / T;
    uint32_t tot = 0, big = 0;
#pragma unroll
    for (uint32_t e = 0; e < kPer; ++e) {
        const uint32_t b = tid * kPer + e;
        const uint32_t c = sm.boff[b];
        tot += c;
        if (b < kNB - 1) big = max(big, c);
    }
    big = block_reduce<T>(big, sm.red32, OpMaxU32());
    if (big > kMaxBucket) return false;
    {
        uint32_t all;
        uint32_t run = block_exclusive_add<T>(tot, sm.red32, &all);
#pragma unroll
        for (uint32_t e = 0; e < kPer; ++e) {
            const uint32_t b = tid * kPer + e;
            const uint32_t c = sm.boff[b];
            sm.boff[b] = run;
            run += c;
        }
    }
    __syncthreads();

    // C: each survivor's term, once: into E (index order; -1 for the rest)
    // and into its bucket of S. E is offset so that the row's 16-byte body
    // stores as float4.
    const uint32_t mis = static_cast<uint32_t>((reinterpret_cast<uintptr_t>(rv.p) >> 2) & 3u);
    const uint32_t head = mis ? min(n, 4u - mis) : 0u;
    const uint32_t n4 = (n - head) / 4u;
    const uint32_t tail0 = head + 4u * n4;
    float *E = E16 + ((4u - head) & 3u);
    auto term_of = [&](float v) -> float {
        if (v == kNegInf) return -1.0f;
        const float d = __fsub_rn(smax, v);
        const float t = expf_ref(-d, tab);  // exp(fl(v - max)): fl(v - max) = -d
        const uint32_t pos = atomicAdd(&sm.boff[dist_bucket(d, inv, kNB)], 1u);
        S[walk::padded<kR>(pos)] = t;
        return t;
    };
    if (tid < head) E[tid] = term_of(rv.value(tid));
    if (tid >= 32 && tid - 32 < n - tail0) E[tail0 + tid - 32] = term_of(rv.value(tail0 + tid - 32));
    {
        const float4 *p4 = reinterpret_cast<const float4 *>(rv.p + head);
        float4 *e4 = reinterpret_cast<float4 *>(E + head);
        constexpr int kB = 4;
        for (uint32_t q0 = 0; q0 < n4; q0 += T * kB) {
            float4 x[kB];
#pragma unroll
            for (int b = 0; b < kB; ++b) {
                const uint32_t q = q0 + b * T + tid;
                if (q < n4) x[b] = p4[q];
            }
#pragma unroll
            for (int b = 0; b < kB; ++b) {
                const uint32_t q = q0 + b * T + tid;
                if (q < n4) {
                    float4 t;
                    t.x = term_of(rv.scaled(x[b].x));
                    t.y = term_of(rv.scaled(x[b].y));
                    t.z = term_of(rv.scaled(x[b].z));
                    t.w = term_of(rv.scaled(x[b].w));
                    e4[q] = t;
                }
            }
        }
    }
    __syncthreads();

    // D: each bucket by term, descending (insertion sort in place; any order
    // of equal terms gives the same sums). Bucket b is [boff[b-1], boff[b])
    // now. Thread t sorts buckets t, t + T, ...: buckets T apart lie far
    // apart in d, so few threads get more than one of the dense ones.
    for (uint32_t b = tid; b < kNB - 1; b += T) {
        const uint32_t st = b ? sm.boff[b - 1] : 0u, en = sm.boff[b];
        for (uint32_t x = st + 1; x < en; ++x) {
            const float key = S[walk::padded<kR>(x)];
            uint32_t y = x;
            while (y > st) {
                const float o = S[walk::padded<kR>(y - 1)];
                if (!(o < key)) break;
                S[walk::padded<kR>(y)] = o;
                --y;
            }
            S[walk::padded<kR>(y)] = key;
        }
    }
    __syncthreads();

    // E, F: exp_sum and the cut-off over the sorted terms (candidates.rs:62-75).
    const float exp_sum = walk::replay_array<T, kR>(S, nsurv, walk::Identity(), Never(), sm.walk).sum;
    const float p = cp.top_p;
    auto over_sum = [exp_sum](float x) { return __fdiv_rn(x, exp_sum); };
    const ReplayResult cs =
        walk::replay_array<T, kR>(S, nsurv, over_sum, [p](float x) { return x > p; }, sm.walk);
    bool cut = false, gsplit = false;
    float tc = 0.0f;
    uint32_t cut_key = 0, cut_idx = 0;
    if (cs.stop >= 0 && static_cast<uint32_t>(cs.stop) + 1 < nsurv) {
        cut = true;
        const uint32_t c = static_cast<uint32_t>(cs.stop);
        tc = S[walk::padded<kR>(c)];
        // The group of survivors whose term equals the cut-off's: how many
        // terms lie above it, and its size.
        uint32_t above = 0, eq = 0;
        for (uint32_t q = tid; q < nsurv; q += T) {
            const float o = S[walk::padded<kR>(q)];
            above += o > tc ? 1u : 0u;
            eq += o == tc ? 1u : 0u;
        }
        above = block_reduce<T>(above, sm.red32, OpAddU32());
        eq = block_reduce<T>(eq, sm.red32, OpAddU32());
        const uint32_t m = c - above + 1u;
        if (m < eq) {
            // The group's first m in the reference's (value desc, index
            // asc) order are kept: gather it, rank it, take the m-th.
            gsplit = true;
            if (tid == 0) sm.bcast[1] = 0;
            __syncthreads();
            uint32_t *gk = G, *gi = G + n;
            for (uint32_t i = tid; i < n; i += T) {
                if (E[i] == tc) {
                    const uint32_t at = atomicAdd(&sm.bcast[1], 1u);
                    gk[at] = total_key(rv.value(i));
                    gi[at] = i;
                }
            }
            __syncthreads();
            const uint32_t gn = sm.bcast[1];
            for (uint32_t a = tid; a < gn; a += T) {
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
        }
    }
    __syncthreads();
    // Kept after top-p: a survivor at or before the cut-off in the
    // reference's order.
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
    for (uint32_t i = tid; i < n; i += T)
        if (kept(i, E[i])) last = max(last, i);
    last = block_reduce<T>(last, sm.red32, OpMaxU32());

    // H: the softmax sum in index order (filters.rs:7-8). Its maximum is the
    // row's (the largest survivor is always kept), so its terms are E. S is
    // free now; its space holds the tiles.
    float *buf = S;
    auto sum_fill = [&](uint32_t base, uint32_t tn, float s, float *b) {
        fill_array<T>(E, base, tn, kept, s, 1.0f, false, b);
    };
    const float sum = walk::replay_fill<T, kR>(n, sum_fill, Never(), buf, sm.walk).sum;

    // I: the draw (sampler.rs:111-121); sum >= 1, finite.
    const float r = block_uniform<T>(cp, row, sm);
    auto draw_fill = [&](uint32_t base, uint32_t tn, float s, float *b) {
        fill_array<T>(E, base, tn, kept, s, sum, true, b);
    };
    const ReplayResult dr =
        walk::replay_fill<T, kR>(n, draw_fill, [r](float x) { return r < x; }, buf, sm.walk);
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
    write_row(row, pos, status, __fdiv_rn(E[pos], sum), out_ids, out_status, out_probs);
    __syncthreads();
    return true;
}

template <int T>
__global__ void __launch_bounds__(T, 1)
whole_kernel(const float *__restrict__ logits, size_t rows, uint32_t vocab, size_t row_stride,
             CallParams cp, uint32_t *__restrict__ out_ids, int32_t *__restrict__ out_status,
             float *__restrict__ out_probs, uint32_t *__restrict__ scratch, uint32_t cap) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    WholeSmem<T> &sm = *reinterpret_cast<WholeSmem<T> *>(smem_raw);
    float *big = reinterpret_cast<float *>(smem_raw + big_offset<T>());
    load_exp_table(sm.exp_tab);
    __syncthreads();
    // The block's scratch slot: 4 * vocab words (E, then the tie group).
    uint32_t *slot = scratch + static_cast<size_t>(blockIdx.x) * 4u * vocab;
    for (size_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const RowView rv{logits + row * row_stride, vocab, cp.scale, false};
        if (!topp_row<T>(cp, rv, row, reinterpret_cast<float *>(slot), slot + vocab + 4u, out_ids,
                         out_status, out_probs, sm, big, cap)) {
            // The large-row code in the same shared memory (its table sits
            // where this kernel's does).
            __syncthreads();
            large::LargeSmem<T> &lsm = *reinterpret_cast<large::LargeSmem<T> *>(smem_raw);
            large::large_row<T>(cp, rv, row, slot, out_ids, out_status, out_probs, lsm);
            __syncthreads();
            load_exp_table(sm.exp_tab);
            __syncthreads();
        }
    }
}

constexpr int kThreads = 1024;

// Dynamic shared memory of a launch: the fixed part, then the larger of the
// sorted terms (padded) and the index-order replays' tile buffer, and at
// least the large-row code's layout for the rows that fall back to it.
constexpr size_t smem_need(uint32_t vocab) {
    const size_t tile = static_cast<size_t>(kThreads) * (kR + 1) * sizeof(float);
    const size_t sorted = (static_cast<size_t>(vocab) + vocab / kR + kR) * sizeof(float);
    const size_t bytes = big_offset<kThreads>() + (sorted > tile ? sorted : tile);
    return bytes < sizeof(large::LargeSmem<kThreads>) ? sizeof(large::LargeSmem<kThreads>) : bytes;
}
static_assert(smem_need(kWholeMaxToppVocab) <= 232448, "top-p rows must fit shared memory");

}  // namespace whole

bool whole_takes(const CallParams &p, size_t vocab) {
    return p.mode == kModeSampleLogits && p.normal_scale && !p.out_nsurv && !p.out_surv &&
           !p.out_survp && !p.row_params && !p.topk_active && p.topp_active &&
           !p.argmax_branch && vocab <= kWholeMaxToppVocab;
}

cudaError_t launch_whole(const float *logits, size_t rows, uint32_t vocab, size_t row_stride,
                         const CallParams &p, uint32_t *out_ids, int32_t *out_status,
                         float *out_probs, uint32_t *scratch, uint32_t slots, int num_sms,
                         cudaStream_t stream) {
    using namespace whole;
    if (rows == 0 || slots == 0) return cudaSuccess;
    const size_t smem = smem_need(vocab);
    cudaError_t e = cudaFuncSetAttribute(whole_kernel<kThreads>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const uint32_t cap = static_cast<uint32_t>((smem - big_offset<kThreads>()) / sizeof(float));
    size_t grid = static_cast<size_t>(num_sms);
    if (grid > slots) grid = slots;
    if (grid > rows) grid = rows;
    whole_kernel<kThreads><<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(
        logits, rows, vocab, row_stride, p, out_ids, out_status, out_probs, scratch, cap);
    return cudaGetLastError();
}

}  // namespace rsc
