// Device helpers shared by the sampling kernels: total-order keys, the
// reference's f32 semantics (NaN folding, temperature scaling), a binary32 exp
// that reproduces glibc's expf bit for bit, the per-row generator, and bounded
// mbarrier waits for the TMA pipelines.
//
// Every floating-point operation that the reference performs in binary32 is
// written with an explicit round-to-nearest intrinsic (__fmul_rn, __fadd_rn,
// __fsub_rn, __fdiv_rn) so that no contraction or reassociation can change a
// result; the library is also built with -fmad=false.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/rusticide_cuda.h"

namespace rsc {

constexpr float kNegInf = -__builtin_huge_valf();
constexpr float kPosInf = __builtin_huge_valf();
// x86-64 SSE writes this "default NaN" (sign set, quiet) for an invalid
// operation such as inf * 0; the reference runs there, and f32::total_cmp
// orders it below -inf. The GPU's own NaN (0x7fffffff) would order above +inf,
// so any NaN that the scaling step creates is rewritten to this pattern.
constexpr uint32_t kX86DefaultNaN = 0xffc00000u;

// Monotone unsigned key of f32::total_cmp (core::f32::total_cmp): negative
// values have every bit flipped, non-negative ones only the sign bit, so that
// unsigned order equals the total order (-NaN < -inf < ... < -0 < +0 < ... <
// +inf < +NaN).
__host__ __device__ __forceinline__ uint32_t total_key(float v) {
#ifdef __CUDA_ARCH__
    uint32_t u = __float_as_uint(v);
#else
    uint32_t u;
    __builtin_memcpy(&u, &v, 4);
#endif
    uint32_t mask = static_cast<uint32_t>(static_cast<int32_t>(u) >> 31) | 0x80000000u;
    return u ^ mask;
}

__host__ __device__ __forceinline__ float key_to_float(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k ^ 0x80000000u) : ~k;
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    float f;
    __builtin_memcpy(&f, &u, 4);
    return f;
#endif
}

constexpr uint32_t kKeyNegInf = 0x007fffffu;   // total_key(-inf)
constexpr uint32_t kKeyNegZero = 0x7fffffffu;  // total_key(-0.0)
constexpr uint32_t kKeyPosZero = 0x80000000u;  // total_key(+0.0)
constexpr uint32_t kKeyPosInf = 0xff800000u;   // total_key(+inf)

// The reference's scaling step, crates/rusticide-sampling/src/candidates.rs:30-37:
// NaN reads as -inf, then one binary32 multiply by `scale`.
__device__ __forceinline__ float scale_logit(float x, float scale) {
    float l = (x != x) ? kNegInf : x;
    float v = __fmul_rn(l, scale);
    if (v != v) v = __uint_as_float(kX86DefaultNaN);
    return v;
}

// The keep test of candidates.rs:48-50 against threshold `thr`:
// value != -inf && value.partial_cmp(&thr) != Some(Less).
__device__ __forceinline__ bool survives(float v, float thr) {
    return v != kNegInf && !(v < thr);
}

// ---------------------------------------------------------------------------
// expf reproducing glibc 2.39's binary32 exp.
//
// Method (the exp2-table method of ARM's optimized-routines, which glibc
// adopted for expf): with N = 32, z = x * N/ln2 is split as k + r with k the
// nearest integer (found by adding 1.5 * 2^52) and |r| <= 1/2;
// exp(x) = 2^(k/N) * 2^(r/N), 2^(k/N) comes from a 32-entry table of 2^(j/N)
// with the exponent (k div N) added to its bits, and 2^(r/N) is a degree-3
// polynomial in r. Everything is binary64 and the result is rounded once to
// binary32. The reduction uses fused multiply-adds, as glibc's x86-64 FMA
// variant does. Checked exhaustively against glibc expf for every binary32
// x in [-104, 0], the only range this path evaluates (x = v - max <= 0):
// 1,120,927,745 inputs, 0 differences.
// ---------------------------------------------------------------------------
struct ExpTable {
    double t[32];
};

// 2^(j/32), j = 0..31, each correctly rounded to binary64.
__host__ __device__ constexpr ExpTable exp2_table() {
    return ExpTable{{
        0x1p+0, 0x1.059b0d3158574p+0, 0x1.0b5586cf9890fp+0, 0x1.11301d0125b51p+0,
        0x1.172b83c7d517bp+0, 0x1.1d4873168b9aap+0, 0x1.2387a6e756238p+0, 0x1.29e9df51fdee1p+0,
        0x1.306fe0a31b715p+0, 0x1.371a7373aa9cbp+0, 0x1.3dea64c123422p+0, 0x1.44e086061892dp+0,
        0x1.4bfdad5362a27p+0, 0x1.5342b569d4f82p+0, 0x1.5ab07dd485429p+0, 0x1.6247eb03a5585p+0,
        0x1.6a09e667f3bcdp+0, 0x1.71f75e8ec5f74p+0, 0x1.7a11473eb0187p+0, 0x1.82589994cce13p+0,
        0x1.8ace5422aa0dbp+0, 0x1.93737b0cdc5e5p+0, 0x1.9c49182a3f09p+0, 0x1.a5503b23e255dp+0,
        0x1.ae89f995ad3adp+0, 0x1.b7f76f2fb5e47p+0, 0x1.c199bdd85529cp+0, 0x1.cb720dcef9069p+0,
        0x1.d5818dcfba487p+0, 0x1.dfc97337b9b5fp+0, 0x1.ea4afa2a490dap+0, 0x1.f50765b6e454p+0}};
}

// The table in constant memory; kernels copy it to shared memory, where the
// lanes of a warp can read different entries in one access.
static __constant__ ExpTable kExp2Table = exp2_table();

__device__ __forceinline__ void load_exp_table(double *dst) {
    if (threadIdx.x < 32) dst[threadIdx.x] = kExp2Table.t[threadIdx.x];
}

// The method's core for x in [-104, 88.72...] (no range checks).
// Attribution: the reduction constant, the 2^(j/32) table and the three
// polynomial coefficients below are the published data of Arm's
// optimized-routines expf (math/expf.c with math/exp2f_data.c, Copyright
// Arm Limited, MIT licence, later MIT OR Apache-2.0 WITH LLVM-exception);
// glibc ships the same data in sysdeps/ieee754/flt-32/e_exp2f_data.c. The
// code around them is this library's own restatement of the method.
__device__ __forceinline__ float expf_core(float x, const double *tab) {
    const double kInvLn2N = 0x1.71547652b82fep+0 * 32.0;
    const double kShift = 0x1.8p+52;
    const double c0 = 0x1.c6af84b912394p-5 / (32.0 * 32.0 * 32.0);
    const double c1 = 0x1.ebfce50fac4f3p-3 / (32.0 * 32.0);
    const double c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    double xd = static_cast<double>(x);
    double kd = __fma_rn(kInvLn2N, xd, kShift);
    uint64_t ki = static_cast<uint64_t>(__double_as_longlong(kd));
    kd = __dsub_rn(kd, kShift);
    double r = __fma_rn(kInvLn2N, xd, -kd);
    uint64_t t = static_cast<uint64_t>(__double_as_longlong(tab[ki & 31]));
    t += ki << 47;  // adds k div 32 to the exponent; the table entry keeps j/32
    t -= (ki & 31) << 47;
    double s = __longlong_as_double(static_cast<long long>(t));
    double z = __fma_rn(c0, r, c1);
    double r2 = __dmul_rn(r, r);
    double y = __fma_rn(c2, r, 1.0);
    y = __fma_rn(z, r2, y);
    y = __dmul_rn(y, s);
    return __double2float_rn(y);
}

// `tab` points at the 32-entry table (shared memory in hot loops).
__device__ __forceinline__ float expf_ref(float x, const double *tab) {
    if (!(x >= -104.0f)) {            // -inf, below the subnormal range, or NaN
        return (x != x) ? x : 0.0f;   // glibc: exp(NaN) = NaN, otherwise +0
    }
    if (x > 88.72283172607421875f) return kPosInf;
    return expf_core(x, tab);
}

// ---------------------------------------------------------------------------
// Per-row generator: fastrand::Rng as the reference's Sampler uses it
// (Rng::with_seed(seed), then f32(); crates/rusticide-sampling/src/
// sampler.rs:17-23,112; fastrand 2.5.0 per Cargo.lock:191-195).
//  - gen_u64 is the wyrand step with the final wyhash v4.2 constants, which
//    fastrand's lib.rs uses since its 2.1 release: the state advances by
//    0x2d358dccaa6c78a5, and the output is the xor of the two halves of the
//    128-bit product s * (s ^ 0x8bb84b93962eacc9).
//  - f32 takes gen_u32 (the low 32 bits of gen_u64), keeps its top 23 bits
//    as the mantissa of a float in [1, 2) and subtracts 1.
// The stream is restated from the crate's published source; it is not
// checked against output of the crate itself (no Rust toolchain here).
// ---------------------------------------------------------------------------
constexpr uint64_t kWyInc = 0x2d358dccaa6c78a5ULL;
constexpr uint64_t kWyXor = 0x8bb84b93962eacc9ULL;

__host__ __device__ __forceinline__ uint64_t wyrand_next(uint64_t *state) {
    uint64_t s = *state + kWyInc;
    *state = s;
    uint64_t b = s ^ kWyXor;
#ifdef __CUDA_ARCH__
    uint64_t hi = __umul64hi(s, b);
#else
    uint64_t hi = static_cast<uint64_t>((static_cast<unsigned __int128>(s) * b) >> 64);
#endif
    uint64_t lo = s * b;
    return hi ^ lo;
}

__host__ __device__ __forceinline__ float wyrand_f32(uint64_t *state) {
    uint32_t x = static_cast<uint32_t>(wyrand_next(state));
    uint32_t bits = 0x3f800000u | (x >> 9);
#ifdef __CUDA_ARCH__
    float f = __uint_as_float(bits);
    return __fsub_rn(f, 1.0f);
#else
    float f;
    __builtin_memcpy(&f, &bits, 4);
    return f - 1.0f;
#endif
}

// ---------------------------------------------------------------------------
// Launch-wide parameters of one sampling call.
// ---------------------------------------------------------------------------
enum Mode : int {
    kModeSampleLogits = 0,   // Sampler::sample_logits
    kModeSampleWithTemp = 1  // Sampler::sample_with_temp (T != 0)
};

struct CallParams {
    float temperature;
    float scale;        // 1/T when T > 0 else 1 (candidates.rs:25-29); 1/T for sample_with_temp
    uint32_t top_k;     // as given
    float top_p;
    bool topk_active;   // 0 < k < vocab
    bool topp_active;   // top_p < 1.0
    bool argmax_branch; // T == 0 || top_k == 1 (src/sampler.rs:48)
    bool normal_scale;  // scale finite and > 0: scaling can create no NaN
    int mode;
    const float *uniforms;   // nullable
    uint64_t *rng_states;    // nullable
    uint32_t *out_nsurv;     // nullable: survivor count per row
    uint32_t *out_surv;      // nullable: rows x surv_cap survivor ids
    uint32_t surv_cap;
    float *out_survp = nullptr;   // nullable: rows x surv_cap survivor probabilities
    const rsc_params *row_params = nullptr;  // one parameter set per row (rsc_sample_rows)
    // Log-sum-exp parts (nullable): for row r and part p of it, lse_parts[r *
    // lse_stride + p] = (total_key of the part's largest scaled logit, sum of
    // exp(v - that maximum) over the part), each part of the row one slot.
    uint2 *lse_parts = nullptr;
    uint32_t lse_stride = 0;
};

// Combines two (maximum, sum of exp(v - maximum)) partial log-sum-exps.
__device__ __forceinline__ void lse_combine(float &m, float &s, float m2, float s2) {
    if (m2 == kNegInf) return;
    if (m == kNegInf) {
        m = m2;
        s = s2;
        return;
    }
    if (m2 > m) {
        s = s * __expf(m - m2) + s2;
        m = m2;
    } else {
        s += s2 * __expf(m2 - m);
    }
}

// Adds one scaled logit v to a partial log-sum-exp (m, s).
__device__ __forceinline__ void lse_add(float &m, float &s, float v) {
    if (v == kNegInf) return;
    if (v > m) {
        s = (m == kNegInf ? 0.0f : s * __expf(m - v)) + 1.0f;
        m = v;
    } else {
        s += __expf(v - m);
    }
}

// The parameters that apply to one row: the call's, or the row's own set,
// derived field by field as the host derives the call's.
__device__ __forceinline__ CallParams for_row(const CallParams &cp, size_t row, size_t vocab) {
    if (!cp.row_params) return cp;
    CallParams r = cp;
    const rsc_params q = cp.row_params[row];
    r.temperature = q.temperature;
    // candidates.rs:25-29: 1/T for T > 0, else 1 (IEEE division, as on the host).
    r.scale = q.temperature > 0.0f ? __fdiv_rn(1.0f, q.temperature) : 1.0f;
    r.top_k = q.top_k;
    r.top_p = q.top_p;
    r.topk_active = q.top_k != 0 && static_cast<size_t>(q.top_k) < vocab;
    r.topp_active = q.top_p < 1.0f;
    r.argmax_branch = q.temperature == 0.0f || q.top_k == 1;
    r.normal_scale = isfinite(r.scale) && r.scale > 0.0f;
    return r;
}

// The uniform for a row that takes the draw branch.
__device__ __forceinline__ float row_uniform(const CallParams &p, size_t row) {
    if (p.uniforms) return p.uniforms[row];
    if (p.rng_states) {
        uint64_t st = p.rng_states[row];
        float u = wyrand_f32(&st);
        p.rng_states[row] = st;
        return u;
    }
    return 0.0f;
}

// ---------------------------------------------------------------------------
// Bounded waits. Every spin in these kernels gives up after a bounded number
// of polls and reports RSC_ROW_INTERNAL instead of hanging the GPU.
// ---------------------------------------------------------------------------
// A wait gives up after this many nanoseconds of the global timer.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

// One potentially blocking test of the barrier: a waiting thread is suspended
// (up to 100 us) rather than spinning, so it takes no issue slots from the
// warps that are working.
__device__ __forceinline__ bool mbar_try(uint32_t addr, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity), "r"(100000u)
        : "memory");
    return done != 0;
}

// Returns true once phase `parity` of the barrier has completed; false if it
// has not after kWaitLimitNs. The timer is read once per 256 polls.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    const uint32_t addr = smem_addr(bar);
    if (mbar_try(addr, parity)) return true;
    const unsigned long long t0 = global_ns();
    while (true) {
        if (mbar_try(addr, parity)) return true;
        if (global_ns() - t0 > kWaitLimitNs) return false;
    }
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// One-dimensional TMA bulk copy global -> shared (no multicast), completing
// on `bar` with a transaction count of `bytes`. Both addresses 16-byte
// aligned, bytes a multiple of 16.
__device__ __forceinline__ void tma_load_1d(void *dst_smem, const void *src_gmem, uint32_t bytes,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Asks the L2 to fetch the 128-byte line holding a global address (no data
// returns to the thread; a hint only).
__device__ __forceinline__ void prefetch_l2(const void *p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// ---------------------------------------------------------------------------
// Small helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t pack_key_index(uint32_t key, uint32_t idx) {
    return (static_cast<uint64_t>(key) << 32) | idx;
}

template <typename T>
__device__ __forceinline__ T warp_max(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        T w = __shfl_xor_sync(0xffffffffu, v, o);
        v = v > w ? v : w;
    }
    return v;
}

template <typename T>
__device__ __forceinline__ T warp_min(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        T w = __shfl_xor_sync(0xffffffffu, v, o);
        v = v < w ? v : w;
    }
    return v;
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace rsc
