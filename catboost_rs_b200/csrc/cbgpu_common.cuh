// cbgpu_common.cuh -- shared device/host primitives for the B200 oblivious-tree path.
//
// TFastRng64 and FastLogf are restated here (product code) from the reference's
// crates/cb-core/src/rng.rs and crates/cb-train/src/fast_approx.rs.  Everything
// that must be bit-exact against the CPU path (bootstrap weights) uses explicit
// round-to-nearest intrinsics so no FMA contraction can change a rounding.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#define CBGPU_HD __host__ __device__ __forceinline__

namespace cbgpu {

constexpr uint64_t kLcgA = 6364136223846793005ULL;  // rng.rs:26

// PCG XSH-RR output mix (rng.rs:31-38).
CBGPU_HD uint32_t pcg_mix(uint64_t x) {
    uint32_t xs = (uint32_t)(((x >> 18) ^ x) >> 27);
    uint32_t rot = (uint32_t)(x >> 59);
    return (xs >> rot) | (xs << ((32u - rot) & 31u));
}

// The multiplier pair of an O(log delta) jump of an LCG stream (rng.rs:45-69):
// delta steps take x to x * apow + c * adiv, for any increment c.
CBGPU_HD void lcg_jump(uint64_t delta, uint64_t& apow, uint64_t& adiv) {
    uint64_t mask = 1;
    while (mask != (1ULL << 63) && (mask << 1) <= delta) mask <<= 1;
    apow = 1;
    adiv = 0;
    while (mask != 0) {
        adiv = adiv * (apow + 1);
        apow = apow * apow;
        if (delta & mask) {
            adiv = adiv + apow;
            apow = apow * kLcgA;
        }
        mask >>= 1;
    }
}

CBGPU_HD uint64_t lcg_advance(uint64_t seed, uint64_t c, uint64_t delta) {
    uint64_t apow, adiv;
    lcg_jump(delta, apow, adiv);
    return seed * apow + c * adiv;
}

CBGPU_HD uint32_t lcg_next32(uint64_t& x, uint64_t c) {
    x = x * kLcgA + c;
    return pcg_mix(x);
}

// Two concatenated PCG streams; stream 1 yields the high word (rng.rs:150-190).
struct Rng64 {
    uint64_t x1, c1, x2, c2;

    CBGPU_HD static Rng64 from_parts(uint64_t s1, uint32_t q1, uint64_t s2, uint32_t q2) {
        const uint32_t m = 0x7fffffffu;  // FixSeq (rng.rs:128-136)
        uint32_t q2f = ((q1 & m) == (q2 & m)) ? ~q2 : q2;
        Rng64 r;
        r.x1 = s1;
        r.c1 = ((uint64_t)q1 << 1) | 1u;
        r.x2 = s2;
        r.c2 = ((uint64_t)q2f << 1) | 1u;
        return r;
    }
    // One-seed constructor: parameters from TReallyFastRng32(seed) (rng.rs:171-179).
    CBGPU_HD static Rng64 from_seed(uint64_t seed) {
        uint64_t x = seed;
        uint64_t lo = lcg_next32(x, 1), hi = lcg_next32(x, 1);
        uint64_t s1 = lo | (hi << 32);
        uint32_t q1 = lcg_next32(x, 1);
        lo = lcg_next32(x, 1);
        hi = lcg_next32(x, 1);
        uint64_t s2 = lo | (hi << 32);
        uint32_t q2 = lcg_next32(x, 1);
        return from_parts(s1, q1, s2, q2);
    }
    CBGPU_HD uint64_t gen() {
        uint64_t hi = lcg_next32(x1, c1);
        uint64_t lo = lcg_next32(x2, c2);
        return (hi << 32) | lo;
    }
    CBGPU_HD void advance(uint64_t d) {
        x1 = lcg_advance(x1, c1, d);
        x2 = lcg_advance(x2, c2, d);
    }
    // a jump by a fixed distance whose (apow, adiv) pair is known (lcg_jump)
    CBGPU_HD void jump(uint64_t apow, uint64_t adiv) {
        x1 = x1 * apow + c1 * adiv;
        x2 = x2 * apow + c2 * adiv;
    }
};

// The per-leaf terms of the SolarL2 / LOOL2 / SatL2 split scores
// (crates/cb-compute/src/score.rs:266-330, after score_calcers.cuh), over a
// leaf's weighted der sum and weight; score = the sum of the terms, no l2.
// score_fn: 2 = SolarL2, 5 = LOOL2, 6 = SatL2.
__device__ __forceinline__ double gpu_score_term(int score_fn, double sum, double weight) {
    const double nss = __dmul_rn(-sum, sum);
    if (score_fn == 2)
        return weight > 1e-20
                   ? __ddiv_rn(__dmul_rn(nss, __dadd_rn(1.0, __dmul_rn(2.0, log(__dadd_rn(weight, 1.0))))), weight)
                   : 0.0;
    double adjust;
    if (score_fn == 5) {
        adjust = weight > 1.0 ? __ddiv_rn(weight, __dsub_rn(weight, 1.0)) : 0.0;
        adjust = __dmul_rn(adjust, adjust);
    } else {
        adjust = weight > 2.0 ? __ddiv_rn(__dmul_rn(weight, __dsub_rn(weight, 2.0)),
                                          __dadd_rn(__dsub_rn(__dmul_rn(weight, weight), __dmul_rn(3.0, weight)), 1.0))
                              : 0.0;
    }
    return weight > 0.0 ? __ddiv_rn(__dmul_rn(adjust, nss), weight) : 0.0;
}

// (GenRand() >> 11) * (1 / (2^53 - 1)) (rng.rs:256-259).
__device__ __forceinline__ double real1(Rng64& r) {
    return __dmul_rn((double)(r.gen() >> 11), 1.0 / 9007199254740991.0);
}

// FastLog2f / FastLogf (fast_approx.rs:154-188): every f32 operation rounded
// separately, in the reference's evaluation order.
__device__ __forceinline__ float fast_log2f(float v) {
    uint32_t vx = __float_as_uint(v);
    float mx = __uint_as_float((vx & 0x007FFFFFu) | 0x3f000000u);
    float y = __fmul_rn(__uint2float_rn(vx), 1.1920928955078125e-7f);
    float t = __fsub_rn(y, 124.22551499f);
    t = __fsub_rn(t, __fmul_rn(1.498030302f, mx));
    return __fsub_rn(t, __fdiv_rn(1.72587999f, __fadd_rn(0.3520887068f, mx)));
}
__device__ __forceinline__ float fast_logf(float v) { return __fmul_rn(0.69314718f, fast_log2f(v)); }

// Bayesian bootstrap weight (bootstrap.rs:141-150): powf(-FastLogf((f32)u + 1e-100f), T).
// The 1e-100 literal is +0.0 in f32.  T == 1 returns w exactly (pow(x, 1) == x).
__device__ __forceinline__ double bayesian_weight(double u, float temp) {
    float w = -fast_logf(__fadd_rn(__double2float_rn(u), 0.0f));
    if (temp == 1.0f) return (double)w;
    return (double)__double2float_rn(pow((double)w, (double)temp));
}

// Device error word bits (read by the host after every tree).
enum : uint32_t {
    kErrNone = 0,
    kErrNoCandidate = 1u << 0,   // no split candidate at some level
    kErrBinRange = 1u << 1,      // a bin index >= n_bins was seen
    kErrOverflow = 1u << 2,      // fixed-point range exceeded
    kErrLeafRange = 1u << 3,     // leaf id out of range
    kErrChunkCap = 1u << 4,      // the histogram work list exceeded its buffer
};

}  // namespace cbgpu
