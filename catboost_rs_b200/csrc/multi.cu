// multi.cu -- the multi-output (MultiClass softmax) arm of the oblivious-tree
// grow, behind the seam's FamilyTreeArgs::MultiOutput
// (crates/cb-compute/src/runtime.rs:935-948): the approximant has K
// dimensions, one tree serves all of them, and each leaf carries a K-vector.
//
// The reference's device session declines every multi-output fit
// (crates/cb-backend/src/gpu_runtime/session.rs:1401-1467); its CPU branch
// (crates/cb-train/src/boosting.rs:7400-8930 at approx_dimension K) is what
// this arm reproduces, one CUDA stream per session:
//
//   per tree   mc_der_kernel       pending leaf update, softmax, weighted der1
//              bootstrap           (the scalar path's kernels)
//              mc_max / mc_pack    K + 1 score channels as int64 fixed point
//   per level  mc_hist_kernel      (feature, channel, row chunk) blocks, the
//                                  level's leaves x bins table in shared memory
//              mc_prefix_kernel    exact int64 bin prefix sums
//              mc_score_kernel     every (feature, border) candidate, multi-dim
//                                  Cosine / L2 in dimension-then-leaf order
//              mc_argmax_kernel    strict first-wins over (feature, border)
//              mc_route_kernel     leaf |= (bin > border) << level (one-hot
//                                  categorical features: bin == value)
//   per tree   mc_leafsum_kernel   int64 per-leaf sums of w*der1 and w*der2
//              mc_newton_kernel    the trace-regularised symmetric Newton
//                                  solve per leaf (Cholesky), x lr
//
// Histogram and leaf sums are exact integer sums of values rounded once to a
// power-of-two fixed point, so results do not depend on the launch geometry or
// atomic order; against the CPU's sequential f64 sums the difference is the
// rounding of each value (2^-40 of the largest value or finer).  The host keeps
// the main TFastRng64 stream replica with cb-train's draw accounting, as the
// scalar session does.  One GPU per session; MVS and document sharding decline.
//
// The same session serves the grouped (ranking) losses QueryRMSE and PairLogit
// at K = 1 (cbgpu_rank_begin_raw): rk_der_kernel computes the grouped ders one
// thread per group in the reference's order, the histogram weight channel is
// PairLogit's pairwise weights, and rk_leafsum / rk_newton give the Newton
// leaves and the PairLogit leaf centring.
#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <vector>

#include "../../include/cbgpu.h"
#include "kernels.cuh"

using namespace cbgpu;

namespace cbgpu {
int record_error(int code, const char* msg);  // session.cu: sets cbgpu_last_error()
}

namespace {

constexpr int kMcMaxK = 16;
constexpr int kMcMaxDepth = 10;
constexpr int kMcChunk = 16384;                  // rows per histogram block
constexpr size_t kMcSmemTable = 96 * 1024;       // shared table budget per block
constexpr int kMcThreads = 256;

enum : uint32_t { kMcErrNoCandidate = 1u << 0, kMcErrNonFinite = 1u << 1, kMcErrLeafRange = 1u << 2 };

int mfail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    return cbgpu::record_error(code, buf);
}

#define MCU(call)                                                                             \
    do {                                                                                      \
        cudaError_t _e = (call);                                                              \
        if (_e != cudaSuccess)                                                                \
            return mfail(_e == cudaErrorMemoryAllocation ? CBGPU_ERR_OOM : CBGPU_ERR_CUDA,    \
                         "%s failed: %s", #call, cudaGetErrorString(_e));                     \
    } while (0)

// Host replica of the main TFastRng64 stream with cb-train's call counter.
struct McRng {
    Rng64 r{};
    uint64_t calls = 0;
    uint64_t gen() {
        ++calls;
        return r.gen();
    }
    double real1() { return (double)(gen() >> 11) * (1.0 / 9007199254740991.0); }
    void advance(uint64_t d) {
        r.advance(d);
        calls += d;
    }
    double std_normal() {  // normal.rs (Marsaglia polar)
        for (;;) {
            double x = real1() * 2.0 - 1.0;
            double y = real1() * 2.0 - 1.0;
            double rr = x * x + y * y;
            if (!(rr > 1.0 || rr <= 0.0)) return x * std::sqrt(-2.0 * std::log(rr) / rr);
        }
    }
};

struct McSplit {
    int32_t feature, bin;
};

// Per-tree device state read back once per tree.
struct McState {
    McSplit split[kMcMaxDepth];
    uint32_t err;
    uint32_t pad;
    unsigned long long maxbits;  // bit pattern of max |score channel| (a non-negative double)
    int32_t hist_shift;          // score channels are llrint(v * 2^hist_shift)
};

// ---- kernels ---------------------------------------------------------------

// Exclusive block-wide scan of one u32 per thread (blockDim a multiple of 32).
__device__ __forceinline__ uint32_t block_excl_scan_u32(uint32_t v, uint32_t* sm) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    uint32_t inc = v;
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
    }
    if (lane == 31) sm[w] = inc;
    __syncthreads();
    if (w == 0) {
        uint32_t x = lane < nw ? sm[lane] : 0u;
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += t;
        }
        sm[lane] = x;
    }
    __syncthreads();
    const uint32_t off = w ? sm[w - 1] : 0u;
    __syncthreads();
    return off + inc - v;
}

// Softmax probabilities of one object (loss.rs:424-455): max-subtracted exp,
// sequential sum, division.
__device__ __forceinline__ void mc_softmax(const double* __restrict__ approx, int64_t n, int64_t i, int K,
                                           double* p) {
    double mx = -INFINITY;
    for (int d = 0; d < K; ++d) {
        const double a = approx[(size_t)d * n + i];
        p[d] = a;
        if (a > mx) mx = a;
    }
    double s = 0.0;
    for (int d = 0; d < K; ++d) {
        p[d] = exp(__dsub_rn(p[d], mx));
        s = __dadd_rn(s, p[d]);
    }
    for (int d = 0; d < K; ++d) p[d] = __ddiv_rn(p[d], s);
}

// sigmoid (loss.rs:54-57): 1 - 1 / (1 + exp(a)).
__device__ __forceinline__ double mc_sigmoid(double a) {
    return __dsub_rn(1.0, __ddiv_rn(1.0, __dadd_rn(1.0, exp(a))));
}

// approx += lr * leaf (the previous tree, when pending); then the weighted der1
// per dimension: softmax wd1[d] = ([d == y] - p[d]) * w; diagonal (loss.rs:501-560)
// wd1[d] = (t_d - sigmoid(a_d)) * w with t_d = tmat[d * n + i], or [d == y]
// without a label matrix (MultiClassOneVsAll).
__global__ void mc_der_kernel(int64_t n, int K, double* __restrict__ approx, const int32_t* __restrict__ target,
                              const double* __restrict__ weight, const uint16_t* __restrict__ leaf,
                              const double* __restrict__ lrv, int L, int pending, int diag,
                              const double* __restrict__ tmat, double* __restrict__ wd1, McState* __restrict__ ms) {
    double p[kMcMaxK];
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        if (pending) {
            const int q = leaf[i];
            for (int d = 0; d < K; ++d)
                approx[(size_t)d * n + i] = __dadd_rn(approx[(size_t)d * n + i], lrv[(size_t)d * L + q]);
        }
        const double w = weight ? weight[i] : 1.0;
        bool finite = true;
        if (diag == 2) {
            // rmse_with_uncertainty_ders (loss.rs:680-720): [w diff, w (diff^2 prec - 1)]
            const double diff = __dsub_rn(tmat[i], approx[i]);
            const double prec = exp(__dmul_rn(-2.0, approx[(size_t)n + i]));
            const double dsp = __dmul_rn(__dmul_rn(diff, diff), prec);
            const double v0 = __dmul_rn(w, diff), v1 = __dmul_rn(w, __dsub_rn(dsp, 1.0));
            wd1[i] = v0;
            wd1[(size_t)n + i] = v1;
            if (!(isfinite(v0) && isfinite(v1))) atomicOr(&ms->err, kMcErrNonFinite);
            continue;
        }
        if (diag) {
            const int y = tmat ? -1 : target[i];
            for (int d = 0; d < K; ++d) {
                const double t = tmat ? tmat[(size_t)d * n + i] : (d == y ? 1.0 : 0.0);
                const double v = __dmul_rn(__dsub_rn(t, mc_sigmoid(approx[(size_t)d * n + i])), w);
                finite &= isfinite(v);
                wd1[(size_t)d * n + i] = v;
            }
            if (!finite) atomicOr(&ms->err, kMcErrNonFinite);
            continue;
        }
        mc_softmax(approx, n, i, K, p);
        const int y = target[i];
        for (int d = 0; d < K; ++d) {
            double d1 = -p[d];
            if (d == y) d1 = __dadd_rn(d1, 1.0);
            const double v = __dmul_rn(d1, w);
            finite &= isfinite(v);
            wd1[(size_t)d * n + i] = v;
        }
        if (!finite) atomicOr(&ms->err, kMcErrNonFinite);
    }
}

// score channels: c < K: wd1[c] * s, c == K: w * s (s = the bootstrap
// multiplier; boosting.rs:7700-7732).  s_mode 0: 1, 1: f32 device sample,
// 2: f64 host sample.
__device__ __forceinline__ double mc_channel(int c, int K, int64_t n, int64_t i, const double* wd1,
                                             const double* weight, int s_mode, const float* sw32,
                                             const double* sw64) {
    const double s = s_mode == 1 ? (double)sw32[i] : (s_mode == 2 ? sw64[i] : 1.0);
    const double v = c < K ? wd1[(size_t)c * n + i] : (weight ? weight[i] : 1.0);
    return __dmul_rn(v, s);
}

__global__ void mc_max_kernel(int64_t n, int K, const double* __restrict__ wd1, const double* __restrict__ weight,
                              int s_mode, const float* __restrict__ sw32, const double* __restrict__ sw64,
                              McState* __restrict__ ms) {
    double mx = 0.0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        for (int c = 0; c <= K; ++c) mx = fmax(mx, fabs(mc_channel(c, K, n, i, wd1, weight, s_mode, sw32, sw64)));
    for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0 && mx > 0.0) atomicMax(&ms->maxbits, (unsigned long long)__double_as_longlong(mx));
}

// hist_shift: max |v| * 2^shift * n < 2^62, so no int64 sum over n rows overflows.
__global__ void mc_shift_kernel(int64_t n, McState* ms) {
    const double mx = __longlong_as_double((long long)ms->maxbits);
    int e = 0;
    if (mx > 0.0) frexp(mx, &e);  // mx < 2^e
    int t = 0;
    while (t < 62 && (1ll << t) < n) ++t;  // n <= 2^t
    int sh = 61 - e - t;
    if (sh > 1000) sh = 1000;
    ms->hist_shift = sh;
}

__global__ void mc_pack_kernel(int64_t n, int K, const double* __restrict__ wd1, const double* __restrict__ weight,
                               int s_mode, const float* __restrict__ sw32, const double* __restrict__ sw64,
                               const McState* __restrict__ ms, long long* __restrict__ q) {
    const int sh = ms->hist_shift;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        for (int c = 0; c <= K; ++c)
            q[(size_t)c * n + i] = llrint(ldexp(mc_channel(c, K, n, i, wd1, weight, s_mode, sw32, sw64), sh));
}

// ---- histograms over leaf-sorted row lists (every mode but the pairwise
// scorers): the score channels are packed in pairs at the scalar path's
// fixed point (max |v| * 2^shift < 2^kPackBits, one shift for all channels),
// each pair is histogrammed by the scalar path's kernel for the built child
// of every parent only, the siblings are derived by subtraction, and the
// level table is laid out as hist[leaf][F][NB][C] for the scorers.

__global__ void mc_shift33_kernel(McState* ms) {
    ms->hist_shift = fixed_shift(__longlong_as_double((long long)ms->maxbits), kPackBits);
}

// qp[p][i] = the (lo, hi) parts of channels 2p and 2p + 1 of row i (pack_gh's split).
__global__ void mc_pack2_kernel(int64_t n, int K, int P, const double* __restrict__ wd1,
                                const double* __restrict__ weight, int s_mode, const float* __restrict__ sw32,
                                const double* __restrict__ sw64, const McState* __restrict__ ms,
                                uint4* __restrict__ qp) {
    const int sh = ms->hist_shift;
    const int C = K + 1;
    const long long mask = (1ll << kPackSplit) - 1;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        for (int p = 0; p < P; ++p) {
            const long long v0 = llrint(ldexp(mc_channel(2 * p, K, n, i, wd1, weight, s_mode, sw32, sw64), sh));
            const long long v1 =
                2 * p + 1 < C ? llrint(ldexp(mc_channel(2 * p + 1, K, n, i, wd1, weight, s_mode, sw32, sw64), sh))
                              : 0ll;
            qp[(size_t)p * n + i] = make_uint4((uint32_t)(v0 & mask), (uint32_t)(int32_t)(v0 >> kPackSplit),
                                               (uint32_t)(v1 & mask), (uint32_t)(int32_t)(v1 >> kPackSplit));
        }
}

// hist[q][f][b][c] = cur[c / 2][f][q][b][c % 2] (pair tables `pair_stride` words apart).
__global__ void mc_gather_kernel(int Q, int F, int NB, int C, const unsigned long long* __restrict__ cur,
                                 size_t pair_stride, unsigned long long* __restrict__ hist) {
    const int64_t total = (int64_t)Q * F * NB * C;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < total; k += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(k % C);
        int64_t t = k / C;
        const int b = (int)(t % NB);
        t /= NB;
        const int f = (int)(t % F);
        const int q = (int)(t / F);
        hist[k] = cur[(size_t)(c >> 1) * pair_stride + (((size_t)f * Q + q) * NB + b) * 2 + (c & 1)];
    }
}

// The next level's build side of each leaf q: the winner's child with no more
// weight (channel K).  Float split: TRUE = bins above the border; one-hot:
// TRUE = the value's own bin, as routing sets the leaf bit.
__global__ void mc_side_kernel(int level, int F, int NB, int C, int K, int F0,
                               const unsigned long long* __restrict__ hist, McState* __restrict__ ms,
                               const TreeState* __restrict__ fts, uint8_t* __restrict__ small_side) {
    const McSplit sp = ms->split[level];
    const int Q = 1 << level;
    for (int q = threadIdx.x; q < Q; q += blockDim.x) {
        const unsigned long long* row = hist + ((size_t)q * F + sp.feature) * NB * C;
        const long long wt = (long long)row[(size_t)(NB - 1) * C + K];
        const long long wp = (long long)row[(size_t)sp.bin * C + K];
        long long tw;
        if (sp.feature >= F0) tw = wp - (sp.bin > 0 ? (long long)row[(size_t)(sp.bin - 1) * C + K] : 0ll);
        else tw = wt - wp;
        small_side[q] = true_child_built((unsigned long long)(wt - tw), (unsigned long long)tw);
    }
    if (threadIdx.x == 0 && fts->err) atomicOr(&ms->err, kMcErrLeafRange);  // a work list outgrew its buffer
}

// Level histogram: block (feature f, channel c, rows [r0, r0 + kMcChunk)) adds
// q[c][row] into cell (leaf, f, bin, c) of hist[leaves][F][NB][C].  The
// leaves x bins table sits in shared memory when it fits (smem > 0), each
// int64 cell as a (lo, hi) pair of 32-bit words added exactly (add_split64):
// 64-bit shared atomics run as compare-and-swap loops, several times slower.
__global__ void __launch_bounds__(kMcThreads)
mc_hist_kernel(int64_t n, int F, int NB, int C, int leaves, const uint8_t* __restrict__ bins_fm,
               const long long* __restrict__ q, const uint16_t* __restrict__ leaf,
               unsigned long long* __restrict__ hist, int use_smem) {
    extern __shared__ uint32_t tab32[];  // [cells] lo words, then [cells] hi words
    const int f = blockIdx.x, c = blockIdx.y;
    const int64_t r0 = (int64_t)blockIdx.z * kMcChunk;
    const int64_t r1 = r0 + kMcChunk < n ? r0 + kMcChunk : n;
    const int cells = leaves * NB;
    uint32_t* tlo = tab32;
    uint32_t* thi = tab32 + cells;
    if (use_smem) {
        for (int k = threadIdx.x; k < 2 * cells; k += blockDim.x) tab32[k] = 0u;
        __syncthreads();
    }
    const uint8_t* col = bins_fm + (size_t)f * (size_t)n;
    const long long* qc = q + (size_t)c * (size_t)n;
    for (int64_t i = r0 + threadIdx.x; i < r1; i += blockDim.x) {
        const int lf = leaf[i];
        const int b = col[i];
        if (lf >= leaves || b >= NB) continue;
        const long long v = qc[i];
        if (v == 0) continue;
        if (use_smem) add_split64(tlo + lf * NB + b, thi + lf * NB + b, v);
        else atomicAdd(&hist[(((size_t)lf * F + f) * NB + b) * C + c], (unsigned long long)v);
    }
    if (use_smem) {
        __syncthreads();
        for (int k = threadIdx.x; k < cells; k += blockDim.x) {
            const unsigned long long v = ((unsigned long long)thi[k] << 32) + tlo[k];
            if (v) {
                const int lf = k / NB, b = k - lf * NB;
                atomicAdd(&hist[(((size_t)lf * F + f) * NB + b) * C + c], v);
            }
        }
    }
}

// Inclusive prefix over bins of every (leaf, feature, channel) row, in place.
__global__ void mc_prefix_kernel(int leaves, int F, int NB, int C, unsigned long long* __restrict__ hist) {
    const int64_t rows = (int64_t)leaves * F * C;
    for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < rows; r += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(r % C);
        const int64_t lfq = r / C;  // leaf * F + f
        unsigned long long* row = hist + (size_t)lfq * NB * C + c;
        unsigned long long run = 0ull;
        for (int b = 0; b < NB; ++b) {
            run += row[(size_t)b * C];
            row[(size_t)b * C] = run;
        }
    }
}

// calc_average (leaf.rs:161-175)
__device__ __forceinline__ double mc_avg(double s, double w, double l2) {
    return w > 0.0 ? __ddiv_rn(s, __dadd_rn(w, l2)) : 0.0;
}

// Score of candidate (f, b) over the 2P children of this level's P leaves:
// multi_dim_split_score_into (score.rs:192-265), false children 0..P-1 then
// true children, dimension-then-leaf order.
// Features f >= F0 are one-hot categorical (scan_and_score_one_hot_bins_into,
// histogram.rs:1160-1290): candidate b is present[f - F0][b], its TRUE
// children the bin's cells (prefix(b) - prefix(b - 1)), its FALSE children the
// parent totals minus them.
// Block = 32 consecutive borders of one feature (lane = border).  The
// 2 K parents terms of each candidate are computed in pieces of 32 by the
// eight compute warps (warps 1-8) into a double-buffered shared table, while
// warp 0 adds the previous piece in order, one lane per candidate: each sum
// sees the CPU's terms in the CPU's sequence, and the terms' loads and
// divisions run in parallel instead of on one thread's dependent chain.
constexpr int kMsCompute = 8;   // compute warps
constexpr int kMsPiece = 32;    // terms per piece
__global__ void __launch_bounds__((kMsCompute + 1) * 32)
mc_score_kernel(int parents, int F, int NB, int K, const unsigned long long* __restrict__ pre,
                const int32_t* __restrict__ border_counts, const McState* __restrict__ ms, double l2, int score_fn,
                int F0, const uint8_t* __restrict__ present, double* __restrict__ scores) {
    __shared__ double tn[2][kMsPiece][32], td[2][kMsPiece][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int groups = (NB + 31) / 32;
    const int f = blockIdx.x / groups;
    const int b = (blockIdx.x % groups) * 32 + lane;
    if (f >= F) return;
    const int C = K + 1;
    const double inv = ldexp(1.0, -ms->hist_shift);
    const bool cat = f >= F0;
    const bool cosine = score_fn == CBGPU_SCORE_COSINE;
    const bool valid = b < NB && (cat ? present[(size_t)(f - F0) * NB + b] != 0
                                      : (b < border_counts[f] && b < NB - 1));
    const int T = 2 * K * parents;  // (dimension, side, leaf) terms, leaf fastest
    const int pieces = (T + kMsPiece - 1) / kMsPiece;
    // terms [t0, t0 + kMsPiece) of this lane's candidate into buffer buf
    auto compute = [&](int t0, int buf) {
        for (int j = warp - 1; j < kMsPiece; j += kMsCompute) {
            const int t = t0 + j;
            double vn = 0.0, vd = 0.0;
            if (t < T && valid) {
                const int d = t / (2 * parents), side = (t / parents) & 1, q = t % parents;
                const unsigned long long* row = pre + ((size_t)q * F + f) * NB * C;
                long long wp = (long long)__ldg(row + (size_t)b * C + K);
                const long long wt = (long long)__ldg(row + (size_t)(NB - 1) * C + K);
                long long sp = (long long)__ldg(row + (size_t)b * C + d);
                const long long stot = (long long)__ldg(row + (size_t)(NB - 1) * C + d);
                double w, sv;
                if (cat) {  // the bin's own cell: TRUE = cell, FALSE = total - cell
                    if (b > 0) {
                        wp -= (long long)__ldg(row + (size_t)(b - 1) * C + K);
                        sp -= (long long)__ldg(row + (size_t)(b - 1) * C + d);
                    }
                    w = __dmul_rn((double)(side ? wp : wt - wp), inv);
                    sv = __dmul_rn((double)(side ? sp : stot - sp), inv);
                } else {
                    w = __dmul_rn((double)(side ? wt - wp : wp), inv);
                    sv = __dmul_rn((double)(side ? stot - sp : sp), inv);
                }
                if (score_fn > 1) {  // SolarL2 / LOOL2 / SatL2: per-leaf terms, no l2
                    vn = gpu_score_term(score_fn, sv, w);
                } else {
                    const double avg = mc_avg(sv, w, l2);
                    vn = __dmul_rn(avg, sv);
                    if (cosine) vd = __dmul_rn(__dmul_rn(avg, avg), w);
                }
            }
            tn[buf][j][lane] = vn;
            td[buf][j][lane] = vd;
        }
    };
    double num = 0.0, den = 1e-100;
    if (warp > 0) compute(0, 0);
    __syncthreads();
    for (int pc = 0; pc < pieces; ++pc) {
        const int buf = pc & 1;
        if (warp > 0) {
            if (pc + 1 < pieces) compute((pc + 1) * kMsPiece, buf ^ 1);
        } else {
            const int cnt = T - pc * kMsPiece < kMsPiece ? T - pc * kMsPiece : kMsPiece;
            if (cnt == kMsPiece) {
#pragma unroll 8
                for (int j = 0; j < kMsPiece; ++j) {
                    num = __dadd_rn(num, tn[buf][j][lane]);
                    if (cosine) den = __dadd_rn(den, td[buf][j][lane]);
                }
            } else {
                for (int j = 0; j < cnt; ++j) {
                    num = __dadd_rn(num, tn[buf][j][lane]);
                    if (cosine) den = __dadd_rn(den, td[buf][j][lane]);
                }
            }
        }
        __syncthreads();
    }
    if (warp == 0 && b < NB)
        scores[(size_t)f * NB + b] = !valid ? -INFINITY : (!cosine ? num : __ddiv_rn(num, sqrt(den)));
}

// Strict first-wins argmax over (feature, border) (tree.rs:355-366): the
// highest score, the lowest candidate index among equal scores.
__global__ void __launch_bounds__(1024) mc_argmax_kernel(int64_t cand, int NB, const double* __restrict__ scores,
                                                         int level, McState* __restrict__ ms) {
    __shared__ double s_best[32];
    __shared__ long long s_idx[32];
    double best = -INFINITY;
    long long idx = -1;
    for (int64_t k = threadIdx.x; k < cand; k += blockDim.x) {
        const double s = scores[k];
        if (s > best) {  // k ascends per thread: the first maximum stays
            best = s;
            idx = k;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const double ob = __shfl_xor_sync(0xffffffffu, best, o);
        const long long oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (oi >= 0 && (idx < 0 || ob > best || (ob == best && oi < idx))) {
            best = ob;
            idx = oi;
        }
    }
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        s_best[w] = best;
        s_idx[w] = idx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < (int)(blockDim.x >> 5); ++k) {
            const double ob = s_best[k];
            const long long oi = s_idx[k];
            if (oi >= 0 && (idx < 0 || ob > best || (ob == best && oi < idx))) {
                best = ob;
                idx = oi;
            }
        }
        if (idx < 0) {
            ms->err |= kMcErrNoCandidate;
            ms->split[level] = McSplit{0, 0};
        } else {
            ms->split[level] = McSplit{(int32_t)(idx / NB), (int32_t)(idx % NB)};
        }
    }
}

// advance_leaf_only (tree.rs:1005-1016): the level's split is leaf bit `level`.
__global__ void mc_route_kernel(int64_t n, int level, const uint8_t* __restrict__ bins_fm, int F0,
                                const McState* __restrict__ ms, uint16_t* __restrict__ leaf) {
    const McSplit sp = ms->split[level];
    const uint8_t* col = bins_fm + (size_t)sp.feature * (size_t)n;
    const bool cat = sp.feature >= F0;  // one-hot: passes on bin == value (tree.rs:1005-1016)
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        if (cat ? (int)col[i] == sp.bin : (int)col[i] > sp.bin) leaf[i] = (uint16_t)(leaf[i] | (1u << level));
}

// Per-leaf sums of w*der1[d] (K) and w*der2 packed (pk) over ALL rows
// (compute_softmax_leaf_deltas, boosting.rs:2610-2700), int64 fixed point at
// 2^leaf_shift; table[L][K + pk] in shared memory when it fits.  Diagonal
// losses fill only the first K der2 slots: w * (-p_d (1 - p_d)) per dimension
// (the per-dimension scalar sums of boosting.rs:8323-8420).
__global__ void __launch_bounds__(kMcThreads)
mc_leafsum_kernel(int64_t n, int K, int L, const double* __restrict__ approx, const double* __restrict__ wd1,
                  const double* __restrict__ weight, const uint16_t* __restrict__ leaf, int leaf_shift_in, int diag,
                  const double* __restrict__ tmat, unsigned long long* __restrict__ sums, int use_smem,
                  McState* __restrict__ ms) {
    // RMSEWithUncertainty's ders are unbounded: its sums take the tree's score
    // shift less 2 (|w der2| <= 2 |w der1_1| + 2 w <= 4 max channel)
    const int leaf_shift = diag == 2 ? ms->hist_shift - 2 : leaf_shift_in;
    // shared table: the (lo, hi) 32-bit words of each int64 cell, lo words
    // first (add_split64; 64-bit shared atomics would be compare-and-swap loops)
    extern __shared__ unsigned long long ltab[];
    const int pk = K * (K + 1) / 2, W = K + pk;
    uint32_t* tlo = (uint32_t*)ltab;
    uint32_t* thi = tlo + (size_t)L * W;
    if (use_smem) {
        for (int k = threadIdx.x; k < L * W; k += blockDim.x) ltab[k] = 0ull;
        __syncthreads();
    }
    auto add = [&](size_t c, double x) {
        const long long v = llrint(ldexp(x, leaf_shift));
        if (use_smem) add_split64(tlo + c, thi + c, v);
        else atomicAdd(&sums[c], (unsigned long long)v);
    };
    double p[kMcMaxK];
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int q = leaf[i];
        if (q >= L) {
            atomicOr(&ms->err, kMcErrLeafRange);
            continue;
        }
        const size_t cell = (size_t)q * W;
        for (int d = 0; d < K; ++d) add(cell + d, wd1[(size_t)d * n + i]);
        const double w = weight ? weight[i] : 1.0;
        if (diag == 2) {
            const double diff = __dsub_rn(tmat[i], approx[i]);
            const double prec = exp(__dmul_rn(-2.0, approx[(size_t)n + i]));
            const double dsp = __dmul_rn(__dmul_rn(diff, diff), prec);
            add(cell + K, -w);
            add(cell + K + 1, __dmul_rn(__dmul_rn(-2.0, w), dsp));
            continue;
        }
        if (diag) {
            for (int d = 0; d < K; ++d) {
                const double pd = mc_sigmoid(approx[(size_t)d * n + i]);
                add(cell + K + d, __dmul_rn(__dmul_rn(-pd, __dsub_rn(1.0, pd)), w));
            }
            continue;
        }
        mc_softmax(approx, n, i, K, p);
        int j = 0;
        for (int dy = 0; dy < K; ++dy) {
            add(cell + K + j++, __dmul_rn(__dmul_rn(p[dy], __dsub_rn(p[dy], 1.0)), w));
            for (int dx = dy + 1; dx < K; ++dx) add(cell + K + j++, __dmul_rn(__dmul_rn(p[dy], p[dx]), w));
        }
    }
    if (use_smem) {
        __syncthreads();
        for (int k = threadIdx.x; k < L * W; k += blockDim.x) {
            const unsigned long long v = ((unsigned long long)thi[k] << 32) | tlo[k];
            if (v) atomicAdd(&sums[k], v);
        }
    }
}

// solve_symmetric_newton (leaf.rs:281-340) for leaf `threadIdx.x`: Rust
// f32::max semantics for the trace regulariser, Cholesky (leaf.rs:360-420),
// zeros on a non-positive pivot; delta x lr for the approximant.
// Diagonal losses: newton_leaf_delta per dimension (leaf.rs:196-232),
// s1 / (-s2 + l2), 0 on a zero denominator.
__global__ void mc_newton_kernel(int K, int L, const unsigned long long* __restrict__ sums, int leaf_shift_in,
                                 double l2, double lr, int diag, const McState* __restrict__ ms,
                                 double* __restrict__ leaf_raw, double* __restrict__ leaf_lrv) {
    const int q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= L) return;
    const int leaf_shift = diag == 2 ? ms->hist_shift - 2 : leaf_shift_in;
    const int pk = K * (K + 1) / 2, W = K + pk;
    const double inv = ldexp(1.0, -leaf_shift);
    if (diag) {
        const unsigned long long* s = sums + (size_t)q * W;
        for (int d = 0; d < K; ++d) {
            const double s1 = __dmul_rn((double)(long long)s[d], inv);
            const double s2 = __dmul_rn((double)(long long)s[K + d], inv);
            const double den = __dadd_rn(-s2, l2);
            const double delta = den == 0.0 ? 0.0 : __ddiv_rn(s1, den);
            leaf_raw[(size_t)q * K + d] = delta;
            leaf_lrv[(size_t)d * L + q] = __dmul_rn(delta, lr);
        }
        return;
    }
    double H[kMcMaxK * kMcMaxK], Lm[kMcMaxK * kMcMaxK], y[kMcMaxK], x[kMcMaxK], g[kMcMaxK];
    const unsigned long long* s = sums + (size_t)q * W;
    for (int d = 0; d < K; ++d) g[d] = __dmul_rn((double)(long long)s[d], inv);
    int j = 0;
    for (int a = 0; a < K; ++a)
        for (int b = a; b < K; ++b) {
            const double v = __dmul_rn((double)(long long)s[K + j++], inv);
            H[a * K + b] = v;
            H[b * K + a] = v;
        }
    float mt = (float)l2;
    for (int d = 0; d < K; ++d) {
        const float t = (float)(-H[d * K + d]);
        if (isnan(mt) || (!isnan(t) && t > mt)) mt = t;
    }
    float l2f = (float)l2, mtl = __fmul_rn(mt, FLT_EPSILON);
    const float adjf = isnan(l2f) ? mtl : (isnan(mtl) ? l2f : (l2f > mtl ? l2f : mtl));
    const double adj = (double)adjf;
    for (int d = 0; d < K; ++d) H[d * K + d] = __dsub_rn(H[d * K + d], adj);
    for (int k = 0; k < K * K; ++k) H[k] = -H[k];
    for (int d = 0; d < K; ++d) g[d] = -g[d];
    bool ok = true;
    for (int k = 0; k < K * K; ++k) Lm[k] = 0.0;
    for (int i = 0; i < K && ok; ++i)
        for (int jj = 0; jj <= i && ok; ++jj) {
            double sum = H[i * K + jj];
            for (int p = 0; p < jj; ++p) sum = __dsub_rn(sum, __dmul_rn(Lm[i * K + p], Lm[jj * K + p]));
            if (i == jj) {
                if (sum <= 0.0) ok = false;
                else Lm[i * K + jj] = sqrt(sum);
            } else {
                const double ljj = Lm[jj * K + jj];
                if (ljj == 0.0) ok = false;
                else Lm[i * K + jj] = __ddiv_rn(sum, ljj);
            }
        }
    for (int i = 0; i < K && ok; ++i) {
        double sum = g[i];
        for (int p = 0; p < i; ++p) sum = __dsub_rn(sum, __dmul_rn(Lm[i * K + p], y[p]));
        if (Lm[i * K + i] == 0.0) ok = false;
        else y[i] = __ddiv_rn(sum, Lm[i * K + i]);
    }
    for (int i = K - 1; i >= 0 && ok; --i) {
        double sum = y[i];
        for (int p = i + 1; p < K; ++p) sum = __dsub_rn(sum, __dmul_rn(Lm[p * K + i], x[p]));
        if (Lm[i * K + i] == 0.0) ok = false;
        else x[i] = __ddiv_rn(sum, Lm[i * K + i]);
    }
    for (int d = 0; d < K; ++d) {
        const double delta = ok ? -x[d] : 0.0;
        leaf_raw[(size_t)q * K + d] = delta;                 // leaf-major, raw (the seam's layout)
        leaf_lrv[(size_t)d * L + q] = __dmul_rn(delta, lr);  // dim-major, x lr (normalize_leaf_values)
    }
}

__global__ void mc_fill2_kernel(int64_t n, double* __restrict__ approx, double b0, double b1) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        approx[i] = b0;
        approx[(size_t)n + i] = b1;
    }
}

__global__ void mc_leaf_export_kernel(int64_t n, const uint16_t* __restrict__ leaf, void* out, int bytes) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t v = leaf[i];
        if (bytes == 1) ((uint8_t*)out)[i] = (uint8_t)v;
        else if (bytes == 2) ((uint16_t*)out)[i] = (uint16_t)v;
        else ((uint32_t*)out)[i] = v;
    }
}

__global__ void mc_apply_pending_kernel(int64_t n, int K, int L, double* __restrict__ approx,
                                        const uint16_t* __restrict__ leaf, const double* __restrict__ lrv) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int q = leaf[i];
        for (int d = 0; d < K; ++d)
            approx[(size_t)d * n + i] = __dadd_rn(approx[(size_t)d * n + i], lrv[(size_t)d * L + q]);
    }
}

// ---- ranking mode (grouped losses, K = 1) ----------------------------------

enum : int { kRankQueryRmse = 0, kRankPairLogit = 1, kRankPairLogitPairwise = 2, kRankQuerySoftMax = 3,
             kRankLambdaMart = 4, kRankYetiRank = 5, kRankStochasticRank = 6, kRankYetiRankPairwise = 7 };

// Per-loss parameters of rk_der_kernel.  LambdaMart's position denominators
// log2(2 + pos) (as log(x) * log2(e), ranking_der.rs:456-467) and each group's
// ideal DCG (lambdamart_ideal_ndcg, ranking_der.rs:616-628) are computed on
// the host once the target is known, so they round exactly as the CPU's.
struct RkLossParams {
    double sm_lambda, sm_beta;
    double lm_sigma;
    int64_t lm_top;
    int32_t lm_norm;
    const double* lm_den;    // [max group size]
    const double* lm_ideal;  // [n_groups]
    int32_t* lm_order;       // [n] group-local sort scratch
    int32_t lm_no_op;        // metric MRR / ERR / MAP: zero ders (ranking_der.rs:574-581)
};
constexpr double kPairwisePrior = 0.1;  // PairwiseNonDiagReg default (oblivious_tree_options.cpp:16)

// Grouped derivatives (calc_ders_for_queries, crates/cb-compute/src/
// ranking_der.rs:139-440), one thread per group in the reference's order, so
// every f64 sum rounds as the CPU's does:
//  QueryRMSE  queryAvrg = sum((t - a) * w) / sum(w); der1 = ((t - a) - queryAvrg) * w,
//             der2 = -1 * w;
//  PairLogit  doc-ascending winners, competitor order: p = e^l / (e^l + e^w),
//             winner += p, loser -= p (der2: p * (p - 1)), pair weight 1.
//  QuerySoftMax (ranking_der.rs:247-320, loss.rs:608-619): max approx and
//             sumWT = sum(w t) over w > 0 (t > 0 terms), ew = e^(beta (a - max)) w,
//             p = ew / sum(ew), der1 = beta (-sumWT p + w t),
//             der2 = beta sumWT (beta p (p - 1) - lambda); 0 when sumWT <= 0 or w <= 0.
//  LambdaMart (lambdamart_group_der, ranking_der.rs:482-606; loss.rs:673-679):
//             stable sort by approx descending, then every ordered pair with
//             t1 > t2 (second position bounded by top) scatters the sigmoid
//             lambda with delta = (t1 - t2) |1/den1 - 1/den2| / idealDCG
//             (/ (0.01 + |a1 - a2|) under norm); norm rescales the group by
//             log2(1 + sumDer1) / sumDer1.  Object weights do not enter.
// The ders carry the weights already (boosting.rs:7453-7490).
__global__ void rk_der_kernel(int n_groups, int mode, const int64_t* __restrict__ goff,
                              const int64_t* __restrict__ cstart, const int64_t* __restrict__ closer,
                              const double* __restrict__ approx, const double* __restrict__ target,
                              const double* __restrict__ weight, RkLossParams lp, double* __restrict__ d1,
                              double* __restrict__ d2, McState* __restrict__ ms) {
    const int g = blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= n_groups) return;
    const int64_t b = goff[g], e = goff[g + 1];
    const double sm_lambda = lp.sm_lambda, sm_beta = lp.sm_beta;
    bool finite = true;
    if (mode == kRankLambdaMart) {
        const int64_t cnt = e - b;
        for (int64_t i = b; i < e; ++i) {
            d1[i] = 0.0;
            d2[i] = 0.0;
        }
        // MRR / ERR / MAP: the reference's arms leave the ders at zero
        if (cnt > 1 && !lp.lm_no_op) {
            int32_t* ord = lp.lm_order + b;
            const double* ap = approx + b;
            const double* tg = target + b;
            for (int64_t k = 0; k < cnt; ++k) ord[k] = (int32_t)k;
            for (int64_t k = 1; k < cnt; ++k) {  // stable insertion sort, approx descending
                const int32_t key = ord[k];
                int64_t j = k - 1;
                while (j >= 0 && ap[ord[j]] < ap[key]) {
                    ord[j + 1] = ord[j];
                    --j;
                }
                ord[j + 1] = key;
            }
            const bool same = fabs(__dsub_rn(ap[ord[0]], ap[ord[cnt - 1]])) == 0.0;
            const int64_t top = (lp.lm_top == -1 || lp.lm_top > cnt) ? cnt : lp.lm_top;
            const double ideal = lp.lm_ideal[g], sigma = lp.lm_sigma;
            double sum_der1 = 0.0;
            for (int64_t fi = 0; fi < cnt; ++fi) {
                const int64_t bound = fi < top ? cnt : top;
                for (int64_t si = 0; si < bound; ++si) {
                    const double ft = tg[ord[fi]], st = tg[ord[si]];
                    if (ft <= st) continue;
                    const double adiff = __dsub_rn(ap[ord[fi]], ap[ord[si]]);
                    const double dnum = __dsub_rn(ft, st);
                    const double dden =
                        fabs(__dsub_rn(__ddiv_rn(1.0, lp.lm_den[fi]), __ddiv_rn(1.0, lp.lm_den[si])));
                    double delta = ideal != 0.0 ? __ddiv_rn(__dmul_rn(dnum, dden), ideal) : 0.0;
                    if (lp.lm_norm && !same) delta = __ddiv_rn(delta, __dadd_rn(0.01, fabs(adiff)));
                    const double sig = __ddiv_rn(1.0, __dadd_rn(1.0, exp(__dmul_rn(sigma, adiff))));
                    const double hess = __dmul_rn(__dmul_rn(sig, __dsub_rn(1.0, sig)),
                                                  __dmul_rn(__dmul_rn(sigma, sigma), delta));
                    const double anti = __dmul_rn(__dmul_rn(-sigma, delta), sig);
                    d1[b + ord[fi]] = __dadd_rn(d1[b + ord[fi]], anti);
                    d2[b + ord[fi]] = __dadd_rn(d2[b + ord[fi]], hess);
                    d1[b + ord[si]] = __dsub_rn(d1[b + ord[si]], anti);
                    d2[b + ord[si]] = __dadd_rn(d2[b + ord[si]], hess);
                    sum_der1 = __dsub_rn(sum_der1, __dmul_rn(2.0, anti));
                }
            }
            if (lp.lm_norm && sum_der1 > 0.0) {
                const double norma = __ddiv_rn(log2(__dadd_rn(1.0, sum_der1)), sum_der1);
                for (int64_t i = b; i < e; ++i) {
                    d1[i] = __dmul_rn(d1[i], norma);
                    d2[i] = __dmul_rn(d2[i], norma);
                }
            }
        }
        for (int64_t i = b; i < e; ++i) finite &= isfinite(d1[i]) && isfinite(d2[i]);
    } else if (mode == kRankQuerySoftMax) {
        double mx = -DBL_MAX, swt = 0.0;
        for (int64_t i = b; i < e; ++i) {
            const double w = weight ? weight[i] : 1.0;
            d1[i] = 0.0;
            d2[i] = 0.0;
            if (w > 0.0) {
                if (approx[i] > mx) mx = approx[i];
                if (target[i] > 0.0) swt = __dadd_rn(swt, __dmul_rn(w, target[i]));
            }
        }
        if (swt > 0.0) {
            double sum_exp = 0.0;
            for (int64_t i = b; i < e; ++i)
                sum_exp = __dadd_rn(sum_exp, __dmul_rn(exp(__dmul_rn(sm_beta, __dsub_rn(approx[i], mx))),
                                                       weight ? weight[i] : 1.0));
            for (int64_t i = b; i < e; ++i) {
                const double w = weight ? weight[i] : 1.0;
                if (!(w > 0.0 && sum_exp > 0.0)) continue;
                const double ew = __dmul_rn(exp(__dmul_rn(sm_beta, __dsub_rn(approx[i], mx))), w);
                const double p = __ddiv_rn(ew, sum_exp);
                d2[i] = __dmul_rn(__dmul_rn(sm_beta, swt),
                                  __dsub_rn(__dmul_rn(__dmul_rn(sm_beta, p), __dsub_rn(p, 1.0)), sm_lambda));
                d1[i] = __dmul_rn(sm_beta, __dadd_rn(__dmul_rn(-swt, p), __dmul_rn(w, target[i])));
            }
        }
        for (int64_t i = b; i < e; ++i) finite &= isfinite(d1[i]) && isfinite(d2[i]);
    } else if (mode == kRankQueryRmse) {
        double num = 0.0, den = 0.0;
        for (int64_t i = b; i < e; ++i) {
            const double w = weight ? weight[i] : 1.0;
            num = __dadd_rn(num, __dmul_rn(__dsub_rn(target[i], approx[i]), w));
        }
        for (int64_t i = b; i < e; ++i) den = __dadd_rn(den, weight ? weight[i] : 1.0);
        const double avg = den > 0.0 ? __ddiv_rn(num, den) : 0.0;
        for (int64_t i = b; i < e; ++i) {
            const double w = weight ? weight[i] : 1.0;
            d1[i] = __dmul_rn(__dsub_rn(__dsub_rn(target[i], approx[i]), avg), w);
            d2[i] = __dmul_rn(-1.0, w);
            finite &= isfinite(d1[i]);
        }
    } else {
        for (int64_t i = b; i < e; ++i) {
            d1[i] = 0.0;
            d2[i] = 0.0;
        }
        for (int64_t wi = b; wi < e; ++wi) {
            double wd = 0.0, wd2 = 0.0;
            const double aw = approx[wi];
            for (int64_t k = cstart[wi]; k < cstart[wi + 1]; ++k) {
                const int64_t li = closer[k];
                const double el = exp(approx[li]), ew = exp(aw);
                const double den = __dadd_rn(el, ew);
                const double p = den > 0.0 ? __ddiv_rn(el, den) : 0.5;
                const double t = __dmul_rn(__dmul_rn(1.0, p), __dsub_rn(p, 1.0));
                wd = __dadd_rn(wd, __dmul_rn(1.0, p));
                wd2 = __dadd_rn(wd2, t);
                d1[li] = __dsub_rn(d1[li], __dmul_rn(1.0, p));
                d2[li] = __dadd_rn(d2[li], t);
            }
            d1[wi] = __dadd_rn(d1[wi], wd);
            d2[wi] = __dadd_rn(d2[wi], wd2);
        }
        for (int64_t i = b; i < e; ++i) finite &= isfinite(d1[i]) && isfinite(d2[i]);
    }
    if (!finite) atomicOr(&ms->err, kMcErrNonFinite);
}

constexpr int kYetiWarps = 4;  // groups per 128-thread block (warp-per-group ranking kernels)

// PairLogit derivatives with one warp per group and one lane per document
// (the PairLogit arm of rk_der_kernel, ranking_der.rs:400-440, restated per
// document).  The sequential loop visits winners in ascending order and each
// winner's competitors in input order: a document's der1 / der2 receive, in
// that order, -w p (and w p (p - 1)) for each pair of weight w it loses to a winner at or
// below its own index -- its own self pairs included, as they come while its
// competitor list runs -- then its own list's sums, then the pairs it loses to
// later winners.  Its loser slots (lstart / lpair, ascending slot index) are
// that order, so each lane's sums round exactly as the loop's.
__global__ void __launch_bounds__(kYetiWarps * 32) rk_pairlogit_der_kernel(
    int n_groups, const int64_t* __restrict__ goff, const int64_t* __restrict__ cstart,
    const int64_t* __restrict__ closer, const int64_t* __restrict__ pwin, const int64_t* __restrict__ lstart,
    const int64_t* __restrict__ lpair, const double* __restrict__ pairw, const double* __restrict__ approx,
    double* __restrict__ ex, double* __restrict__ d1, double* __restrict__ d2, McState* __restrict__ ms) {
    const int lane = threadIdx.x & 31;
    const int gi = blockIdx.x * kYetiWarps + (threadIdx.x >> 5);
    if (gi >= n_groups) return;  // warp-uniform
    const int64_t b = goff[gi], e = goff[gi + 1];
    for (int64_t i = b + lane; i < e; i += 32) ex[i] = exp(approx[i]);
    __syncwarp();
    bool finite = true;
    for (int64_t x = b + lane; x < e; x += 32) {
        const double exx = ex[x];
        double a1 = 0.0, a2 = 0.0;
        auto lose = [&](int64_t k) {  // x loses pair k: p = e^x / (e^x + e^winner), weight w
            const double den = __dadd_rn(exx, ex[pwin[k]]);
            const double p = den > 0.0 ? __ddiv_rn(exx, den) : 0.5;
            const double wp = __dmul_rn(pairw[k], p);
            a1 = __dsub_rn(a1, wp);
            a2 = __dadd_rn(a2, __dmul_rn(wp, __dsub_rn(p, 1.0)));
        };
        int64_t j = lstart[x];
        const int64_t je = lstart[x + 1];
        for (; j < je && pwin[lpair[j]] <= x; ++j) lose(lpair[j]);
        double wd = 0.0, wd2 = 0.0;
        for (int64_t k = cstart[x]; k < cstart[x + 1]; ++k) {
            const double el = ex[closer[k]];
            const double den = __dadd_rn(el, exx);
            const double p = den > 0.0 ? __ddiv_rn(el, den) : 0.5;
            const double wp = __dmul_rn(pairw[k], p);
            wd = __dadd_rn(wd, wp);
            wd2 = __dadd_rn(wd2, __dmul_rn(wp, __dsub_rn(p, 1.0)));
        }
        a1 = __dadd_rn(a1, wd);
        a2 = __dadd_rn(a2, wd2);
        for (; j < je; ++j) lose(lpair[j]);
        d1[x] = a1;
        d2[x] = a2;
        finite &= isfinite(a1) && isfinite(a2);
    }
    if (__any_sync(0xffffffffu, !finite) && lane == 0) atomicOr(&ms->err, kMcErrNonFinite);
}

// Ranking-mode leaf sums: per leaf the sums of der1, der2 (unit leaf weights
// for Newton, boosting.rs:8345-8380) -- or, for Gradient leaves (count = 1),
// the row count -- and of the object weight (normalize_leaf_values' leaf
// weights, boosting.rs:8525-8540), sums[leaf][3], each accumulated in f64 in
// object order exactly as the CPU's `sum[leaf[i]] += v[i]` loop does, so the
// leaf values round as the CPU's (exact ties in the approximants survive,
// which LambdaMart's pair order depends on).  Through a stable counting sort
// by leaf: rows are counted per
// (tile, leaf), the counts scanned (leaf-major, then by tile), each tile
// writes its rows' three values to its leaves' runs in object order (warps in
// order, lanes in order within a warp), and one thread per leaf adds its run
// front to back -- the CPU's additions in the CPU's order, with each row
// read a bounded number of times.
constexpr int kLsTile = 4096;      // rows per tile (256 threads x 16)
constexpr int kLsThreads = 256;
constexpr int kLsMaxLeaves = 1024;

__global__ void __launch_bounds__(kLsThreads) rk_leafcount_kernel(int64_t n, int L, const uint16_t* __restrict__ leaf,
                                                                  uint32_t* __restrict__ counts,
                                                                  McState* __restrict__ ms) {
    __shared__ uint32_t c[kLsMaxLeaves];
    for (int q = threadIdx.x; q < L; q += blockDim.x) c[q] = 0u;
    __syncthreads();
    const int64_t r0 = (int64_t)blockIdx.x * kLsTile;
    bool bad = false;
    for (int64_t i = r0 + threadIdx.x; i < r0 + kLsTile && i < n; i += blockDim.x) {
        const uint32_t q = leaf[i];
        if (q < (uint32_t)L) atomicAdd(&c[q], 1u);
        else bad = true;
    }
    if (bad) atomicOr(&ms->err, kMcErrLeafRange);
    __syncthreads();
    for (int q = threadIdx.x; q < L; q += blockDim.x) counts[(size_t)blockIdx.x * L + q] = c[q];
}

// offs[tile][q] = start of tile's rows of leaf q in the leaf-major order;
// begin[q] / len[q] = leaf q's run.  One block; a thread per leaf walks the tiles.
__global__ void __launch_bounds__(kLsMaxLeaves) rk_leafscan_kernel(int tiles, int L, const uint32_t* __restrict__ counts,
                                                                   uint32_t* __restrict__ offs,
                                                                   uint32_t* __restrict__ begin,
                                                                   uint32_t* __restrict__ len) {
    __shared__ uint32_t s_scan[40];
    const int q = threadIdx.x;
    uint32_t tot = 0;
    if (q < L)
        for (int t = 0; t < tiles; ++t) tot += counts[(size_t)t * L + q];
    const uint32_t base = block_excl_scan_u32(q < L ? tot : 0u, s_scan);
    if (q < L) {
        begin[q] = base;
        len[q] = tot;
        uint32_t at = base;
        for (int t = 0; t < tiles; ++t) {
            offs[(size_t)t * L + q] = at;
            at += counts[(size_t)t * L + q];
        }
    }
}

__global__ void __launch_bounds__(kLsThreads) rk_leafscatter_kernel(int64_t n, int L, const uint16_t* __restrict__ leaf,
                                                                    const uint32_t* __restrict__ offs,
                                                                    const double* __restrict__ d1,
                                                                    const double* __restrict__ d2,
                                                                    const double* __restrict__ weight, int count,
                                                                    double* __restrict__ v1, double* __restrict__ v2,
                                                                    double* __restrict__ v3) {
    constexpr int kW = kLsThreads / 32, kRows = kLsTile / kW;  // each warp: kRows consecutive rows
    __shared__ uint32_t wc[kW][kLsMaxLeaves];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    for (int k = threadIdx.x; k < kW * L; k += blockDim.x) wc[k / L][k % L] = 0u;
    __syncthreads();
    const int64_t r0 = (int64_t)blockIdx.x * kLsTile + (int64_t)w * kRows;
    for (int j = 0; j < kRows; j += 32) {  // this warp's counts per leaf
        const int64_t i = r0 + j + lane;
        const uint32_t q = i < n ? leaf[i] : 0xffffu;
        const unsigned m = __match_any_sync(0xffffffffu, q);
        if (q < (uint32_t)L && (m & ((1u << lane) - 1u)) == 0u) wc[w][q] += (uint32_t)__popc(m);
        __syncwarp();
    }
    __syncthreads();
    for (int q = threadIdx.x; q < L; q += blockDim.x) {  // warp starts in row order
        uint32_t at = offs[(size_t)blockIdx.x * L + q];
        for (int k = 0; k < kW; ++k) {
            const uint32_t c = wc[k][q];
            wc[k][q] = at;
            at += c;
        }
    }
    __syncthreads();
    for (int j = 0; j < kRows; j += 32) {
        const int64_t i = r0 + j + lane;
        const uint32_t q = i < n ? leaf[i] : 0xffffu;
        const unsigned m = __match_any_sync(0xffffffffu, q);
        if (q < (uint32_t)L) {
            const uint32_t pos = wc[w][q] + (uint32_t)__popc(m & ((1u << lane) - 1u));
            v1[pos] = d1[i];
            v2[pos] = count ? 1.0 : __dmul_rn(d2[i], 1.0);
            v3[pos] = weight ? weight[i] : 1.0;
        }
        __syncwarp();
        if (q < (uint32_t)L && (m & ((1u << lane) - 1u)) == 0u) wc[w][q] += (uint32_t)__popc(m);
        __syncwarp();
    }
}

// One block per leaf: the run is staged into shared memory a chunk at a time
// (coalesced loads by every thread, the next chunk's loads in flight while
// thread 0 adds the current one in order).
constexpr int kLsRunChunk = 2048;

__global__ void __launch_bounds__(kLsThreads) rk_leafsum_runs_kernel(int L, const uint32_t* __restrict__ begin,
                                                                     const uint32_t* __restrict__ len,
                                                                     const double* __restrict__ v1,
                                                                     const double* __restrict__ v2,
                                                                     const double* __restrict__ v3,
                                                                     double* __restrict__ sums) {
    __shared__ double c1[2][kLsRunChunk / 2], c2[2][kLsRunChunk / 2], c3[2][kLsRunChunk / 2];
    constexpr int kC = kLsRunChunk / 2;  // values per stage
    const int q = blockIdx.x;
    const uint32_t b = begin[q], m = len[q];
    double s1 = 0.0, s2 = 0.0, s3 = 0.0;
    auto stage = [&](uint32_t at, int buf) {
        for (uint32_t k = threadIdx.x; k < kC && at + k < m; k += blockDim.x) {
            c1[buf][k] = v1[b + at + k];
            c2[buf][k] = v2[b + at + k];
            c3[buf][k] = v3[b + at + k];
        }
    };
    if (m > 0) stage(0, 0);
    __syncthreads();
    int buf = 0;
    for (uint32_t at = 0; at < m; at += kC) {
        if (at + kC < m) stage(at + kC, buf ^ 1);  // the next chunk, while thread 0 adds this one
        if (threadIdx.x == 0) {
            const uint32_t cnt = m - at < (uint32_t)kC ? m - at : (uint32_t)kC;
            uint32_t k = 0;
            // 8 values' loads issue ahead of their (ordered) additions
            for (; k + 8 <= cnt; k += 8) {
                double x1[8], x2[8], x3[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    x1[u] = c1[buf][k + u];
                    x2[u] = c2[buf][k + u];
                    x3[u] = c3[buf][k + u];
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    s1 = __dadd_rn(s1, x1[u]);
                    s2 = __dadd_rn(s2, x2[u]);
                    s3 = __dadd_rn(s3, x3[u]);
                }
            }
            for (; k < cnt; ++k) {
                s1 = __dadd_rn(s1, c1[buf][k]);
                s2 = __dadd_rn(s2, c2[buf][k]);
                s3 = __dadd_rn(s3, c3[buf][k]);
            }
        }
        __syncthreads();
        buf ^= 1;
    }
    if (threadIdx.x == 0) {
        sums[3 * q] = s1;
        sums[3 * q + 1] = s2;
        sums[3 * q + 2] = s3;
    }
}

// Newton leaves sum(der1) / (-sum(der2) + scaled_l2) (leaf.rs:223-232), or
// Gradient leaves sum(der1) / (count + scaled_l2) (calc_average,
// leaf.rs:161-194); the raw deltas go back through the seam; the approximant
// gets normalize_leaf_values' result (PairLogit: minus the document-weighted
// mean, boosting.rs:2844-2880) x lr.  One thread: L <= 1024 leaves.
__global__ void rk_newton_kernel(int L, int pairwise, int gradient, const double* __restrict__ sums, double l2,
                                 double lr, double* __restrict__ leaf_raw, double* __restrict__ leaf_lrv) {
    if (blockIdx.x != 0 || threadIdx.x != 0) return;
    for (int q = 0; q < L; ++q) {
        const double s1 = sums[3 * q];
        const double s2 = sums[3 * q + 1];
        if (gradient) {
            leaf_raw[q] = s2 > 0.0 ? __ddiv_rn(s1, __dadd_rn(s2, l2)) : 0.0;
        } else {
            const double den = __dadd_rn(-s2, l2);
            leaf_raw[q] = den == 0.0 ? 0.0 : __ddiv_rn(s1, den);
        }
    }
    double avg = 0.0;
    bool centre = false;
    if (pairwise) {
        double total = 0.0;
        for (int q = 0; q < L; ++q) total = __dadd_rn(total, sums[3 * q + 2]);
        if (fabs(total) > 1e-9) {
            double acc = 0.0;
            for (int q = 0; q < L; ++q) acc = __dadd_rn(acc, __dmul_rn(leaf_raw[q], sums[3 * q + 2]));
            avg = __ddiv_rn(acc, total);
            centre = true;
        }
    }
    for (int q = 0; q < L; ++q) {
        double v = leaf_raw[q];
        if (centre) {
            const double w = sums[3 * q + 2];
            v = fabs(w) > 1e-9 ? __dsub_rn(v, avg) : 0.0;
        }
        leaf_lrv[q] = __dmul_rn(v, lr);
    }
}

// ---- StochasticRank: Monte-Carlo DCG / NDCG ders on the device -------------

// Marsaglia polar standard normal over a TFastRng64 (normal.rs; the same draw
// sequence as the host replica).
__device__ double srk_std_normal(Rng64& r) {
    for (;;) {
        const double x = __dsub_rn(__dmul_rn(real1(r), 2.0), 1.0);
        const double y = __dsub_rn(__dmul_rn(real1(r), 2.0), 1.0);
        const double rr = __dadd_rn(__dmul_rn(x, x), __dmul_rn(y, y));
        if (!(rr > 1.0 || rr <= 0.0)) return __dmul_rn(x, sqrt(__ddiv_rn(__dmul_rn(-2.0, log(rr)), rr)));
    }
}

// normal_density (ranking_der.rs:640-655)
__device__ __forceinline__ double srk_density(double x, double mean, double sigma) {
    const double t = __ddiv_rn(__dsub_rn(x, mean), sigma);
    const double z = __dmul_rn(t, t);
    return __ddiv_rn(__dmul_rn(exp(__ddiv_rn(-z, 2.0)), 0.398942280401432677939946), sigma);
}

// stochastic_rank_group_der (ranking_der.rs:710-910), one thread per group:
// group-mean centring, the Mu tie shift, num_est samples of TFastRng64(base +
// group) noise with a stable descending sort, the DCG cumulative statistics
// and the per-position density-weighted metric diffs, then the SFA mean
// removal and approx-direction projection (Nu 0.01, Lambda 1).  Position
// denominators and the NDCG ideal come from the host.  der2 = 0.
// ws: 9 g + 3 doubles per group at ws + 9 b + 3 gi (8 g + 3 used); ord: n int32.
__global__ void rk_srank_kernel(int n_groups, const int64_t* __restrict__ goff, const double* __restrict__ approx,
                                const double* __restrict__ target, int ndcg, double sigma_p, double mu, int num_est,
                                uint64_t base, const double* __restrict__ den, const double* __restrict__ ideal,
                                double* __restrict__ wsall, int32_t* __restrict__ ordall, double* __restrict__ d1,
                                double* __restrict__ d2, McState* __restrict__ ms) {
    const int gi = blockIdx.x * blockDim.x + threadIdx.x;
    if (gi >= n_groups) return;
    const int64_t b = goff[gi], cnt = goff[gi + 1] - b;
    double* o1 = d1 + b;
    double* o2 = d2 + b;
    for (int64_t i = 0; i < cnt; ++i) {
        o1[i] = 0.0;
        o2[i] = 0.0;
    }
    if (cnt <= 1) return;
    const double* tg = target + b;
    double* ap = wsall + 9 * b + 3 * (int64_t)gi;
    double* sh = ap + cnt;
    double* pw = sh + cnt;
    double* noise = pw + cnt;
    double* sc = noise + cnt;
    double* cs = sc + cnt;
    double* csu = cs + cnt + 1;
    double* csl = csu + cnt + 1;
    int32_t* ord = ordall + b;
    const double fc = (double)cnt;
    double acc = 0.0;
    for (int64_t i = 0; i < cnt; ++i) acc = __dadd_rn(acc, approx[b + i]);
    const double am = __ddiv_rn(acc, fc);
    for (int64_t i = 0; i < cnt; ++i) ap[i] = __dsub_rn(approx[b + i], am);
    acc = 0.0;
    for (int64_t i = 0; i < cnt; ++i) {
        sh[i] = __dsub_rn(ap[i], __dmul_rn(__dmul_rn(sigma_p, mu), tg[i]));
        acc = __dadd_rn(acc, sh[i]);
    }
    const double avs = __ddiv_rn(acc, fc);
    for (int64_t i = 0; i < cnt; ++i) sh[i] = __dsub_rn(sh[i], avs);
    const double idl = ideal[gi];
    for (int64_t p = 0; p < cnt; ++p) {
        pw[p] = __ddiv_rn(1.0, den[p]);
        if (ndcg && idl > DBL_EPSILON) pw[p] = __ddiv_rn(pw[p], idl);
    }
    Rng64 rng = Rng64::from_seed(base + (uint64_t)gi);
    const double sigma = __dmul_rn(sigma_p, sqrt(__ddiv_rn(fc, __dsub_rn(fc, 1.0))));
    const int ne = num_est < 1 ? 1 : num_est;
    for (int s = 0; s < ne; ++s) {
        double noise_sum = 0.0;
        for (int64_t d = 0; d < cnt; ++d) {
            noise[d] = srk_std_normal(rng);
            sc[d] = __dadd_rn(sh[d], __dmul_rn(sigma_p, noise[d]));
            noise_sum = __dadd_rn(noise_sum, noise[d]);
        }
        for (int64_t i = 0; i < cnt; ++i) ord[i] = (int32_t)i;
        for (int64_t i = 1; i < cnt; ++i) {  // stable, descending by score
            const int32_t key = ord[i];
            int64_t j = i - 1;
            while (j >= 0 && sc[ord[j]] < sc[key]) {
                ord[j + 1] = ord[j];
                --j;
            }
            ord[j + 1] = key;
        }
        for (int64_t p = 0; p <= cnt; ++p) {
            cs[p] = 0.0;
            csu[p] = 0.0;
            csl[p] = 0.0;
        }
        for (int64_t p = 0; p < cnt; ++p) {  // CalcDCGCumulativeStatistics
            const double gain = tg[ord[p]];
            cs[p + 1] = __dadd_rn(cs[p], __dmul_rn(gain, pw[p]));
            if (p + 1 < cnt) csl[p + 1] = __dadd_rn(csl[p], __dmul_rn(gain, pw[p + 1]));
            if (p > 0) csu[p + 1] = __dadd_rn(csu[p], __dmul_rn(gain, pw[p - 1]));
        }
        csl[cnt] = csl[cnt - 1];
        for (int64_t p = 0; p < cnt; ++p) {
            const int32_t doc = ord[p];
            const double score = sc[doc], a = ap[doc];
            const double mean = __dadd_rn(a, __ddiv_rn(__dsub_rn(noise_sum, __dsub_rn(score, a)), __dsub_rn(fc, 1.0)));
            const double gain = tg[doc];
            double der_sum = 0.0;
            for (int64_t np = 0; np < cnt; ++np) {
                if (np == p) continue;
                // calc_dcg_metric_diff (ranking_der.rs:920-965)
                const double doc_diff = __dmul_rn(gain, __dsub_rn(pw[np], pw[p]));
                double mid;
                if (np < p) mid = __dsub_rn(__dsub_rn(csl[p], csl[np]), __dsub_rn(cs[p], cs[np]));
                else mid = __dsub_rn(__dsub_rn(csu[np + 1], csu[p + 1]), __dsub_rn(cs[np + 1], cs[p + 1]));
                const double md = __dadd_rn(doc_diff, mid);
                double dd;
                if (np == 0) dd = srk_density(sc[ord[0]], mean, sigma);
                else if (np + 1 == cnt) dd = -srk_density(sc[ord[cnt - 1]], mean, sigma);
                else if (np < p)
                    dd = __dsub_rn(srk_density(sc[ord[np]], mean, sigma), srk_density(sc[ord[np - 1]], mean, sigma));
                else
                    dd = __dsub_rn(srk_density(sc[ord[np + 1]], mean, sigma), srk_density(sc[ord[np]], mean, sigma));
                der_sum = __dadd_rn(der_sum, __dmul_rn(md, dd));
            }
            o1[doc] = __dadd_rn(o1[doc], __ddiv_rn(der_sum, (double)ne));
        }
    }
    acc = 0.0;
    for (int64_t i = 0; i < cnt; ++i) acc = __dadd_rn(acc, o1[i]);
    const double avg_der = __ddiv_rn(acc, fc);
    for (int64_t i = 0; i < cnt; ++i) o1[i] = __dsub_rn(o1[i], avg_der);
    if (cnt > 2) {
        acc = 0.0;
        for (int64_t i = 0; i < cnt; ++i) acc = __dadd_rn(acc, ap[i]);
        const double aa = __ddiv_rn(acc, fc);
        double sq = 0.0, dot = 0.0;
        for (int64_t i = 0; i < cnt; ++i) {
            sh[i] = __dsub_rn(ap[i], aa);
            sq = __dadd_rn(sq, __dmul_rn(sh[i], sh[i]));
        }
        for (int64_t i = 0; i < cnt; ++i) dot = __dadd_rn(dot, __dmul_rn(o1[i], sh[i]));
        const double nr = __dadd_rn(sqrt(sq), 0.01);
        const double norm_sqr = __dmul_rn(nr, nr);
        if (norm_sqr > 0.0) {
            const double k = __ddiv_rn(__dmul_rn(1.0, dot), norm_sqr);
            for (int64_t i = 0; i < cnt; ++i) o1[i] = __dsub_rn(o1[i], __dmul_rn(k, sh[i]));
        }
    }
    bool finite = true;
    for (int64_t i = 0; i < cnt; ++i) finite &= isfinite(o1[i]);
    if (!finite) atomicOr(&ms->err, kMcErrNonFinite);
}

// ---- YetiRank: per-tree pair sampling on the device --------------------------

// sample_pairs (crates/cb-train/src/yetirank.rs:75-171), one warp per group:
// per permutation one TFastRng64 draw per document (cast to f32, ratio
// u / (1.000001 - u) in f32) multiplies exp(approx), a stable descending sort,
// and the Classic decayed weights 0.15 * decay^k * |rel_a - rel_b| (f32) go to
// the higher-relevance document's row of the group's dense f32 matrix
// cw[winner][loser].  Each lane jumps its own copy of the group's stream to
// its documents' draws (draw p * g + i); the sort is a rank count (position of
// i = documents with a larger key, or an equal key and a smaller index: the
// stable descending order); within one permutation the adjacent pairs touch
// distinct cells, so lanes add them at once, and permutations follow each
// other in order -- every rounding is the sequential loop's.  decay_pow[k] =
// decay^k formed by k successive multiplications.  idx / boot are n-sized
// scratch indexed by object.
constexpr int kYetiSmemDocs = 256;  // groups up to this size keep their sort keys in shared memory

// The sampler for a group of g <= 32 * kSlots documents with its keys, exps,
// order and relevances in shared memory: each lane keeps the RNG states of its
// documents' first draw and moves them by fixed jumps (32 documents within a
// permutation, g between permutations), and counts the ranks of its kSlots
// documents in one pass over the keys.
template <int kSlots>
__device__ __forceinline__ void yeti_sample_smem(int64_t g, int lane, const Rng64& base, int perms,
                                                 const double* __restrict__ apg, const double* __restrict__ tg,
                                                 const double* __restrict__ decay_pow, float* __restrict__ cwg,
                                                 double* __restrict__ key, double* __restrict__ ex,
                                                 int32_t* __restrict__ ix, float* __restrict__ rel) {
    for (int64_t i = lane; i < g; i += 32) {
        ex[i] = exp(apg[i]);
        rel[i] = __double2float_rn(tg[i]);
    }
    uint64_t a32, d32, ag, dg;
    lcg_jump(32, a32, d32);
    lcg_jump((uint64_t)g, ag, dg);
    Rng64 first = base;  // draw (permutation p, document lane)
    first.advance((uint64_t)lane);
    // the decay weights of this lane's adjacent positions d = 1 + lane + 32 sl
    double dpw[kSlots];
#pragma unroll
    for (int sl = 0; sl < kSlots; ++sl) dpw[sl] = 1 + lane + 32 * sl < g ? decay_pow[lane + 32 * sl] : 0.0;
    __syncwarp();
    for (int p = 0; p < perms; ++p) {
        double k[kSlots];
        Rng64 r = first;
#pragma unroll
        for (int sl = 0; sl < kSlots; ++sl) {
            const int64_t i = lane + 32 * sl;
            Rng64 d = r;
            const float u = __double2float_rn(real1(d));
            const float ratio = __fdiv_rn(u, __fsub_rn(1.000001f, u));
            k[sl] = i < g ? __dmul_rn(ex[i], (double)ratio) : 0.0;
            if (i < g) key[i] = k[sl];
            r.jump(a32, d32);
        }
        first.jump(ag, dg);
        __syncwarp();
        // position of i = documents with a larger key, or an equal key and a
        // smaller index (the stable descending order)
        int pos[kSlots];
#pragma unroll
        for (int sl = 0; sl < kSlots; ++sl) pos[sl] = 0;
        for (int64_t j = 0; j < g; ++j) {
            const double o = key[j];
#pragma unroll
            for (int sl = 0; sl < kSlots; ++sl)
                pos[sl] += (o > k[sl] || (o == k[sl] && j < lane + 32 * sl)) ? 1 : 0;
        }
#pragma unroll
        for (int sl = 0; sl < kSlots; ++sl)
            if (lane + 32 * sl < g) ix[pos[sl]] = lane + 32 * sl;
        __syncwarp();
        // a permutation's adjacent pairs are distinct, so are their cells:
        // all of a lane's loads go out before its stores
        int64_t cell[kSlots];
        float pwv[kSlots], old[kSlots];
#pragma unroll
        for (int sl = 0; sl < kSlots; ++sl) {
            const int64_t d = 1 + lane + 32 * sl;
            cell[sl] = -1;
            pwv[sl] = 0.0f;
            if (d < g) {
                const int32_t fi = ix[d - 1], se = ix[d];
                const float rf = rel[fi], rs = rel[se];
                pwv[sl] = __double2float_rn(__dmul_rn(__dmul_rn(0.15, dpw[sl]), (double)fabsf(__fsub_rn(rf, rs))));
                if (rf > rs) cell[sl] = (int64_t)fi * g + se;
                else if (rf < rs) cell[sl] = (int64_t)se * g + fi;
            }
        }
#pragma unroll
        for (int sl = 0; sl < kSlots; ++sl) old[sl] = cell[sl] >= 0 ? cwg[cell[sl]] : 0.0f;
#pragma unroll
        for (int sl = 0; sl < kSlots; ++sl)
            if (cell[sl] >= 0) cwg[cell[sl]] = __fadd_rn(old[sl], pwv[sl]);
        __syncwarp();
    }
}

__global__ void __launch_bounds__(kYetiWarps * 32, 6) rk_yeti_sample_kernel(
    int n_groups, const int64_t* __restrict__ goff, const double* __restrict__ ap, const double* __restrict__ target,
    int perms, const double* __restrict__ decay_pow, const uint64_t* __restrict__ seeds,
    const int64_t* __restrict__ cwoff, float* __restrict__ cw, int32_t* __restrict__ idx,
    double* __restrict__ boot) {
    __shared__ double skey[kYetiWarps][kYetiSmemDocs], sex[kYetiWarps][kYetiSmemDocs];
    __shared__ int32_t six[kYetiWarps][kYetiSmemDocs];
    __shared__ float srel[kYetiWarps][kYetiSmemDocs];
    const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
    const int gi = blockIdx.x * kYetiWarps + wp;
    if (gi >= n_groups) return;  // warp-uniform
    const int64_t b = goff[gi], g = goff[gi + 1] - b;
    float* cwg = cw + cwoff[gi];
    for (int64_t k = lane; k < g * g; k += 32) cwg[k] = 0.0f;
    if (g == 0) return;
    const Rng64 base = Rng64::from_seed(seeds[gi]);
    if (g <= kYetiSmemDocs) {
        __syncwarp();
#define CBGPU_YS(S) yeti_sample_smem<S>(g, lane, base, perms, ap + b, target + b, decay_pow, cwg, skey[wp], \
                                        sex[wp], six[wp], srel[wp])
        switch ((g + 31) / 32) {
            case 1: CBGPU_YS(1); break;
            case 2: CBGPU_YS(2); break;
            case 3: CBGPU_YS(3); break;
            case 4: CBGPU_YS(4); break;
            case 5: CBGPU_YS(5); break;
            case 6: CBGPU_YS(6); break;
            case 7: CBGPU_YS(7); break;
            default: CBGPU_YS(8); break;
        }
#undef CBGPU_YS
        return;
    }
    // larger groups: keys and order in the n-sized scratch
    int32_t* ix = idx + b;
    double* bt = boot + b;
    __syncwarp();
    for (int p = 0; p < perms; ++p) {
        for (int64_t i = lane; i < g; i += 32) {
            Rng64 r = base;
            r.advance((uint64_t)p * (uint64_t)g + (uint64_t)i);
            const float u = __double2float_rn(real1(r));
            const float ratio = __fdiv_rn(u, __fsub_rn(1.000001f, u));
            bt[i] = __dmul_rn(exp(ap[b + i]), (double)ratio);
        }
        __syncwarp();
        for (int64_t i = lane; i < g; i += 32) {
            const double key = bt[i];
            int64_t pos = 0;
#pragma unroll 4
            for (int64_t j = 0; j < g; ++j) {
                const double o = bt[j];
                pos += (o > key || (o == key && j < i)) ? 1 : 0;
            }
            ix[pos] = (int32_t)i;
        }
        __syncwarp();
        for (int64_t d = 1 + lane; d < g; d += 32) {
            const int32_t first = ix[d - 1], second = ix[d];
            const float rf = __double2float_rn(target[b + first]), rs = __double2float_rn(target[b + second]);
            const float pw =
                __double2float_rn(__dmul_rn(__dmul_rn(0.15, decay_pow[d - 1]), (double)fabsf(__fsub_rn(rf, rs))));
            if (rf > rs) cwg[first * g + second] = __fadd_rn(cwg[first * g + second], pw);
            else if (rf < rs) cwg[second * g + first] = __fadd_rn(cwg[second * g + first], pw);
        }
        __syncwarp();
    }
}

// One pair cell's contribution, shared by both walks: the pair weight
// wf = qw * cv / perms (f32) and the loser's probability p = e_l / (e_l + e_w);
// returns false for a skipped cell (wf == 0).
__device__ __forceinline__ bool yeti_cell(float cv, float qw, float den, double el, double ew, double& c,
                                          double& cp, double& q) {
    const float wf = __fdiv_rn(__fmul_rn(qw, cv), den);
    if (wf == 0.0f) return false;
    c = (double)wf;
    const double dn = __dadd_rn(el, ew);
    const double p = dn > 0.0 ? __ddiv_rn(el, dn) : 0.5;
    cp = __dmul_rn(c, p);
    q = __dmul_rn(cp, __dsub_rn(p, 1.0));
    return true;
}

constexpr int kYetiMaskDocs = 128;  // groups up to this size take the sparse walk
constexpr int kYetiMaskWords = kYetiMaskDocs / 32;

// The sparse walk for a group of g <= kYetiMaskDocs documents with a finite
// weight (where zero cells are skipped): non-zero masks of the pair matrix are
// built from coalesced row reads (row masks in shared memory, each lane's
// column masks in registers), then lane x visits only its non-zero cells, in
// the dense walk's order: winners w < x of its column, its own row's losers,
// winners w > x.  The sums are the dense walk's, term for term.
__device__ __forceinline__ void yeti_der_sparse(int64_t g, const float* __restrict__ cwg,
                                                const double* __restrict__ exg, float qw, float den,
                                                uint32_t* __restrict__ rmask, uint32_t* __restrict__ cmask_s,
                                                double* __restrict__ d1, double* __restrict__ d2,
                                                double* __restrict__ eff, int lane, bool& finite) {
    const int W = (int)((g + 31) >> 5);
    uint32_t cmask[kYetiMaskWords][kYetiMaskWords];  // [column slot][row word]
#pragma unroll
    for (int k = 0; k < kYetiMaskWords; ++k)
#pragma unroll
        for (int w = 0; w < kYetiMaskWords; ++w) cmask[k][w] = 0u;
    // rows in batches of 4 whose loads issue before their ballots
    constexpr int kRowBatch = 4;
#pragma unroll
    for (int rw = 0; rw < kYetiMaskWords; ++rw) {
        if (rw >= W) break;
        for (int ri0 = 0; ri0 < 32 && rw * 32 + ri0 < g; ri0 += kRowBatch) {
            float v[kRowBatch][kYetiMaskWords];
#pragma unroll
            for (int j = 0; j < kRowBatch; ++j) {
                const int64_t r = rw * 32 + ri0 + j;
#pragma unroll
                for (int k = 0; k < kYetiMaskWords; ++k) {
                    const int64_t c = lane + 32 * k;
                    v[j][k] = (k < W && r < g && c < g) ? cwg[r * g + c] : 0.0f;
                }
            }
#pragma unroll
            for (int j = 0; j < kRowBatch; ++j) {
                const int64_t r = rw * 32 + ri0 + j;
                if (r >= g) break;
#pragma unroll
                for (int k = 0; k < kYetiMaskWords; ++k) {
                    if (k >= W) break;
                    const bool nz = v[j][k] != 0.0f;
                    const uint32_t bal = __ballot_sync(0xffffffffu, nz);
                    if (lane == 0) rmask[r * kYetiMaskWords + k] = bal;
                    cmask[k][rw] |= (nz ? 1u : 0u) << (ri0 + j);
                }
            }
        }
    }
    // column masks to shared memory, so the walk below indexes them at run
    // time instead of unrolling (the unrolled walk overflowed the
    // instruction cache)
#pragma unroll
    for (int k = 0; k < kYetiMaskWords; ++k)
#pragma unroll
        for (int w = 0; w < kYetiMaskWords; ++w) cmask_s[(lane + 32 * k) * kYetiMaskWords + w] = cmask[k][w];
    __syncwarp();
#pragma unroll 1
    for (int k = 0; k < W; ++k) {
        const int64_t x = lane + 32 * k;
        if (x >= g) continue;
        const double ewx = exg[x];
        double a1 = 0.0, a2 = 0.0, ae = 0.0, wd = 0.0, wd2 = 0.0, c, cp, q;
        // phases: 0 = winners w < x of column x, 1 = row x's losers, 2 = winners w > x
#pragma unroll 1
        for (int ph = 0; ph < 3; ++ph) {
#pragma unroll 1
            for (int rw = 0; rw < W; ++rw) {
                uint32_t m;
                if (ph == 1) {
                    m = rmask[x * kYetiMaskWords + rw];
                } else {
                    m = cmask_s[x * kYetiMaskWords + rw];
                    const int64_t cut = x - rw * 32;  // bit index of x in this word
                    if (ph == 0) m = cut <= 0 ? 0u : (cut >= 32 ? m : m & ((1u << cut) - 1u));
                    else m = cut < 0 ? m : (cut >= 31 ? 0u : m & ~((2u << cut) - 1u));
                }
                while (m) {
                    const int o = rw * 32 + __ffs(m) - 1;  // loser (row) or winner (column)
                    m &= m - 1;
                    const bool row = ph == 1;
                    const float cv = row ? cwg[x * g + o] : cwg[(int64_t)o * g + x];
                    if (yeti_cell(cv, qw, den, row ? exg[o] : ewx, row ? ewx : exg[o], c, cp, q)) {
                        if (row) {
                            wd = __dadd_rn(wd, cp);
                            wd2 = __dadd_rn(wd2, q);
                        } else {
                            a1 = __dsub_rn(a1, cp);
                            a2 = __dadd_rn(a2, q);
                        }
                        ae = __dadd_rn(ae, c);
                    }
                }
            }
            if (ph == 1) {  // the winner row ends
                a1 = __dadd_rn(a1, wd);
                a2 = __dadd_rn(a2, wd2);
            }
        }
        d1[x] = a1;
        d2[x] = a2;
        if (eff) eff[x] = ae;
        finite &= isfinite(a1) && isfinite(a2);
    }
}

// The PairLogit der over one phase's sampled pairs (pairlogit_group_der,
// ranking_der.rs:400-440), winner rows ascending, losers ascending, pair
// weight (qw * cw / perms) in f32; eff (when given) gets the pairwise weights
// (calc_pairwise_weights, boosting.rs:1761-1780) in the same order.  One warp
// per group, one lane per document: a document's der1 / der2 / eff receive
// its terms in the sequential loop's order (by winner row; its own winner row
// adds its loser sum at that point), so every sum rounds as the CPU's.  ex is
// n-sized scratch for exp(approx).
__global__ void __launch_bounds__(kYetiWarps * 32) rk_yeti_der_kernel(
    int n_groups, const int64_t* __restrict__ goff, const double* __restrict__ ap, const double* __restrict__ gw,
    int perms, const int64_t* __restrict__ cwoff, const float* __restrict__ cw, double* __restrict__ d1,
    double* __restrict__ d2, double* __restrict__ eff, double* __restrict__ ex, McState* __restrict__ ms) {
    __shared__ uint32_t s_rmask[kYetiWarps][kYetiMaskDocs * kYetiMaskWords];
    __shared__ uint32_t s_cmask[kYetiWarps][kYetiMaskDocs * kYetiMaskWords];
    const int lane = threadIdx.x & 31;
    const int gi = blockIdx.x * kYetiWarps + (threadIdx.x >> 5);
    if (gi >= n_groups) return;  // warp-uniform
    const int64_t b = goff[gi], g = goff[gi + 1] - b;
    const float* cwg = cw + cwoff[gi];
    const float qw = __double2float_rn(gw[gi]), den = (float)perms;
    // a zero cell gives wf == 0 (skipped) whenever qw is finite: skip it before dividing
    const bool qw_finite = isfinite(qw);
    for (int64_t i = lane; i < g; i += 32) ex[b + i] = exp(ap[b + i]);
    __syncwarp();
    bool finite = true;
    if (qw_finite && g <= kYetiMaskDocs) {
        yeti_der_sparse(g, cwg, ex + b, qw, den, s_rmask[threadIdx.x >> 5], s_cmask[threadIdx.x >> 5], d1 + b,
                        d2 + b, eff ? eff + b : nullptr, lane, finite);
        if (__any_sync(0xffffffffu, !finite) && lane == 0) atomicOr(&ms->err, kMcErrNonFinite);
        return;
    }
    // Lane x walks 2g - 1 steps: column cells (x as the loser of wl) for
    // wl < x, then its own winner row (losers ascending, summed apart and
    // added to der1 / der2 when the row ends), then column cells for wl > x.
    // Every lane takes the same step count, so no lane waits on another's
    // row, and each sum still takes its terms in the sequential loop's order.
    for (int64_t x0 = 0; x0 < g; x0 += 32) {
        const int64_t x = x0 + lane;
        const bool act = x < g;
        double a1 = 0.0, a2 = 0.0, ae = 0.0, wd = 0.0, wd2 = 0.0;
        const double ewx = act ? ex[b + x] : 0.0;
        for (int64_t st = 0; st < 2 * g - 1; ++st) {
            if (!act) continue;
            const bool row = st >= x && st < x + g;
            const int64_t o = row ? st - x : (st < x ? st : st - g + 1);  // loser (row) or winner (column)
            const float cv = row ? cwg[x * g + o] : cwg[o * g + x];
            if (!(cv == 0.0f && qw_finite)) {
                const float wf = __fdiv_rn(__fmul_rn(qw, cv), den);
                if (wf != 0.0f) {
                    const double c = (double)wf;
                    const double eo = ex[b + o];
                    if (row) {
                        const double dn = __dadd_rn(eo, ewx);
                        const double p = dn > 0.0 ? __ddiv_rn(eo, dn) : 0.5;
                        const double cp = __dmul_rn(c, p);
                        wd = __dadd_rn(wd, cp);
                        wd2 = __dadd_rn(wd2, __dmul_rn(cp, __dsub_rn(p, 1.0)));
                    } else {
                        const double dn = __dadd_rn(ewx, eo);
                        const double p = dn > 0.0 ? __ddiv_rn(ewx, dn) : 0.5;
                        const double cp = __dmul_rn(c, p);
                        a1 = __dsub_rn(a1, cp);
                        a2 = __dadd_rn(a2, __dmul_rn(cp, __dsub_rn(p, 1.0)));
                    }
                    ae = __dadd_rn(ae, c);
                }
            }
            if (st == x + g - 1) {  // the winner row ends
                a1 = __dadd_rn(a1, wd);
                a2 = __dadd_rn(a2, wd2);
            }
        }
        if (act) {
            d1[b + x] = a1;
            d2[b + x] = a2;
            if (eff) eff[b + x] = ae;
            finite &= isfinite(a1) && isfinite(a2);
        }
    }
    if (__any_sync(0xffffffffu, !finite) && lane == 0) atomicOr(&ms->err, kMcErrNonFinite);
}

// ---- PairLogitPairwise: pairwise split scoring and Cholesky pairwise leaves
//
// The reference scores a candidate border b of feature f at a level with P
// leaves by building a running 2P x 2P pair-weight system over the border
// buckets 0..b (calculate_pairwise_score, crates/cb-compute/src/
// pairwise_scoring.rs:367-580) and solving it with a Cholesky factor per
// border.  With unit pair weights every entry of that system is an integer
// pair count, so the system at border b equals one built directly from the
// bin-prefix pair statistics: candidates are independent here, one block each.

constexpr int kPwThreads = 128;
constexpr int kPwMaxDepth = 8;                 // P <= 128 leaves at the last level
constexpr int kPwSmemMaxN2 = 64;               // systems up to 64 x 64 stay in shared memory
constexpr int kPwGlobalBlocks = 148 * 2;       // global-scratch slots for larger systems
constexpr size_t kPwMaxStatBytes = (size_t)16 << 30;

// doubles of scratch one candidate needs: ws (n2^2), the factor (m^2) and
// dsum, lv, y, x, term (n2 each)
__host__ __device__ inline size_t pw_scratch_doubles(int n2) {
    const size_t m = (size_t)(n2 > 1 ? n2 - 1 : 1);
    return (size_t)n2 * n2 + m * m + 5 * (size_t)n2;
}

// Pair weights enter the statistics as int64 fixed point at 2^pw_shift
// (llrint(w * 2^pw_shift)); the host bounds pw_shift so every sum stays below
// 2^61.  Unit weights are exact, and any order gives the same sums.
__device__ __forceinline__ void pw_add(long long* p, long long v) {
    atomicAdd(reinterpret_cast<unsigned long long*>(p), (unsigned long long)v);
}

// One pair's statistics (compute_pair_weight_statistics,
// pairwise_scoring.rs:163-198), buckets = bins:
//   wb > lb: smaller[ll][wl][lb] -= w, greater[ll][wl][wb] -= w
//   else:    smaller[wl][ll][wb] -= w, greater[wl][ll][lb] -= w
// st[a][c][bin][2] = (smaller, greater) of one feature.
__device__ __forceinline__ void pw_stat_pair(int wb, int lb, int wl, int ll, int P, int NB, long long q,
                                             long long* st) {
    if (wl >= P || ll >= P || wb >= NB || lb >= NB) return;
    if (wb > lb) {
        pw_add(&st[(((size_t)ll * P + wl) * NB + lb) * 2 + 0], -q);
        pw_add(&st[(((size_t)ll * P + wl) * NB + wb) * 2 + 1], -q);
    } else {
        pw_add(&st[(((size_t)wl * P + ll) * NB + wb) * 2 + 0], -q);
        pw_add(&st[(((size_t)wl * P + ll) * NB + lb) * 2 + 1], -q);
    }
}

// The statistics of one level over a pair list: explicit pairs of unit weight
// (pq null), or YetiRank's compacted samples with their fixed-point weights
// pq and their count in n_dev (n_pairs then bounds it).
__global__ void rk_pairstat_kernel(int64_t n_pairs, int64_t n, int P, int NB, const int64_t* __restrict__ pw,
                                   const int64_t* __restrict__ pl, const uint8_t* __restrict__ bins_fm,
                                   const uint16_t* __restrict__ leaf, int pw_shift, long long* __restrict__ stats,
                                   const long long* __restrict__ pq, const unsigned long long* __restrict__ n_dev) {
    const int f = blockIdx.y;
    const uint8_t* col = bins_fm + (size_t)f * (size_t)n;
    long long* st = stats + (size_t)f * P * P * NB * 2;
    const long long unit = 1ll << pw_shift;
    const int64_t np = n_dev ? (int64_t)min(*n_dev, (unsigned long long)n_pairs) : n_pairs;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < np; k += (int64_t)gridDim.x * blockDim.x) {
        const int64_t w = pw[k], l = pl[k];
        if (w == l) continue;
        pw_stat_pair(col[w], col[l], leaf[w], leaf[l], P, NB, pq ? pq[k] : unit, st);
    }
}

// The same statistics at levels of at most kPsSmemLeaves parents, where one
// feature's whole table (P^2 NB (smaller, greater) cells) fits in shared
// memory: a block takes one feature and a share of the pairs, adds exactly
// into (lo, hi) 32-bit word pairs (add_split64), and flushes its table with
// one global atomic per non-zero cell -- instead of two contended global
// atomics per (pair, feature).  Integer sums: the same result in any order.
constexpr int kPsSmemLeaves = 8;
constexpr int kPsThreads = 1024;
__global__ void __launch_bounds__(kPsThreads) rk_pairstat_smem_kernel(
    int64_t n_pairs, int64_t n, int P, int NB, const int64_t* __restrict__ pw, const int64_t* __restrict__ pl,
    const uint8_t* __restrict__ bins_fm, const uint16_t* __restrict__ leaf, int pw_shift,
    long long* __restrict__ stats, const long long* __restrict__ pq, const unsigned long long* __restrict__ n_dev) {
    extern __shared__ uint32_t pst[];  // lo words [cells], then hi words [cells]
    const int f = blockIdx.y;
    const uint8_t* col = bins_fm + (size_t)f * (size_t)n;
    const int cells = P * P * NB * 2;
    uint32_t* lo = pst;
    uint32_t* hi = pst + cells;
    for (int k = threadIdx.x; k < 2 * cells; k += blockDim.x) pst[k] = 0u;
    __syncthreads();
    const long long unit = -(1ll << pw_shift);
    const int64_t np = n_dev ? (int64_t)min(*n_dev, (unsigned long long)n_pairs) : n_pairs;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < np; k += (int64_t)gridDim.x * blockDim.x) {
        const int64_t w = pw[k], l = pl[k];
        if (w == l) continue;
        const long long q = pq ? -pq[k] : unit;
        const int wb = col[w], lb = col[l], wl = leaf[w], ll = leaf[l];
        if (wl >= P || ll >= P || wb >= NB || lb >= NB) continue;
        int c0, c1;  // pw_stat_pair's two cells
        if (wb > lb) {
            c0 = ((ll * P + wl) * NB + lb) * 2;
            c1 = ((ll * P + wl) * NB + wb) * 2 + 1;
        } else {
            c0 = ((wl * P + ll) * NB + wb) * 2;
            c1 = ((wl * P + ll) * NB + lb) * 2 + 1;
        }
        add_split64(lo + c0, hi + c0, q);
        add_split64(lo + c1, hi + c1, q);
    }
    __syncthreads();
    unsigned long long* st = reinterpret_cast<unsigned long long*>(stats + (size_t)f * cells);
    for (int k = threadIdx.x; k < cells; k += blockDim.x) {
        const unsigned long long v = ((unsigned long long)hi[k] << 32) | lo[k];
        if (v) atomicAdd(st + k, v);
    }
}

// YetiRank's sampled pairs as a list, once per resample: a warp per group
// walks its dense matrix and appends every cell that is a pair of the
// pairwise statistics (weight wf = qw * cw / perms in f32, non-zero, winner
// != loser; compute_pair_weight_statistics, pairwise_scoring.rs:163-198)
// with its fixed-point weight llrint(wf * 2^pw_shift); the level kernels then
// take the list like explicit pairs.  List order does not matter: the statistics are
// integer sums.  A list longer than cap (possible only with a non-finite
// group weight) is cut and flagged.
__global__ void __launch_bounds__(kYetiWarps * 32) rk_yeti_compact_kernel(
    int n_groups, const int64_t* __restrict__ goff, const int64_t* __restrict__ cwoff, const float* __restrict__ cw,
    const double* __restrict__ gw, int perms, int pw_shift, int64_t cap, int64_t* __restrict__ out_w,
    int64_t* __restrict__ out_l, long long* __restrict__ out_q, unsigned long long* __restrict__ count,
    McState* __restrict__ ms) {
    const int lane = threadIdx.x & 31;
    const int gi = blockIdx.x * kYetiWarps + (threadIdx.x >> 5);
    if (gi >= n_groups) return;  // warp-uniform
    const int64_t b = goff[gi], g = goff[gi + 1] - b;
    const float* cwg = cw + cwoff[gi];
    const float qw = __double2float_rn(gw[gi]), den = (float)perms;
    for (int64_t c0 = 0; c0 < g * g; c0 += 32) {
        const int64_t c = c0 + lane;
        bool keep = false;
        long long q = 0;
        int64_t wl = 0, ll = 0;
        if (c < g * g) {
            wl = c / g;
            ll = c - wl * g;
            const float wf = __fdiv_rn(__fmul_rn(qw, cwg[c]), den);
            keep = !(wf == 0.0f || wl == ll);
            if (keep) q = llrint(ldexp((double)wf, pw_shift));
        }
        const unsigned m = __ballot_sync(0xffffffffu, keep);
        if (!m) continue;
        unsigned long long base = 0;
        if (lane == 0) base = atomicAdd(count, (unsigned long long)__popc(m));
        base = __shfl_sync(0xffffffffu, base, 0);
        if (keep) {
            const unsigned long long at = base + (unsigned long long)__popc(m & ((1u << lane) - 1u));
            if (at < (unsigned long long)cap) {
                out_w[at] = b + wl;
                out_l[at] = b + ll;
                out_q[at] = q;
            } else {
                atomicOr(&ms->err, kMcErrNonFinite);
            }
        }
    }
}

// Inclusive prefix over bins of every (feature, leaf, leaf, kind) row.
__global__ void rk_pairprefix_kernel(int64_t rows, int NB, long long* __restrict__ st) {
    for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < rows; r += (int64_t)gridDim.x * blockDim.x) {
        long long* row = st + (size_t)(r >> 1) * NB * 2 + (r & 1);
        long long run = 0;
        for (int b = 0; b < NB; ++b) {
            run += row[(size_t)b * 2];
            row[(size_t)b * 2] = run;
        }
    }
}

// make_zero_average (crates/cb-train/src/pairwise_leaves.rs:202-212), one thread.
__device__ void pw_zero_average(double* v, int n) {
    double s = 0.0;
    for (int i = 0; i < n; ++i) s = __dadd_rn(s, v[i]);
    const double avg = __ddiv_rn(s, (double)n);
    for (int i = 0; i < n; ++i) v[i] = __dsub_rn(v[i], avg);
}

// cholesky_solve (crates/cb-compute/src/leaf.rs:360-420) by the whole block:
// A (m x m, lower triangle) is factored in place, right-looking, but every
// entry subtracts its products in ascending column order and is divided by
// the same pivot, so each value rounds as in the reference's left-looking
// loops; the substitutions run on thread 0 in the reference's order.  The
// result is block-uniform: false on a non-positive pivot.
__device__ bool pw_cholesky_block(double* A, const double* rhs, int m, double* y, double* x, int* s_flag) {
    const int tid = threadIdx.x, nt = blockDim.x;
    if (tid == 0) *s_flag = 0;
    __syncthreads();
    for (int j = 0; j < m; ++j) {
        if (tid == 0) {
            const double d = A[(size_t)j * m + j];
            if (d <= 0.0) *s_flag = 1;
            else A[(size_t)j * m + j] = sqrt(d);
        }
        __syncthreads();
        if (*s_flag) return false;
        const double piv = A[(size_t)j * m + j];
        for (int i = j + 1 + tid; i < m; i += nt) A[(size_t)i * m + j] = __ddiv_rn(A[(size_t)i * m + j], piv);
        __syncthreads();
        const int rem = m - j - 1;
        for (int idx = tid; idx < rem * rem; idx += nt) {
            const int ii = idx / rem, kk = idx - ii * rem;
            if (kk > ii) continue;
            const int i = j + 1 + ii, k = j + 1 + kk;
            A[(size_t)i * m + k] = __dsub_rn(A[(size_t)i * m + k], __dmul_rn(A[(size_t)i * m + j], A[(size_t)k * m + j]));
        }
        __syncthreads();
    }
    if (tid == 0) {
        for (int i = 0; i < m; ++i) {
            double sum = rhs[i];
            for (int p = 0; p < i; ++p) sum = __dsub_rn(sum, __dmul_rn(A[(size_t)i * m + p], y[p]));
            y[i] = __ddiv_rn(sum, A[(size_t)i * m + i]);
        }
        for (int i = m - 1; i >= 0; --i) {
            double sum = y[i];
            for (int p = i + 1; p < m; ++p) sum = __dsub_rn(sum, __dmul_rn(A[(size_t)p * m + i], x[p]));
            x[i] = __ddiv_rn(sum, A[(size_t)i * m + i]);
        }
    }
    __syncthreads();
    return true;
}

// calculate_pairwise_leaf_values (pairwise_leaves.rs:113-200) by the whole
// block: w is n x n, out gets n zero-averaged values; A holds (n-1)^2, y and
// x (n-1) each.
__device__ void pw_leaf_values_block(const double* w, const double* der, int n, double l2, double* out, double* A,
                                     double* y, double* x, int* s_flag) {
    const int tid = threadIdx.x;
    if (n <= 2) {
        if (tid == 0) {
            if (n == 1) {
                out[0] = 0.0;
            } else {
                const double cp = __ddiv_rn(1.0, 2.0);
                const double dg = __dadd_rn(__dmul_rn(kPairwisePrior, __dsub_rn(1.0, cp)), l2);
                const double den = __dadd_rn(w[0], dg);
                out[0] = den != 0.0 ? __ddiv_rn(der[0], den) : 0.0;
                out[1] = 0.0;
                pw_zero_average(out, 2);
            }
        }
        __syncthreads();
        return;
    }
    const double cp = __ddiv_rn(1.0, (double)n);
    const double nd = __dmul_rn(-kPairwisePrior, cp);
    const double dg = __dadd_rn(__dmul_rn(kPairwisePrior, __dsub_rn(1.0, cp)), l2);
    const int m = n - 1;
    // the system's lower triangle mirrored (the reference reads w[r][c], c < r)
    for (int idx = tid; idx < m * m; idx += blockDim.x) {
        const int r = idx / m, c = idx - r * m;
        const int hi = r > c ? r : c, lo = r > c ? c : r;
        A[idx] = r == c ? __dadd_rn(w[(size_t)r * n + r], dg) : __dadd_rn(w[(size_t)hi * n + lo], nd);
    }
    __syncthreads();
    const bool ok = pw_cholesky_block(A, der, m, y, x, s_flag);
    if (tid == 0) {
        for (int i = 0; i < m; ++i) out[i] = ok ? x[i] : 0.0;
        out[m] = 0.0;
        pw_zero_average(out, n);
    }
    __syncthreads();
}

// One off-diagonal entry (r != c) of the pair-weight system of border b
// (the running sums of pairwise_scoring.rs:420-540 evaluated in closed
// form); leaf a of row r = r / 2, its side r % 2 (1: bins above b).
// Every off-diagonal entry is minus a pair-weight sum (<= 0), so each
// diagonal, minus its row sum, is exact in the int64 fixed point too.
__device__ __forceinline__ long long pw_offdiag(int r, int c, int P, int NB, int b, const long long* __restrict__ st) {
    auto S = [&](int u, int v, int bin) -> long long { return st[(((size_t)u * P + v) * NB + bin) * 2 + 0]; };
    auto G = [&](int u, int v, int bin) -> long long { return st[(((size_t)u * P + v) * NB + bin) * 2 + 1]; };
    const int a = r >> 1, sa = r & 1, d = c >> 1, sd = c & 1;
    if (a == d) return S(a, a, b) - G(a, a, b);  // the two sides of one leaf
    const int y = a < d ? a : d, x = a < d ? d : a;
    const int sy = a < d ? sa : sd, sx = a < d ? sd : sa;
    if (sy == 1 && sx == 1)  // every pair between the leaves minus those at or below b
        return (S(x, y, NB - 1) + S(y, x, NB - 1)) - (S(x, y, b) + S(y, x, b));
    if (sy == 0 && sx == 0) return G(x, y, b) + G(y, x, b);
    if (sx == 0) return S(x, y, b) - G(x, y, b);  // x below, y above
    return S(y, x, b) - G(y, x, b);               // x above, y below
}

// Scores of every candidate (feature, border) at a level with P leaves
// (calculate_pairwise_score + calculate_score, pairwise_scoring.rs:367-580):
// block per candidate, the der sums from the level histogram's bin prefix of
// channel 0 (exact int64), the pair counts from the prefixed statistics.
// Scratch: dynamic shared memory when 2P <= 64, else a global slot per block.
__global__ void __launch_bounds__(kPwThreads)
rk_pairscore_kernel(int P, int F, int NB, int C, const unsigned long long* __restrict__ pre,
                    const long long* __restrict__ stats, const int32_t* __restrict__ border_counts,
                    const McState* __restrict__ ms, double l2, int pw_shift, int use_smem,
                    double* __restrict__ gscratch, double* __restrict__ scores) {
    extern __shared__ double pw_smem[];
    __shared__ int s_flag;
    const int n2 = 2 * P, m = n2 - 1, tid = threadIdx.x;
    double* ws = use_smem ? pw_smem : gscratch + (size_t)blockIdx.x * pw_scratch_doubles(n2);
    double* A = ws + (size_t)n2 * n2;
    double* dsum = A + (size_t)(m > 0 ? m : 1) * (m > 0 ? m : 1);
    double* lv = dsum + n2;
    double* y = lv + n2;
    double* x = y + n2;
    double* term = x + n2;
    const double inv = ldexp(1.0, -ms->hist_shift);
    const double winv = ldexp(1.0, -pw_shift);
    const int64_t cand = (int64_t)F * NB;
    for (int64_t k = blockIdx.x; k < cand; k += gridDim.x) {
        const int f = (int)(k / NB), b = (int)(k - (int64_t)f * NB);
        if (b >= border_counts[f] || b >= NB - 1) {  // block-uniform
            if (tid == 0) scores[k] = -INFINITY;
            continue;
        }
        const long long* st = stats + (size_t)f * P * P * NB * 2;
        for (int idx = tid; idx < n2 * n2; idx += blockDim.x) {
            const int r = idx / n2, c = idx - r * n2;
            if (r == c) {  // rows sum to zero: minus the exact int64 row sum
                long long s = 0;
                for (int cc = 0; cc < n2; ++cc)
                    if (cc != r) s += pw_offdiag(r, cc, P, NB, b, st);
                ws[idx] = __dmul_rn((double)(-s), winv);
            } else {
                ws[idx] = __dmul_rn((double)pw_offdiag(r, c, P, NB, b, st), winv);
            }
        }
        for (int q = tid; q < P; q += blockDim.x) {
            const unsigned long long* row = pre + ((size_t)q * F + f) * NB * C;
            const long long below = (long long)row[(size_t)b * C], all = (long long)row[(size_t)(NB - 1) * C];
            dsum[2 * q] = __dmul_rn((double)below, inv);
            dsum[2 * q + 1] = __dmul_rn((double)(all - below), inv);
        }
        __syncthreads();
        pw_leaf_values_block(ws, dsum, n2, l2, lv, A, y, x, &s_flag);
        for (int xr = tid; xr < n2; xr += blockDim.x) {
            double sub = 0.0;
            for (int yc = 0; yc < n2; ++yc) sub = __dadd_rn(sub, __dmul_rn(lv[yc], ws[(size_t)xr * n2 + yc]));
            term[xr] = __dmul_rn(lv[xr], __dsub_rn(dsum[xr], __dmul_rn(0.5, sub)));
        }
        __syncthreads();
        if (tid == 0) {
            double outer = 0.0;
            for (int xr = 0; xr < n2; ++xr) outer = __dadd_rn(outer, term[xr]);
            scores[k] = outer;
        }
        __syncthreads();
    }
}

// The leaf pair-weight matrix of the grown tree (compute_pairwise_weight_sums,
// pairwise_leaves.rs:51-91), int64 fixed point at 2^pw_shift: exact in any order.
__device__ __forceinline__ void pw_leafw_pair(int wl, int ll, int L, long long q, long long* wsum) {
    if (wl == ll || wl >= L || ll >= L) return;
    pw_add(&wsum[(size_t)wl * L + ll], -q);
    pw_add(&wsum[(size_t)ll * L + wl], -q);
    pw_add(&wsum[(size_t)wl * L + wl], q);
    pw_add(&wsum[(size_t)ll * L + ll], q);
}

__global__ void rk_pairleafw_kernel(int64_t n_pairs, int L, const int64_t* __restrict__ pw,
                                    const int64_t* __restrict__ pl, const uint16_t* __restrict__ leaf, int pw_shift,
                                    long long* __restrict__ wsum) {
    const long long unit = 1ll << pw_shift;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < n_pairs; k += (int64_t)gridDim.x * blockDim.x)
        pw_leafw_pair(leaf[pw[k]], leaf[pl[k]], L, unit, wsum);
}

// The same over YetiRank's sampled pairs (dense per-group matrices).
__global__ void rk_yeti_pairleafw_kernel(int n_groups, const int64_t* __restrict__ goff,
                                         const int64_t* __restrict__ cwoff, const float* __restrict__ cw,
                                         const double* __restrict__ gw, int perms, int L,
                                         const uint16_t* __restrict__ leaf, int pw_shift,
                                         long long* __restrict__ wsum) {
    const int gi = blockIdx.x * blockDim.x + threadIdx.x;
    if (gi >= n_groups) return;
    const int64_t b = goff[gi], g = goff[gi + 1] - b;
    const float* cwg = cw + cwoff[gi];
    const float qw = __double2float_rn(gw[gi]), den = (float)perms;
    for (int64_t wl = 0; wl < g; ++wl)
        for (int64_t ll = 0; ll < g; ++ll) {
            const float wf = __fdiv_rn(__fmul_rn(qw, cwg[wl * g + ll]), den);
            if (wf == 0.0f) continue;
            pw_leafw_pair(leaf[b + wl], leaf[b + ll], L, llrint(ldexp((double)wf, pw_shift)), wsum);
        }
}

// Cholesky pairwise leaves (compute_pairwise_leaf_deltas, pairwise_leaves.rs:
// 219-242) from the leaf der sums (rk_leafsums' channel 0) with the raw
// l2, one block; the seam gets these deltas, the approximant
// normalize_leaf_values' document-weighted centring x lr (boosting.rs:
// 2844-2880).  scratch: pw_scratch_doubles(L).
__global__ void __launch_bounds__(kPwThreads)
rk_pairleaf_kernel(int L, const long long* __restrict__ wsum, const double* __restrict__ sums, double l2, double lr,
                   int pw_shift, int centre_on, double* __restrict__ scratch, double* __restrict__ leaf_raw,
                   double* __restrict__ leaf_lrv) {
    __shared__ int s_flag;
    const int m = L - 1, tid = threadIdx.x;
    const double winv = ldexp(1.0, -pw_shift);
    double* w = scratch;
    double* A = w + (size_t)L * L;
    double* der = A + (size_t)(m > 0 ? m : 1) * (m > 0 ? m : 1);
    double* y = der + L;
    double* x = y + L;
    for (int k = tid; k < L * L; k += blockDim.x) w[k] = __dmul_rn((double)wsum[k], winv);
    for (int q = tid; q < L; q += blockDim.x) der[q] = sums[3 * q];
    __syncthreads();
    pw_leaf_values_block(w, der, L, l2, leaf_raw, A, y, x, &s_flag);
    if (tid != 0) return;
    double total = 0.0;
    for (int q = 0; q < L; ++q) total = __dadd_rn(total, sums[3 * q + 2]);
    double avg = 0.0;
    const bool centre = centre_on && fabs(total) > 1e-9;
    if (centre) {
        double acc = 0.0;
        for (int q = 0; q < L; ++q) acc = __dadd_rn(acc, __dmul_rn(leaf_raw[q], sums[3 * q + 2]));
        avg = __ddiv_rn(acc, total);
    }
    for (int q = 0; q < L; ++q) {
        double v = leaf_raw[q];
        if (centre) {
            const double wq = sums[3 * q + 2];
            v = fabs(wq) > 1e-9 ? __dsub_rn(v, avg) : 0.0;
        }
        leaf_lrv[q] = __dmul_rn(v, lr);
    }
}

unsigned grid_for(int64_t n, int threads = kMcThreads) {
    int64_t b = (n + threads - 1) / threads;
    if (b > 148 * 16) b = 148 * 16;
    return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace

struct cbgpu_multi_session {
    int device = 0, K = 0, depth = 0, F = 0, NB = 0, score_fn = 0, boot = 0, sample_from_host = 0;
    int F0 = 0;                    // float features; F0..F-1 are one-hot categorical
    int loss = 0;                  // cbgpu_loss of a multi-output session
    int diag = 0;                  // 1: the diagonal losses (OneVsAll, MultiLogloss, MultiCrossEntropy)
    double* d_tmat = nullptr;      // [K][n] label matrix of MultiLogloss / MultiCrossEntropy
    uint8_t* d_present = nullptr;  // [F - F0][NB] learn-set bins of each categorical feature
    float sample_rate = 1.0f, temp = 1.0f;
    double lr = 0.0, l2 = 0.0;
    int64_t n = 0;
    int leaf_shift = 0;
    bool target_ready = false, pending = false;
    McRng rng;
    cudaStream_t st = nullptr;
    uint8_t* bins_fm = nullptr;
    int32_t* d_bc = nullptr;
    std::vector<int32_t> bc;
    double *approx = nullptr, *weight = nullptr, *wd1 = nullptr, *sw64 = nullptr;
    float* sw32 = nullptr;
    int32_t* target = nullptr;
    long long* q = nullptr;
    uint16_t* leaf = nullptr;
    unsigned long long *hist = nullptr, *sums = nullptr;
    double *scores = nullptr, *leaf_raw = nullptr, *leaf_lrv = nullptr;
    McState *d_ms = nullptr, *h_ms = nullptr;
    TreeParams *d_tp = nullptr, *h_tp = nullptr;
    double* h_raw = nullptr;
    void* leaf_export = nullptr;
    size_t hist_cells = 0;
    // histograms over leaf-sorted row lists (all modes but the pairwise scorers)
    bool fast = false;
    int fast_pairs = 0, F_pad = 0;
    // When the one-hot features' values widen the table past the float
    // features' bins (NBf), the histogram takes two launches over the same
    // rows: features [0, wide_col) at NBf bins in the narrower-table shape,
    // [wide_col, F) (the last F0 mod 32 float features, then the one-hot
    // features, which fill a 32-lane tile's idle lanes) at NB bins.  wide_col
    // is a multiple of 32, so both launches' row slices stay 16-byte aligned;
    // 0 means one launch over all F features.
    int NBf = 0, wide_col = 0;
    uint32_t chunk_rows = kChunkRows;  // rows per histogram work item (hist_chunk_rows)
    uint8_t* bins_rm = nullptr;            // u8 [n][F_pad]
    uint4* qpairs = nullptr;               // [fast_pairs][n] packed channel pairs
    unsigned long long* fbuilt = nullptr;  // [fast_pairs][F][slots][NB][2] built children
    unsigned long long* fcur[2] = {nullptr, nullptr};  // [fast_pairs][F][L/2][NB][2] prefix, two levels
    size_t fbuilt_cells = 0, fcur_cells = 0;            // per pair
    uint32_t *flist = nullptr, *fcursor = nullptr, *fseg_rows = nullptr, *fseg_base = nullptr;
    uint8_t* fside = nullptr;
    HistChunk *fchunks0 = nullptr, *fchunks = nullptr;
    uint32_t *fn_chunks0 = nullptr, *fn_chunks = nullptr;
    size_t fchunk_cap = 0;
    TreeState* fts = nullptr;  // partition bookkeeping: first cursor, work-list errors
    // ranking mode (grouped losses, K = 1)
    int rank_mode = -1;  // -1: MultiClass; kRankQueryRmse / kRankPairLogit / kRankPairLogitPairwise
    int n_groups = 0;
    int64_t *d_goff = nullptr, *d_cstart = nullptr, *d_closer = nullptr;
    double *d_eff = nullptr, *d_der2 = nullptr, *d_tgt = nullptr;
    // PairLogitPairwise: winner per competitor slot (losers are d_closer),
    // the level's pair statistics, the leaf pair-weight matrix, scratch
    int64_t n_pairs = 0;
    int64_t* d_pwin = nullptr;
    // PairLogit: each document's loser slots (competitor indices k with
    // closer[k] == doc, ascending), their offsets, exp(approx) scratch
    int64_t *d_lstart = nullptr, *d_lpair = nullptr;
    double* d_pex = nullptr;
    double* d_pairw = nullptr;  // [n_pairs] pair weight per competitor slot (closer order)
    // YetiRankPairwise: the tree's sampled pairs as a list (rk_yeti_compact_kernel)
    int64_t *d_ypw = nullptr, *d_ypl = nullptr;
    long long* d_ypq = nullptr;
    unsigned long long* d_ypn = nullptr;
    int64_t ycap = 0;
    long long *d_pstat = nullptr, *d_pwsum = nullptr;
    int pw_shift = 0;  // pair weights in the statistics: llrint(w * 2^pw_shift)
    double* d_pwscratch = nullptr;
    double raw_l2 = 0.0;
    double sm_lambda = 0.01, sm_beta = 1.0;
    // LambdaMart: sigma / top / norm, position denominators, per-group ideal
    // DCG (filled at the first grow, when the target arrives), sort scratch
    double lm_sigma = 1.0;
    int64_t lm_top = -1;
    int32_t lm_norm = 1;
    int32_t lm_no_op = 0;  // LambdaMart metric MRR / ERR / MAP
    std::vector<int64_t> h_goff;
    double *d_lmden = nullptr, *d_lmideal = nullptr;
    int32_t* d_lmorder = nullptr;
    // YetiRank: the seeder's context stream, group weights, per-tree query
    // seeds (deriv, learning fold, leaf values), the dense per-group pair
    // matrices, sort scratch, the learning-fold approximant and its deltas
    McRng yeti_rng;
    int yeti_perms = 10;
    double yeti_decay = 0.85;
    double* d_gw = nullptr;
    uint64_t *d_yseeds = nullptr, *h_yseeds = nullptr;
    int64_t* d_cwoff = nullptr;
    float* d_cw = nullptr;
    double *d_yboot = nullptr, *d_lapprox = nullptr, *d_ylf_raw = nullptr, *d_ylf_lrv = nullptr;
    double* d_ydecay = nullptr;  // decay^k by successive multiplications, k < largest group
    // ranking leaf sums through a stable sort by leaf: per-(tile, leaf) counts
    // and offsets, leaf runs, the three value arrays
    uint32_t *d_lscnt = nullptr, *d_lsoff = nullptr, *d_lsrun = nullptr;
    double* d_lsval = nullptr;
    // StochasticRank: metric / sigma / mu / samples and per-group scratch
    int srank_ndcg = 1, srank_num_est = 1;
    double srank_sigma = 1.0, srank_mu = 0.0;
    double* d_srank_ws = nullptr;

    ~cbgpu_multi_session() {
        if (st) cudaStreamSynchronize(st);
        cudaFree(d_srank_ws);
        cudaFree(d_tmat);
        cudaFree(d_present);
        cudaFree(d_gw);
        cudaFree(d_yseeds);
        if (h_yseeds) cudaFreeHost(h_yseeds);
        cudaFree(d_cwoff);
        cudaFree(d_cw);
        cudaFree(d_yboot);
        cudaFree(d_ydecay);
        cudaFree(d_lscnt);
        cudaFree(d_lsoff);
        cudaFree(d_lsrun);
        cudaFree(d_lsval);
        cudaFree(d_lapprox);
        cudaFree(d_ylf_raw);
        cudaFree(d_ylf_lrv);
        cudaFree(d_lmden);
        cudaFree(d_lmideal);
        cudaFree(d_lmorder);
        cudaFree(d_pwin);
        cudaFree(d_lstart);
        cudaFree(d_lpair);
        cudaFree(d_pex);
        cudaFree(d_pairw);
        cudaFree(d_ypw);
        cudaFree(d_ypl);
        cudaFree(d_ypq);
        cudaFree(d_ypn);
        cudaFree(d_pstat);
        cudaFree(d_pwsum);
        cudaFree(d_pwscratch);
        cudaFree(d_goff);
        cudaFree(d_cstart);
        cudaFree(d_closer);
        cudaFree(d_eff);
        cudaFree(d_der2);
        cudaFree(d_tgt);
        cudaFree(bins_fm);
        cudaFree(bins_rm);
        cudaFree(qpairs);
        cudaFree(fbuilt);
        cudaFree(fcur[0]);
        cudaFree(fcur[1]);
        cudaFree(flist);
        cudaFree(fcursor);
        cudaFree(fseg_rows);
        cudaFree(fseg_base);
        cudaFree(fside);
        cudaFree(fchunks0);
        cudaFree(fchunks);
        cudaFree(fn_chunks0);
        cudaFree(fn_chunks);
        cudaFree(fts);
        cudaFree(d_bc);
        cudaFree(approx);
        cudaFree(weight);
        cudaFree(wd1);
        cudaFree(sw64);
        cudaFree(sw32);
        cudaFree(target);
        cudaFree(q);
        cudaFree(leaf);
        cudaFree(hist);
        cudaFree(sums);
        cudaFree(scores);
        cudaFree(leaf_raw);
        cudaFree(leaf_lrv);
        cudaFree(d_ms);
        cudaFree(d_tp);
        cudaFree(leaf_export);
        if (h_ms) cudaFreeHost(h_ms);
        if (h_tp) cudaFreeHost(h_tp);
        if (h_raw) cudaFreeHost(h_raw);
        if (st) cudaStreamDestroy(st);
    }
};

namespace {

template <typename T>
int mdalloc(T** p, size_t count) {
    cudaError_t e = cudaMalloc((void**)p, sizeof(T) * (count ? count : 1));
    if (e != cudaSuccess)
        return mfail(e == cudaErrorMemoryAllocation ? CBGPU_ERR_OOM : CBGPU_ERR_CUDA, "cudaMalloc(%zu bytes): %s",
                     sizeof(T) * count, cudaGetErrorString(e));
    return CBGPU_OK;
}

#define MDA(p, count)                        \
    do {                                     \
        int _rc = mdalloc(&(p), (count));    \
        if (_rc) return _rc;                 \
    } while (0)

template <typename T>
int mhalloc(T** p, size_t count) {
    cudaError_t e = cudaMallocHost((void**)p, sizeof(T) * (count ? count : 1));
    if (e != cudaSuccess) return mfail(CBGPU_ERR_OOM, "cudaMallocHost: %s", cudaGetErrorString(e));
    memset((void*)*p, 0, sizeof(T) * (count ? count : 1));
    return CBGPU_OK;
}

int begin_impl(const cbgpu_begin_args* a, int32_t K, const float* const* cols, const double* borders_flat,
               const int32_t* border_counts, int32_t n_cat, const uint32_t* const* cat_cols,
               cbgpu_multi_session* s) {
    s->device = a->device;
    s->K = K;
    s->depth = a->depth;
    s->F0 = a->n_features;
    s->F = a->n_features + n_cat;
    s->loss = a->loss;
    s->diag = a->loss == CBGPU_LOSS_RMSE_WITH_UNCERTAINTY
                  ? 2
                  : (a->loss == CBGPU_LOSS_MULTICLASS_ONE_VS_ALL || a->loss == CBGPU_LOSS_MULTILOGLOSS ||
                     a->loss == CBGPU_LOSS_MULTICROSSENTROPY);
    s->score_fn = a->score_function;
    s->boot = a->bootstrap_type;
    s->sample_from_host = a->sample_from_host;
    s->sample_rate = a->sample_rate;
    s->temp = a->bagging_temperature;
    s->lr = a->learning_rate;
    s->l2 = a->scaled_l2;
    s->n = a->n;
    s->rng.r = Rng64::from_seed(a->rng_seed);
    s->bc.assign(border_counts, border_counts + s->F0);
    int maxb = 0;
    for (int f = 0; f < s->F0; ++f) maxb = std::max(maxb, (int)s->bc[(size_t)f]);
    s->NB = maxb + 1;
    // one-hot columns: u8 bins and the learn-set presence of each bin
    std::vector<uint8_t> cat_u8((size_t)n_cat * (size_t)std::max<int64_t>(a->n, 0));
    for (int c = 0; c < n_cat; ++c) {
        uint32_t mx = 0;
        for (int64_t i = 0; i < a->n; ++i) {
            const uint32_t v = cat_cols[c][i];
            if (v > 255) return mfail(CBGPU_DECLINED, "multi_begin: categorical feature %d has bin %u (> 255)", c, v);
            mx = std::max(mx, v);
            cat_u8[(size_t)c * a->n + i] = (uint8_t)v;
        }
        s->bc.push_back((int32_t)mx + 1);
        s->NB = std::max(s->NB, (int)mx + 1);
    }
    const int64_t n = s->n;
    const int F = s->F, C = K + 1, L = 1 << s->depth, pk = K * (K + 1) / 2;
    MCU(cudaSetDevice(s->device));
    MCU(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking));
    MDA(s->bins_fm, (size_t)F * n);
    MDA(s->d_bc, F);
    if (n_cat > 0) {
        std::vector<uint8_t> present((size_t)n_cat * s->NB, 0);
        for (int c = 0; c < n_cat; ++c)
            for (int64_t i = 0; i < n; ++i) present[(size_t)c * s->NB + cat_u8[(size_t)c * n + i]] = 1;
        MDA(s->d_present, present.size());
        MCU(cudaMemcpy(s->d_present, present.data(), present.size(), cudaMemcpyHostToDevice));
        MCU(cudaMemcpy(s->bins_fm + (size_t)s->F0 * n, cat_u8.data(), cat_u8.size(), cudaMemcpyHostToDevice));
    } else {
        MDA(s->d_present, 1);
    }
    MDA(s->approx, (size_t)K * n);
    MDA(s->wd1, (size_t)K * n);
    MDA(s->q, (size_t)C * n);
    MDA(s->target, n);
    if (a->loss == CBGPU_LOSS_MULTILOGLOSS || a->loss == CBGPU_LOSS_MULTICROSSENTROPY) MDA(s->d_tmat, (size_t)K * n);
    if (a->loss == CBGPU_LOSS_RMSE_WITH_UNCERTAINTY) MDA(s->d_tmat, n);
    MDA(s->leaf, n);
    MDA(s->sw32, n);
    MDA(s->sw64, n);
    s->hist_cells = (size_t)(L / 2) * F * s->NB * C;  // the deepest level has L/2 parents
    MDA(s->hist, s->hist_cells);
    MDA(s->scores, (size_t)F * s->NB);
    MDA(s->sums, (size_t)L * std::max(K + pk, 3));  // the ranking mode keeps 3 sums per leaf
    MDA(s->leaf_raw, (size_t)L * K);
    MDA(s->leaf_lrv, (size_t)L * K);
    MDA(s->d_ms, 1);
    MDA(s->d_tp, 1);
    {
        int rc = mhalloc(&s->h_ms, 1);
        if (rc) return rc;
        rc = mhalloc(&s->h_tp, 1);
        if (rc) return rc;
        rc = mhalloc(&s->h_raw, (size_t)L * K);
        if (rc) return rc;
    }
    MCU(cudaMemcpyAsync(s->d_bc, s->bc.data(), sizeof(int32_t) * F, cudaMemcpyHostToDevice, s->st));
    MCU(cudaMemsetAsync(s->approx, 0, sizeof(double) * (size_t)K * n, s->st));  // bias 0 (boost_from_average off)
    MCU(cudaMemsetAsync(s->leaf, 0, sizeof(uint16_t) * (size_t)n, s->st));
    double max_w = 1.0;
    if (a->weight) {
        MDA(s->weight, n);
        MCU(cudaMemcpyAsync(s->weight, a->weight, sizeof(double) * n, cudaMemcpyHostToDevice, s->st));
        max_w = 0.0;
        for (int64_t i = 0; i < n; ++i) max_w = std::max(max_w, std::fabs(a->weight[i]));
    }
    // leaf sums: |w * der1| <= max|w|, |w * der2| <= max|w| / 4: max * 2^shift * n < 2^62
    {
        int e = 0;
        if (max_w > 0.0) std::frexp(max_w, &e);
        int t = 0;
        while (t < 62 && (1ll << t) < n) ++t;
        s->leaf_shift = 61 - e - t;
    }
    // device quantization of each column (histogram.rs:159-165 bin_of)
    float* d_col = nullptr;
    double* d_b = nullptr;
    uint32_t* d_err = nullptr;
    MDA(d_col, n);
    MDA(d_b, 256);
    MDA(d_err, 1);
    MCU(cudaMemsetAsync(d_err, 0, sizeof(uint32_t), s->st));
    int64_t off = 0;
    int rc = CBGPU_OK;
    for (int f = 0; f < s->F0 && rc == CBGPU_OK; ++f) {
        const int nb = s->bc[(size_t)f];
        cudaError_t e = cudaMemcpyAsync(d_col, cols[f], sizeof(float) * n, cudaMemcpyHostToDevice, s->st);
        if (e == cudaSuccess && nb > 0)
            e = cudaMemcpyAsync(d_b, borders_flat + off, sizeof(double) * nb, cudaMemcpyHostToDevice, s->st);
        if (e != cudaSuccess) rc = mfail(CBGPU_ERR_CUDA, "column upload: %s", cudaGetErrorString(e));
        else launch_quantize_column(d_col, n, d_b, nb, s->bins_fm + (size_t)f * n, d_err, s->st);
        off += nb;
        // the staging buffers are reused by the next column: wait for this one
        if (rc == CBGPU_OK && cudaStreamSynchronize(s->st) != cudaSuccess)
            rc = mfail(CBGPU_ERR_CUDA, "quantize column %d failed", f);
    }
    cudaFree(d_col);
    cudaFree(d_b);
    cudaFree(d_err);
    if (rc) return rc;
    MCU(cudaStreamSynchronize(s->st));
    return CBGPU_OK;
}

// Per-leaf sequential f64 sums (der1, der2 or the row count, weight) of the
// ranking arm in object order, through the stable sort by leaf.
int rk_leafsums(cbgpu_multi_session* s, int count, double* sums, cudaStream_t st) {
    const int64_t n = s->n;
    const int L = 1 << s->depth;
    const int tiles = (int)((n + kLsTile - 1) / kLsTile);
    if (tiles == 0) {
        MCU(cudaMemsetAsync(sums, 0, sizeof(double) * 3 * (size_t)L, st));
        return CBGPU_OK;
    }
    if (!s->d_lscnt) {
        MDA(s->d_lscnt, (size_t)tiles * L);
        MDA(s->d_lsoff, (size_t)tiles * L);
        MDA(s->d_lsrun, 2 * (size_t)L);
        MDA(s->d_lsval, 3 * (size_t)n);
    }
    double* v = s->d_lsval;
    rk_leafcount_kernel<<<tiles, kLsThreads, 0, st>>>(n, L, s->leaf, s->d_lscnt, s->d_ms);
    rk_leafscan_kernel<<<1, kLsMaxLeaves, 0, st>>>(tiles, L, s->d_lscnt, s->d_lsoff, s->d_lsrun, s->d_lsrun + L);
    rk_leafscatter_kernel<<<tiles, kLsThreads, 0, st>>>(n, L, s->leaf, s->d_lsoff, s->wd1, s->d_der2, s->weight, count,
                                                        v, v + n, v + 2 * n);
    rk_leafsum_runs_kernel<<<L, kLsThreads, 0, st>>>(L, s->d_lsrun, s->d_lsrun + L, v, v + n, v + 2 * n, sums);
    MCU(cudaGetLastError());
    return CBGPU_OK;
}

// Buffers of the list-based histograms: row-major bins, packed channel pairs,
// the built / level tables of every pair, the row list with its per-parent
// segments, the work lists.  Called once, at the first tree of a mode that
// uses them.
int fast_setup(cbgpu_multi_session* s) {
    const int64_t n = s->n;
    const int F = s->F, NB = s->NB, C = s->K + 1, L = 1 << s->depth;
    cudaStream_t st = s->st;
    s->fast_pairs = (C + 1) / 2;
    const int F0 = s->F0;
    int maxb = 0;
    for (int f = 0; f < F0; ++f) maxb = std::max(maxb, (int)s->bc[(size_t)f]);
    s->NBf = maxb + 1;
    s->wide_col = F0 < F && hist_lane_features(s->NBf) > hist_lane_features(NB) ? F0 / 32 * 32 : 0;
    s->F_pad = (F + 31) / 32 * 32;
    {
        int sms = 0;
        MCU(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, s->device));
        const int tiles = (s->wide_col ? hist_tiles(s->wide_col, s->NBf) : 0) + hist_tiles(F - s->wide_col, NB);
        s->chunk_rows = hist_chunk_rows(n, tiles, s->fast_pairs, sms);
    }
    MDA(s->bins_rm, (size_t)std::max<int64_t>(n, 1) * s->F_pad);
    MDA(s->qpairs, (size_t)s->fast_pairs * std::max<int64_t>(n, 1));
    s->fbuilt_cells = (size_t)F * std::max(1, L / 4) * NB * 2;
    s->fcur_cells = (size_t)F * std::max(1, L / 2) * NB * 2;
    MDA(s->fbuilt, s->fbuilt_cells * s->fast_pairs);
    MDA(s->fcur[0], s->fcur_cells * s->fast_pairs);
    MDA(s->fcur[1], s->fcur_cells * s->fast_pairs);
    MDA(s->flist, std::max<int64_t>(n, 1));
    MDA(s->fcursor, 2 * kSegMax);
    MDA(s->fseg_rows, 2 * kSegMax);
    MDA(s->fseg_base, 2 * kSegMax);
    MDA(s->fside, kSegMax);
    s->fchunk_cap = (size_t)(n / s->chunk_rows) + (L / 2) + 2;
    MDA(s->fchunks, s->fchunk_cap);
    MDA(s->fn_chunks, 1);
    MDA(s->fchunks0, (size_t)(n / s->chunk_rows) + 2);
    MDA(s->fn_chunks0, 1);
    MDA(s->fts, 1);
    MCU(cudaMemsetAsync(s->fts, 0, sizeof(TreeState), st));
    if (n > 0) launch_transpose_fm_to_rm(s->bins_fm, n, n, F, s->bins_rm, s->F_pad, st);
    launch_level0_chunks(n, s->fchunks0, (uint32_t)(n / s->chunk_rows) + 2, s->fn_chunks0,
                         (uint32_t*)((char*)s->fts + offsetof(TreeState, err)), s->chunk_rows, st);
    MCU(cudaGetLastError());
    MCU(cudaStreamSynchronize(st));
    s->fast = true;
    return CBGPU_OK;
}

}  // namespace

int cbgpu_multi_begin_raw(const cbgpu_begin_args* a, int32_t approx_dim, const float* const* float_columns,
                          const double* borders_flat, const int32_t* border_counts, cbgpu_multi_session** out) {
    return cbgpu_multi_begin_cat_raw(a, approx_dim, float_columns, borders_flat, border_counts, 0, nullptr, out);
}

int cbgpu_multi_begin_cat_raw(const cbgpu_begin_args* a, int32_t approx_dim, const float* const* float_columns,
                              const double* borders_flat, const int32_t* border_counts, int32_t n_cat,
                              const uint32_t* const* cat_columns, cbgpu_multi_session** out) {
    if (!out) return mfail(CBGPU_ERR_INVALID, "multi_begin: out is NULL");
    *out = nullptr;
    if (!a || !border_counts || (a->n > 0 && a->n_features > 0 && !float_columns) || n_cat < 0 ||
        (n_cat > 0 && a->n > 0 && !cat_columns))
        return mfail(CBGPU_ERR_INVALID, "multi_begin: bad arguments");
    if (n_cat > 0) {
        for (int c = 0; c < n_cat; ++c)
            if (!cat_columns[c]) return mfail(CBGPU_ERR_INVALID, "multi_begin: categorical column %d is NULL", c);
        // upstream rejects one-hot columns whenever draws are active (tree.rs:1403-1420)
        if (a->bootstrap_type != CBGPU_BOOT_NO || a->sample_from_host)
            return mfail(CBGPU_DECLINED, "multi_begin: one-hot categorical features need bootstrap No");
    }
    // the coverage this arm accepts; everything else declines to the CPU grower
    const bool labels = a->loss == CBGPU_LOSS_MULTILOGLOSS || a->loss == CBGPU_LOSS_MULTICROSSENTROPY;
    const bool uncertainty = a->loss == CBGPU_LOSS_RMSE_WITH_UNCERTAINTY;
    if (a->loss != CBGPU_LOSS_MULTICLASS && a->loss != CBGPU_LOSS_MULTICLASS_ONE_VS_ALL && !labels && !uncertainty)
        return mfail(CBGPU_DECLINED, "multi_begin: loss %d is not a covered multi-output loss", a->loss);
    // its leaf sums take the tree's score shift, which a bootstrap sample would shrink
    if (uncertainty && (approx_dim != 2 || a->bootstrap_type != CBGPU_BOOT_NO || a->sample_from_host))
        return mfail(CBGPU_DECLINED, "multi_begin: RMSEWithUncertainty needs approx_dim 2 and bootstrap No");
    if (a->grow_policy != CBGPU_GROW_SYMMETRIC || !a->boosting_type_is_plain || a->fold_count != 1)
        return mfail(CBGPU_DECLINED, "multi_begin: only Plain SymmetricTree with one fold");
    if (a->score_function != CBGPU_SCORE_COSINE && a->score_function != CBGPU_SCORE_L2 &&
        a->score_function != CBGPU_SCORE_SOLAR_L2 && a->score_function != CBGPU_SCORE_LOO_L2 &&
        a->score_function != CBGPU_SCORE_SAT_L2)
        return mfail(CBGPU_DECLINED, "multi_begin: score function not covered");
    if (a->random_strength != 0.0) return mfail(CBGPU_DECLINED, "multi_begin: random_strength != 0");
    if (a->bootstrap_type == CBGPU_BOOT_MVS || a->bootstrap_type == CBGPU_BOOT_POISSON)
        return mfail(CBGPU_DECLINED, "multi_begin: MVS / Poisson not covered on this arm");
    if (a->world_size != 1) return mfail(CBGPU_DECLINED, "multi_begin: one GPU per multi-output session");
    if (approx_dim < (labels ? 1 : 2) || approx_dim > kMcMaxK)
        return mfail(CBGPU_DECLINED, "multi_begin: approx_dim %d outside %d..%d", approx_dim, labels ? 1 : 2,
                     kMcMaxK);
    if (a->depth < 1 || a->depth > kMcMaxDepth)
        return mfail(CBGPU_DECLINED, "multi_begin: depth %d outside 1..%d", a->depth, kMcMaxDepth);
    // histogram grids index row chunks in gridDim.z (at most 65535 chunks)
    if (a->n < 1 || a->n > (int64_t)65535 * kMcChunk || a->n_features < 0 || a->n_features + n_cat < 1 ||
        a->n_features + n_cat > 65535)
        return mfail(CBGPU_ERR_INVALID, "multi_begin: n must be 1..%lld and features 1..65535",
                     (long long)65535 * kMcChunk);
    for (int f = 0; f < a->n_features; ++f)
        if (border_counts[f] < 0 || border_counts[f] > 255)
            return mfail(CBGPU_DECLINED, "multi_begin: feature %d has %d borders (> 255)", f, border_counts[f]);
    {
        int64_t off = 0;
        for (int f = 0; f < a->n_features; ++f) {
            for (int k = 1; k < border_counts[f]; ++k)
                if (!(borders_flat[off + k - 1] < borders_flat[off + k]))
                    return mfail(CBGPU_ERR_INVALID, "multi_begin: borders of feature %d are not ascending", f);
            off += border_counts[f];
        }
    }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return mfail(CBGPU_ERR_NO_DEVICE, "no CUDA device");
    if (a->device < 0 || a->device >= ndev) return mfail(CBGPU_ERR_INVALID, "multi_begin: bad device");
    auto* s = new cbgpu_multi_session();
    const int rc = begin_impl(a, approx_dim, float_columns, borders_flat, border_counts, n_cat, cat_columns, s);
    if (rc) {
        delete s;
        return rc;
    }
    *out = s;
    return CBGPU_OK;
}

int cbgpu_rank_begin_raw(const cbgpu_begin_args* a, const int64_t* group_offsets, int32_t n_groups,
                         const int64_t* pair_winner, const int64_t* pair_loser, int64_t n_pairs,
                         const cbgpu_rank_params* params, const float* const* float_columns, const double* borders_flat, const int32_t* border_counts,
                         cbgpu_multi_session** out) {
    if (!out) return mfail(CBGPU_ERR_INVALID, "rank_begin: out is NULL");
    *out = nullptr;
    if (!a || !border_counts || !group_offsets || (a->n > 0 && !float_columns) ||
        (n_pairs > 0 && (!pair_winner || !pair_loser)) || n_pairs < 0)
        return mfail(CBGPU_ERR_INVALID, "rank_begin: bad arguments");
    int mode;
    if (a->loss == CBGPU_LOSS_QUERYRMSE) mode = kRankQueryRmse;
    else if (a->loss == CBGPU_LOSS_PAIRLOGIT) mode = kRankPairLogit;
    else if (a->loss == CBGPU_LOSS_PAIRLOGIT_PAIRWISE) mode = kRankPairLogitPairwise;
    else if (a->loss == CBGPU_LOSS_QUERYSOFTMAX) mode = kRankQuerySoftMax;
    else if (a->loss == CBGPU_LOSS_LAMBDAMART) mode = kRankLambdaMart;
    else if (a->loss == CBGPU_LOSS_YETIRANK) mode = kRankYetiRank;
    else if (a->loss == CBGPU_LOSS_STOCHASTICRANK) mode = kRankStochasticRank;
    else if (a->loss == CBGPU_LOSS_YETIRANK_PAIRWISE) mode = kRankYetiRankPairwise;
    else return mfail(CBGPU_DECLINED, "rank_begin: loss %d is not a covered grouped loss", a->loss);
    const double l2_leaf_reg = params && params->l2_leaf_reg >= 0.0 ? params->l2_leaf_reg : a->scaled_l2;
    const double sm_lambda = params ? params->softmax_lambda : 0.01;
    const double sm_beta = params ? params->softmax_beta : 1.0;
    if (mode == kRankQuerySoftMax && !(std::isfinite(sm_lambda) && sm_lambda >= 0.0 && std::isfinite(sm_beta) &&
                                       sm_beta > 0.0))  // LossFunction validation (runtime.rs:698-715)
        return mfail(CBGPU_ERR_INVALID, "rank_begin: QuerySoftMax needs lambda >= 0 and beta > 0, finite");
    const double lm_sigma = params ? params->lambdamart_sigma : 1.0;
    const int64_t lm_top = params ? params->lambdamart_top : -1;
    const int yeti_perms = params ? params->yeti_permutations : 10;
    const double yeti_decay = params ? params->yeti_decay : 0.85;
    if (mode == kRankYetiRank || mode == kRankYetiRankPairwise) {
        if (yeti_perms < 1 || !std::isfinite(yeti_decay))
            return mfail(CBGPU_ERR_INVALID, "rank_begin: YetiRank needs permutations >= 1 and a finite decay");
        int64_t cells = 0;
        for (int g = 0; g < n_groups; ++g) {
            const int64_t sz = group_offsets[g + 1] - group_offsets[g];
            cells += sz * sz;
        }
        if (cells > ((int64_t)1 << 31))
            return mfail(CBGPU_DECLINED, "rank_begin: YetiRank pair matrices need %lld cells (> 2^31)",
                         (long long)cells);
    }
    if (mode == kRankStochasticRank && params) {
        if (params->srank_metric != 0 && params->srank_metric != 1)
            return mfail(CBGPU_DECLINED, "rank_begin: StochasticRank covers the NDCG / DCG metrics");
        if (!(std::isfinite(params->srank_sigma) && params->srank_sigma > 0.0) ||
            !(std::isfinite(params->srank_mu) && params->srank_mu >= 0.0) || params->srank_num_estimations < 1)
            return mfail(CBGPU_ERR_INVALID, "rank_begin: StochasticRank needs sigma > 0, mu >= 0 and "
                                            "num_estimations >= 1");
    }
    if (mode == kRankLambdaMart) {
        if (params && (params->lambdamart_metric < 0 || params->lambdamart_metric > 4))
            return mfail(CBGPU_ERR_INVALID, "rank_begin: LambdaMart metric %d is not NDCG / DCG / MRR / ERR / MAP",
                         params->lambdamart_metric);
        if (!(std::isfinite(lm_sigma) && lm_sigma > 0.0) || !(lm_top == -1 || lm_top > 0))
            return mfail(CBGPU_ERR_INVALID, "rank_begin: LambdaMart needs sigma > 0 and top > 0 or -1");
    }
    if (a->grow_policy != CBGPU_GROW_SYMMETRIC || !a->boosting_type_is_plain || a->fold_count != 1)
        return mfail(CBGPU_DECLINED, "rank_begin: only Plain SymmetricTree with one fold");
    if (a->score_function != CBGPU_SCORE_COSINE && a->score_function != CBGPU_SCORE_L2 &&
        a->score_function != CBGPU_SCORE_SOLAR_L2 && a->score_function != CBGPU_SCORE_LOO_L2 &&
        a->score_function != CBGPU_SCORE_SAT_L2)
        return mfail(CBGPU_DECLINED, "rank_begin: score function not covered");
    if (a->random_strength != 0.0 || a->bootstrap_type != CBGPU_BOOT_NO || a->sample_from_host)
        return mfail(CBGPU_DECLINED, "rank_begin: bootstrap / random_strength not covered on this arm");
    if (a->world_size != 1) return mfail(CBGPU_DECLINED, "rank_begin: one GPU per ranking session");
    if (a->depth < 1 || a->depth > kMcMaxDepth)
        return mfail(CBGPU_DECLINED, "rank_begin: depth %d outside 1..%d", a->depth, kMcMaxDepth);
    if (mode == kRankPairLogitPairwise || mode == kRankYetiRankPairwise) {
        if (a->depth > kPwMaxDepth)
            return mfail(CBGPU_DECLINED, "rank_begin: pairwise scoring covers depth 1..%d, got %d", kPwMaxDepth,
                         a->depth);
        if (!(l2_leaf_reg >= 0.0) || !std::isfinite(l2_leaf_reg))
            return mfail(CBGPU_ERR_INVALID, "rank_begin: l2_leaf_reg must be finite and >= 0");
        if (n_pairs >= ((int64_t)1 << 31) || a->n_features > 65535)
            return mfail(CBGPU_DECLINED, "rank_begin: pairwise scoring counts pairs in int32 and features in "
                                         "gridDim.y");
        int maxb = 0;
        for (int f = 0; f < a->n_features; ++f) maxb = std::max(maxb, (int)border_counts[f]);
        const size_t P = (size_t)1 << (a->depth - 1);
        const size_t bytes = (size_t)a->n_features * P * P * (size_t)(maxb + 1) * 2 * sizeof(long long);
        if (bytes > kPwMaxStatBytes)
            return mfail(CBGPU_DECLINED, "rank_begin: pair statistics need %zu bytes (> %zu)", bytes,
                         kPwMaxStatBytes);
    }
    const int64_t n = a->n;
    if (n < 1 || n > (int64_t)65535 * kMcChunk || a->n_features < 1)
        return mfail(CBGPU_ERR_INVALID, "rank_begin: bad n / n_features");
    for (int f = 0; f < a->n_features; ++f)
        if (border_counts[f] < 0 || border_counts[f] > 255)
            return mfail(CBGPU_DECLINED, "rank_begin: feature %d has %d borders (> 255)", f, border_counts[f]);
    {
        int64_t off = 0;
        for (int f = 0; f < a->n_features; ++f) {
            for (int k = 1; k < border_counts[f]; ++k)
                if (!(borders_flat[off + k - 1] < borders_flat[off + k]))
                    return mfail(CBGPU_ERR_INVALID, "rank_begin: borders of feature %d are not ascending", f);
            off += border_counts[f];
        }
    }
    // contiguous groups over object order (query.h:48-67)
    if (n_groups < 1 || group_offsets[0] != 0 || group_offsets[n_groups] != n)
        return mfail(CBGPU_ERR_INVALID, "rank_begin: group offsets must run from 0 to n");
    std::vector<int32_t> group_of((size_t)n);
    for (int g = 0; g < n_groups; ++g) {
        if (group_offsets[g + 1] < group_offsets[g])
            return mfail(CBGPU_ERR_INVALID, "rank_begin: group offsets decrease at group %d", g);
        for (int64_t i = group_offsets[g]; i < group_offsets[g + 1]; ++i) group_of[(size_t)i] = g;
    }
    // competitors (query_info.rs:205-250): pairs in input order on their
    // winner's row, weight 1; the pairwise weights count the incident pairs
    // (calc_pairwise_weights, boosting.rs:1761-1780)
    std::vector<int64_t> cstart((size_t)n + 1, 0), closer((size_t)std::max<int64_t>(n_pairs, 1));
    std::vector<double> eff((size_t)n, 0.0);
    std::vector<int64_t> win, lstart, lpair;
    std::vector<double> slot_w;
    const double* pair_weight = params ? params->pair_weight : nullptr;
    if (pair_weight && (mode == kRankPairLogit || mode == kRankPairLogitPairwise)) {
        for (int64_t k = 0; k < n_pairs; ++k) {
            if (!std::isfinite(pair_weight[k]))
                return mfail(CBGPU_ERR_INVALID, "rank_begin: pair %lld has a non-finite weight", (long long)k);
            if (mode == kRankPairLogitPairwise && pair_weight[k] != 1.0)
                return mfail(CBGPU_DECLINED, "rank_begin: PairLogitPairwise covers unit pair weights");
        }
    }
    if (mode == kRankPairLogit || mode == kRankPairLogitPairwise) {
        for (int64_t k = 0; k < n_pairs; ++k) {
            const int64_t wv = pair_winner[k], lv = pair_loser[k];
            if (wv < 0 || wv >= n || lv < 0 || lv >= n || group_of[(size_t)wv] != group_of[(size_t)lv])
                return mfail(CBGPU_ERR_INVALID, "rank_begin: pair (%lld, %lld) is out of range or crosses group "
                                                "boundaries", (long long)wv, (long long)lv);
            cstart[(size_t)wv + 1]++;
        }
        for (int64_t i = 0; i < n; ++i) cstart[(size_t)i + 1] += cstart[(size_t)i];
        std::vector<int64_t> fill(cstart.begin(), cstart.end() - 1);
        slot_w.assign(closer.size(), 1.0);
        for (int64_t k = 0; k < n_pairs; ++k) {
            const int64_t at = fill[(size_t)pair_winner[k]]++;
            closer[(size_t)at] = pair_loser[k];
            if (pair_weight) slot_w[(size_t)at] = pair_weight[k];
        }
        win.assign(closer.size(), 0);
        for (int64_t i = 0; i < n; ++i)
            for (int64_t k = cstart[(size_t)i]; k < cstart[(size_t)i + 1]; ++k) win[(size_t)k] = i;
        // calc_pairwise_weights: each pair adds its weight to both documents
        for (int g = 0; g < n_groups; ++g)
            for (int64_t wi = group_offsets[g]; wi < group_offsets[g + 1]; ++wi)
                for (int64_t k = cstart[(size_t)wi]; k < cstart[(size_t)wi + 1]; ++k) {
                    eff[(size_t)wi] += slot_w[(size_t)k];
                    eff[(size_t)closer[(size_t)k]] += slot_w[(size_t)k];
                }
        if (mode == kRankPairLogit) {
            // loser slots by document, ascending k: by winner, then input order
            lstart.assign((size_t)n + 1, 0);
            lpair.assign(closer.size(), 0);
            for (int64_t k = 0; k < n_pairs; ++k) lstart[(size_t)closer[(size_t)k] + 1]++;
            for (int64_t i = 0; i < n; ++i) lstart[(size_t)i + 1] += lstart[(size_t)i];
            std::vector<int64_t> lfill(lstart.begin(), lstart.end() - 1);
            for (int64_t k = 0; k < n_pairs; ++k) lpair[(size_t)lfill[(size_t)closer[(size_t)k]]++] = k;
        }
    } else {
        for (int64_t i = 0; i < n; ++i) eff[(size_t)i] = a->weight ? a->weight[i] : 1.0;
    }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return mfail(CBGPU_ERR_NO_DEVICE, "no CUDA device");
    if (a->device < 0 || a->device >= ndev) return mfail(CBGPU_ERR_INVALID, "rank_begin: bad device");
    auto* s = new cbgpu_multi_session();
    int rc = begin_impl(a, 1, float_columns, borders_flat, border_counts, 0, nullptr, s);
    if (!rc) {
        s->rank_mode = mode;
        s->n_groups = n_groups;
        s->sm_lambda = sm_lambda;
        s->sm_beta = sm_beta;
        s->lm_sigma = lm_sigma;
        s->lm_top = lm_top;
        s->lm_norm = params ? (params->lambdamart_norm ? 1 : 0) : 1;
        s->lm_no_op = params && params->lambdamart_metric >= 2 ? 1 : 0;
        s->h_goff.assign(group_offsets, group_offsets + n_groups + 1);
        s->yeti_perms = yeti_perms;
        s->yeti_decay = yeti_decay;
        s->yeti_rng.r = Rng64::from_seed(a->rng_seed);
        if (params) {
            s->srank_ndcg = params->srank_metric == 0 ? 1 : 0;
            s->srank_num_est = params->srank_num_estimations;
            s->srank_sigma = params->srank_sigma;
            s->srank_mu = params->srank_mu;
        }
        rc = mdalloc(&s->d_goff, (size_t)n_groups + 1);
        if (!rc) rc = mdalloc(&s->d_cstart, (size_t)n + 1);
        if (!rc) rc = mdalloc(&s->d_closer, closer.size());
        if (!rc) rc = mdalloc(&s->d_eff, (size_t)n);
        if (!rc) rc = mdalloc(&s->d_der2, (size_t)n);
        if (!rc) rc = mdalloc(&s->d_tgt, (size_t)n);
        if (!rc && mode == kRankPairLogit) {
            s->n_pairs = n_pairs;
            rc = mdalloc(&s->d_pwin, win.size());
            if (!rc) rc = mdalloc(&s->d_lstart, lstart.size());
            if (!rc) rc = mdalloc(&s->d_lpair, lpair.size());
            if (!rc) rc = mdalloc(&s->d_pex, (size_t)std::max<int64_t>(n, 1));
            if (!rc) rc = mdalloc(&s->d_pairw, slot_w.size());
        }
        if (!rc && (mode == kRankYetiRank || mode == kRankYetiRankPairwise)) {
            // group weight: the mean member weight (query_info.rs:180-187)
            std::vector<double> gw((size_t)n_groups);
            std::vector<int64_t> cwoff((size_t)n_groups);
            int64_t cells = 0;
            for (int g = 0; g < n_groups; ++g) {
                const int64_t b = group_offsets[g], e = group_offsets[g + 1];
                double acc = 0.0;
                for (int64_t i = b; i < e; ++i) acc += a->weight ? a->weight[i] : 1.0;
                gw[(size_t)g] = e > b ? acc / (double)(e - b) : 1.0;
                cwoff[(size_t)g] = cells;
                cells += (e - b) * (e - b);
            }
            rc = mdalloc(&s->d_gw, (size_t)n_groups);
            if (!rc) rc = mdalloc(&s->d_yseeds, 3 * (size_t)n_groups);
            if (!rc) rc = mhalloc(&s->h_yseeds, 3 * (size_t)n_groups);
            if (!rc) rc = mdalloc(&s->d_cwoff, (size_t)n_groups);
            if (!rc) rc = mdalloc(&s->d_cw, (size_t)std::max<int64_t>(cells, 1));
            if (!rc && mode == kRankYetiRankPairwise) {
                // a permutation adds at most g - 1 cells per group: perms * n bounds the list
                s->ycap = std::max<int64_t>(1, std::min<int64_t>(cells, (int64_t)std::max(yeti_perms, 1) * n));
                rc = mdalloc(&s->d_ypw, (size_t)s->ycap);
                if (!rc) rc = mdalloc(&s->d_ypl, (size_t)s->ycap);
                if (!rc) rc = mdalloc(&s->d_ypq, (size_t)s->ycap);
                if (!rc) rc = mdalloc(&s->d_ypn, 1);
            }
            if (!rc) rc = mdalloc(&s->d_lmorder, (size_t)n);
            if (!rc) rc = mdalloc(&s->d_yboot, (size_t)n);
            if (!rc) {
                int64_t maxg = 1;
                for (int g = 0; g < n_groups; ++g) maxg = std::max(maxg, group_offsets[g + 1] - group_offsets[g]);
                std::vector<double> dp((size_t)maxg);
                double dc = 1.0;  // the sampler's running product, one multiplication per position
                for (int64_t k = 0; k < maxg; ++k) {
                    dp[(size_t)k] = dc;
                    dc = dc * s->yeti_decay;
                }
                rc = mdalloc(&s->d_ydecay, (size_t)maxg);
                if (!rc && cudaMemcpy(s->d_ydecay, dp.data(), sizeof(double) * dp.size(), cudaMemcpyHostToDevice) !=
                               cudaSuccess)
                    rc = mfail(CBGPU_ERR_CUDA, "rank_begin: upload failed");
            }
            if (!rc) rc = mdalloc(&s->d_lapprox, (size_t)n);
            if (!rc) rc = mdalloc(&s->d_ylf_raw, (size_t)1 << a->depth);
            if (!rc) rc = mdalloc(&s->d_ylf_lrv, (size_t)1 << a->depth);
            if (!rc && (cudaMemcpy(s->d_gw, gw.data(), sizeof(double) * gw.size(), cudaMemcpyHostToDevice) !=
                            cudaSuccess ||
                        cudaMemcpy(s->d_cwoff, cwoff.data(), sizeof(int64_t) * cwoff.size(),
                                   cudaMemcpyHostToDevice) != cudaSuccess ||
                        cudaMemset(s->d_lapprox, 0, sizeof(double) * (size_t)n) != cudaSuccess))
                rc = mfail(CBGPU_ERR_CUDA, "rank_begin: upload failed");
        }
        if (!rc && mode == kRankStochasticRank) {
            rc = mdalloc(&s->d_srank_ws, 9 * (size_t)n + 3 * (size_t)n_groups);
        }
        if (!rc && (mode == kRankLambdaMart || mode == kRankStochasticRank)) {
            int64_t maxg = 1;
            for (int g = 0; g < n_groups; ++g) maxg = std::max(maxg, group_offsets[g + 1] - group_offsets[g]);
            std::vector<double> den((size_t)maxg);
            for (int64_t p = 0; p < maxg; ++p) den[(size_t)p] = std::log(2.0 + (double)p) * 1.4426950408889634;
            rc = mdalloc(&s->d_lmden, den.size());
            if (!rc) rc = mdalloc(&s->d_lmideal, (size_t)n_groups);
            if (!rc) rc = mdalloc(&s->d_lmorder, (size_t)n);
            if (!rc && cudaMemcpy(s->d_lmden, den.data(), sizeof(double) * den.size(), cudaMemcpyHostToDevice) !=
                           cudaSuccess)
                rc = mfail(CBGPU_ERR_CUDA, "rank_begin: upload failed");
        }
        if (!rc && (mode == kRankPairLogitPairwise || mode == kRankYetiRankPairwise)) {
            const int L = 1 << a->depth, P = L / 2;
            s->raw_l2 = l2_leaf_reg;
            const size_t leaf_scratch = pw_scratch_doubles(L);
            const size_t score_scratch = L > kPwSmemMaxN2 ? (size_t)kPwGlobalBlocks * pw_scratch_doubles(L) : 0;
            if (mode == kRankPairLogitPairwise) {
                // unit weights: sums of at most n_pairs units stay below 2^60
                s->n_pairs = n_pairs;
                int t = 0;
                while (t < 62 && ((int64_t)1 << t) < n_pairs + 1) ++t;
                s->pw_shift = 59 - t;
                rc = mdalloc(&s->d_pwin, win.size());
            }
            if (!rc) rc = mdalloc(&s->d_pstat, (size_t)a->n_features * P * P * s->NB * 2);
            if (!rc) rc = mdalloc(&s->d_pwsum, (size_t)L * L);
            if (!rc) rc = mdalloc(&s->d_pwscratch, std::max(leaf_scratch, score_scratch));
            const size_t smem = pw_scratch_doubles(std::min(L, kPwSmemMaxN2)) * sizeof(double);
            if (!rc && smem > 48 * 1024 &&
                cudaFuncSetAttribute(rk_pairscore_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
                    cudaSuccess)
                rc = mfail(CBGPU_ERR_CUDA, "rank_begin: pairwise scorer shared memory (%zu bytes)", smem);
        }
    }
    if (!rc) {
        cudaError_t e = cudaMemcpy(s->d_goff, group_offsets, sizeof(int64_t) * ((size_t)n_groups + 1),
                                   cudaMemcpyHostToDevice);
        if (e == cudaSuccess)
            e = cudaMemcpy(s->d_cstart, cstart.data(), sizeof(int64_t) * cstart.size(), cudaMemcpyHostToDevice);
        if (e == cudaSuccess)
            e = cudaMemcpy(s->d_closer, closer.data(), sizeof(int64_t) * closer.size(), cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(s->d_eff, eff.data(), sizeof(double) * (size_t)n, cudaMemcpyHostToDevice);
        if (e == cudaSuccess && s->d_pwin)
            e = cudaMemcpy(s->d_pwin, win.data(), sizeof(int64_t) * win.size(), cudaMemcpyHostToDevice);
        if (e == cudaSuccess && s->d_lstart)
            e = cudaMemcpy(s->d_lstart, lstart.data(), sizeof(int64_t) * lstart.size(), cudaMemcpyHostToDevice);
        if (e == cudaSuccess && s->d_lpair)
            e = cudaMemcpy(s->d_lpair, lpair.data(), sizeof(int64_t) * lpair.size(), cudaMemcpyHostToDevice);
        if (e == cudaSuccess && s->d_pairw)
            e = cudaMemcpy(s->d_pairw, slot_w.data(), sizeof(double) * slot_w.size(), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) rc = mfail(CBGPU_ERR_CUDA, "rank_begin: upload failed: %s", cudaGetErrorString(e));
    }
    if (rc) {
        delete s;
        return rc;
    }
    *out = s;
    return CBGPU_OK;
}

int cbgpu_multi_grow_tree(cbgpu_multi_session* s, const double* approx_k, const double* target, int64_t n,
                          const double* sample, int64_t sample_len, int32_t* split_feature, int32_t* split_bin,
                          int32_t* n_splits, double* leaf_values, void* leaf_of, int32_t leaf_of_bytes) {
    if (!s) return mfail(CBGPU_ERR_INVALID, "multi_grow: no session");
    if (n != s->n) return mfail(CBGPU_ERR_INVALID, "LengthMismatch: n %lld != session n %lld", (long long)n,
                                (long long)s->n);
    if (sample_len != 0 && sample_len != n)
        return mfail(CBGPU_ERR_INVALID, "LengthMismatch: sample length %lld", (long long)sample_len);
    if (sample_len != 0 && !s->sample_from_host)
        return mfail(CBGPU_ERR_INVALID, "Degenerate: a host sample without sample_from_host");
    if (sample_len == 0 && s->sample_from_host)
        return mfail(CBGPU_ERR_INVALID, "Degenerate: sample_from_host without a sample");
    if (leaf_of && leaf_of_bytes != 0 && leaf_of_bytes != 1 && leaf_of_bytes != 2 && leaf_of_bytes != 4)
        return mfail(CBGPU_ERR_INVALID, "multi_grow: leaf_of_bytes must be 1, 2 or 4");
    const int K = s->K, D = s->depth, L = 1 << D, F = s->F, NB = s->NB, C = K + 1;
    const int pk = K * (K + 1) / 2;
    cudaStream_t st = s->st;
    MCU(cudaSetDevice(s->device));
    if (!s->target_ready && s->rank_mode >= 0) {
        if (!target) return mfail(CBGPU_ERR_INVALID, "multi_grow: the first call needs the target");
        if (s->rank_mode == kRankLambdaMart || s->rank_mode == kRankStochasticRank) {
            // lambdamart_ideal_ndcg / compute_dcg_pos_weights' ideal per group:
            // the DCG of the relevance-sorted order over the top positions,
            // summed in position order (StochasticRank: the whole group, as
            // relevance x (1 / denominator))
            const int G = s->n_groups;
            std::vector<double> ideal((size_t)G), ts;
            for (int g = 0; g < G; ++g) {
                const int64_t b = s->h_goff[(size_t)g], e = s->h_goff[(size_t)g + 1], cnt = e - b;
                ts.assign(target + b, target + e);
                std::stable_sort(ts.begin(), ts.end(), [](double x, double y) { return x > y; });
                const bool srank = s->rank_mode == kRankStochasticRank;
                const int64_t top = (srank || s->lm_top == -1 || s->lm_top > cnt) ? cnt : s->lm_top;
                double acc = 0.0;
                for (int64_t p = 0; p < top; ++p) {
                    const double dn = std::log(2.0 + (double)p) * 1.4426950408889634;
                    acc += srank ? ts[(size_t)p] * (1.0 / dn) : ts[(size_t)p] / dn;
                }
                ideal[(size_t)g] = acc;
            }
            MCU(cudaMemcpyAsync(s->d_lmideal, ideal.data(), sizeof(double) * (size_t)G, cudaMemcpyHostToDevice, st));
            MCU(cudaStreamSynchronize(st));
        }
        if (s->rank_mode == kRankYetiRankPairwise) {
            // a bound on any sampled pair weight: qw * 0.15 * |rel_a - rel_b| *
            // decay^k per permutation, averaged over the permutations
            // (yetirank.rs:450-514), and on the pair count: the cells of the
            // groups' dense matrices; their product stays below 2^60
            double tmin = INFINITY, tmax = -INFINITY, gwmax = 0.0, cells = 0.0;
            int64_t maxg = 1;
            for (int64_t i = 0; i < n; ++i) {
                tmin = std::min(tmin, (double)(float)target[i]);
                tmax = std::max(tmax, (double)(float)target[i]);
            }
            std::vector<double> gw((size_t)s->n_groups);
            MCU(cudaMemcpy(gw.data(), s->d_gw, sizeof(double) * gw.size(), cudaMemcpyDeviceToHost));
            for (int g = 0; g < s->n_groups; ++g) {
                const int64_t sz = s->h_goff[(size_t)g + 1] - s->h_goff[(size_t)g];
                gwmax = std::max(gwmax, std::fabs(gw[(size_t)g]));
                maxg = std::max(maxg, sz);
                cells += (double)sz * (double)sz;
            }
            const double decay_max = s->yeti_decay > 1.0 ? std::pow(s->yeti_decay, (double)std::max<int64_t>(maxg - 2, 0))
                                                         : 1.0;
            const double bound = std::max(1e-300, 1.01 * gwmax * 0.15 * (tmax - tmin) * decay_max);
            int e = 0, t = 0;
            std::frexp(bound, &e);
            while (t < 62 && std::ldexp(1.0, t) < cells + 1.0) ++t;
            s->pw_shift = std::min(60 - e - t, 1000);
            if (s->pw_shift < 0) return mfail(CBGPU_DECLINED, "YetiRankPairwise: pair weights too large (%g)", bound);
        }
        MCU(cudaMemcpyAsync(s->d_tgt, target, sizeof(double) * n, cudaMemcpyHostToDevice, st));
        MCU(cudaStreamSynchronize(st));
        s->target_ready = true;
    }
    if (!s->target_ready && s->diag == 2) {
        if (!target) return mfail(CBGPU_ERR_INVALID, "multi_grow: the first call needs the target");
        for (int64_t i = 0; i < n; ++i)
            if (!std::isfinite(target[i]))
                return mfail(CBGPU_ERR_INVALID, "multi_grow: target %g at row %lld is not finite", target[i],
                             (long long)i);
        // the starting approximant [f32 mean, 0.5 ln f32 var] (boosting.rs:1895-1914)
        double acc = 0.0;
        for (int64_t i = 0; i < n; ++i) acc += target[i];
        const double mean = (double)(float)(acc / (double)n);
        double sq = 0.0;
        for (int64_t i = 0; i < n; ++i) sq += (target[i] - mean) * (target[i] - mean);
        const double log_scale = 0.5 * std::log((double)(float)(sq / (double)n));
        MCU(cudaMemcpyAsync(s->d_tmat, target, sizeof(double) * n, cudaMemcpyHostToDevice, st));
        mc_fill2_kernel<<<(unsigned)std::min<int64_t>((n + kMcThreads - 1) / kMcThreads, 148 * 8), kMcThreads, 0,
                          st>>>(n, s->approx, mean, log_scale);
        MCU(cudaGetLastError());
        MCU(cudaStreamSynchronize(st));
        s->target_ready = true;
    }
    if (!s->target_ready && s->d_tmat) {
        // MultiLogloss {0, 1} / MultiCrossEntropy [0, 1] labels (Loss::validate)
        if (!target) return mfail(CBGPU_ERR_INVALID, "multi_grow: the first call needs the target");
        const bool binary = s->loss == CBGPU_LOSS_MULTILOGLOSS;
        for (int64_t k = 0; k < (int64_t)K * n; ++k) {
            const double t = target[k];
            if (binary ? !(t == 0.0 || t == 1.0) : !(t >= 0.0 && t <= 1.0))
                return mfail(CBGPU_ERR_INVALID, "multi_grow: label %g of dimension %lld row %lld is outside %s", t,
                             (long long)(k / n), (long long)(k % n), binary ? "{0, 1}" : "[0, 1]");
        }
        MCU(cudaMemcpyAsync(s->d_tmat, target, sizeof(double) * (size_t)K * n, cudaMemcpyHostToDevice, st));
        MCU(cudaStreamSynchronize(st));
        s->target_ready = true;
    }
    if (!s->target_ready) {
        if (!target) return mfail(CBGPU_ERR_INVALID, "multi_grow: the first call needs the target");
        std::vector<int32_t> cls((size_t)n);
        for (int64_t i = 0; i < n; ++i) {
            const double t = target[i];
            if (!(t >= 0.0 && t < (double)K) || t != std::floor(t))
                return mfail(CBGPU_ERR_INVALID, "multi_grow: target %g at row %lld is not a class index in 0..%d", t,
                             (long long)i, K - 1);
            cls[(size_t)i] = (int32_t)t;
        }
        MCU(cudaMemcpyAsync(s->target, cls.data(), sizeof(int32_t) * n, cudaMemcpyHostToDevice, st));
        MCU(cudaStreamSynchronize(st));
        s->target_ready = true;
    }
    if (approx_k) {
        MCU(cudaMemcpyAsync(s->approx, approx_k, sizeof(double) * (size_t)K * n, cudaMemcpyHostToDevice, st));
        s->pending = false;
    }
    // bootstrap: the host stream replica decides the draws (boosting.rs:6568-6660)
    TreeParams& tp = *s->h_tp;
    tp = TreeParams{};
    int s_mode = 0, boot_mode = 0;
    if (s->sample_from_host) {
        MCU(cudaMemcpyAsync(s->sw64, sample, sizeof(double) * n, cudaMemcpyHostToDevice, st));
        s_mode = 2;
    } else if (s->boot != CBGPU_BOOT_NO) {
        s->rng.gen();  // PRE_TREE_DRAWS = 2 (boosting.rs:59)
        s->rng.gen();
        if (s->boot == CBGPU_BOOT_BAYESIAN && s->temp != 0.0f) {
            tp.boot_seed = s->rng.gen();
            boot_mode = 1;
            s_mode = 1;
        } else if (s->boot == CBGPU_BOOT_BERNOULLI && (double)s->sample_rate < 1.0) {
            tp.boot_base = s->rng.r;
            s->rng.advance((uint64_t)n);
            boot_mode = 2;
            s_mode = 1;
        }
    }
    MCU(cudaMemcpyAsync(s->d_tp, s->h_tp, sizeof(TreeParams), cudaMemcpyHostToDevice, st));
    MCU(cudaMemsetAsync(s->d_ms, 0, sizeof(McState), st));
    const unsigned g = grid_for(n);
    const bool yeti = s->rank_mode == kRankYetiRank || s->rank_mode == kRankYetiRankPairwise;
    const bool srank = s->rank_mode == kRankStochasticRank;
    const unsigned yg = (unsigned)((s->n_groups + 127) / 128);
    const unsigned yw = (unsigned)((s->n_groups + kYetiWarps - 1) / kYetiWarps);  // a warp per group
    uint64_t srank_base[2] = {0, 0};
    if (yeti || srank) {
        // YetiRankTreeSeeder::next_tree (yetirank.rs:340-430) on the host: the
        // per-group query seeds of the three resamples of this tree
        const int G = s->n_groups;
        McRng& yr = s->yeti_rng;
        auto first_gen = [](uint64_t seed) { Rng64 t = Rng64::from_seed(seed); return t.gen(); };
        auto fill = [&](uint64_t recalc, uint64_t* out) {
            Rng64 t = Rng64::from_seed(recalc);
            for (int q = 0; q < G; ++q) out[q] = first_gen(t.gen());
        };
        (void)yr.gen();  // structure-fold selection
        const uint64_t drs = first_gen(yr.gen());
        for (int l = 0; l < D; ++l) {
            for (int f = 0; f < F; ++f) (void)yr.real1();
            (void)yr.gen();
            for (int f = 0; f < F; ++f) (void)yr.std_normal();
        }
        const uint64_t lrs = first_gen(first_gen(yr.gen()));
        const uint64_t vb = yr.gen();
        if (yeti) {
            fill(drs, s->h_yseeds);
            fill(lrs, s->h_yseeds + G);
            fill(vb, s->h_yseeds + 2 * (size_t)G);
            MCU(cudaMemcpyAsync(s->d_yseeds, s->h_yseeds, sizeof(uint64_t) * 3 * (size_t)G, cudaMemcpyHostToDevice,
                                st));
        }
        srank_base[0] = drs;  // StochasticRank: the derivative and leaf-value bases
        srank_base[1] = vb;
    }
    if (s->rank_mode >= 0) {
        if (s->pending)
            mc_apply_pending_kernel<<<g, kMcThreads, 0, st>>>(n, 1, L, s->approx, s->leaf, s->leaf_lrv);
    }
    if (yeti) {
        // gradient / split ders and the histogram's pairwise weights from pairs
        // sampled off the learning-fold approximant
        rk_yeti_sample_kernel<<<yw, kYetiWarps * 32, 0, st>>>(s->n_groups, s->d_goff, s->d_lapprox, s->d_tgt, s->yeti_perms,
                                                 s->d_ydecay, s->d_yseeds, s->d_cwoff, s->d_cw, s->d_lmorder,
                                                 s->d_yboot);
        rk_yeti_der_kernel<<<yw, kYetiWarps * 32, 0, st>>>(s->n_groups, s->d_goff, s->d_lapprox, s->d_gw, s->yeti_perms,
                                              s->d_cwoff, s->d_cw, s->wd1, s->d_der2, s->d_eff, s->d_yboot, s->d_ms);
        if (s->rank_mode == kRankYetiRankPairwise) {  // the split search's pairs, as a list
            MCU(cudaMemsetAsync(s->d_ypn, 0, sizeof(unsigned long long), st));
            rk_yeti_compact_kernel<<<yw, kYetiWarps * 32, 0, st>>>(s->n_groups, s->d_goff, s->d_cwoff, s->d_cw,
                                                                   s->d_gw, s->yeti_perms, s->pw_shift, s->ycap,
                                                                   s->d_ypw, s->d_ypl, s->d_ypq, s->d_ypn, s->d_ms);
        }
    } else if (srank) {
        rk_srank_kernel<<<yg, 128, 0, st>>>(s->n_groups, s->d_goff, s->approx, s->d_tgt, s->srank_ndcg, s->srank_sigma,
                                           s->srank_mu, s->srank_num_est, srank_base[0], s->d_lmden, s->d_lmideal,
                                           s->d_srank_ws, s->d_lmorder, s->wd1, s->d_der2, s->d_ms);
    } else if (s->rank_mode == kRankPairLogit) {
        rk_pairlogit_der_kernel<<<yw, kYetiWarps * 32, 0, st>>>(s->n_groups, s->d_goff, s->d_cstart, s->d_closer,
                                                                s->d_pwin, s->d_lstart, s->d_lpair, s->d_pairw,
                                                                s->approx, s->d_pex, s->wd1, s->d_der2, s->d_ms);
    } else if (s->rank_mode >= 0) {
        rk_der_kernel<<<(unsigned)((s->n_groups + 127) / 128), 128, 0, st>>>(
            s->n_groups, s->rank_mode, s->d_goff, s->d_cstart, s->d_closer, s->approx, s->d_tgt, s->weight,
            RkLossParams{s->sm_lambda, s->sm_beta, s->lm_sigma, s->lm_top, s->lm_norm, s->d_lmden, s->d_lmideal,
                         s->d_lmorder, s->lm_no_op},
            s->wd1, s->d_der2, s->d_ms);
    } else {
        mc_der_kernel<<<g, kMcThreads, 0, st>>>(n, K, s->approx, s->target, s->weight, s->leaf, s->leaf_lrv, L,
                                                s->pending ? 1 : 0, s->diag, s->d_tmat, s->wd1, s->d_ms);
    }
    MCU(cudaGetLastError());
    s->pending = false;
    // the previous tree's leaf ids are consumed: every row starts this tree in leaf 0
    MCU(cudaMemsetAsync(s->leaf, 0, sizeof(uint16_t) * (size_t)n, st));
    if (boot_mode) launch_bootstrap(boot_mode, n, 0, s->d_tp, (double)s->sample_rate, s->temp, s->sw32, st);
    // the histogram weight channel: PairLogit's pairwise weights, else the object weights
    const double* hw = s->rank_mode >= 0 ? s->d_eff : s->weight;
    mc_max_kernel<<<g, kMcThreads, 0, st>>>(n, K, s->wd1, hw, s_mode, s->sw32, s->sw64, s->d_ms);
    const unsigned chunks = (unsigned)((n + kMcChunk - 1) / kMcChunk);
    const bool pairwise = s->rank_mode == kRankPairLogitPairwise || s->rank_mode == kRankYetiRankPairwise;
    if (!pairwise && !s->fast) {
        int rc = fast_setup(s);
        if (rc) return rc;
    }
    if (!pairwise) {
        // histograms of the built children over leaf-sorted row lists
        const int P = s->fast_pairs;
        mc_shift33_kernel<<<1, 1, 0, st>>>(s->d_ms);
        mc_pack2_kernel<<<g, kMcThreads, 0, st>>>(n, K, P, s->wd1, hw, s_mode, s->sw32, s->sw64, s->d_ms,
                                                  s->qpairs);
        MCU(cudaMemsetAsync(s->fts, 0, sizeof(TreeState), st));
        MCU(cudaGetLastError());
        const int32_t* mc_splits = (const int32_t*)((char*)s->d_ms + offsetof(McState, split));
        int cur = 0;
        for (int l = 0; l < D; ++l) {
            const int Q = 1 << l;
            const size_t slots = l == 0 ? 1 : (size_t)Q / 2;
            const size_t bcells = (size_t)F * slots * NB * 2;
            MCU(cudaMemsetAsync(s->fbuilt, 0, sizeof(unsigned long long) * s->fbuilt_cells * P, st));
            const uint32_t max_chunks = (uint32_t)(n / s->chunk_rows + slots + 1);
            // fbuilt is zeroed above, so a float feature's cells past its NBf
            // bins stay 0 when only those bins are built
            // (every channel pair in one launch: grid z)
            const int Fw = s->wide_col;
            if (Fw > 0)
                launch_hist_sets(s->bins_rm, s->F_pad, Fw, s->NBf, s->qpairs, l == 0 ? nullptr : s->flist,
                                 l == 0 ? s->fchunks0 : s->fchunks, l == 0 ? s->fn_chunks0 : s->fn_chunks,
                                 max_chunks, s->fbuilt, (int64_t)slots * NB * 2, (int64_t)NB * 2, P, n,
                                 (int64_t)bcells, st);
            launch_hist_sets(s->bins_rm + Fw, s->F_pad, F - Fw, NB, s->qpairs, l == 0 ? nullptr : s->flist,
                             l == 0 ? s->fchunks0 : s->fchunks, l == 0 ? s->fn_chunks0 : s->fn_chunks, max_chunks,
                             s->fbuilt + (size_t)Fw * slots * NB * 2, (int64_t)slots * NB * 2, (int64_t)NB * 2, P,
                             n, (int64_t)bcells, st);
            launch_derive_prefix_sets(l, F, NB, s->fbuilt, s->fcur[cur ^ 1], s->fcur[cur], s->fside, P,
                                      (int64_t)bcells, (int64_t)s->fcur_cells, st);
            mc_gather_kernel<<<grid_for((int64_t)Q * F * NB * C), kMcThreads, 0, st>>>(Q, F, NB, C, s->fcur[cur],
                                                                                     s->fcur_cells, s->hist);
            mc_score_kernel<<<(unsigned)(F * ((NB + 31) / 32)), (kMsCompute + 1) * 32, 0, st>>>(
                Q, F, NB, K, s->hist, s->d_bc, s->d_ms, s->l2, s->score_fn, s->F0, s->d_present, s->scores);
            mc_argmax_kernel<<<1, 1024, 0, st>>>((int64_t)F * NB, NB, s->scores, l, s->d_ms);
            if (l + 1 < D) {
                mc_side_kernel<<<1, 1024, 0, st>>>(l, F, NB, C, K, s->F0, s->hist, s->d_ms, s->fts, s->fside);
                const int pp = l & 1, np = pp ^ 1;
                uint32_t* cur_l = l == 0 ? (uint32_t*)((char*)s->fts + offsetof(TreeState, cursor0))
                                         : s->fcursor + (size_t)pp * kSegMax;
                const bool more = l + 2 < D;
                launch_partition(l, n, s->bins_fm, n, s->leaf, s->fside, cur_l, s->flist, mc_splits, 2, s->F0, st);
                launch_segments(l, n, l == 0 ? nullptr : s->fseg_rows + (size_t)pp * kSegMax,
                                l == 0 ? nullptr : s->fseg_base + (size_t)pp * kSegMax, cur_l, s->fside,
                                more ? s->fseg_rows + (size_t)np * kSegMax : nullptr,
                                more ? s->fseg_base + (size_t)np * kSegMax : nullptr,
                                more ? s->fcursor + (size_t)np * kSegMax : nullptr, s->fchunks,
                                (uint32_t)s->fchunk_cap, s->fn_chunks, s->fts, s->chunk_rows, st);
            } else {
                mc_route_kernel<<<g, kMcThreads, 0, st>>>(n, l, s->bins_fm, s->F0, s->d_ms, s->leaf);
            }
            MCU(cudaGetLastError());
            cur ^= 1;
        }
    }
    if (pairwise) {
        mc_shift_kernel<<<1, 1, 0, st>>>(n, s->d_ms);
        mc_pack_kernel<<<g, kMcThreads, 0, st>>>(n, K, s->wd1, hw, s_mode, s->sw32, s->sw64, s->d_ms, s->q);
        MCU(cudaGetLastError());
    }
    for (int l = 0; l < D && pairwise; ++l) {
        const int leaves = 1 << l;
        const size_t cells = (size_t)leaves * F * NB * C;
        MCU(cudaMemsetAsync(s->hist, 0, sizeof(unsigned long long) * cells, st));
        const size_t tab = (size_t)leaves * NB * sizeof(unsigned long long);
        const int use_smem = tab <= kMcSmemTable ? 1 : 0;
        if (use_smem && tab > 48 * 1024)
            MCU(cudaFuncSetAttribute(mc_hist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tab));
        // the pairwise scorer reads only the der channel
        mc_hist_kernel<<<dim3((unsigned)F, pairwise ? 1u : (unsigned)C, chunks), kMcThreads, use_smem ? tab : 0,
                         st>>>(n, F, NB, C, leaves, s->bins_fm, s->q, s->leaf, s->hist, use_smem);
        MCU(cudaGetLastError());
        mc_prefix_kernel<<<grid_for((int64_t)leaves * F * C), kMcThreads, 0, st>>>(leaves, F, NB, C, s->hist);
        if (pairwise) {
            const int64_t rows = (int64_t)F * leaves * leaves * 2;
            MCU(cudaMemsetAsync(s->d_pstat, 0, sizeof(long long) * (size_t)rows * NB, st));
            // YetiRankPairwise: the tree's compacted samples with their
            // weights; PairLogitPairwise: the explicit pairs, unit weights
            const int64_t* PW = yeti ? s->d_ypw : s->d_pwin;
            const int64_t* PL = yeti ? s->d_ypl : s->d_closer;
            const long long* PQ = yeti ? s->d_ypq : nullptr;
            const unsigned long long* ND = yeti ? s->d_ypn : nullptr;
            const int64_t NP = yeti ? s->ycap : s->n_pairs;
            const size_t psm = sizeof(uint32_t) * 2 * (size_t)leaves * leaves * NB * 2;
            if (leaves <= kPsSmemLeaves && psm <= (size_t)220 * 1024) {
                if (psm > 48 * 1024)
                    MCU(cudaFuncSetAttribute(rk_pairstat_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)psm));
                // a few shares of the pairs per feature: each block flushes its whole table
                const unsigned shares = (unsigned)std::max<int64_t>(1, std::min<int64_t>(4, NP >> 20));
                rk_pairstat_smem_kernel<<<dim3(shares, (unsigned)F), kPsThreads, psm, st>>>(
                    NP, n, leaves, NB, PW, PL, s->bins_fm, s->leaf, s->pw_shift, s->d_pstat, PQ, ND);
            } else {
                rk_pairstat_kernel<<<dim3(grid_for(NP), (unsigned)F), kMcThreads, 0, st>>>(
                    NP, n, leaves, NB, PW, PL, s->bins_fm, s->leaf, s->pw_shift, s->d_pstat, PQ, ND);
            }
            rk_pairprefix_kernel<<<grid_for(rows), kMcThreads, 0, st>>>(rows, NB, s->d_pstat);
            const int n2 = 2 * leaves;
            const int pw_smem = n2 <= kPwSmemMaxN2 ? 1 : 0;
            const int64_t cand = (int64_t)F * NB;
            const int64_t blocks = std::min<int64_t>(cand, pw_smem ? (int64_t)148 * 8 : (int64_t)kPwGlobalBlocks);
            rk_pairscore_kernel<<<(unsigned)blocks, kPwThreads, pw_smem ? pw_scratch_doubles(n2) * sizeof(double) : 0,
                                  st>>>(leaves, F, NB, C, s->hist, s->d_pstat, s->d_bc, s->d_ms, s->raw_l2,
                                        s->pw_shift, pw_smem, s->d_pwscratch, s->scores);
        } else {
            mc_score_kernel<<<(unsigned)(F * ((NB + 31) / 32)), (kMsCompute + 1) * 32, 0, st>>>(
                leaves, F, NB, K, s->hist, s->d_bc, s->d_ms, s->l2, s->score_fn, s->F0, s->d_present, s->scores);
        }
        mc_argmax_kernel<<<1, 1024, 0, st>>>((int64_t)F * NB, NB, s->scores, l, s->d_ms);
        mc_route_kernel<<<g, kMcThreads, 0, st>>>(n, l, s->bins_fm, s->F0, s->d_ms, s->leaf);
        MCU(cudaGetLastError());
    }
    if (s->rank_mode >= 0) {
        // Newton leaves over the grouped ders, then normalize_leaf_values; the
        // leaf-value recomputes come first so the leaf fixed point sees their ders
        if (yeti) {  // the stored leaves come from pairs sampled off the model approximant
            rk_yeti_sample_kernel<<<yw, kYetiWarps * 32, 0, st>>>(s->n_groups, s->d_goff, s->approx, s->d_tgt, s->yeti_perms,
                                                     s->d_ydecay, s->d_yseeds + 2 * (size_t)s->n_groups, s->d_cwoff,
                                                     s->d_cw, s->d_lmorder, s->d_yboot);
            rk_yeti_der_kernel<<<yw, kYetiWarps * 32, 0, st>>>(s->n_groups, s->d_goff, s->approx, s->d_gw, s->yeti_perms,
                                                  s->d_cwoff, s->d_cw, s->wd1, s->d_der2, nullptr, s->d_yboot, s->d_ms);
        }
        if (srank)  // the leaf-value recompute with the leaf-value base
            rk_srank_kernel<<<yg, 128, 0, st>>>(s->n_groups, s->d_goff, s->approx, s->d_tgt, s->srank_ndcg,
                                               s->srank_sigma, s->srank_mu, s->srank_num_est, srank_base[1],
                                               s->d_lmden, s->d_lmideal, s->d_srank_ws, s->d_lmorder, s->wd1,
                                               s->d_der2, s->d_ms);
        const int gradient = (s->rank_mode == kRankQuerySoftMax || srank) ? 1 : 0;
        double* rsum = reinterpret_cast<double*>(s->sums);  // 3 f64 per leaf in the ranking mode
        {
            int rc = rk_leafsums(s, gradient, rsum, st);
            if (rc) return rc;
        }
        if (pairwise) {
            MCU(cudaMemsetAsync(s->d_pwsum, 0, sizeof(long long) * (size_t)L * L, st));
            if (yeti)
                rk_yeti_pairleafw_kernel<<<yg, 128, 0, st>>>(s->n_groups, s->d_goff, s->d_cwoff, s->d_cw, s->d_gw,
                                                            s->yeti_perms, L, s->leaf, s->pw_shift, s->d_pwsum);
            else
                rk_pairleafw_kernel<<<grid_for(s->n_pairs), kMcThreads, 0, st>>>(
                    s->n_pairs, L, s->d_pwin, s->d_closer, s->leaf, s->pw_shift, s->d_pwsum);
            rk_pairleaf_kernel<<<1, kPwThreads, 0, st>>>(L, s->d_pwsum, rsum, s->raw_l2, s->lr, s->pw_shift, 1,
                                                         s->d_pwscratch, s->leaf_raw, s->leaf_lrv);
        } else {
            rk_newton_kernel<<<1, 1, 0, st>>>(L, (s->rank_mode == kRankPairLogit || yeti) ? 1 : 0, gradient, rsum,
                                              s->l2, s->lr, s->leaf_raw, s->leaf_lrv);
        }
        if (yeti) {
            // the learning fold: its own resample, Newton deltas x lr, no centring
            rk_yeti_sample_kernel<<<yw, kYetiWarps * 32, 0, st>>>(s->n_groups, s->d_goff, s->d_lapprox, s->d_tgt, s->yeti_perms,
                                                     s->d_ydecay, s->d_yseeds + (size_t)s->n_groups, s->d_cwoff,
                                                     s->d_cw, s->d_lmorder, s->d_yboot);
            rk_yeti_der_kernel<<<yw, kYetiWarps * 32, 0, st>>>(s->n_groups, s->d_goff, s->d_lapprox, s->d_gw, s->yeti_perms,
                                                  s->d_cwoff, s->d_cw, s->wd1, s->d_der2, nullptr, s->d_yboot, s->d_ms);
            {
                int rc = rk_leafsums(s, 0, rsum, st);
                if (rc) return rc;
            }
            if (pairwise) {  // YetiRankPairwise: Cholesky deltas for the learning fold too
                MCU(cudaMemsetAsync(s->d_pwsum, 0, sizeof(long long) * (size_t)L * L, st));
                rk_yeti_pairleafw_kernel<<<yg, 128, 0, st>>>(s->n_groups, s->d_goff, s->d_cwoff, s->d_cw, s->d_gw,
                                                            s->yeti_perms, L, s->leaf, s->pw_shift, s->d_pwsum);
                rk_pairleaf_kernel<<<1, kPwThreads, 0, st>>>(L, s->d_pwsum, rsum, s->raw_l2, s->lr, s->pw_shift, 0,
                                                             s->d_pwscratch, s->d_ylf_raw, s->d_ylf_lrv);
            } else {
                rk_newton_kernel<<<1, 1, 0, st>>>(L, 0, 0, rsum, s->l2, s->lr, s->d_ylf_raw, s->d_ylf_lrv);
            }
            mc_apply_pending_kernel<<<g, kMcThreads, 0, st>>>(n, 1, L, s->d_lapprox, s->leaf, s->d_ylf_lrv);
        }
        MCU(cudaGetLastError());
    } else {
        // leaf values from the unsampled channels (boosting.rs:2610-2700)
        const size_t ltab = (size_t)L * (K + pk) * sizeof(unsigned long long);
        const int luse = ltab <= kMcSmemTable ? 1 : 0;
        MCU(cudaMemsetAsync(s->sums, 0, ltab, st));
        if (luse && ltab > 48 * 1024)
            MCU(cudaFuncSetAttribute(mc_leafsum_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ltab));
        mc_leafsum_kernel<<<g, kMcThreads, luse ? ltab : 0, st>>>(n, K, L, s->approx, s->wd1, s->weight, s->leaf,
                                                                 s->leaf_shift, s->diag, s->d_tmat, s->sums, luse,
                                                                 s->d_ms);
        mc_newton_kernel<<<(L + 63) / 64, 64, 0, st>>>(K, L, s->sums, s->leaf_shift, s->l2, s->lr, s->diag, s->d_ms,
                                                       s->leaf_raw, s->leaf_lrv);
        MCU(cudaGetLastError());
    }
    MCU(cudaMemcpyAsync(s->h_raw, s->leaf_raw, sizeof(double) * (size_t)L * K, cudaMemcpyDeviceToHost, st));
    MCU(cudaMemcpyAsync(s->h_ms, s->d_ms, sizeof(McState), cudaMemcpyDeviceToHost, st));
    if (leaf_of && leaf_of_bytes) {
        if (!s->leaf_export) MDA(*(uint32_t**)&s->leaf_export, n);
        mc_leaf_export_kernel<<<g, kMcThreads, 0, st>>>(n, s->leaf, s->leaf_export, leaf_of_bytes);
        MCU(cudaMemcpyAsync(leaf_of, s->leaf_export, (size_t)leaf_of_bytes * n, cudaMemcpyDeviceToHost, st));
    }
    // the RNG phase after the tree (boosting.rs:7267-7300, device_draw_replay.rs)
    if (!s->sample_from_host && s->boot != CBGPU_BOOT_NO) {
        for (int l = 0; l < D; ++l) {
            for (int f = 0; f < F; ++f) (void)s->rng.real1();
            (void)s->rng.gen();
            for (int f = 0; f < F; ++f) (void)s->rng.std_normal();
        }
        s->rng.gen();  // POST_TREE_EXTRA_DRAWS = 2
        s->rng.gen();
    }
    MCU(cudaStreamSynchronize(st));
    const McState& m = *s->h_ms;
    if (m.err & kMcErrNoCandidate) return mfail(CBGPU_ERR_DEVICE, "Degenerate: no split candidate available");
    if (m.err) return mfail(CBGPU_ERR_DEVICE, "multi_grow: device error word 0x%x", m.err);
    for (int l = 0; l < D; ++l) {
        if (split_feature) split_feature[l] = m.split[l].feature;
        if (split_bin) split_bin[l] = m.split[l].bin;
    }
    if (n_splits) *n_splits = D;
    if (leaf_values) memcpy(leaf_values, s->h_raw, sizeof(double) * (size_t)L * K);
    s->pending = true;
    return CBGPU_OK;
}

int cbgpu_multi_approx(cbgpu_multi_session* s, double* out_dim_major, int64_t n) {
    if (!s || !out_dim_major || n != s->n) return mfail(CBGPU_ERR_INVALID, "multi_approx: bad arguments");
    MCU(cudaSetDevice(s->device));
    if (s->pending) {
        mc_apply_pending_kernel<<<grid_for(n), kMcThreads, 0, s->st>>>(n, s->K, 1 << s->depth, s->approx, s->leaf,
                                                                         s->leaf_lrv);
        MCU(cudaGetLastError());
        s->pending = false;
    }
    MCU(cudaMemcpyAsync(out_dim_major, s->approx, sizeof(double) * (size_t)s->K * n, cudaMemcpyDeviceToHost, s->st));
    MCU(cudaStreamSynchronize(s->st));
    return CBGPU_OK;
}

int cbgpu_multi_end(cbgpu_multi_session* s) {
    if (!s) return CBGPU_OK;
    cudaSetDevice(s->device);
    delete s;
    return CBGPU_OK;
}
