// kernels.cu -- sm_100a kernels of the oblivious-tree training path.
//
// Per tree: bootstrap -> fused apply/derivative -> fixed-point scales, then per
// level: histogram (smaller children only) -> derive siblings + bin prefix ->
// score + argmax -> stable partition of the leaf-sorted row order; the last
// level routes and reduces the leaf sums.  Every reduction whose result feeds a
// split decision is an exact int64 fixed-point sum, so results do not depend on
// launch geometry, atomic order or the number of GPUs.
//
// Compiled with -fmad=false: every f64 expression rounds each operation as the
// reference's Rust code does (no FMA contraction).
#include <algorithm>
#include <cfloat>
#include <cstdio>
#include <map>
#include <mutex>
#include <utility>

#include "kernels.cuh"

#include <cub/block/block_reduce.cuh>
#include <cub/block/block_scan.cuh>
#include <cub/device/device_radix_sort.cuh>

namespace cbgpu {

// Raises a kernel's dynamic shared-memory limit on the current device to at
// least `bytes`.  The attribute is per (kernel, device); the record of what
// was set is shared by all host threads under one lock and only grows, so a
// thread launching with fewer bytes, or on another device, never skips a
// setting it needs.
int ensure_dyn_smem(const void* kernel, int bytes) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    std::lock_guard<std::mutex> lk(mu);
    int& cur = done[{kernel, dev}];
    if (cur >= bytes) return 0;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) cur = bytes;
    return (int)e;
}

namespace {

constexpr unsigned kFull = 0xffffffffu;

template <typename T>
__device__ __forceinline__ T warp_incl_scan(T v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        T y = __shfl_up_sync(kFull, v, o);
        if (lane >= o) v += y;
    }
    return v;
}

// Exclusive block scan (blockDim multiple of 32, <= 1024).  `sm` holds >= 33 T.
template <typename T>
__device__ __forceinline__ T block_excl_scan(T v, T* sm, T* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    T inc = warp_incl_scan(v);
    if (lane == 31) sm[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        T s = lane < nw ? sm[lane] : T(0);
        s = warp_incl_scan(s);
        sm[lane] = s;
    }
    __syncthreads();
    T off = warp ? sm[warp - 1] : T(0);
    if (total) *total = sm[nw - 1];
    __syncthreads();
    return off + inc - v;
}

__device__ __forceinline__ double nan_to_neg_inf(double s) { return s == s ? s : -INFINITY; }

__device__ __forceinline__ bool better(double s, int i, double bs, int bi) { return better_split(s, i, bs, bi); }

}  // namespace

// ============================================================================
// begin: quantization and layout
// ============================================================================

// bin = #{k : borders[k] < value} over ascending borders (histogram.rs:159-165);
// NaN -> 0, or the top bin when the last border is the f32::MAX sentinel.
__global__ void quantize_column_kernel(const float* __restrict__ col, int64_t n,
                                       const double* __restrict__ borders, int32_t nb,
                                       uint8_t* __restrict__ out, uint32_t* err) {
    __shared__ double sb[256];
    for (int k = threadIdx.x; k < nb; k += blockDim.x) sb[k] = borders[k];
    __syncthreads();
    const bool nan_top = nb > 0 && sb[nb - 1] == (double)FLT_MAX;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        float v = col[i];
        uint32_t b;
        if (v != v) {
            b = nan_top ? (uint32_t)nb : 0u;
        } else {
            double x = (double)v;
            int lo = 0, hi = nb;
            while (lo < hi) {
                int mid = (lo + hi) >> 1;
                if (sb[mid] < x) lo = mid + 1; else hi = mid;
            }
            b = (uint32_t)lo;
        }
        out[i] = (uint8_t)b;
    }
    (void)err;
}

void launch_quantize_column(const float* col, int64_t n, const double* borders, int32_t nb,
                            uint8_t* out, uint32_t* err, cudaStream_t st) {
    int64_t blocks = (n + 1023) / 1024;
    if (blocks > 4096) blocks = 4096;
    if (blocks < 1) blocks = 1;
    quantize_column_kernel<<<(unsigned)blocks, 256, 0, st>>>(col, n, borders, nb, out, err);
}

__global__ void u32_to_u8_kernel(const uint32_t* __restrict__ col, int64_t n, int32_t n_bins,
                                 uint8_t* __restrict__ out, uint32_t* err) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        uint32_t b = col[i];
        if (b >= (uint32_t)n_bins) {
            atomicOr(err, kErrBinRange);
            b = 0;
        }
        out[i] = (uint8_t)b;
    }
}

void launch_u32_to_u8_column(const uint32_t* col, int64_t n, int32_t n_bins, uint8_t* out,
                             uint32_t* err, cudaStream_t st) {
    int64_t blocks = (n + 1023) / 1024;
    if (blocks > 4096) blocks = 4096;
    if (blocks < 1) blocks = 1;
    u32_to_u8_kernel<<<(unsigned)blocks, 256, 0, st>>>(col, n, n_bins, out, err);
}

// Feature-major [F][n_stride] -> row-major [n][F_pad] via a 32-feature x 128-row
// shared tile; padding features are written as 0.
__global__ void transpose_fm_rm_kernel(const uint8_t* __restrict__ fm, int64_t n, int64_t n_stride,
                                       int32_t F, uint8_t* __restrict__ rm, int32_t F_pad) {
    __shared__ uint8_t tile[32][128 + 4];
    const int64_t r0 = (int64_t)blockIdx.x * 128;
    const int f0 = blockIdx.y * 32;
    for (int k = threadIdx.x; k < 32 * 128; k += blockDim.x) {
        int fl = k / 128, rl = k % 128;
        int64_t r = r0 + rl;
        int f = f0 + fl;
        tile[fl][rl] = (f < F && r < n) ? fm[(int64_t)f * n_stride + r] : (uint8_t)0;
    }
    __syncthreads();
    for (int k = threadIdx.x; k < 32 * 128; k += blockDim.x) {
        int rl = k / 32, fl = k % 32;
        int64_t r = r0 + rl;
        if (r < n) rm[r * F_pad + f0 + fl] = tile[fl][rl];
    }
}

void launch_transpose_fm_to_rm(const uint8_t* fm, int64_t n, int64_t n_stride, int32_t F,
                               uint8_t* rm, int32_t F_pad, cudaStream_t st) {
    // columns [0, round_up(F, 32)) of each F_pad-byte row: the F features, zeros after
    dim3 grid((unsigned)((n + 127) / 128), (unsigned)((F + 31) / 32));
    if (grid.x == 0) return;
    transpose_fm_rm_kernel<<<grid, 256, 0, st>>>(fm, n, n_stride, F, rm, F_pad);
}

__global__ void transpose_rm_fm_kernel(const uint8_t* __restrict__ rm, int64_t n, int32_t F,
                                       int32_t F_src, uint8_t* __restrict__ fm, int64_t n_stride) {
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < n * F;
         k += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = k / F;
        int f = (int)(k % F);
        fm[(int64_t)f * n_stride + r] = rm[r * F_src + f];
    }
}

void launch_transpose_rm_to_fm(const uint8_t* rm, int64_t n, int32_t F, int32_t F_src,
                               uint8_t* fm, int64_t n_stride, cudaStream_t st) {
    int64_t blocks = (n * F + 1023) / 1024;
    if (blocks > 8192) blocks = 8192;
    if (blocks < 1) blocks = 1;
    transpose_rm_fm_kernel<<<(unsigned)blocks, 256, 0, st>>>(rm, n, F, F_src, fm, n_stride);
}

// ============================================================================
// bootstrap (crates/cb-train/src/bootstrap.rs)
// ============================================================================

// Bayesian: 1000-row blocks, block b draws from from_seed(rand_seed + b)
// advanced 10 then one gen_rand_real1 per row (bootstrap.rs:152-175).
// Bernoulli: the main stream continues across rows: row g uses the base state
// advanced g draws (set_sampled_control, bootstrap.rs:178-184).  A thread
// jumps once and steps kBootRun consecutive rows; the Bayesian jumps (10 to
// 1009 steps) use the session's table of jump multipliers when given.
__device__ __forceinline__ void jump_rng(Rng64& r, uint64_t d, const ull* __restrict__ jump) {
    if (jump) {
        const ull p = __ldg(jump + 2 * d), c = __ldg(jump + 2 * d + 1);
        r.x1 = r.x1 * p + r.c1 * c;
        r.x2 = r.x2 * p + r.c2 * c;
    } else {
        r.advance(d);
    }
}

// Sample weights of rows i0 .. i0 + kBootRun - 1 (global row g0 = row_offset +
// i0); rows at or past n get 0.
__device__ __forceinline__ void boot_run(int mode, int64_t i0, int64_t g0, int64_t n,
                                         const TreeParams* __restrict__ tp, double rate, float temp,
                                         const ull* __restrict__ jump, float (&v)[kBootRun]) {
    if (mode == 1) {
        const uint64_t rand_seed = tp->boot_seed;
        const uint64_t blk = (uint64_t)(g0 / 1000);
        const int rem = (int)(g0 - (int64_t)blk * 1000);
        Rng64 r = Rng64::from_seed(rand_seed + blk);
        jump_rng(r, 10 + (uint64_t)rem, jump);
#pragma unroll
        for (int j = 0; j < kBootRun; ++j) {
            if (j > 0 && j == 1000 - rem) {  // the run crosses into the next 1000-row block
                r = Rng64::from_seed(rand_seed + blk + 1);
                jump_rng(r, 10, jump);
            }
            v[j] = i0 + j < n ? (float)bayesian_weight(real1(r), temp) : 0.0f;
        }
    } else {
        Rng64 r = tp->boot_base;
        r.advance((uint64_t)g0);
#pragma unroll
        for (int j = 0; j < kBootRun; ++j) v[j] = i0 + j < n && real1(r) < rate ? 1.0f : 0.0f;
    }
}

// x -> x * A^d + c * (A^(d-1) + ... + 1) for d < kJumpSteps: jump[2d] = A^d,
// jump[2d + 1] = the sum (the multipliers lcg_advance forms, rng.rs:45-69).
__global__ void jump_table_kernel(ull* __restrict__ jump) {
    const int d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= kJumpSteps) return;
    jump[2 * d] = lcg_advance(1, 0, (uint64_t)d);
    jump[2 * d + 1] = lcg_advance(0, 1, (uint64_t)d);
}

void launch_jump_table(ull* jump, cudaStream_t st) {
    jump_table_kernel<<<(kJumpSteps + 255) / 256, 256, 0, st>>>(jump);
}

__global__ void bootstrap_kernel(int mode, int64_t n, int64_t row_offset, const TreeParams* __restrict__ tp,
                                 double rate, float temp, const ull* __restrict__ jump, float* __restrict__ out) {
    static_assert(kBootRun == 8, "a run is stored as two float4");
    int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    int64_t i0 = t * kBootRun;
    if (i0 >= n) return;
    float v[kBootRun];
    boot_run(mode, i0, row_offset + i0, n, tp, rate, temp, jump, v);
    if (i0 + kBootRun <= n) {  // i0 is a multiple of 8 floats: 32-byte aligned
        ((float4*)(out + i0))[0] = make_float4(v[0], v[1], v[2], v[3]);
        ((float4*)(out + i0))[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
        for (int j = 0; i0 + j < n; ++j) out[i0 + j] = v[j];
    }
}

void launch_bootstrap(int mode, int64_t n, int64_t row_offset, const TreeParams* tp, double rate, float temp,
                      float* out_sw, cudaStream_t st) {
    int64_t threads = (n + kBootRun - 1) / kBootRun;
    int64_t blocks = (threads + 255) / 256;
    if (blocks < 1) return;
    bootstrap_kernel<<<(unsigned)blocks, 256, 0, st>>>(mode, n, row_offset, tp, rate, temp, nullptr, out_sw);
}

// ---- MVS (bootstrap.rs:186-300): per 8192-row block a threshold from the
// quickselect-style recursion with SEQUENTIAL f64 partial sums, then per row
// p = min(1, sqrt(der^2 + lambda) / threshold), one draw per row with p > eps.

constexpr int kMvsBlock = 8192;
constexpr int kMvsThreads = 256;

__device__ __forceinline__ double mvs_der_obj(double wd) { return sqrt(__dmul_rn(wd, wd)); }

__global__ void __launch_bounds__(kMvsThreads) mvs_threshold_kernel(
    int64_t n, const double* __restrict__ wd1, const TreeParams* __restrict__ tp, double rate,
    double* __restrict__ thresholds) {
    // the block's values stay in place (val); the recursion partitions 16-bit
    // indices between two buffers (96 KB in all: two blocks per SM, so one
    // block's sequential sum overlaps the other's partition)
    extern __shared__ double msm[];
    double* val = msm;
    uint16_t* bufA = (uint16_t*)(msm + kMvsBlock);
    uint16_t* bufB = bufA + kMvsBlock;
    __shared__ int s_scan[40];
    __shared__ double s_state[4];  // sum_small_cur, n_large_cur, result
    __shared__ int s_ctl[4];       // len, which buffer/offset, done
    const double lambda = tp->mvs_lambda;
    const int64_t beg = (int64_t)blockIdx.x * kMvsBlock;
    const int64_t end = beg + kMvsBlock < n ? beg + kMvsBlock : n;
    const int bs = (int)(end - beg);
    for (int k = threadIdx.x; k < bs; k += blockDim.x) {
        double d = mvs_der_obj(wd1[beg + k]);
        val[k] = sqrt(__dadd_rn(lambda, __dmul_rn(d, d)));
        bufA[k] = (uint16_t)k;
    }
    const double sample_size = (double)__fmul_rn((float)rate, (float)bs);
    if (threadIdx.x == 0) {
        s_state[0] = 0.0;
        s_state[1] = 0.0;
        s_ctl[0] = bs;
        s_ctl[1] = 0;  // cur buffer = A, offset 0
        s_ctl[2] = 0;  // done
    }
    __syncthreads();
    for (;;) {
        const int len = s_ctl[0];
        const uint16_t* cur = (s_ctl[1] & 1 ? bufB : bufA) + (s_ctl[1] >> 1);
        uint16_t* oth = (s_ctl[1] & 1) ? bufA : bufB;
        if (len == 0) {
            if (threadIdx.x == 0) thresholds[blockIdx.x] = 0.0;
            return;
        }
        const double thr = val[cur[0]];
        const int per = (len + blockDim.x - 1) / blockDim.x;
        const int k0 = threadIdx.x * per;
        const int k1 = k0 + per < len ? k0 + per : len;
        int cs = 0, cm = 0, cl = 0;
        for (int k = k0; k < k1; ++k) {
            double c = val[cur[k]];
            if (c < thr) ++cs; else if (c <= thr) ++cm; else ++cl;
        }
        int ts, tl;
        int ps = block_excl_scan<int>(cs, s_scan, &ts);
        int pl = block_excl_scan<int>(cl, s_scan, &tl);
        int tm_dummy;
        (void)block_excl_scan<int>(cm, s_scan, &tm_dummy);
        const int tm = tm_dummy;
        for (int k = k0; k < k1; ++k) {
            const uint16_t ik = cur[k];
            double c = val[ik];
            if (c < thr) oth[ps++] = ik;
            else if (!(c <= thr)) oth[ts + pl++] = ik;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            double sum_small_upd = 0.0;
            int k = 0;
            for (; k + 8 <= ts; k += 8) {  // 8 loads ahead of their (ordered) additions
                double x[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) x[u] = val[oth[k + u]];
#pragma unroll
                for (int u = 0; u < 8; ++u) sum_small_upd = __dadd_rn(sum_small_upd, x[u]);
            }
            for (; k < ts; ++k) sum_small_upd = __dadd_rn(sum_small_upd, val[oth[k]]);
            const double s_cur = s_state[0], nl_cur = s_state[1];
            const double nl_upd = (double)tl, n_mid = (double)tm;
            const double sum_mid = __dmul_rn(n_mid, thr);
            double est;
            if (thr != 0.0)
                est = __dadd_rn(__dadd_rn(__dadd_rn(__ddiv_rn(__dadd_rn(s_cur, sum_small_upd), thr), nl_cur),
                                          nl_upd), n_mid);
            else
                est = INFINITY;
            const int oth_id = (s_ctl[1] & 1) ? 0 : 1;
            if (tl == len || ts == len) {
                // no progress (a NaN pivot puts every element in `large`): stop
                // with the pivot; the derivative kernel has flagged the NaN.
                s_state[2] = thr;
                s_ctl[2] = 1;
            } else if (est > sample_size) {
                if (tl > 0) {
                    s_state[0] = __dadd_rn(__dadd_rn(s_cur, sum_mid), sum_small_upd);
                    s_ctl[0] = tl;
                    s_ctl[1] = oth_id | (ts << 1);
                } else {
                    double denom = __dsub_rn(sample_size, nl_cur);
                    s_state[2] = denom != 0.0
                                     ? __ddiv_rn(__dadd_rn(__dadd_rn(s_cur, sum_small_upd), sum_mid), denom)
                                     : thr;
                    s_ctl[2] = 1;
                }
            } else if (ts > 0) {
                s_state[1] = __dadd_rn(__dadd_rn(nl_cur, nl_upd), n_mid);
                s_ctl[0] = ts;
                s_ctl[1] = oth_id;
            } else {
                double denom = __dsub_rn(__dsub_rn(__dsub_rn(sample_size, nl_cur), n_mid), nl_upd);
                s_state[2] = denom != 0.0 ? __ddiv_rn(s_cur, denom) : thr;
                s_ctl[2] = 1;
            }
        }
        __syncthreads();
        if (s_ctl[2]) {
            if (threadIdx.x == 0) thresholds[blockIdx.x] = s_state[2];
            return;
        }
    }
}

__global__ void __launch_bounds__(kMvsThreads) mvs_weights_kernel(
    int64_t n, int64_t row_offset, const double* __restrict__ wd1, const TreeParams* __restrict__ tp,
    const double* __restrict__ thresholds, float* __restrict__ out) {
    __shared__ int s_scan[40];
    const double lambda = tp->mvs_lambda;
    const uint64_t rand_seed = tp->boot_seed;
    const int64_t beg = (int64_t)blockIdx.x * kMvsBlock;
    const int64_t end = beg + kMvsBlock < n ? beg + kMvsBlock : n;
    const int bs = (int)(end - beg);
    const double thr = thresholds[blockIdx.x];
    const int per = kMvsBlock / kMvsThreads;  // 32 rows per thread, contiguous
    const int k0 = threadIdx.x * per;
    int cnt = 0;
    for (int k = k0; k < k0 + per && k < bs; ++k) {
        double d = mvs_der_obj(wd1[beg + k]);
        double x = sqrt(__dadd_rn(__dmul_rn(d, d), lambda));
        double p = x > thr ? 1.0 : (thr > 0.0 ? __ddiv_rn(x, thr) : 0.0);
        cnt += p > DBL_EPSILON;
    }
    int tot;
    int idx = block_excl_scan<int>(cnt, s_scan, &tot);
    const uint64_t gblk = (uint64_t)((row_offset + beg) / kMvsBlock);
    Rng64 r = Rng64::from_seed(rand_seed + gblk);
    r.advance(10 + (uint64_t)idx);
    for (int k = k0; k < k0 + per && k < bs; ++k) {
        double d = mvs_der_obj(wd1[beg + k]);
        double x = sqrt(__dadd_rn(__dmul_rn(d, d), lambda));
        double p = x > thr ? 1.0 : (thr > 0.0 ? __ddiv_rn(x, thr) : 0.0);
        float w = 0.0f;
        if (p > DBL_EPSILON) {
            double weight = __ddiv_rn(1.0, p);
            double u = real1(r);
            w = __double2float_rn(__dmul_rn(weight, u < p ? 1.0 : 0.0));
        }
        out[beg + k] = w;
    }
}

void launch_mvs(int64_t n, int64_t row_offset, const double* wd1, const TreeParams* tp, double rate,
                double* thresholds, float* out_sw, cudaStream_t st) {
    int64_t blocks = (n + kMvsBlock - 1) / kMvsBlock;
    if (blocks < 1) return;
    size_t smem = sizeof(double) * kMvsBlock + 2 * sizeof(uint16_t) * kMvsBlock;
    static_assert(kMvsBlock <= 65536, "16-bit indices");
    ensure_dyn_smem((const void*)mvs_threshold_kernel, (int)smem);
    mvs_threshold_kernel<<<(unsigned)blocks, kMvsThreads, smem, st>>>(n, wd1, tp, rate, thresholds);
    mvs_weights_kernel<<<(unsigned)blocks, kMvsThreads, 0, st>>>(n, row_offset, wd1, tp, thresholds, out_sw);
}

// ============================================================================
// fused apply + derivatives (loss.rs:35-80, boosting.rs:7450-7732)
// ============================================================================

__device__ __forceinline__ void block_max4(double m[4], TreeState* ts) {
    __shared__ double sm[4][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        double v = m[c];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(kFull, v, o));
        if (lane == 0) sm[c][warp] = v;
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            double v = lane < nw ? sm[c][lane] : 0.0;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(kFull, v, o));
            if (lane == 0 && v > 0.0) atomicMax(&ts->maxbits[c], (ull)__double_as_longlong(v));
        }
    }
}

__device__ __forceinline__ double sample_of(int s_mode, const float* sw32, const double* sw64, int64_t i) {
    return s_mode == 0 ? 1.0 : (s_mode == 1 ? (double)sw32[i] : sw64[i]);
}

// approx += lr * leaf value of the previous tree (when pending), then
// der1 (RMSE t - a; Logloss t - (1 - 1/(1 + e^a))), wd1 = der1 * w, and the
// maxima of |g| = |wd1 * s|, |h| = |w * s|, |wd1|, |w| for the fixed-point scales.
// MAE / Quantile (loss ids 15, 16): quantile_der1 (loss.rs:166-175), 0 inside
// |t - a| < delta, else alpha above and -(1 - alpha) below.
__device__ __forceinline__ double der1_of(int loss, double a, double t, double qa, double qd) {
    if (loss == 0) return __dsub_rn(t, a);
    if (loss >= 15) {
        const double v = __dsub_rn(t, a);
        return fabs(v) < qd ? 0.0 : (v > 0.0 ? qa : -__dsub_rn(1.0, qa));
    }
    const double e = exp(a);
    const double p = __dsub_rn(1.0, __ddiv_rn(1.0, __dadd_rn(1.0, e)));
    return __dsub_rn(t, p);
}

// kDerHalf consecutive doubles from p + i (32-byte aligned when the half is
// full), `fill` past n.
constexpr int kDerHalf = kBootRun / 2;  // rows a thread carries through the derivative math at once

__device__ __forceinline__ void load_half(const double* __restrict__ p, int64_t i, int64_t n, bool full, double fill,
                                          double (&v)[kDerHalf]) {
    if (full) {
#pragma unroll
        for (int k = 0; k < kDerHalf; k += 2) {
            const double2 x = *(const double2*)(p + i + k);
            v[k] = x.x;
            v[k + 1] = x.y;
        }
    } else {
#pragma unroll
        for (int k = 0; k < kDerHalf; ++k) v[k] = i + k < n ? p[i + k] : fill;
    }
}

__device__ __forceinline__ void store_half(double* __restrict__ p, int64_t i, int64_t n, bool full,
                                           const double (&v)[kDerHalf]) {
    if (full) {
#pragma unroll
        for (int k = 0; k < kDerHalf; k += 2) *(double2*)(p + i + k) = make_double2(v[k], v[k + 1]);
    } else {
#pragma unroll
        for (int k = 0; k < kDerHalf; ++k)
            if (i + k < n) p[i + k] = v[k];
    }
}

// Each thread takes runs of kBootRun consecutive rows.  kBoot 1 / 2 draws the
// run's Bayesian / Bernoulli sample here (boot_run, one RNG jump per run) and
// stores it to sw32 as the bootstrap kernel would; otherwise the sample is
// read as s_mode says (unless deferred to MVS).  The derivative math then
// runs over the run's two halves in turn (fewer live registers, more warps
// per SM).  kWeight: per-row weights.
template <bool kWeight, int kBoot>
__global__ void __launch_bounds__(256, 3) der_kernel(
    int64_t n, int loss, double* __restrict__ approx, const double* __restrict__ target,
    const double* __restrict__ weight, const uint16_t* __restrict__ leaf,
    const double* __restrict__ lrv_in, const TreeParams* __restrict__ tp, int s_mode, float* __restrict__ sw32,
    const double* __restrict__ sw64, double* __restrict__ wd1, TreeState* ts, bool defer,
    int64_t row_offset, double rate, float temp, const ull* __restrict__ jump) {
    static_assert(kBootRun == 8, "a run's leaf ids are one 16-byte load");
    const double* lrv = tp->pending ? lrv_in : nullptr;
    const double qa = tp->q_alpha, qd = tp->q_delta;
    double m[4] = {0.0, 0.0, 0.0, 0.0};
    bool bad = false;
    const int64_t runs = (n + kBootRun - 1) / kBootRun;
    for (int64_t run = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; run < runs;
         run += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i0 = run * kBootRun;
        const bool full = i0 + kBootRun <= n;
        float sv32[kBootRun];
        if (kBoot) {
            boot_run(kBoot, i0, row_offset + i0, n, tp, rate, temp, jump, sv32);
            if (full) {
                ((float4*)(sw32 + i0))[0] = make_float4(sv32[0], sv32[1], sv32[2], sv32[3]);
                ((float4*)(sw32 + i0))[1] = make_float4(sv32[4], sv32[5], sv32[6], sv32[7]);
            } else {
                for (int k = 0; i0 + k < n; ++k) sw32[i0 + k] = sv32[k];
            }
        }
        uint32_t pw[4] = {0u, 0u, 0u, 0u};  // the run's leaf ids, two per word
        if (lrv) {
            if (full) {
                const uint4 p = *(const uint4*)(leaf + i0);
                pw[0] = p.x; pw[1] = p.y; pw[2] = p.z; pw[3] = p.w;
            } else {
                for (int k = 0; i0 + k < n; ++k) pw[k >> 1] |= (uint32_t)leaf[i0 + k] << ((k & 1) * 16);
            }
        }
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
            const int64_t i = i0 + h * kDerHalf;
            double a[kDerHalf], t[kDerHalf], w[kDerHalf], sv[kDerHalf], wd[kDerHalf];
            load_half(approx, i, n, full, 0.0, a);
            load_half(target, i, n, full, 0.0, t);
            if (kWeight) {
                load_half(weight, i, n, full, 1.0, w);
            } else {
#pragma unroll
                for (int k = 0; k < kDerHalf; ++k) w[k] = 1.0;
            }
            if (lrv) {
                const uint32_t hw[2] = {h ? pw[2] : pw[0], h ? pw[3] : pw[1]};  // this half's ids
#pragma unroll
                for (int k = 0; k < kDerHalf; ++k) {
                    const uint32_t id = (hw[k >> 1] >> ((k & 1) * 16)) & 0xffffu;
                    if (i + k < n) a[k] = __dadd_rn(a[k], __ldg(lrv + id));
                }
                store_half(approx, i, n, full, a);
            }
            if (kBoot) {
#pragma unroll
                for (int k = 0; k < kDerHalf; ++k) sv[k] = (double)(h ? sv32[kDerHalf + k] : sv32[k]);
            } else if (!defer && s_mode == 2) {
                load_half(sw64, i, n, full, 1.0, sv);
            } else {
#pragma unroll
                for (int k = 0; k < kDerHalf; ++k)
                    sv[k] = (!defer && s_mode == 1 && i + k < n) ? (double)sw32[i + k] : 1.0;
            }
#pragma unroll
            for (int k = 0; k < kDerHalf; ++k) {
                wd[k] = 0.0;
                if (i + k >= n) continue;
                wd[k] = __dmul_rn(der1_of(loss, a[k], t[k], qa, qd), w[k]);
                m[2] = fmax(m[2], fabs(wd[k]));
                m[3] = fmax(m[3], fabs(w[k]));
                bad |= !isfinite(wd[k]);
                if (!defer) {
                    const double g = __dmul_rn(wd[k], sv[k]), hh = __dmul_rn(w[k], sv[k]);
                    m[0] = fmax(m[0], fabs(g));
                    m[1] = fmax(m[1], fabs(hh));
                    bad |= !isfinite(g) || !isfinite(hh);
                }
            }
            store_half(wd1, i, n, full, wd);
        }
    }
    if (bad) atomicOr(&ts->err, kErrOverflow);
    block_max4(m, ts);
}

void launch_der(int64_t n, int loss, double* approx, const double* target, const double* weight,
                const uint16_t* leaf, const double* lrv, const TreeParams* tp, int s_mode, float* sw32,
                const double* sw64, double* wd1, TreeState* ts, bool defer, int boot_mode, int64_t row_offset,
                double rate, float temp, const ull* jump, cudaStream_t st) {
    const int64_t runs = (n + kBootRun - 1) / kBootRun;
    int64_t blocks = (runs + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks < 1) blocks = 1;
#define CBGPU_DER(W, K)                                                                                        \
    der_kernel<W, K><<<(unsigned)blocks, 256, 0, st>>>(n, loss, approx, target, weight, leaf, lrv, tp, s_mode, sw32, \
                                                       sw64, wd1, ts, defer, row_offset, rate, temp, jump)
    const int k = boot_mode == 1 ? 1 : (boot_mode == 2 ? 2 : 0);
    if (weight) {
        if (k == 1) CBGPU_DER(true, 1);
        else if (k == 2) CBGPU_DER(true, 2);
        else CBGPU_DER(true, 0);
    } else {
        if (k == 1) CBGPU_DER(false, 1);
        else if (k == 2) CBGPU_DER(false, 2);
        else CBGPU_DER(false, 0);
    }
#undef CBGPU_DER
}

// Maxima of |g| and |h| once an MVS sample exists.
__global__ void __launch_bounds__(256) max_gh_kernel(int64_t n, const double* __restrict__ wd1,
                                                     const double* __restrict__ weight,
                                                     const float* __restrict__ sw32, TreeState* ts) {
    double m[4] = {0.0, 0.0, 0.0, 0.0};
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const double w = weight ? weight[i] : 1.0;
        const double s = (double)sw32[i];
        m[0] = fmax(m[0], fabs(__dmul_rn(wd1[i], s)));
        m[1] = fmax(m[1], fabs(__dmul_rn(w, s)));
    }
    block_max4(m, ts);
}

void launch_max_gh(int64_t n, const double* wd1, const double* weight, const float* sw32, TreeState* ts,
                   cudaStream_t st) {
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks < 1) blocks = 1;
    max_gh_kernel<<<(unsigned)blocks, 256, 0, st>>>(n, wd1, weight, sw32, ts);
}

// Fixed-point scales.  Score channels (g, h): 2^s with max|v| * 2^s < 2^33, so a
// row value splits into hi = v >> 17 (|hi| <= 2^16) and lo = v & (2^17 - 1) whose
// 32-bit sums over a kChunkRows-row work item cannot overflow; resolution is
// 2^-33 of the largest value.  Leaf channels: max|v| * n_total * 2^s < 2^62.
// The fixed-point exponent of channel c from the tree's maxima.
__device__ __forceinline__ int channel_shift(const TreeState* ts, int c, int64_t n_total) {
    const double m = __longlong_as_double((long long)ts->maxbits[c]);
    // score channels: max |v| * 2^s < 2^kPackBits; leaf channels: any sum
    // over n_total rows stays below 2^62
    return c < 2 ? fixed_shift(m, kPackBits) : fixed_shift(__dmul_rn(m, (double)(n_total > 0 ? n_total : 1)), 62);
}

__device__ __forceinline__ void write_scales(TreeState* ts, int64_t n_total, int64_t n_local) {
    ts->hist_rows[0] = (uint32_t)n_local;  // level 0 histograms every row
    for (int c = 0; c < 4; ++c) {
        const int sh = channel_shift(ts, c, n_total);
        ts->sc.scale[c] = pow2_of(sh);
        ts->sc.inv[c] = pow2_of(-sh);
    }
}

// Per row: g = wd1 * s, h = w * s (the CPU's score channels, boosting.rs:7700-7732),
// rounded once to fixed point and split into the (lo, hi) parts the histogram
// accumulates: {g_lo, g_hi, h_lo, h_hi} (pack_gh).

__global__ void __launch_bounds__(256) pack_stats_kernel(int64_t n, const double* __restrict__ wd1,
                                                         const double* __restrict__ weight, int s_mode,
                                                         const float* __restrict__ sw32,
                                                         const double* __restrict__ sw64, TreeState* ts,
                                                         int64_t n_total, uint4* __restrict__ qstats) {
    // every block derives the score channels' scales from the tree's maxima;
    // block 0 also records all four for the later kernels
    if (blockIdx.x == 0 && threadIdx.x == 0) write_scales(ts, n_total, n);
    const Pow2 sg = pow2_of(channel_shift(ts, 0, n_total)), sh = pow2_of(channel_shift(ts, 1, n_total));
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const double w = weight ? weight[i] : 1.0;
        const double s = sample_of(s_mode, sw32, sw64, i);
        qstats[i] = pack_gh(__dmul_rn(wd1[i], s), __dmul_rn(w, s), sg, sh);
    }
}

void launch_pack_stats(int64_t n, const double* wd1, const double* weight, int s_mode, const float* sw32,
                       const double* sw64, TreeState* ts, int64_t n_total, uint4* qstats, cudaStream_t st) {
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks < 1) blocks = 1;
    pack_stats_kernel<<<(unsigned)blocks, 256, 0, st>>>(n, wd1, weight, s_mode, sw32, sw64, ts, n_total, qstats);
}

__global__ void apply_kernel(int64_t n, double* __restrict__ approx, const uint16_t* __restrict__ leaf,
                             const double* __restrict__ lrv) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        approx[i] = __dadd_rn(approx[i], lrv[leaf[i]]);
}

void launch_apply(int64_t n, double* approx, const uint16_t* leaf, const double* lrv,
                  cudaStream_t st) {
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks < 1) return;
    apply_kernel<<<(unsigned)blocks, 256, 0, st>>>(n, approx, leaf, lrv);
}

// ============================================================================
// histogram (the hot kernel)
// ============================================================================
//
// Grid (work item, feature tile).  A block owns one work item (<= kChunkRows
// rows of ONE leaf) and one 32-feature tile; lane f of every warp owns feature
// tile*32+f.  Shared memory holds the tile histogram as u32 words laid out
// [bin][part][lane] (part = g_lo, g_hi, h_lo, h_hi), so lane f always touches
// bank f: the 32 updates of a warp are bank-conflict free whatever the bins.
// Each update is four 32-bit shared reductions of the row's pre-split fixed
// point parts; the parts of a work item cannot overflow 32 bits, and the flush
// recombines them into exact int64 sums merged with global atomics.  Integer
// sums make the result independent of ordering, launch geometry and GPU count.

void launch_zero(void* p, size_t bytes, cudaStream_t st) {
    if (bytes) cudaMemsetAsync(p, 0, bytes, st);
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// Tiles: as many 64-feature tiles as fit (each lane owns 2 features), then
// one 32-feature tile if 32+ features remain, then a narrow tail of < 32
// features whose warp step consumes 32 / width rows.  All tiles of a row
// chunk run in one launch (blockIdx.x = tile, fastest) and share L2 lines.
struct TileInfo {
    int f0, nf, kind;  // kind: 2 = 64-feature tile, 1 = 32-feature tile, 0 = narrow tail
};

__host__ __device__ __forceinline__ int hist_n_tiles(int F, int fpl) {
    const int w = 32 * fpl;
    const int nfull = F / w, rem = F % w;
    return nfull + (fpl == 2 && rem >= 32 ? 1 : 0) + ((fpl == 2 ? rem % 32 : rem) > 0 ? 1 : 0);
}

__device__ __forceinline__ TileInfo hist_tile(int F, int fpl, int t) {
    const int w = 32 * fpl;
    const int nfull = F / w, rem = F % w;
    if (t < nfull) return TileInfo{t * w, w, fpl};
    int f0 = nfull * w;
    if (fpl == 2 && rem >= 32) {
        if (t == nfull) return TileInfo{f0, 32, 1};
        f0 += 32;
    }
    return TileInfo{f0, F - f0, 0};
}

// One staged group of up to 32 rows for a tile whose lanes each own kFpl
// features and whose warp step covers kRows = 32 / kWt rows.
template <int kFpl, int kWt, bool kFull = false>
__device__ __forceinline__ void hist_group(uint32_t* __restrict__ hs, const uint8_t* __restrict__ sb,
                                           const uint4* __restrict__ ss, uint32_t cnt, int lane, int nf) {
    constexpr int kRows = 32 / kWt;
    constexpr int kCols = 32 * kFpl;  // u32 columns per (bin, part) row of the table
    constexpr int kUnroll = 8;        // rows whose loads issue before their reductions
    const int sub = lane / kWt, fl = lane % kWt;
    if (!kFull && fl * kFpl >= nf) return;
    const bool second = kFull || (kFpl == 2 && fl * 2 + 1 < nf);
    uint32_t* my = hs + lane;
    uint32_t u = sub;
    for (; u + (kUnroll - 1) * kRows < cnt; u += kUnroll * kRows) {
        uint32_t b[kUnroll][kFpl];
        uint4 s[kUnroll];
#pragma unroll
        for (int v = 0; v < kUnroll; ++v) {
            const uint32_t r = u + v * kRows;
            if (kFpl == 2) {
                const uint32_t two = *(const uint16_t*)(sb + r * 64 + fl * 2);
                b[v][0] = two & 0xffu;
                b[v][kFpl - 1] = two >> 8;
            } else {
                b[v][0] = sb[r * 32 + fl];
            }
            s[v] = ss[r];
        }
#pragma unroll
        for (int v = 0; v < kUnroll; ++v) {
#pragma unroll
            for (int j = 0; j < kFpl; ++j) {
                if (j == 1 && !second) continue;
                uint32_t* cc = my + b[v][j] * (4 * kCols) + j * 32;
                atomicAdd(cc, s[v].x);
                atomicAdd(cc + kCols, s[v].y);
                atomicAdd(cc + 2 * kCols, s[v].z);
                atomicAdd(cc + 3 * kCols, s[v].w);
            }
        }
    }
    for (; u < cnt; u += kRows) {
        uint32_t b0, b1 = 0;
        if (kFpl == 2) {
            const uint32_t two = *(const uint16_t*)(sb + u * 64 + fl * 2);
            b0 = two & 0xffu;
            b1 = two >> 8;
        } else {
            b0 = sb[u * 32 + fl];
        }
        const uint4 s = ss[u];
#pragma unroll
        for (int j = 0; j < kFpl; ++j) {
            if (j == 1 && !second) continue;
            uint32_t* cc = my + (j ? b1 : b0) * (4 * kCols) + j * 32;
            atomicAdd(cc, s.x);
            atomicAdd(cc + kCols, s.y);
            atomicAdd(cc + 2 * kCols, s.z);
            atomicAdd(cc + 3 * kCols, s.w);
        }
    }
}

// Flush: column j*32 + lane of a kFpl tile holds feature lane*kFpl + j; for a
// narrow tile (kFpl 1, width kWt) the columns r*kWt + f (r < 32/kWt) all hold
// feature f and are summed.  Each column's (lo, hi) parts recombine exactly.
template <int kFpl, int kWt>
__device__ __forceinline__ void hist_flush(const uint32_t* __restrict__ hs, int B, int nf,
                                           ull* __restrict__ out, int64_t feat_stride) {
    constexpr int kRows = 32 / kWt;
    constexpr int kCols = 32 * kFpl;
    for (int k = threadIdx.x; k < B * 32 * kFpl; k += blockDim.x) {
        const int b = k / (32 * kFpl), c = k % (32 * kFpl);
        int f;  // feature within the tile
        if (kFpl == 2) f = (c & 31) * 2 + (c >> 5);
        else f = c;
        if (kWt < 32 && c >= kWt) continue;
        if (f >= nf) continue;
        long long gsum = 0, hsum = 0;
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
            const uint32_t* cc = hs + b * 4 * kCols + r * kWt + c;
            gsum += (long long)(int32_t)cc[kCols] * (1ll << kPackSplit) + (long long)cc[0];
            hsum += (long long)(int32_t)cc[3 * kCols] * (1ll << kPackSplit) + (long long)cc[2 * kCols];
        }
        ull* o = out + (int64_t)f * feat_stride + b * 2;
        if (gsum) atomicAdd(o, (ull)gsum);
        if (hsum) atomicAdd(o + 1, (ull)hsum);
    }
}

// Each warp streams its rows in groups of 32 through a kStages-deep ring
// of shared-memory stages: lane l copies row l's tile slice (16-byte pieces)
// and its 16-byte packed stats with cp.async, so one warp instruction moves
// 512 B and several groups are in flight.  A staged group is then consumed
// with lane = (row slot, features): one byte (or u16) load per lane, one load
// of the row's stats, and four conflict-free 32-bit shared reductions per
// feature into the lane's own column (bank = lane).  Reductions and shared
// loads issue through the MIO queue, which bounds this kernel: owning two
// features per lane spends the two loads on eight reductions instead of four.
template <bool kGather, int kFplFull, int kWarps, int kStages>
__global__ void __launch_bounds__(kWarps * 32, 1) hist_kernel(
    const uint8_t* __restrict__ bins_rm, int32_t F_pad, int32_t F, int32_t B,
    const uint4* __restrict__ qstats, const uint32_t* __restrict__ perm,
    const HistChunk* __restrict__ chunks, const uint32_t* __restrict__ n_chunks,
    ull* __restrict__ built, int64_t feat_stride, int64_t slot_stride, int64_t set_qstride,
    int64_t set_built_stride) {
    extern __shared__ __align__(16) uint32_t hs[];  // table [B][4][32*fpl] then the staging ring
    // blockIdx.z = stat set: sets share the rows and their bins, each has its
    // own packed stats and output table
    qstats += (int64_t)blockIdx.z * set_qstride;
    built += (int64_t)blockIdx.z * set_built_stride;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int kSlice = 32 * kFplFull;  // staged bytes per row
    const size_t table_words = (size_t)B * 128 * kFplFull;
    uint8_t* sbins = (uint8_t*)(hs + table_words) + (size_t)warp * kStages * 32 * kSlice;
    uint4* sstat = (uint4*)((uint8_t*)(hs + table_words) + (size_t)kWarps * kStages * 32 * kSlice) +
                   (size_t)warp * kStages * 32;
    // grid: x = feature tile (fastest, so the tiles of a chunk run together and
    // share the chunk's rows in L2), y = chunk (striding when there are more
    // chunks than grid rows)
    const TileInfo ti = hist_tile(F, kFplFull, blockIdx.x);
    // 16-byte pieces of the row slice this tile needs
    const int pieces = ti.kind == 2 ? 4 : (ti.kind == 1 ? 2 : (ti.nf > 16 ? 2 : 1));
    const int narrow_w = ti.nf > 16 ? 32 : ti.nf > 8 ? 16 : ti.nf > 4 ? 8 : ti.nf > 2 ? 4 : ti.nf > 1 ? 2 : 1;
    const uint8_t* tile_base = bins_rm + ti.f0;
    const uint32_t nch = n_chunks[0];
    for (uint32_t c = blockIdx.y; c < nch; c += gridDim.y) {
    const HistChunk ck = chunks[c];
    for (size_t k = threadIdx.x; k < table_words / 4; k += blockDim.x) ((uint4*)hs)[k] = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();

    const uint32_t start = ck.start, len = ck.len;
    const uint32_t n_groups = (len + 31) >> 5;

    // groups of this warp: g = warp, warp + kWarps, ...
    auto row_of = [&](uint32_t g) -> uint32_t {  // row index for lane's row of group g (or ~0)
        const uint32_t r = (g << 5) + lane;
        if (g >= n_groups || r >= len) return 0xffffffffu;
        return kGather ? __ldg(perm + start + r) : start + r;
    };
    auto issue = [&](uint32_t i, int st) {
        if (i != 0xffffffffu) {
            uint8_t* d = sbins + ((size_t)st * 32 + lane) * kSlice;
            const uint8_t* src = tile_base + (size_t)i * F_pad;
            for (int p = 0; p < pieces; ++p) cp_async16(d + 16 * p, src + 16 * p);
            cp_async16(sstat + st * 32 + lane, qstats + i);
        }
        cp_async_commit();
    };
    uint32_t g = warp;
    uint32_t inext = row_of(g);
#pragma unroll
    for (int p = 0; p < kStages - 1; ++p) {
        issue(inext, p);
        inext = row_of(g + (p + 1) * kWarps);
    }
    int st = 0;
    for (; g < n_groups; g += kWarps) {
        // keep kStages - 1 groups in flight
        issue(inext, (st + kStages - 1) % kStages);
        inext = row_of(g + kStages * kWarps);
        cp_async_wait<kStages - 1>();
        __syncwarp();
        const uint32_t cnt = len - (g << 5) < 32u ? len - (g << 5) : 32u;
        const uint8_t* sb = sbins + (size_t)st * 32 * kSlice;
        const uint4* ss = sstat + st * 32;
        // staged rows are kSlice bytes apart; the narrow / 32-wide bodies index
        // rows 32 bytes apart, so they read the ring through a 32-byte view
        if (kFplFull == 2 && ti.kind == 2) {
            hist_group<2, 32, true>(hs, sb, ss, cnt, lane, ti.nf);
        } else {
            // kFplFull == 2 stages 64-byte rows: re-point the row stride
            const uint8_t* sb32 = sb;
            uint32_t* tab = hs;
            if (kFplFull == 2) {
                // compact this group's 32-byte slices in place (rows 64 B apart -> 32 B apart)
                __syncwarp();
                uint8_t* w = (uint8_t*)sb;
                const uint4 lo = *(const uint4*)(sb + lane * 64), hi = *(const uint4*)(sb + lane * 64 + 16);
                __syncwarp();
                *(uint4*)(w + lane * 32) = lo;
                *(uint4*)(w + lane * 32 + 16) = hi;
                __syncwarp();
            }
            if (ti.kind == 1 || narrow_w == 32) hist_group<1, 32>(tab, sb32, ss, cnt, lane, ti.nf);
            else if (narrow_w == 16) hist_group<1, 16>(tab, sb32, ss, cnt, lane, ti.nf);
            else if (narrow_w == 8) hist_group<1, 8>(tab, sb32, ss, cnt, lane, ti.nf);
            else if (narrow_w == 4) hist_group<1, 4>(tab, sb32, ss, cnt, lane, ti.nf);
            else if (narrow_w == 2) hist_group<1, 2>(tab, sb32, ss, cnt, lane, ti.nf);
            else hist_group<1, 1>(tab, sb32, ss, cnt, lane, ti.nf);
        }
        __syncwarp();  // the stage is refilled next iteration
        st = (st + 1) % kStages;
    }
    cp_async_wait<0>();
    __syncthreads();
    ull* out = built + (int64_t)ck.slot * slot_stride + (int64_t)ti.f0 * feat_stride;
    if (kFplFull == 2 && ti.kind == 2) hist_flush<2, 32>(hs, B, ti.nf, out, feat_stride);
    else if (ti.kind == 1 || narrow_w == 32) hist_flush<1, 32>(hs, B, ti.nf, out, feat_stride);
    else if (narrow_w == 16) hist_flush<1, 16>(hs, B, ti.nf, out, feat_stride);
    else if (narrow_w == 8) hist_flush<1, 8>(hs, B, ti.nf, out, feat_stride);
    else if (narrow_w == 4) hist_flush<1, 4>(hs, B, ti.nf, out, feat_stride);
    else if (narrow_w == 2) hist_flush<1, 2>(hs, B, ti.nf, out, feat_stride);
    else hist_flush<1, 1>(hs, B, ti.nf, out, feat_stride);
    __syncthreads();  // the table is zeroed again for the next chunk
    }
}

// Launch shapes: a lane owning two features doubles the table, so that shape
// runs one 16-warp block per SM with a 2-deep ring; the one-feature shape
// keeps 8-warp blocks with a 3-deep ring (two blocks per SM at 129 bins).
struct HistShape {
    int fpl, warps, stages;
};

static size_t hist_shape_bytes(int32_t B, const HistShape& h) {
    return sizeof(uint32_t) * (size_t)B * 128 * h.fpl + (size_t)h.warps * h.stages * 32 * (32 * h.fpl + 16);
}

static HistShape hist_shape(int32_t B) {
    const HistShape two{2, 16, 2};
    if (hist_shape_bytes(B, two) + 1024 <= kHistSmemMax) return two;  // 1 KB left for static shared memory
    return HistShape{1, 8, 3};
}

size_t hist_smem_bytes(int32_t B) { return hist_shape_bytes(B, hist_shape(B)); }

template <bool kGather, int kFpl, int kWarps, int kStages>
static void launch_hist_variant(unsigned gy, unsigned gz, cudaStream_t st, const uint8_t* bins_rm, int32_t F_pad,
                                int32_t F, int32_t B, const uint4* qstats, const uint32_t* perm,
                                const HistChunk* chunks, const uint32_t* n_chunks, ull* built, int64_t feat_stride,
                                int64_t slot_stride, int64_t set_qstride, int64_t set_built_stride) {
    ensure_dyn_smem((const void*)hist_kernel<kGather, kFpl, kWarps, kStages>, (int)hist_smem_bytes(B));
    const dim3 grid((unsigned)hist_n_tiles(F, kFpl), gy, gz);
    hist_kernel<kGather, kFpl, kWarps, kStages><<<grid, kWarps * 32, hist_smem_bytes(B), st>>>(
        bins_rm, F_pad, F, B, qstats, perm, chunks, n_chunks, built, feat_stride, slot_stride, set_qstride,
        set_built_stride);
}

int hist_tiles(int32_t F, int32_t B) { return hist_n_tiles(F, hist_shape(B).fpl); }
int hist_lane_features(int32_t B) { return hist_shape(B).fpl; }

void launch_hist_sets(const uint8_t* bins_rm, int32_t F_pad, int32_t F, int32_t B, const uint4* qstats,
                      const uint32_t* perm, const HistChunk* chunks, const uint32_t* n_chunks, uint32_t max_chunks,
                      ull* built, int64_t feat_stride, int64_t slot_stride, int32_t n_sets, int64_t set_qstride,
                      int64_t set_built_stride, cudaStream_t st) {
    if (max_chunks == 0 || n_sets <= 0 || F <= 0) return;
    const unsigned gy = max_chunks < 65535u ? max_chunks : 65535u;
    const unsigned gz = (unsigned)n_sets;
    const bool two = hist_shape(B).fpl == 2;
#define CBGPU_HIST_ARGS gy, gz, st, bins_rm, F_pad, F, B, qstats, perm, chunks, n_chunks, built, feat_stride, \
                        slot_stride, set_qstride, set_built_stride
    if (perm) {
        if (two) launch_hist_variant<true, 2, 16, 2>(CBGPU_HIST_ARGS);
        else launch_hist_variant<true, 1, 8, 3>(CBGPU_HIST_ARGS);
    } else {
        if (two) launch_hist_variant<false, 2, 16, 2>(CBGPU_HIST_ARGS);
        else launch_hist_variant<false, 1, 8, 3>(CBGPU_HIST_ARGS);
    }
#undef CBGPU_HIST_ARGS
}

void launch_hist(const uint8_t* bins_rm, int32_t F_pad, int32_t F, int32_t B, const uint4* qstats,
                 const uint32_t* perm, const HistChunk* chunks, const uint32_t* n_chunks, uint32_t max_chunks,
                 ull* built, int64_t feat_stride, int64_t slot_stride, cudaStream_t st) {
    launch_hist_sets(bins_rm, F_pad, F, B, qstats, perm, chunks, n_chunks, max_chunks, built, feat_stride,
                     slot_stride, 1, 0, 0, st);
}

// The level-0 work list: rows [0, n) in cr-row items (cr <= kChunkRows; built once per
// session: the row count does not change).
__global__ void level0_chunks_kernel(int64_t n, HistChunk* __restrict__ chunks, uint32_t cap,
                                     uint32_t* __restrict__ n_chunks, uint32_t* __restrict__ err, uint32_t cr) {
    uint32_t nch = (uint32_t)((n + cr - 1) / cr);
    if (nch > cap) {  // cannot happen with the session's sizing; never write past the buffer
        if (threadIdx.x == 0) atomicOr(err, kErrChunkCap);
        nch = cap;
    }
    for (uint32_t k = threadIdx.x; k < nch; k += blockDim.x) {
        const uint32_t st = k * cr;
        chunks[k] = HistChunk{0u, st, (uint32_t)(n - st < cr ? n - st : cr), 0u};
    }
    if (threadIdx.x == 0) n_chunks[0] = nch;
}

void launch_level0_chunks(int64_t n, HistChunk* chunks, uint32_t cap, uint32_t* n_chunks, uint32_t* err,
                          uint32_t chunk_rows, cudaStream_t st) {
    if (chunk_rows == 0 || chunk_rows > (uint32_t)kChunkRows) chunk_rows = kChunkRows;
    level0_chunks_kernel<<<1, 1024, 0, st>>>(n, chunks, cap, n_chunks, err, chunk_rows);
}

uint32_t hist_chunk_rows(int64_t n, int tiles, int sets, int sms) {
    // kChunkRows, or half of it when the level-0 launch would give fewer than
    // 8 blocks per SM: small shards with few stat sets otherwise leave the
    // last of a few waves of one-block-per-SM launches mostly empty (measured:
    // 1M rows x 136 features, 406 -> 454 trees/s); smaller items cost more in
    // table flushes than they gain (a quarter: 5% slower at 1.25M x 200)
    const int64_t want = 8ll * (sms > 0 ? sms : 148);
    uint32_t cr = kChunkRows;
    if ((n / cr) * (int64_t)tiles * (sets > 0 ? sets : 1) < want) cr >>= 1;
    return cr;
}

// ============================================================================
// derive siblings + bin prefix: cur[q][f][*] = inclusive prefix over bins.
// Level 0: prefix(built[0]).  Level l: parent p = q mod 2^(l-1); the built child
// of p is copied, the other is prev[p] - prefix(built[p]) (exact integers; the
// subtraction trick of tree.rs:1075-1131 applied to prefix sums, which are linear).
// One warp per (leaf, feature) row.  All three arrays are feature-major over
// this rank's feature slice of Fs features: built[f][slot][B][2] (slots =
// 2^(level-1) parents, 1 at level 0), prev[f][Q/2][B][2], cur[f][Q][B][2].
// ============================================================================
// kDeriveRounds = ceil(B / 32) rounds of 32 bins (B <= 256).
template <int kDeriveRounds>
__global__ void __launch_bounds__(256) derive_prefix_kernel(int level, int32_t Fs, int32_t B, const ull* __restrict__ built,
                                     const ull* __restrict__ prev, ull* __restrict__ cur,
                                     const uint8_t* __restrict__ small_side, int64_t set_built_stride,
                                     int64_t set_cur_stride) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    // blockIdx.y = stat set (prev and cur share a stride)
    built += (int64_t)blockIdx.y * set_built_stride;
    prev += (int64_t)blockIdx.y * set_cur_stride;
    cur += (int64_t)blockIdx.y * set_cur_stride;
    const int64_t Q = 1ll << level;
    const int64_t slots = level > 0 ? Q >> 1 : 1;
    if (row >= Q * Fs) return;
    const int f = (int)(row / Q);
    const int64_t q = row % Q;
    int64_t p = 0;
    bool is_built = true;
    if (level > 0) {
        const int64_t half = Q >> 1;
        p = q & (half - 1);
        is_built = ((q >> (level - 1)) & 1) == (int64_t)small_side[p];
    }
    const ulonglong2* src = (const ulonglong2*)(built + ((size_t)f * slots + p) * B * 2);
    const ulonglong2* par = (level > 0) ? (const ulonglong2*)(prev + ((size_t)f * slots + p) * B * 2) : nullptr;
    ulonglong2* dst = (ulonglong2*)(cur + ((size_t)f * Q + q) * B * 2);
    // bins b = 32k + lane: coalesced 16-byte (g, h) pairs, all loads issued
    // first, then the prefix carried across rounds
    ulonglong2 v[kDeriveRounds], pv[kDeriveRounds];
#pragma unroll
    for (int k = 0; k < kDeriveRounds; ++k) {
        const int b = 32 * k + lane;
        v[k] = make_ulonglong2(0ull, 0ull);
        pv[k] = make_ulonglong2(0ull, 0ull);
        if (b < B) {
            v[k] = src[b];
            if (!is_built) pv[k] = par[b];
        }
    }
    long long cg = 0, ch = 0;
#pragma unroll
    for (int k = 0; k < kDeriveRounds; ++k) {
        const int b = 32 * k + lane;
        const long long ig = warp_incl_scan<long long>((long long)v[k].x) + cg;
        const long long ih = warp_incl_scan<long long>((long long)v[k].y) + ch;
        cg = __shfl_sync(kFull, ig, 31);
        ch = __shfl_sync(kFull, ih, 31);
        if (b < B) {
            ulonglong2 o = make_ulonglong2((ull)ig, (ull)ih);
            if (!is_built) o = make_ulonglong2((ull)((long long)pv[k].x - ig), (ull)((long long)pv[k].y - ih));
            dst[b] = o;
        }
    }
}

void launch_derive_prefix_sets(int level, int32_t Fs, int32_t B, const ull* built, const ull* prev, ull* cur,
                               const uint8_t* small_side, int32_t n_sets, int64_t set_built_stride,
                               int64_t set_cur_stride, cudaStream_t st) {
    int64_t rows = (1ll << level) * Fs;
    int64_t blocks = (rows * 32 + 255) / 256;
    if (blocks < 1 || n_sets <= 0) return;
    const dim3 g((unsigned)blocks, (unsigned)n_sets);
#define CBGPU_DERIVE(K) derive_prefix_kernel<K><<<g, 256, 0, st>>>(level, Fs, B, built, prev, cur, small_side, \
                                                                   set_built_stride, set_cur_stride)
    switch ((B + 31) / 32) {
        case 1: CBGPU_DERIVE(1); break;
        case 2: CBGPU_DERIVE(2); break;
        case 3: CBGPU_DERIVE(3); break;
        case 4: CBGPU_DERIVE(4); break;
        case 5: CBGPU_DERIVE(5); break;
        case 6: CBGPU_DERIVE(6); break;
        case 7: CBGPU_DERIVE(7); break;
        default: CBGPU_DERIVE(8); break;
    }
#undef CBGPU_DERIVE
}

void launch_derive_prefix(int level, int32_t Fs, int32_t B, const ull* built, const ull* prev,
                          ull* cur, const uint8_t* small_side, cudaStream_t st) {
    launch_derive_prefix_sets(level, Fs, B, built, prev, cur, small_side, 1, 0, 0, st);
}

// ============================================================================
// scoring (score.rs:39-265, histogram.rs:1007-1171) + argmax (tree.rs:355-366)
// Block (border group g, feature f) scores up to 32 consecutive borders
// (lane = border, so the (g, h) pairs of a child load as one 512-byte run).
// The per-child terms avg*swd and avg^2*sw are independent, so the 4 warps
// compute a piece of kScorePiece children into shared memory; then warp 0 adds
// them to each border's running sums in the CPU's canonical order (false
// children 0..Q-1, then true), so the sums round as the CPU's do.  The true
// children's totals (bin B-1 of each leaf's prefix row) are staged once per
// block.  The last block to finish reduces the per-group winners in (feature,
// border) order, which is the CPU's first-wins strict-> scan (no spin wait).
// ============================================================================
constexpr int kScoreWarps = 4;
constexpr int kScorePiece = 32;      // children per piece, kScorePiece / kScoreWarps per warp
constexpr int kScoreTotSmem = 256;   // leaves whose totals are staged in shared memory

__global__ void __launch_bounds__(kScoreWarps * 32, 8) score_kernel(int level, int32_t Fs, int32_t f0, int32_t F,
                                                                    int32_t B, const ull* __restrict__ cur,
                                                                    const int32_t* __restrict__ border_counts,
                                                                    double l2, int score_fn,
                                                                    double* __restrict__ grp_score,
                                                                    int32_t* __restrict__ grp_bin, TreeState* ts,
                                                                    ull* __restrict__ rank_best,
                                                                    uint8_t* __restrict__ small_side) {
    __shared__ double2 s_t[kScorePiece][32];  // (num, den) terms of a piece
    __shared__ ulonglong2 s_tot[kScoreTotSmem];
    __shared__ double s_sc[kScoreWarps];
    __shared__ int s_bi[kScoreWarps];
    __shared__ bool s_last;
    const int g = blockIdx.x, fl = blockIdx.y, G = gridDim.x;
    const int f = f0 + fl;  // global feature
    const int nb = f < F ? border_counts[f] : 0;
    const int Q = 1 << level;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int b = g * 32 + lane;
    const bool in = b < nb;
    const Pow2 ig = ts->sc.inv[0], ih = ts->sc.inv[1];
    const ulonglong2* rows = (const ulonglong2*)(cur + (size_t)fl * Q * B * 2);  // row q at rows + q * B
    const bool tot_smem = Q <= kScoreTotSmem;
    double num = 0.0, den = 1e-100;
    if (g * 32 < B - 1) {  // nb <= B - 1: groups past every feature's borders do nothing
        constexpr int kPer = kScorePiece / kScoreWarps;
        ulonglong2 v[kPer];
        // piece c0's values for this warp's children; the first piece's loads
        // go out together with the totals' staging
        auto load_piece = [&](int c0, int pc) {
#pragma unroll
            for (int k = 0; k < kPer; ++k) {
                const int cc = warp + k * kScoreWarps;
                v[k] = make_ulonglong2(0ull, 0ull);
                if (cc < pc && b < B) {  // every row has B bins: no need to wait for nb
                    const int ch = c0 + cc;  // canonical child index: side * Q + q
                    const int q = ch >= Q ? ch - Q : ch;
                    v[k] = rows[(size_t)q * B + b];
                }
            }
        };
        load_piece(0, 2 * Q < kScorePiece ? 2 * Q : kScorePiece);
        if (tot_smem) {
            for (int q = threadIdx.x; q < Q; q += blockDim.x) s_tot[q] = rows[(size_t)q * B + B - 1];
            __syncthreads();
        }
        for (int c0 = 0; c0 < 2 * Q; c0 += kScorePiece) {
            const int pc = 2 * Q - c0 < kScorePiece ? 2 * Q - c0 : kScorePiece;
#pragma unroll
            for (int k = 0; k < kPer; ++k) {
                const int cc = warp + k * kScoreWarps;
                if (cc < pc && in) {
                    const int ch = c0 + cc;
                    long long pg = (long long)v[k].x, ph = (long long)v[k].y;
                    if (ch >= Q) {
                        const int q = ch - Q;
                        const ulonglong2 t = tot_smem ? s_tot[q] : rows[(size_t)q * B + B - 1];
                        pg = (long long)t.x - pg;
                        ph = (long long)t.y - ph;
                    }
                    const double swd = from_fixed(pg, ig);
                    const double sw = from_fixed(ph, ih);
                    double2 term;
                    if (score_fn <= 1) {  // Cosine / L2
                        const double avg = sw > 0.0 ? __ddiv_rn(swd, __dadd_rn(sw, l2)) : 0.0;
                        term = make_double2(__dmul_rn(avg, swd), __dmul_rn(__dmul_rn(avg, avg), sw));
                    } else {  // SolarL2 / LOOL2 / SatL2: the sum of per-leaf terms
                        term = make_double2(gpu_score_term(score_fn, swd, sw), 0.0);
                    }
                    s_t[cc][lane] = term;
                }
            }
            if (c0 + kScorePiece < 2 * Q) {  // the next piece's loads overlap the ordered sum
                const int nc = c0 + kScorePiece;
                load_piece(nc, 2 * Q - nc < kScorePiece ? 2 * Q - nc : kScorePiece);
            }
            __syncthreads();
            if (warp == 0 && in) {
                int cc = 0;
                if (score_fn == 0) {
                    for (; cc + 8 <= pc; cc += 8) {
                        double2 t[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k) t[k] = s_t[cc + k][lane];
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            num = __dadd_rn(num, t[k].x);
                            den = __dadd_rn(den, t[k].y);
                        }
                    }
                    for (; cc < pc; ++cc) {
                        const double2 t = s_t[cc][lane];
                        num = __dadd_rn(num, t.x);
                        den = __dadd_rn(den, t.y);
                    }
                } else {
                    for (; cc + 8 <= pc; cc += 8) {
                        double t[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k) t[k] = s_t[cc + k][lane].x;
#pragma unroll
                        for (int k = 0; k < 8; ++k) num = __dadd_rn(num, t[k]);
                    }
                    for (; cc < pc; ++cc) num = __dadd_rn(num, s_t[cc][lane].x);
                }
            }
            __syncthreads();
        }
    }
    if (warp == 0) {
        double best = -INFINITY;
        int bbin = 0x7fffffff;
        if (in) {
            best = nan_to_neg_inf(score_fn == 0 ? __ddiv_rn(num, sqrt(den)) : num);
            bbin = b;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            double os = __shfl_xor_sync(kFull, best, o);
            int ob = __shfl_xor_sync(kFull, bbin, o);
            if (better(os, ob, best, bbin)) { best = os; bbin = ob; }
        }
        if (lane == 0) {
            grp_score[(size_t)fl * G + g] = best;
            grp_bin[(size_t)fl * G + g] = bbin;
            __threadfence();
            const unsigned done = atomicAdd(&ts->score_done, 1u);
            s_last = (done == gridDim.x * gridDim.y - 1);
        }
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // (feature, border) order: key f * 256 + border, lowest key wins ties.
    // The other blocks' records are read from L2 (ld.cg), a batch of loads
    // in flight per thread.
    double fb = -INFINITY;
    int fk = 0x7fffffff;
    constexpr int kBatch = 8;
    for (int e0 = threadIdx.x; e0 < Fs * G; e0 += blockDim.x * kBatch) {
        double sc[kBatch];
        int bin[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const int e = e0 + j * blockDim.x;
            sc[j] = -INFINITY;
            bin[j] = 0x7fffffff;
            if (e < Fs * G) {
                sc[j] = __ldcg(grp_score + e);
                bin[j] = __ldcg(grp_bin + e);
            }
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const int e = e0 + j * blockDim.x;
            if (bin[j] == 0x7fffffff) continue;
            const int key = (f0 + e / G) * 256 + bin[j];
            if (better(sc[j], key, fb, fk)) { fb = sc[j]; fk = key; }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        double os = __shfl_xor_sync(kFull, fb, o);
        int ok = __shfl_xor_sync(kFull, fk, o);
        if (better(os, ok, fb, fk)) { fb = os; fk = ok; }
    }
    if (lane == 0) { s_sc[warp] = fb; s_bi[warp] = fk; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kScoreWarps; ++w)
            if (better(s_sc[w], s_bi[w], fb, fk)) { fb = s_sc[w]; fk = s_bi[w]; }
        ts->score_done = 0;
        if (rank_best) {  // this rank's feature slice: (score bits, key) for the all-gather
            rank_best[0] = (ull)__double_as_longlong(fb);
            rank_best[1] = (ull)(uint32_t)fk;
            s_bi[0] = fk;
        }
    }
    if (rank_best) {
        // ... followed by the slice winner's per-leaf (false, true) weight
        // channel sums, from which every rank picks the smaller child to build
        __syncthreads();
        const int k = s_bi[0];
        for (int q = threadIdx.x; q < Q; q += blockDim.x) {
            ull fm = 0ull, tm = 0ull;
            if (k != 0x7fffffff) {
                const ull* row = cur + ((size_t)((k >> 8) - f0) * Q + q) * B * 2;
                fm = row[2 * (k & 255) + 1];
                tm = row[2 * (B - 1) + 1] - fm;
            }
            rank_best[2 + 2 * q] = fm;
            rank_best[3 + 2 * q] = tm;
        }
        return;
    }
    if (threadIdx.x == 0) {
        SplitRec rec;
        if (fk == 0x7fffffff || fb == -INFINITY) {
            rec.feature = -1;
            rec.bin = -1;
            rec.score = -INFINITY;
            atomicOr(&ts->err, kErrNoCandidate);
        } else {
            rec.feature = fk >> 8;
            rec.bin = fk & 255;
            rec.score = fb;
        }
        ts->split[level] = rec;
        s_bi[0] = fk;
    }
    if (small_side) {  // the next level builds, per leaf, the winner's lighter child
        __syncthreads();
        const int k = s_bi[0];
        for (int q = threadIdx.x; q < Q; q += blockDim.x) {
            uint8_t side = 1;
            if (k != 0x7fffffff) {
                const ull* row = cur + ((size_t)((k >> 8) - f0) * Q + q) * B * 2;
                const ull fm = row[2 * (k & 255) + 1];
                side = true_child_built(fm, row[2 * (B - 1) + 1] - fm);
            }
            small_side[q] = side;
        }
    }
}

void launch_score(int level, int32_t Fs, int32_t f0, int32_t F, int32_t B, const ull* cur,
                  const int32_t* border_counts, double l2, int score_fn, double* grp_score, int32_t* grp_bin,
                  TreeState* ts, ull* rank_best, uint8_t* small_side, cudaStream_t st) {
    const unsigned G = (unsigned)((B - 1 + 31) / 32);  // border groups: borders <= B - 1
    score_kernel<<<dim3(G > 0 ? G : 1, (unsigned)Fs), kScoreWarps * 32, 0, st>>>(
        level, Fs, f0, F, B, cur, border_counts, l2, score_fn, grp_score, grp_bin, ts, rank_best,
        rank_best ? nullptr : small_side);
}

// The winner over the ranks' slice winners, gathered as (score bits, key,
// per-leaf (false, true) weight sums) records of `stride` words: max score,
// then lowest key, as the single-device scan would pick.  When a next level
// follows, small_side[q] = 1 when leaf q's true child carries no more weight
// than its false child (the rows to histogram; which child is built changes
// no result, the sums are exact), replacing an all-reduce of child counts.
__global__ void select_split_kernel(int level, int world, int stride, const ull* __restrict__ all_best,
                                    TreeState* ts, uint8_t* __restrict__ small_side) {
    __shared__ int s_r;
    if (threadIdx.x == 0) {
        double fb;
        int fk;
        const int fr = pick_split(all_best, world, stride, &fb, &fk);
        SplitRec rec;
        if (fr < 0) {
            rec.feature = -1;
            rec.bin = -1;
            rec.score = -INFINITY;
            atomicOr(&ts->err, kErrNoCandidate);
        } else {
            rec.feature = fk >> 8;
            rec.bin = fk & 255;
            rec.score = fb;
        }
        ts->split[level] = rec;
        s_r = fr;
    }
    __syncthreads();
    if (!small_side) return;
    const int Q = 1 << level;
    const ull* rec = s_r >= 0 ? all_best + (size_t)s_r * stride : nullptr;
    for (int q = threadIdx.x; q < Q; q += blockDim.x) small_side[q] = build_true_side(rec, q);
}

void launch_select_split(int level, int world, int stride, const ull* all_best, TreeState* ts,
                         uint8_t* small_side, cudaStream_t st) {
    select_split_kernel<<<1, 256, 0, st>>>(level, world, stride, all_best, ts, small_side);
}

// ============================================================================
// the chosen split of a level: the feature's column and its border
// ============================================================================

struct PartView {
    const uint8_t* col;
    int32_t bin;
    bool eq;        // one-hot feature: the row passes on bin == value, else on bin > border
    bool vec;       // the column rows can be read 16 at a time (16-byte aligned)
};

__device__ __forceinline__ PartView make_part_view(int32_t feature, int32_t bin, int32_t f_eq,
                                                   const uint8_t* bins_fm, int64_t n_stride) {
    PartView v;
    const int f = feature < 0 ? 0 : feature;
    v.col = bins_fm + (int64_t)f * n_stride;
    v.bin = feature < 0 ? 0x7fffffff : bin;
    v.eq = feature >= f_eq;
    v.vec = (n_stride & 15) == 0;
    return v;
}

__device__ __forceinline__ PartView part_view(const TreeState* ts, int level, const uint8_t* bins_fm,
                                              int64_t n_stride) {
    const SplitRec s = ts->split[level];
    return make_part_view(s.feature, s.bin, 0x7fffffff, bins_fm, n_stride);
}

// The split of `level` from a record array of `stride` 32-bit words per level
// whose first two words are (feature, bin); features >= f_eq route by equality.
__device__ __forceinline__ PartView part_view_of(const int32_t* splits, int stride, int f_eq, int level,
                                                 const uint8_t* bins_fm, int64_t n_stride) {
    return make_part_view(splits[level * stride], splits[level * stride + 1], f_eq, bins_fm, n_stride);
}

__device__ __forceinline__ uint32_t passes(const PartView& pv, uint32_t b) {
    return pv.eq ? (uint32_t)((int32_t)b == pv.bin) : (uint32_t)((int32_t)b > pv.bin);
}

// ============================================================================
// partition: route and list in one pass
// ============================================================================
// After split l is chosen every row's leaf id gains bit l (routing,
// tree.rs:1005-1016), and the next level needs, for each of its 2^l parents,
// the rows of the child it builds (the sibling is derived by subtraction,
// tree.rs:1075-1131).  Which child is built changes no result -- the sums are
// exact -- so the side is chosen before routing, from the split's (false,
// true) weight sums that the score kernel (one GPU) or select_split (ranks)
// already holds: the child with no more weight than its sibling.  Every
// parent q owns a segment [base[q], base[q] + rows[q]) of the row list, laid
// out in parent order from the parents' row counts, so its built child's
// rows (at most rows[q]) fit without a counting pass.  Two kernels:
//  partition: leaf[i] |= (bin[f][i] > b) << l over rows in natural order (16
//             consecutive rows per thread, 16-byte loads); each block writes
//             its built-child rows to a range of each parent's segment
//             reserved with one atomic per (block, parent);
//  segments:  the built children's extents become the next level's
//             histogram work list; the 2^(l+1) children's row counts (built:
//             listed rows; sibling: parent minus built) lay out the next
//             partition's segments.
// Rows of a segment appear in block-scheduling order; the histograms, exact
// integer sums, do not depend on it.

constexpr int kRouteThreads = 256;
constexpr int kRouteRows = 16;  // consecutive rows per thread
constexpr int kRouteTile = kRouteThreads * kRouteRows;
constexpr int kPartSmemParents = 256;  // deeper levels reserve one slot per row

// Leaf ids of the thread's 16 rows after split `level`: lv[k] = old id | side
// << level (the old id is not read at level 0); written back.  Rows past n
// get ~0.
__device__ __forceinline__ void route_rows(int level, int64_t n, int64_t r0, const PartView& pv,
                                           uint16_t* __restrict__ leaf, uint32_t (&lv)[kRouteRows]) {
    if (pv.vec && r0 + kRouteRows <= n) {
        const uint4 v = __ldg((const uint4*)(pv.col + r0));  // n_stride and r0 are multiples of 16
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        if (level > 0) {
            const uint4 a = ((const uint4*)(leaf + r0))[0], b = ((const uint4*)(leaf + r0))[1];
            const uint32_t p[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int k = 0; k < kRouteRows; ++k) lv[k] = (p[k >> 1] >> ((k & 1) * 16)) & 0xffffu;
        } else {
#pragma unroll
            for (int k = 0; k < kRouteRows; ++k) lv[k] = 0u;
        }
#pragma unroll
        for (int k = 0; k < kRouteRows; ++k)
            lv[k] |= passes(pv, (w[k >> 2] >> ((k & 3) * 8)) & 0xffu) << level;
        uint4 o0, o1;
        o0.x = lv[0] | (lv[1] << 16); o0.y = lv[2] | (lv[3] << 16);
        o0.z = lv[4] | (lv[5] << 16); o0.w = lv[6] | (lv[7] << 16);
        o1.x = lv[8] | (lv[9] << 16); o1.y = lv[10] | (lv[11] << 16);
        o1.z = lv[12] | (lv[13] << 16); o1.w = lv[14] | (lv[15] << 16);
        ((uint4*)(leaf + r0))[0] = o0;
        ((uint4*)(leaf + r0))[1] = o1;
    } else {
#pragma unroll
        for (int k = 0; k < kRouteRows; ++k) {
            const int64_t i = r0 + k;
            lv[k] = 0xffffffffu;
            if (i < n) {
                lv[k] = (level > 0 ? (uint32_t)leaf[i] : 0u) | (passes(pv, pv.col[i]) << level);
                leaf[i] = (uint16_t)lv[k];
            }
        }
    }
}

// Route, then list the built-child rows.  A row goes to parent q's segment
// when its new bit is the side small_side[q].  Ranks within the block: kQ > 0
// (levels 0 and 1, kQ = 2^level parents) one ballot per (row, parent); kQ ==
// 0 per-warp shared counters (at most kPartSmemParents parents), else one
// global slot per row.  The block then reserves one range per parent and
// writes its rows there.
template <int kQ>
__global__ void __launch_bounds__(kRouteThreads, 6) partition_kernel(int level, int64_t n,
                                                                     const uint8_t* __restrict__ bins_fm,
                                                                     int64_t n_stride,
                                                                     const int32_t* __restrict__ splits,
                                                                     int split_stride, int f_eq,
                                                                     uint16_t* __restrict__ leaf,
                                                                     const uint8_t* __restrict__ small_side,
                                                                     uint32_t* __restrict__ cursor,
                                                                     uint32_t* __restrict__ list) {
    constexpr int kWarps = kRouteThreads / 32;
    constexpr int kP = kQ > 0 ? kQ : kPartSmemParents;
    __shared__ uint32_t s_w[kWarps][kP];  // per-warp counts, then write bases
    __shared__ uint8_t s_side[kP];
    const uint32_t Q = 1u << level;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const bool smem = Q <= (uint32_t)kP;
    if (smem) {
        for (uint32_t q = threadIdx.x; q < Q; q += blockDim.x) s_side[q] = small_side[q];
        for (uint32_t k = threadIdx.x; k < kWarps * Q; k += blockDim.x) s_w[k >> level][k & (Q - 1u)] = 0u;
    }
    const PartView pv = part_view_of(splits, split_stride, f_eq, level, bins_fm, n_stride);
    const int64_t r0 = (int64_t)blockIdx.x * kRouteTile + (int64_t)threadIdx.x * kRouteRows;
    uint32_t lv[kRouteRows];
    route_rows(level, n, r0, pv, leaf, lv);
    if (!smem) {  // deep levels: one reserved slot per row
#pragma unroll
        for (int k = 0; k < kRouteRows; ++k) {
            if (lv[k] == 0xffffffffu) continue;
            const uint32_t q = lv[k] & (Q - 1u);
            if ((lv[k] >> level) == (uint32_t)small_side[q]) list[atomicAdd(&cursor[q], 1u)] = (uint32_t)(r0 + k);
        }
        return;
    }
    __syncthreads();
    // per row: parent << 16 | rank among the warp's rows of that parent (a
    // warp has 512 rows), or ~0 when the row is not listed
    uint32_t pr[kRouteRows];
    if (Q <= 64) {  // build sides as a bit mask in registers
        const unsigned long long sides =
            (unsigned long long)__ballot_sync(kFull, (uint32_t)lane < Q && s_side[lane]) |
            (Q > 32 ? (unsigned long long)__ballot_sync(kFull, (uint32_t)lane + 32 < Q && s_side[lane + 32]) << 32
                    : 0ull);
#pragma unroll
        for (int k = 0; k < kRouteRows; ++k) {
            const uint32_t q = lv[k] & (Q - 1u);
            const bool sel = lv[k] != 0xffffffffu && (lv[k] >> level) == (uint32_t)(sides >> q & 1ull);
            pr[k] = sel ? q << 16 : 0xffffffffu;
        }
    } else {
#pragma unroll
        for (int k = 0; k < kRouteRows; ++k) {
            const uint32_t q = lv[k] & (Q - 1u);
            const bool sel = lv[k] != 0xffffffffu && (lv[k] >> level) == (uint32_t)s_side[q];
            pr[k] = sel ? q << 16 : 0xffffffffu;
        }
    }
    if (kQ > 0) {
        const uint32_t lt = (1u << lane) - 1u;
        uint32_t run[kQ > 0 ? kQ : 1];
#pragma unroll
        for (int v = 0; v < (kQ > 0 ? kQ : 1); ++v) run[v] = 0u;
#pragma unroll
        for (int k = 0; k < kRouteRows; ++k) {
#pragma unroll
            for (int v = 0; v < (kQ > 0 ? kQ : 1); ++v) {
                const bool mine = pr[k] == ((uint32_t)v << 16);
                const uint32_t m = __ballot_sync(kFull, mine);
                if (mine) pr[k] |= run[v] + (uint32_t)__popc(m & lt);
                run[v] += (uint32_t)__popc(m);
            }
        }
        if (lane == 0) {
#pragma unroll
            for (int v = 0; v < (kQ > 0 ? kQ : 1); ++v)
                if ((uint32_t)v < Q) s_w[warp][v] = run[v];
        }
    } else {
#pragma unroll
        for (int k = 0; k < kRouteRows; ++k)
            if (pr[k] != 0xffffffffu) pr[k] |= atomicAdd(&s_w[warp][pr[k] >> 16], 1u);
    }
    __syncthreads();
    for (uint32_t q = threadIdx.x; q < Q; q += blockDim.x) {
        uint32_t tot = 0;
        for (int w = 0; w < kWarps; ++w) tot += s_w[w][q];
        uint32_t at = tot ? atomicAdd(&cursor[q], tot) : 0u;
        for (int w = 0; w < kWarps; ++w) {
            const uint32_t c = s_w[w][q];
            s_w[w][q] = at;
            at += c;
        }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kRouteRows; ++k)
        if (pr[k] != 0xffffffffu) list[s_w[warp][pr[k] >> 16] + (pr[k] & 0xffffu)] = (uint32_t)(r0 + k);
}

// One block, after the partition of split `level` (Q = 2^level parents):
// parent q's built child holds cursor[q] - base[q] listed rows (rows_in null:
// one parent of n rows; base_in null: base 0).  Writes the next level's
// histogram work list (each built segment cut into cr-row items, cr <= kChunkRows, in
// parent order, cap items at most) and ts->hist_rows[level + 1]; when rows_out
// is not null, the 2Q children's row counts (child q + side * Q) with their
// segments (exclusive prefix in child order) as rows_out / base_out, and
// cursor_out = base_out for the next partition.
constexpr uint32_t kSegItemSmem = 2048;  // parents whose work items all threads write

__global__ void __launch_bounds__(1024) segments_kernel(int level, int64_t n, const uint32_t* __restrict__ rows_in,
                                                        const uint32_t* __restrict__ base_in,
                                                        const uint32_t* __restrict__ cursor,
                                                        const uint8_t* __restrict__ small_side,
                                                        uint32_t* __restrict__ rows_out, uint32_t* __restrict__ base_out,
                                                        uint32_t* __restrict__ cursor_out, HistChunk* __restrict__ chunks,
                                                        uint32_t cap, uint32_t* __restrict__ n_chunks, TreeState* ts,
                                                        uint32_t cr) {
    __shared__ uint32_t s_scan[40];
    __shared__ uint32_t s_first[kSegItemSmem];  // first work item of each parent
    const uint32_t Q = 1u << level;
    const uint32_t per = (Q + blockDim.x - 1) / blockDim.x;
    const uint32_t q0 = threadIdx.x * per;
    auto base_of = [&](uint32_t q) { return base_in ? base_in[q] : 0u; };
    uint32_t rows = 0, items = 0;
    for (uint32_t q = q0; q < q0 + per && q < Q; ++q) {
        const uint32_t cnt = cursor[q] - base_of(q);
        rows += cnt;
        items += (cnt + cr - 1) / cr;
    }
    uint32_t rows_tot, items_tot;
    (void)block_excl_scan<uint32_t>(rows, s_scan, &rows_tot);
    uint32_t item = block_excl_scan<uint32_t>(items, s_scan, &items_tot);
    if (Q <= kSegItemSmem) {
        // few parents, many items each: every thread writes items, finding
        // an item's parent by binary search over the parents' first items
        for (uint32_t q = q0; q < q0 + per && q < Q; ++q) {
            s_first[q] = item;
            item += (cursor[q] - base_of(q) + cr - 1) / cr;
        }
        __syncthreads();
        const uint32_t lim = items_tot < cap ? items_tot : cap;
        for (uint32_t it = threadIdx.x; it < lim; it += blockDim.x) {
            uint32_t lo = 0, hi = Q - 1;  // last parent whose first item <= it
            while (lo < hi) {
                const uint32_t mid = (lo + hi + 1) >> 1;
                if (s_first[mid] <= it) lo = mid;
                else hi = mid - 1;
            }
            const uint32_t b = base_of(lo), cnt = cursor[lo] - b, st = (it - s_first[lo]) * cr;
            chunks[it] = HistChunk{lo, b + st, cnt - st < cr ? cnt - st : cr, 0u};
        }
    } else {
        for (uint32_t q = q0; q < q0 + per && q < Q; ++q) {
            const uint32_t b = base_of(q), cnt = cursor[q] - b;
            for (uint32_t st = 0; st < cnt; st += cr) {
                if (item < cap) chunks[item] = HistChunk{q, b + st, cnt - st < cr ? cnt - st : cr, 0u};
                ++item;
            }
        }
    }
    if (threadIdx.x == 0) {
        if (items_tot > cap) {  // cannot happen with the session's sizing; never write past the buffer
            atomicOr(&ts->err, kErrChunkCap);
            items_tot = cap;
        }
        n_chunks[0] = items_tot;
        ts->hist_rows[level + 1] = rows_tot;
    }
    if (!rows_out) return;
    // children j < 2Q in order: j = q + side * Q
    const uint32_t per2 = (2 * Q + blockDim.x - 1) / blockDim.x;
    const uint32_t j0 = threadIdx.x * per2;
    auto child_rows = [&](uint32_t j) {
        const uint32_t q = j & (Q - 1u), side = j >> level;
        const uint32_t built = cursor[q] - base_of(q);
        const uint32_t parent = rows_in ? rows_in[q] : (uint32_t)n;
        return side == (uint32_t)small_side[q] ? built : parent - built;
    };
    uint32_t sum = 0;
    for (uint32_t j = j0; j < j0 + per2 && j < 2 * Q; ++j) sum += child_rows(j);
    uint32_t off = block_excl_scan<uint32_t>(sum, s_scan, nullptr);
    for (uint32_t j = j0; j < j0 + per2 && j < 2 * Q; ++j) {
        const uint32_t c = child_rows(j);
        rows_out[j] = c;
        base_out[j] = off;
        cursor_out[j] = off;
        off += c;
    }
}

void launch_partition(int level, int64_t n, const uint8_t* bins_fm, int64_t n_stride, uint16_t* leaf,
                      const uint8_t* small_side, uint32_t* cursor, uint32_t* list, const int32_t* splits,
                      int split_stride, int f_eq, cudaStream_t st) {
    const int64_t tiles = (n + kRouteTile - 1) / kRouteTile;
    if (tiles <= 0) return;
    const unsigned g = (unsigned)tiles;
#define CBGPU_PART(K)                                                                                        \
    partition_kernel<K><<<g, kRouteThreads, 0, st>>>(level, n, bins_fm, n_stride, splits, split_stride, f_eq, \
                                                     leaf, small_side, cursor, list)
    if (level == 0) CBGPU_PART(1);
    else if (level == 1) CBGPU_PART(2);
    else CBGPU_PART(0);
#undef CBGPU_PART
}

void launch_segments(int level, int64_t n, const uint32_t* rows_in, const uint32_t* base_in, const uint32_t* cursor,
                     const uint8_t* small_side, uint32_t* rows_out, uint32_t* base_out, uint32_t* cursor_out,
                     HistChunk* chunks, uint32_t cap, uint32_t* n_chunks, TreeState* ts, uint32_t chunk_rows,
                     cudaStream_t st) {
    if (chunk_rows == 0 || chunk_rows > (uint32_t)kChunkRows) chunk_rows = kChunkRows;
    segments_kernel<<<1, 1024, 0, st>>>(level, n, rows_in, base_in, cursor, small_side, rows_out, base_out,
                                        cursor_out, chunks, cap, n_chunks, ts, chunk_rows);
}

// ============================================================================
// last split: the final leaf id of every row (natural order) and, in the same
// pass, the unsampled leaf sums (boosting.rs:2470-2517 Gradient leaves over
// the full w*der1 / w channels) as exact int64 sums.
// ============================================================================
constexpr int kLeafSmemDepth = 10;  // deeper trees add into the global sums per row
constexpr int kLeafsumBlocksPerSm = 4;

__global__ void __launch_bounds__(kRouteThreads) route_leafsum_kernel(int level, int64_t n,
                                                                      const uint8_t* __restrict__ bins_fm,
                                                                      int64_t n_stride,
                                                                      const TreeState* __restrict__ ts,
                                                                      uint16_t* __restrict__ leaf,
                                                                      const double* __restrict__ wd1,
                                                                      const double* __restrict__ weight,
                                                                      ull* __restrict__ leaf_sums) {
    // shared: [L] lo and [L] hi of w*der1, then of w (with weights) or [L] row
    // counts (without: every row adds the same fixed-point 1)
    extern __shared__ uint32_t lsm[];
    const int L = 2 << level;
    const bool smem = level + 1 <= kLeafSmemDepth;
    const int parts = weight ? 4 : 3;
    if (smem) {
        for (int k = threadIdx.x; k < parts * L; k += blockDim.x) lsm[k] = 0u;
        __syncthreads();
    }
    const Pow2 sd = ts->sc.scale[2], sw = ts->sc.scale[3];
    const long long one = to_fixed(1.0, sw);
    const PartView pv = part_view(ts, level, bins_fm, n_stride);
    const int64_t tiles = (n + kRouteTile - 1) / kRouteTile;
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
        const int64_t r0 = t * kRouteTile + (int64_t)threadIdx.x * kRouteRows;
        uint32_t lv[kRouteRows];
        route_rows(level, n, r0, pv, leaf, lv);
        double d[kRouteRows];
        if (r0 + kRouteRows <= n) {
#pragma unroll
            for (int k = 0; k < kRouteRows; k += 2) {
                const double2 v = *(const double2*)(wd1 + r0 + k);  // r0 is a multiple of 16 rows
                d[k] = v.x;
                d[k + 1] = v.y;
            }
        } else {
#pragma unroll
            for (int k = 0; k < kRouteRows; ++k) d[k] = r0 + k < n ? wd1[r0 + k] : 0.0;
        }
#pragma unroll
        for (int k = 0; k < kRouteRows; ++k) {
            if (lv[k] == 0xffffffffu) continue;
            const uint32_t q = lv[k];
            const long long vd = to_fixed(d[k], sd);
            if (smem) {
                add_split64(lsm + q, lsm + L + q, vd);
                if (weight) add_split64(lsm + 2 * L + q, lsm + 3 * L + q, to_fixed(weight[r0 + k], sw));
                else atomicAdd(lsm + 2 * L + q, 1u);
            } else {
                atomicAdd(leaf_sums + 2 * q, (ull)vd);
                atomicAdd(leaf_sums + 2 * q + 1, (ull)(weight ? to_fixed(weight[r0 + k], sw) : one));
            }
        }
    }
    if (!smem) return;
    __syncthreads();
    for (int q = threadIdx.x; q < L; q += blockDim.x) {
        const ull sdv = ((ull)lsm[L + q] << 32) + lsm[q];
        const ull swv = weight ? ((ull)lsm[3 * L + q] << 32) + lsm[2 * L + q]
                               : (ull)lsm[2 * L + q] * (ull)one;
        if (sdv) atomicAdd(leaf_sums + 2 * q, sdv);
        if (swv) atomicAdd(leaf_sums + 2 * q + 1, swv);
    }
}

void launch_route_leafsum(int level, int64_t n, const uint8_t* bins_fm, int64_t n_stride, uint16_t* leaf,
                          const double* wd1, const double* weight, TreeState* ts, ull* leaf_sums, cudaStream_t st) {
    const int64_t tiles = (n + kRouteTile - 1) / kRouteTile;
    if (tiles <= 0) return;
    int64_t blocks = tiles < 148 * kLeafsumBlocksPerSm ? tiles : 148 * kLeafsumBlocksPerSm;
    const size_t smem = level + 1 <= kLeafSmemDepth ? sizeof(uint32_t) * (weight ? 4 : 3) * ((size_t)2 << level) : 0;
    route_leafsum_kernel<<<(unsigned)blocks, kRouteThreads, smem, st>>>(level, n, bins_fm, n_stride, ts, leaf, wd1,
                                                                        weight, leaf_sums);
}

// Gradient leaf delta calc_average(sum w*der1, sum w, scaled_l2) (leaf.rs:161-199),
// then x learning rate for the resident approx (normalize_leaf_values).
__global__ void leaf_values_kernel(int depth, const ull* __restrict__ leaf_sums, double l2, double lr,
                                   const TreeState* __restrict__ ts, double* __restrict__ raw,
                                   double* __restrict__ lrv) {
    const int L = 1 << depth;
    const Pow2 id = ts->sc.inv[2], iw = ts->sc.inv[3];
    for (int q = blockIdx.x * blockDim.x + threadIdx.x; q < L; q += gridDim.x * blockDim.x) {
        const double sd = from_fixed((long long)leaf_sums[2 * q], id);
        const double sw = from_fixed((long long)leaf_sums[2 * q + 1], iw);
        const double v = sw > 0.0 ? __ddiv_rn(sd, __dadd_rn(sw, l2)) : 0.0;
        raw[q] = v;
        lrv[q] = __dmul_rn(v, lr);
    }
}

void launch_leaf_values(int depth, int n_splits_expected, const ull* leaf_sums, double l2, double lr,
                        TreeState* ts, double* leaf_raw, double* leaf_lrv, cudaStream_t st) {
    (void)n_splits_expected;
    int L = 1 << depth;
    leaf_values_kernel<<<(L + 255) / 256, 256, 0, st>>>(depth, leaf_sums, l2, lr, ts, leaf_raw,
                                                        leaf_lrv);
}

__global__ void leaf_export_kernel(int64_t n, const uint16_t* __restrict__ leaf, void* out, int bytes) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        uint16_t v = leaf[i];
        if (bytes == 1) ((uint8_t*)out)[i] = (uint8_t)v;
        else if (bytes == 2) ((uint16_t*)out)[i] = v;
        else ((uint32_t*)out)[i] = v;
    }
}

void launch_leaf_export(int64_t n, const uint16_t* leaf, void* out, int bytes, cudaStream_t st) {
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks < 1) return;
    leaf_export_kernel<<<(unsigned)blocks, 256, 0, st>>>(n, leaf, out, bytes);
}

__global__ void gradients_kernel(int64_t n, int loss, const double* __restrict__ approx,
                                 const double* __restrict__ target, double* __restrict__ d1,
                                 double* __restrict__ d2) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const double a = approx[i], t = target[i];
        if (loss == 0) {
            d1[i] = __dsub_rn(t, a);
            if (d2) d2[i] = -1.0;
        } else {
            const double e = exp(a);
            const double p = __dsub_rn(1.0, __ddiv_rn(1.0, __dadd_rn(1.0, e)));
            d1[i] = __dsub_rn(t, p);
            if (d2) d2[i] = -__dmul_rn(p, __dsub_rn(1.0, p));
        }
    }
}

void launch_gradients(int64_t n, int loss, const double* approx, const double* target, double* d1,
                      double* d2, cudaStream_t st) {
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks < 1) return;
    gradients_kernel<<<(unsigned)blocks, 256, 0, st>>>(n, loss, approx, target, d1, d2);
}


// ---- Exact leaves: MAE / Quantile (leaf.rs:445-520, boosting.rs:2561-2606) ----

// f32 bit pattern -> an unsigned key in f32::total_cmp order
__device__ __forceinline__ uint32_t f32_total_order(float v) {
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float f32_from_total_order(uint32_t u) {
    return __uint_as_float((u & 0x80000000u) ? (u ^ 0x80000000u) : ~u);
}

// keys[i] = leaf << 32 | order(f32(t - a)) (the residuals the CPU collects
// through f32, collect_leaf_residuals), w[i] = the object weight
__global__ void exact_keys_kernel(int64_t n, const double* __restrict__ approx, const double* __restrict__ target,
                                  const double* __restrict__ weight, const uint16_t* __restrict__ leaf,
                                  ull* __restrict__ keys, double* __restrict__ w) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float r = __double2float_rn(__dsub_rn(target[i], approx[i]));
        keys[i] = ((ull)leaf[i] << 32) | f32_total_order(r);
        w[i] = weight ? weight[i] : 1.0;
    }
}

constexpr int kExactThreads = 512;

// first index in [lo, hi) whose key's leaf part is >= q
__device__ __forceinline__ int64_t exact_leaf_start(const ull* keys, int64_t lo, int64_t hi, ull q) {
    while (lo < hi) {
        const int64_t mid = lo + (hi - lo) / 2;
        if ((keys[mid] >> 32) < q) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

// One block per leaf over its sorted members: total weight, the first member
// whose running weight reaches total * alpha - DBL_EPSILON (the last member if
// none), then the delta adjustment from the weights below / equal to it.  The
// block sums add in tree order, so they equal the CPU's sequential sums when
// the partial sums are exact in f64 (unit, integer or dyadic weights) and
// differ by rounding otherwise.
__global__ void __launch_bounds__(kExactThreads)
exact_leaf_kernel(int64_t n, const ull* __restrict__ keys, const double* __restrict__ w, double alpha,
                  double delta, double lr, double* __restrict__ leaf_raw, double* __restrict__ leaf_lrv) {
    using Reduce = cub::BlockReduce<double, kExactThreads>;
    using Scan = cub::BlockScan<double, kExactThreads>;
    __shared__ union {
        typename Reduce::TempStorage r;
        typename Scan::TempStorage s;
    } tmp;
    __shared__ int64_t s_lo, s_hi, s_hit;
    __shared__ double s_val;
    const ull q = blockIdx.x;
    if (threadIdx.x == 0) {
        s_lo = exact_leaf_start(keys, 0, n, q);
        s_hi = exact_leaf_start(keys, s_lo, n, q + 1);
        s_hit = INT64_MAX;
    }
    __syncthreads();
    const int64_t lo = s_lo, hi = s_hi;
    double out = 0.0;
    if (hi > lo && alpha <= 0.0) {
        out = (double)f32_from_total_order((uint32_t)keys[lo]);  // the minimum element
    } else if (hi > lo) {
        double part = 0.0;
        for (int64_t i = lo + threadIdx.x; i < hi; i += kExactThreads) part = __dadd_rn(part, w[i]);
        const double total = Reduce(tmp.r).Sum(part);
        if (threadIdx.x == 0) s_val = total;
        __syncthreads();
        const double need = __dmul_rn(s_val, alpha);
        const double bar = __dsub_rn(need, DBL_EPSILON);
        double carry = 0.0;
        for (int64_t base = lo; base < hi; base += kExactThreads) {
            const int64_t i = base + threadIdx.x;
            const double v = i < hi ? w[i] : 0.0;
            double inc, chunk;
            Scan(tmp.s).InclusiveSum(v, inc, chunk);
            __syncthreads();
            if (i < hi && __dadd_rn(carry, inc) >= bar) atomicMin((unsigned long long*)&s_hit, (unsigned long long)i);
            __syncthreads();
            if (s_hit != INT64_MAX) break;
            carry = __dadd_rn(carry, chunk);
        }
        const int64_t j = s_hit != INT64_MAX ? s_hit : hi - 1;
        const float qf = f32_from_total_order((uint32_t)keys[j]);
        double qv = (double)qf;
        if (delta > 0.0) {
            double less = 0.0, equal = 0.0;
            for (int64_t i = lo + threadIdx.x; i < hi; i += kExactThreads) {
                const float v = f32_from_total_order((uint32_t)keys[i]);
                if (v < qf) less = __dadd_rn(less, w[i]);
                else if (v == qf) equal = __dadd_rn(equal, w[i]);
            }
            __syncthreads();
            const double ls = Reduce(tmp.r).Sum(less);
            __syncthreads();
            const double es = Reduce(tmp.r).Sum(equal);
            if (threadIdx.x == 0) s_val = __dadd_rn(ls, __dmul_rn(es, alpha)) >= bar ? 1.0 : 0.0;
            __syncthreads();
            qv = s_val != 0.0 ? __dsub_rn(qv, delta) : __dadd_rn(qv, delta);
        }
        out = qv;
    }
    if (threadIdx.x == 0) {
        leaf_raw[q] = out;
        leaf_lrv[q] = __dmul_rn(out, lr);
    }
}

size_t exact_sort_scratch_bytes(int64_t n) {
    size_t bytes = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, bytes, (const ull*)nullptr, (ull*)nullptr, (const double*)nullptr,
                                    (double*)nullptr, (int)(n > 0 ? n : 1), 0, 48);
    return bytes;
}

void launch_exact_leaves(int depth, int64_t n, const double* approx, const double* target, const double* weight,
                         const uint16_t* leaf, ull* keys, ull* keys_sorted, double* w, double* w_sorted, void* tmp,
                         size_t tmp_bytes, double alpha, double delta, double lr, double* leaf_raw,
                         double* leaf_lrv, cudaStream_t st) {
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks < 1) blocks = 1;
    exact_keys_kernel<<<(unsigned)blocks, 256, 0, st>>>(n, approx, target, weight, leaf, keys, w);
    size_t bytes = tmp_bytes;
    cub::DeviceRadixSort::SortPairs(tmp, bytes, (const ull*)keys, keys_sorted, (const double*)w, w_sorted, (int)n, 0,
                                    32 + depth, st);
    exact_leaf_kernel<<<1u << depth, kExactThreads, 0, st>>>(n, keys_sorted, w_sorted, alpha, delta, lr, leaf_raw,
                                                             leaf_lrv);
}

}  // namespace cbgpu
