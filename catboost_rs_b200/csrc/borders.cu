// borders.cu -- float-feature border selection on the device.
//
// Restates catboost_rs's cb-data binarizers (crates/cb-data/src/borders.rs,
// border_types.rs) together with the builder's per-column NaN rule
// (crates/catboost-rs/src/builder.rs:1677-1720) so that fit preparation can
// pick the quantization borders next to the data instead of on the host:
//
//   1. host: the fixed-seed 200,000-object sample of borders.rs:504-520
//      (a partial Fisher-Yates with TFastRng64::from_seed(0); it depends only
//      on the row count, so every column shares it);
//   2. device, per batch of staged columns: a NaN scan of the full column
//      (the builder's has_nan test) and the gather of the sampled values as
//      order-preserving u32 keys (NaN -> 0xFFFFFFFF sorts last, -0.0 -> +0.0);
//   3. device, one 1024-thread block per feature: a stable 4-pass LSD radix
//      sort of the keys in global memory (ranks from __match_any_sync and
//      per-warp digit counts, so no atomics decide an order);
//   4. device, one warp per feature: the binarizer over the sorted values
//      (GreedyLogSum / GreedyMinEntropy heap, Median, Uniform,
//      UniformAndQuantiles), then the -0 -> +0 / sort / dedup finalisation and
//      the NaN sentinel.
//
// Border values are f32 computed with explicit round-to-nearest intrinsics;
// split scores are f64 (the reference's discipline, borders.rs:20-24).  The
// greedy penalty calls the device `log`, which may differ from the host libm
// in the last bit; a border can only differ from the CPU's where two candidate
// split scores agree to within that last bit.
#include <algorithm>
#include <cfloat>
#include <cstdarg>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/cbgpu.h"
#include "cbgpu_common.cuh"

using namespace cbgpu;

namespace cbgpu {
int record_error(int code, const char* msg);  // session.cu: sets cbgpu_last_error()
}

namespace {

constexpr int64_t kBorderSample = 200000;   // borders.rs:46 MAX_SUBSET_SIZE_FOR_BUILD_BORDERS
constexpr int kMaxBorderCount = 1024;       // per feature, sentinel included
constexpr int kSortThreads = 1024;
constexpr int kSortWarps = kSortThreads / 32;
constexpr uint32_t kNanKey = 0xFFFFFFFFu;

enum : uint32_t { kBErrCapacity = 1u << 0 };

int bfail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    return cbgpu::record_error(code, buf);
}

#define BCU(call)                                                                            \
    do {                                                                                     \
        cudaError_t _e = (call);                                                             \
        if (_e != cudaSuccess) {                                                             \
            rc = bfail(_e == cudaErrorMemoryAllocation ? CBGPU_ERR_OOM : CBGPU_ERR_CUDA,     \
                       "%s failed: %s", #call, cudaGetErrorString(_e));                      \
            goto done;                                                                       \
        }                                                                                    \
    } while (0)

// ---- keys -----------------------------------------------------------------

// Total-order key of a non-NaN f32 (the reference's radix key, borders.rs:448-456).
__device__ __forceinline__ uint32_t f32_key(float v) {
    uint32_t b = __float_as_uint(v);
    if ((b & 0x7FFFFFFFu) == 0u) b = 0u;  // -0.0 and +0.0 are one value everywhere downstream
    return (b & 0x80000000u) ? ~b : (b ^ 0x80000000u);
}

__device__ __forceinline__ float key_f32(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k ^ 0x80000000u) : ~k);
}

// has_nan[f0 + y] |= any NaN in staged column y (the builder's test over the
// FULL column, builder.rs:1684).
__global__ void border_nan_scan_kernel(const float* __restrict__ cols, int64_t n, int f0,
                                       uint32_t* __restrict__ has_nan) {
    const float* col = cols + (size_t)blockIdx.y * (size_t)n;
    bool any = false;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        any |= isnan(col[i]);
    any = __any_sync(0xffffffffu, any);
    if (any && (threadIdx.x & 31) == 0) atomicOr(&has_nan[f0 + blockIdx.y], 1u);
}

// keys[f][j] = key of the j-th sampled value (idx == nullptr: row j); counts
// the NaNs the sample holds.
__global__ void border_gather_kernel(const float* __restrict__ cols, int64_t n, int f0,
                                     const uint32_t* __restrict__ idx, int64_t m,
                                     uint32_t* __restrict__ keys, uint32_t* __restrict__ nan_cnt) {
    const int f = f0 + blockIdx.y;
    const float* col = cols + (size_t)blockIdx.y * (size_t)n;
    uint32_t* out = keys + (size_t)f * (size_t)m;
    uint32_t nans = 0;
    for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < m;
         j += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = idx ? (int64_t)idx[j] : j;
        const float v = row < n ? col[row] : __uint_as_float(0x7FC00000u);
        uint32_t k;
        if (isnan(v)) {
            k = kNanKey;
            ++nans;
        } else {
            k = f32_key(v);
        }
        out[j] = k;
    }
    for (int o = 16; o > 0; o >>= 1) nans += __shfl_xor_sync(0xffffffffu, nans, o);
    if ((threadIdx.x & 31) == 0 && nans) atomicAdd(&nan_cnt[f], nans);
}

// ---- stable LSD radix sort, one block per feature --------------------------
// Pass p moves keys by digit (key >> 8p) & 255.  Each 1024-key tile is ranked
// exactly: a key's position is base[digit] + (keys of that digit in earlier
// warps of the tile) + (keys of that digit in earlier lanes of its warp), so
// equal digits keep their input order.  Four passes leave the result in `a`.
__global__ void __launch_bounds__(kSortThreads, 1)
border_sort_kernel(uint32_t* __restrict__ keys_a, uint32_t* __restrict__ keys_b, int64_t m) {
    __shared__ uint32_t s_wc[kSortWarps][256];
    __shared__ uint32_t s_base[256];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t* src = keys_a + (size_t)blockIdx.x * (size_t)m;
    uint32_t* dst = keys_b + (size_t)blockIdx.x * (size_t)m;
    const uint32_t lt = (1u << lane) - 1u;
    for (int k = tid; k < kSortWarps * 256; k += kSortThreads) (&s_wc[0][0])[k] = 0u;
    for (int pass = 0; pass < 4; ++pass) {
        const int sh = pass * 8;
        if (tid < 256) s_base[tid] = 0u;
        __syncthreads();
        for (int64_t i = tid; i < m; i += kSortThreads) atomicAdd(&s_base[(src[i] >> sh) & 255u], 1u);
        __syncthreads();
        if (tid == 0) {
            uint32_t run = 0;
            for (int d = 0; d < 256; ++d) {
                const uint32_t c = s_base[d];
                s_base[d] = run;
                run += c;
            }
        }
        __syncthreads();
        for (int64_t t0 = 0; t0 < m; t0 += kSortThreads) {
            const int64_t i = t0 + tid;
            const bool valid = i < m;
            const uint32_t key = valid ? src[i] : 0u;
            const uint32_t d = valid ? ((key >> sh) & 255u) : 256u;
            const uint32_t peers = __match_any_sync(0xffffffffu, d);
            const uint32_t rank = __popc(peers & lt);
            if (valid && rank == 0) s_wc[warp][d] = (uint32_t)__popc(peers);
            __syncthreads();
            if (tid < 256) {
                uint32_t run = s_base[tid];
                for (int w = 0; w < kSortWarps; ++w) {
                    const uint32_t c = s_wc[w][tid];
                    s_wc[w][tid] = run;
                    run += c;
                }
                s_base[tid] = run;
            }
            __syncthreads();
            if (valid) {
                const uint32_t pos = s_wc[warp][d] + rank;
                if (pos < (uint64_t)m) dst[pos] = key;
            }
            __syncthreads();
            for (int k = tid; k < kSortWarps * 256; k += kSortThreads) (&s_wc[0][0])[k] = 0u;
            __syncthreads();
        }
        uint32_t* t = src;
        src = dst;
        dst = t;
    }
}

// ---- binarizers over the sorted values (lane 0 of one warp per feature) ---

struct GBin {
    int32_t start, end, best;
    uint32_t seq;
    double score;
};

struct Sorted {
    const uint32_t* k;
    __device__ __forceinline__ float operator[](int64_t i) const { return key_f32(k[i]); }
};

// penalties (borders.rs:51-63)
__device__ __forceinline__ double border_penalty(bool min_entropy, double w) {
    const double l = log(__dadd_rn(w, 1e-8));
    return min_entropy ? __dmul_rn(w, l) : -l;
}

// CalcSplitScore (borders.rs:157-170)
__device__ double split_score(const GBin& b, int32_t pos, bool me) {
    if (pos == b.start || pos == b.end) return -INFINITY;
    const double left = -border_penalty(me, (double)(pos - b.start));
    const double right = -border_penalty(me, (double)(b.end - pos));
    const double curr = -border_penalty(me, (double)(b.end - b.start));
    return __dsub_rn(__dadd_rn(left, right), curr);
}

// first index in [lo, hi) whose value is >= t (else hi)
__device__ int32_t lower_bound_v(const Sorted& v, int32_t lo, int32_t hi, float t) {
    while (lo < hi) {
        const int32_t mid = lo + (hi - lo) / 2;
        if (v[mid] < t) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

// first index in [lo, hi) whose value is > t (else hi)
__device__ int32_t upper_bound_v(const Sorted& v, int32_t lo, int32_t hi, float t) {
    while (lo < hi) {
        const int32_t mid = lo + (hi - lo) / 2;
        if (v[mid] <= t) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

// UpdateBestSplitProperties (borders.rs:178-198)
__device__ void update_best(GBin& b, const Sorted& v, bool me) {
    const int32_t mid = b.start + (b.end - b.start) / 2;
    const float mv = v[mid];
    const int32_t lb = lower_bound_v(v, b.start, mid, mv);
    const int32_t ub = upper_bound_v(v, mid, b.end, mv);
    const double sl = split_score(b, lb, me), sr = split_score(b, ub, me);
    if (sl >= sr) {
        b.best = lb;
        b.score = sl;
    } else {
        b.best = ub;
        b.score = sr;
    }
}

// queue order: higher score first, then earlier insertion (borders.rs:640-660)
__device__ __forceinline__ bool above(const GBin& a, const GBin& b) {
    if (a.score != b.score) return a.score > b.score;
    return a.seq < b.seq;
}

__device__ void heap_push(GBin* h, int& n, const GBin& x) {
    int i = n++;
    h[i] = x;
    while (i > 0) {
        const int p = (i - 1) / 2;
        if (!above(h[i], h[p])) break;
        const GBin t = h[i];
        h[i] = h[p];
        h[p] = t;
        i = p;
    }
}

__device__ GBin heap_pop(GBin* h, int& n) {
    const GBin top = h[0];
    h[0] = h[--n];
    int i = 0;
    for (;;) {
        const int l = 2 * i + 1, r = l + 1;
        int m = i;
        if (l < n && above(h[l], h[m])) m = l;
        if (r < n && above(h[r], h[m])) m = r;
        if (m == i) break;
        const GBin t = h[i];
        h[i] = h[m];
        h[m] = t;
        i = m;
    }
    return top;
}

// GreedySplit (borders.rs:572-619); left borders 0.5f*v[s-1] + 0.5f*v[s]
// (borders.rs:216-225).  Returns the number of borders written to out.
__device__ int greedy_borders(const Sorted& v, int32_t m, int max_b, bool me, GBin* heap, float* out) {
    if (m < 2) return 0;
    int hn = 0;
    uint32_t seq = 0;
    GBin root{0, m, 0, seq++, 0.0};
    update_best(root, v, me);
    heap_push(heap, hn, root);
    while (hn <= max_b) {
        const GBin& t = heap[0];
        if (!(t.start != t.best && t.end != t.best)) break;
        GBin top = heap_pop(heap, hn);
        GBin left{top.start, top.best, top.start, 0u, 0.0};
        update_best(left, v, me);
        top.start = top.best;
        update_best(top, v, me);
        left.seq = seq++;
        heap_push(heap, hn, left);
        top.seq = seq++;
        heap_push(heap, hn, top);
    }
    int k = 0;
    for (int i = 0; i < hn; ++i) {
        if (heap[i].start == 0) continue;
        const int32_t s = heap[i].start;
        out[k++] = __fadd_rn(__fmul_rn(0.5f, v[s - 1]), __fmul_rn(0.5f, v[s]));
    }
    return k;
}

// RegularBorder (border_types.rs:350-378)
__device__ float regular_border(float border, const Sorted& v, int32_t m) {
    const float front = v[0], back = v[m - 1];
    const int32_t idx = lower_bound_v(v, 0, m, border);
    if (idx == m) return fmaxf(__fmul_rn(2.0f, back), __fadd_rn(back, 1.0f));
    if (idx == 0) return fminf(__fmul_rn(0.5f, front), __fmul_rn(2.0f, front));
    const float hi = v[idx], lo = v[idx - 1];
    float res = __fmul_rn(__fadd_rn(hi, lo), 0.5f);
    if (res == hi) res = lo;
    return res;
}

// GenerateMedianBorders (border_types.rs:279-305)
__device__ int median_borders(const Sorted& v, int32_t m, int max_b, float* out) {
    if (m == 0) return 0;
    const float first = v[0];
    if (first == v[m - 1]) return 0;
    int k = 0;
    for (int i = 0; i < max_b; ++i) {
        uint64_t i1 = (uint64_t)(i + 1) * (uint64_t)m / (uint64_t)(max_b + 1);
        if (i1 > (uint64_t)(m - 1)) i1 = (uint64_t)(m - 1);
        const float val = v[(int64_t)i1];
        if (val != first) out[k++] = regular_border(val, v, m);
    }
    return k;
}

// TUniformBinarizer (border_types.rs:238-261); min and max of the values
__device__ int uniform_borders(const Sorted& v, int32_t m, int max_b, float* out) {
    if (m == 0) return 0;
    const float mn = v[0], mx = v[m - 1];
    if (mn == mx) return 0;
    const float span = __fsub_rn(mx, mn);
    for (int i = 0; i < max_b; ++i) {
        const float step = __fmul_rn((float)(i + 1), span);
        out[i] = __fadd_rn(mn, __fdiv_rn(step, (float)(max_b + 1)));
    }
    return max_b;
}

// TMedianPlusUniformBinarizer (border_types.rs:319-337)
__device__ int median_plus_uniform(const Sorted& v, int32_t m, int max_b, float* out) {
    if (m == 0) return 0;
    const float mn = v[0], mx = v[m - 1];
    if (mn == mx) return 0;
    const int half = max_b / 2;
    int k = median_borders(v, m, max_b - half, out);
    const float span = __fsub_rn(mx, mn);
    for (int i = 0; i < half; ++i) {
        const float step = __fmul_rn((float)(i + 1), span);
        const float val = __fadd_rn(mn, __fdiv_rn(step, (float)(half + 1)));
        out[k++] = regular_border(val, v, m);
    }
    return k;
}

struct SelectParams {
    int64_t m;            // sampled values per feature (key stride)
    int32_t border_count; // total budget per feature, sentinel included
    int32_t type;         // cbgpu_border_type
    int32_t nan_mode;     // cbgpu_nan_mode
};

__global__ void __launch_bounds__(32)
border_select_kernel(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ has_nan,
                     const uint32_t* __restrict__ nan_cnt, SelectParams p, double* __restrict__ out,
                     int32_t* __restrict__ counts, uint32_t* __restrict__ err) {
    __shared__ GBin s_heap[kMaxBorderCount + 3];
    __shared__ float s_b[kMaxBorderCount + 2];
    if (threadIdx.x != 0) return;
    const int f = blockIdx.x;
    const bool nan_col = has_nan[f] != 0u;
    const uint32_t sample_nans = nan_cnt[f];
    const int32_t m = (int32_t)(p.m - (int64_t)(sample_nans < (uint64_t)p.m ? sample_nans : p.m));
    const Sorted v{keys + (size_t)f * (size_t)p.m};
    // the builder's NaN rule: Min spends a slot on the prepended sentinel,
    // Max selects border_count - 1 and appends f32::MAX (builder.rs:1686-1710)
    const bool sentinel_min = nan_col && p.nan_mode == CBGPU_NAN_MIN;
    const bool sentinel_max = nan_col && p.nan_mode == CBGPU_NAN_MAX;
    const int max_b = (sentinel_min || sentinel_max) ? p.border_count - 1 : p.border_count;
    int k = 0;
    switch (p.type) {
    case CBGPU_BORDER_GREEDY_LOGSUM:
        k = greedy_borders(v, m, max_b, false, s_heap, s_b);
        break;
    case CBGPU_BORDER_GREEDY_MIN_ENTROPY:
        k = greedy_borders(v, m, max_b, true, s_heap, s_b);
        break;
    case CBGPU_BORDER_MEDIAN:
        k = median_borders(v, m, max_b, s_b);
        break;
    case CBGPU_BORDER_UNIFORM:
        k = uniform_borders(v, m, max_b, s_b);
        break;
    case CBGPU_BORDER_UNIFORM_AND_QUANTILES:
        k = median_plus_uniform(v, m, max_b, s_b);
        break;
    default:
        k = 0;
    }
    // finalize_border_set (borders.rs:403-424): -0 -> +0, ascending, dedup
    for (int i = 0; i < k; ++i)
        if ((__float_as_uint(s_b[i]) & 0x7FFFFFFFu) == 0u) s_b[i] = 0.0f;
    for (int i = 1; i < k; ++i) {
        const float x = s_b[i];
        int j = i - 1;
        while (j >= 0 && s_b[j] > x) {
            s_b[j + 1] = s_b[j];
            --j;
        }
        s_b[j + 1] = x;
    }
    double* o = out + (size_t)f * (size_t)p.border_count;
    int c = 0;
    if (sentinel_min) o[c++] = (double)(-FLT_MAX);
    for (int i = 0; i < k; ++i) {
        if (i > 0 && s_b[i] == s_b[i - 1]) continue;
        if (c >= p.border_count) {
            atomicOr(err, kBErrCapacity);
            break;
        }
        o[c++] = (double)s_b[i];
    }
    if (sentinel_max) {
        if (c < p.border_count) o[c++] = (double)FLT_MAX;
        else atomicOr(err, kBErrCapacity);
    }
    counts[f] = c;
}

// ---- host: the shared object sample (borders.rs:504-520) ------------------
// Partial Fisher-Yates over the implicit identity array; only touched
// positions are stored.  Returns the sorted sample.
std::vector<uint32_t> sample_indices(int64_t n, int64_t take) {
    std::unordered_map<uint64_t, uint32_t> moved;
    moved.reserve((size_t)(2 * take + 16));
    auto at = [&](uint64_t p) -> uint32_t {
        auto it = moved.find(p);
        return it == moved.end() ? (uint32_t)p : it->second;
    };
    Rng64 r = Rng64::from_seed(0);
    for (int64_t i = 0; i < take; ++i) {
        const uint64_t bound = (uint64_t)(n - i);
        const uint64_t randmax = UINT64_MAX - (UINT64_MAX % bound);  // Uniform (rng.rs:269-292)
        uint64_t x;
        do {
            x = r.gen();
        } while (x >= randmax);
        const uint64_t j = (uint64_t)i + x % bound;
        const uint32_t a = at((uint64_t)i), b = at(j);
        moved[(uint64_t)i] = b;
        moved[j] = a;
    }
    std::vector<uint32_t> out((size_t)take);
    for (int64_t i = 0; i < take; ++i) out[(size_t)i] = at((uint64_t)i);
    std::sort(out.begin(), out.end());
    return out;
}

}  // namespace

int cbgpu_select_borders(const float* const* float_columns, int64_t n, int32_t n_features,
                         int32_t border_count, int32_t border_type, int32_t nan_mode, int32_t device,
                         double* borders_out, int32_t* counts_out) {
    if (n < 0 || n > (int64_t)UINT32_MAX || n_features < 1 || !borders_out || !counts_out ||
        (n > 0 && !float_columns))
        return bfail(CBGPU_ERR_INVALID, "select_borders: bad arguments");
    if (border_count < 1 || border_count > kMaxBorderCount)
        return bfail(CBGPU_ERR_INVALID, "select_borders: border_count %d outside 1..%d", border_count,
                     kMaxBorderCount);
    if (nan_mode < CBGPU_NAN_MIN || nan_mode > CBGPU_NAN_FORBIDDEN)
        return bfail(CBGPU_ERR_INVALID, "select_borders: unknown nan_mode %d", nan_mode);
    switch (border_type) {
    case CBGPU_BORDER_MEDIAN:
    case CBGPU_BORDER_GREEDY_LOGSUM:
    case CBGPU_BORDER_UNIFORM_AND_QUANTILES:
    case CBGPU_BORDER_UNIFORM:
    case CBGPU_BORDER_GREEDY_MIN_ENTROPY:
        break;
    case CBGPU_BORDER_MIN_ENTROPY:
    case CBGPU_BORDER_MAX_LOGSUM:
        return bfail(CBGPU_DECLINED, "select_borders: the exact binarizers (MinEntropy, MaxLogSum) "
                                     "stay with cb-data");
    default:
        return bfail(CBGPU_ERR_INVALID, "select_borders: unknown border_type %d", border_type);
    }
    for (int f = 0; f < n_features && n > 0; ++f)
        if (!float_columns[f]) return bfail(CBGPU_ERR_INVALID, "select_borders: column %d is NULL", f);
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
        return bfail(CBGPU_ERR_NO_DEVICE, "no CUDA device");
    if (device < 0 || device >= ndev) return bfail(CBGPU_ERR_INVALID, "select_borders: bad device %d", device);
    if (n == 0) {
        for (int f = 0; f < n_features; ++f) counts_out[f] = 0;
        return CBGPU_OK;
    }

    int rc = CBGPU_OK;
    const int64_t m = std::min<int64_t>(n, kBorderSample);
    const int F = n_features;
    // columns staged per batch: about 1 GiB, at most 65535 (the grid's y extent)
    const int batch = (int)std::max<int64_t>(
        1, std::min<int64_t>(std::min<int64_t>(F, 65535), (int64_t)(1ll << 30) / (4 * n)));
    std::vector<uint32_t> sample;
    if (n > kBorderSample) sample = sample_indices(n, kBorderSample);

    cudaStream_t st = nullptr;
    float* d_cols = nullptr;
    uint32_t *d_idx = nullptr, *d_a = nullptr, *d_b = nullptr, *d_has = nullptr, *d_nan = nullptr, *d_err = nullptr;
    double* d_out = nullptr;
    int32_t* d_cnt = nullptr;
    uint32_t h_err = 0;
    std::vector<uint32_t> h_has((size_t)F, 0u);
    const SelectParams sp{m, border_count, border_type, nan_mode};
    int gx = (int)std::min<int64_t>(1024, (n + 255) / 256);
    int gm = (int)std::min<int64_t>(1024, (m + 255) / 256);

    BCU(cudaSetDevice(device));
    BCU(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    BCU(cudaMalloc((void**)&d_cols, sizeof(float) * (size_t)n * (size_t)batch));
    BCU(cudaMalloc((void**)&d_a, sizeof(uint32_t) * (size_t)m * (size_t)F));
    BCU(cudaMalloc((void**)&d_b, sizeof(uint32_t) * (size_t)m * (size_t)F));
    BCU(cudaMalloc((void**)&d_has, sizeof(uint32_t) * (size_t)F));
    BCU(cudaMalloc((void**)&d_nan, sizeof(uint32_t) * (size_t)F));
    BCU(cudaMalloc((void**)&d_err, sizeof(uint32_t)));
    BCU(cudaMalloc((void**)&d_out, sizeof(double) * (size_t)F * (size_t)border_count));
    BCU(cudaMalloc((void**)&d_cnt, sizeof(int32_t) * (size_t)F));
    BCU(cudaMemsetAsync(d_has, 0, sizeof(uint32_t) * (size_t)F, st));
    BCU(cudaMemsetAsync(d_nan, 0, sizeof(uint32_t) * (size_t)F, st));
    BCU(cudaMemsetAsync(d_err, 0, sizeof(uint32_t), st));
    if (!sample.empty()) {
        BCU(cudaMalloc((void**)&d_idx, sizeof(uint32_t) * sample.size()));
        BCU(cudaMemcpyAsync(d_idx, sample.data(), sizeof(uint32_t) * sample.size(), cudaMemcpyHostToDevice, st));
    }
    for (int f0 = 0; f0 < F; f0 += batch) {
        const int nb = std::min(batch, F - f0);
        for (int y = 0; y < nb; ++y)
            BCU(cudaMemcpyAsync(d_cols + (size_t)y * (size_t)n, float_columns[f0 + y], sizeof(float) * (size_t)n,
                                cudaMemcpyHostToDevice, st));
        border_nan_scan_kernel<<<dim3((unsigned)gx, (unsigned)nb), 256, 0, st>>>(d_cols, n, f0, d_has);
        BCU(cudaGetLastError());
        border_gather_kernel<<<dim3((unsigned)gm, (unsigned)nb), 256, 0, st>>>(d_cols, n, f0, d_idx, m, d_a, d_nan);
        BCU(cudaGetLastError());
    }
    border_sort_kernel<<<F, kSortThreads, 0, st>>>(d_a, d_b, m);
    BCU(cudaGetLastError());
    border_select_kernel<<<F, 32, 0, st>>>(d_a, d_has, d_nan, sp, d_out, d_cnt, d_err);
    BCU(cudaGetLastError());
    BCU(cudaMemcpyAsync(h_has.data(), d_has, sizeof(uint32_t) * (size_t)F, cudaMemcpyDeviceToHost, st));
    BCU(cudaMemcpyAsync(counts_out, d_cnt, sizeof(int32_t) * (size_t)F, cudaMemcpyDeviceToHost, st));
    BCU(cudaMemcpyAsync(borders_out, d_out, sizeof(double) * (size_t)F * (size_t)border_count,
                        cudaMemcpyDeviceToHost, st));
    BCU(cudaMemcpyAsync(&h_err, d_err, sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
    BCU(cudaStreamSynchronize(st));
    if (h_err) {
        rc = bfail(CBGPU_ERR_DEVICE, "select_borders: device error word 0x%x", h_err);
        goto done;
    }
    if (nan_mode == CBGPU_NAN_FORBIDDEN) {
        for (int f = 0; f < F; ++f)
            if (h_has[(size_t)f]) {
                // builder.rs:1660-1672: nan_mode=Forbidden refuses a NaN-bearing column
                rc = bfail(CBGPU_ERR_INVALID, "Feature #%d: There are nan factors and nan values for float "
                                              "features are not allowed. Set nan_mode != Forbidden.", f);
                goto done;
            }
    }
done:
    if (st) cudaStreamSynchronize(st);
    cudaFree(d_cols);
    cudaFree(d_idx);
    cudaFree(d_a);
    cudaFree(d_b);
    cudaFree(d_has);
    cudaFree(d_nan);
    cudaFree(d_err);
    cudaFree(d_out);
    cudaFree(d_cnt);
    if (st) cudaStreamDestroy(st);
    return rc;
}
