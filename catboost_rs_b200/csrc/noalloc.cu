// noalloc.cu -- a histogram entry point that allocates no device memory.
//
// Some callers cannot call cudaMalloc at the moment they need a histogram:
// serving processes whose device memory is fully reserved by their own pool
// allocator and who hand out only pre-owned buffers, plugins hosted in
// frameworks that forbid allocation on their hot path, and latency-bound
// loops that cannot afford an allocator call (or its failure) per request.
// cbgpu_histogram_noalloc serves them: the caller passes device pointers for
// the inputs and the output, and every piece of intermediate state lives in
// one file-scope device array below, fixed in size when the library is
// loaded.
#include <cfloat>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/cbgpu.h"
#include "kernels.cuh"

using namespace cbgpu;

namespace {

constexpr int64_t kNaMaxRows = 262144;                 // rows per call
constexpr int64_t kNaMaxCells = 256 * 256;             // n_features * n_bins per call
constexpr int64_t kNaMaxChunks = kNaMaxRows / kChunkRows + 1;

// Layout of the scratch array (byte offsets, each 256-aligned).
constexpr size_t kOffQstats = 0;                                              // uint4 [kNaMaxRows]
constexpr size_t kOffAcc = kOffQstats + sizeof(uint4) * kNaMaxRows;           // ull [kNaMaxCells][2]
constexpr size_t kOffChunks = kOffAcc + sizeof(ull) * 2 * kNaMaxCells;        // HistChunk [kNaMaxChunks]
constexpr size_t kOffNChunks = kOffChunks + 256 * ((sizeof(HistChunk) * kNaMaxChunks + 255) / 256);
constexpr size_t kOffMax = kOffNChunks + 256;  // ull [2] max |g|, |h| bits, then the u32 error word
constexpr size_t kOffErr = kOffMax + 2 * sizeof(unsigned long long);
constexpr size_t kScratchBytes = kOffMax + 256;

// Error word bits: the call then builds no histogram and writes NaN.
constexpr uint32_t kNaBadBin = 1u;      // some bin >= n_bins in the first n_features columns
constexpr uint32_t kNaNonFinite = 2u;   // some g or h is NaN or infinite

// The scratch: ~5.1 MiB held by every GPU that loads the library until exit.
// Host code must not use this name as a pointer (it is a host-side stand-in);
// the host obtains the device address with cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_na_scratch[kScratchBytes];

std::mutex g_na_mu;
void* g_na_addr[256] = {};  // per device ordinal, filled on the first call on that device

}  // namespace

namespace cbgpu {
int record_error(int code, const char* msg);  // session.cu: sets cbgpu_last_error()
}

namespace {

int na_fail(int code, const std::string& msg) { return cbgpu::record_error(code, msg.c_str()); }

// Zeroes what must start at zero (the int64 accumulators and the maxima) and
// writes the all-rows work list: the array keeps the previous call's contents.
__global__ void na_init_kernel(int64_t n, int64_t cells) {
    ull* acc = (ull*)(g_na_scratch + kOffAcc);
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < 2 * cells;
         k += (int64_t)gridDim.x * blockDim.x)
        acc[k] = 0ull;
    if (blockIdx.x == 0) {
        HistChunk* ch = (HistChunk*)(g_na_scratch + kOffChunks);
        const uint32_t nch = (uint32_t)((n + kChunkRows - 1) / kChunkRows);
        for (uint32_t k = threadIdx.x; k < nch; k += blockDim.x) {
            const uint32_t st = k * kChunkRows;
            ch[k] = HistChunk{0u, st, (uint32_t)(n - st < kChunkRows ? n - st : kChunkRows), 0u};
        }
        if (threadIdx.x == 0) {
            *(uint32_t*)(g_na_scratch + kOffNChunks) = nch;
            ull* mx = (ull*)(g_na_scratch + kOffMax);
            mx[0] = 0ull;
            mx[1] = 0ull;
            *(uint32_t*)(g_na_scratch + kOffErr) = 0u;
        }
    }
}

// Range check of the bins the histogram will index: the histogram kernel
// adds into a shared-memory table of n_bins rows per feature, so a larger
// bin would write outside it.  16-byte loads over each row's first
// n_features bytes (the padding past them is not read by the histogram).
__global__ void na_check_bins_kernel(int64_t n, int32_t n_features, int32_t row_stride, int32_t n_bins,
                                     const uint8_t* __restrict__ bins) {
    const int32_t pieces = (n_features + 15) / 16;
    const int64_t work = n * pieces;
    bool bad = false;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < work;
         k += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = k / pieces;
        const int32_t p = (int32_t)(k % pieces);
        const uint4 v = *(const uint4*)(bins + r * row_stride + 16 * p);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 16; ++j)
            bad |= 16 * p + j < n_features && ((w[j >> 2] >> (8 * (j & 3))) & 0xffu) >= (uint32_t)n_bins;
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0)
        atomicOr((uint32_t*)(g_na_scratch + kOffErr), kNaBadBin);
}

// max |g|, |h| for the fixed-point scales; NaN or infinity sets the error word
// (fmax would drop a NaN, and an infinite maximum has no scale).
__global__ void na_max_kernel(int64_t n, const double* __restrict__ g, const double* __restrict__ h) {
    double mg = 0.0, mh = 0.0;
    bool bad = false;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const double a = g[i], b = h[i];
        bad |= !isfinite(a) || !isfinite(b);
        mg = fmax(mg, fabs(a));
        mh = fmax(mh, fabs(b));
    }
    for (int o = 16; o > 0; o >>= 1) {
        mg = fmax(mg, __shfl_xor_sync(0xffffffffu, mg, o));
        mh = fmax(mh, __shfl_xor_sync(0xffffffffu, mh, o));
    }
    bad = __any_sync(0xffffffffu, bad);
    ull* mx = (ull*)(g_na_scratch + kOffMax);
    if ((threadIdx.x & 31) == 0) {
        if (mg > 0.0) atomicMax(&mx[0], (ull)__double_as_longlong(mg));
        if (mh > 0.0) atomicMax(&mx[1], (ull)__double_as_longlong(mh));
        if (bad) atomicOr((uint32_t*)(g_na_scratch + kOffErr), kNaNonFinite);
    }
}

// The session's score-channel scale rule (fixed_shift, pow2_of): max |v| * 2^s < 2^kPackBits.
__device__ __forceinline__ Pow2 na_scale(int c, bool inverse) {
    const double m = __longlong_as_double((long long)((ull*)(g_na_scratch + kOffMax))[c]);
    const int s = fixed_shift(m, kPackBits);
    return pow2_of(inverse ? -s : s);
}

// Packs the rows; when the checks failed, empties the work list instead so
// the histogram kernel does nothing.
__global__ void na_pack_kernel(int64_t n, const double* __restrict__ g, const double* __restrict__ h) {
    if (*(const volatile uint32_t*)(g_na_scratch + kOffErr) != 0u) {
        if (blockIdx.x == 0 && threadIdx.x == 0) *(uint32_t*)(g_na_scratch + kOffNChunks) = 0u;
        return;
    }
    const Pow2 sg = na_scale(0, false), sh = na_scale(1, false);
    uint4* qs = (uint4*)(g_na_scratch + kOffQstats);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        qs[i] = pack_gh(g[i], h[i], sg, sh);
}

__global__ void na_convert_kernel(int64_t cells, double* __restrict__ out) {
    const bool failed = *(const volatile uint32_t*)(g_na_scratch + kOffErr) != 0u;
    const Pow2 ig = na_scale(0, true), ih = na_scale(1, true);
    const ull* acc = (const ull*)(g_na_scratch + kOffAcc);
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < 2 * cells;
         k += (int64_t)gridDim.x * blockDim.x)
        out[k] = failed ? __longlong_as_double(0x7ff8000000000000ll) : from_fixed((long long)acc[k], (k & 1) ? ih : ig);
}

// Device address of the scratch array on the current device (set up once per device).
int na_scratch_addr(unsigned char** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 256)
        return na_fail(CBGPU_ERR_NO_DEVICE, std::string("no current CUDA device: ") + cudaGetErrorString(e));
    std::lock_guard<std::mutex> lk(g_na_mu);
    if (!g_na_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_na_scratch);
        if (e != cudaSuccess || !p)
            return na_fail(CBGPU_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch) failed: ") +
                                               cudaGetErrorString(e));
        g_na_addr[dev] = p;
    }
    *out = (unsigned char*)g_na_addr[dev];
    return CBGPU_OK;
}

unsigned grid_for(int64_t work) {
    int64_t b = (work + 255) / 256;
    if (b > 148 * 4) b = 148 * 4;
    return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace

extern "C" {

int cbgpu_histogram_noalloc(const uint8_t* d_bins_row_major, int64_t n, int32_t n_features,
                            int32_t row_stride, int32_t n_bins, const double* d_g, const double* d_h,
                            double* d_out_hist, void* stream) {
    if (n < 0 || n > kNaMaxRows)
        return na_fail(CBGPU_ERR_INVALID, "cbgpu_histogram_noalloc: n = " + std::to_string(n) +
                                              " rows is outside 0.." + std::to_string(kNaMaxRows));
    if (n_features < 1 || n_bins < 1 || n_bins > 256 || (int64_t)n_features * n_bins > kNaMaxCells)
        return na_fail(CBGPU_ERR_INVALID, "cbgpu_histogram_noalloc: n_features * n_bins must be in 1.." +
                                              std::to_string(kNaMaxCells) + " with n_bins <= 256");
    const int32_t f_pad = (n_features + 31) / 32 * 32;
    if (row_stride < f_pad || row_stride % 32 != 0)
        return na_fail(CBGPU_ERR_INVALID, "cbgpu_histogram_noalloc: row_stride must be a multiple of 32 "
                                          "and >= n_features rounded up to 32 (got " +
                                              std::to_string(row_stride) + ")");
    if (!d_out_hist || (n > 0 && (!d_bins_row_major || !d_g || !d_h)))
        return na_fail(CBGPU_ERR_INVALID, "cbgpu_histogram_noalloc: null pointer");
    if (((uintptr_t)d_bins_row_major & 15) != 0 || ((uintptr_t)d_g & 7) != 0 || ((uintptr_t)d_h & 7) != 0)
        return na_fail(CBGPU_ERR_INVALID, "cbgpu_histogram_noalloc: bins must be 16-byte aligned, g/h 8-byte");
    unsigned char* base = nullptr;
    int rc = na_scratch_addr(&base);
    if (rc) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t cells = (int64_t)n_features * n_bins;
    na_init_kernel<<<grid_for(2 * cells), 256, 0, st>>>(n, cells);
    if (n > 0) {
        if (n_bins < 256)
            na_check_bins_kernel<<<grid_for(n * ((n_features + 15) / 16)), 256, 0, st>>>(n, n_features, row_stride,
                                                                                      n_bins, d_bins_row_major);
        na_max_kernel<<<grid_for(n), 256, 0, st>>>(n, d_g, d_h);
        na_pack_kernel<<<grid_for(n), 256, 0, st>>>(n, d_g, d_h);
        launch_hist(d_bins_row_major, row_stride, n_features, n_bins, (const uint4*)(base + kOffQstats),
                    nullptr, (const HistChunk*)(base + kOffChunks), (const uint32_t*)(base + kOffNChunks),
                    (uint32_t)((n + kChunkRows - 1) / kChunkRows), (ull*)(base + kOffAcc), (int64_t)n_bins * 2,
                    (int64_t)n_features * n_bins * 2, st);
    }
    na_convert_kernel<<<grid_for(2 * cells), 256, 0, st>>>(cells, d_out_hist);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return na_fail(CBGPU_ERR_CUDA, std::string("cbgpu_histogram_noalloc launch failed: ") + cudaGetErrorString(e));
    // The checks' verdict: read the error word behind the work on `stream`
    // (into host stack memory, so nothing is allocated) and wait for it.
    uint32_t err = 0;
    e = cudaMemcpyAsync(&err, base + kOffErr, sizeof(err), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess)
        return na_fail(CBGPU_ERR_CUDA, std::string("cbgpu_histogram_noalloc: ") + cudaGetErrorString(e));
    if (err & kNaBadBin)
        return na_fail(CBGPU_ERR_DEVICE, "cbgpu_histogram_noalloc: a bin >= n_bins = " + std::to_string(n_bins) +
                                             " (no histogram was built; the output is NaN)");
    if (err & kNaNonFinite)
        return na_fail(CBGPU_ERR_DEVICE, "cbgpu_histogram_noalloc: g or h holds NaN or infinity "
                                         "(no histogram was built; the output is NaN)");
    return CBGPU_OK;
}

}  // extern "C"
