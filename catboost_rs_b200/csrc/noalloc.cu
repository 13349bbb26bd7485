// noalloc.cu -- a histogram entry point that allocates no device memory.
//
// Some callers cannot call cudaMalloc at the moment they need a histogram:
// code that runs while a CUDA graph is being captured (an allocation there
// breaks or invalidates the capture), serving processes whose device memory
// is fully reserved by their own pool allocator and who hand out only
// pre-owned buffers, and plugins hosted in frameworks that forbid allocation
// on their hot path.  cbgpu_histogram_noalloc serves them: the caller passes
// device pointers for the inputs and the output, and every piece of
// intermediate state lives in one file-scope device array below, fixed in
// size when the library is loaded.
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
constexpr size_t kOffMax = kOffNChunks + 256;                                 // ull [2] max |g|, |h| bits
constexpr size_t kScratchBytes = kOffMax + 256;

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
        }
    }
}

__global__ void na_max_kernel(int64_t n, const double* __restrict__ g, const double* __restrict__ h) {
    double mg = 0.0, mh = 0.0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        mg = fmax(mg, fabs(g[i]));
        mh = fmax(mh, fabs(h[i]));
    }
    for (int o = 16; o > 0; o >>= 1) {
        mg = fmax(mg, __shfl_xor_sync(0xffffffffu, mg, o));
        mh = fmax(mh, __shfl_xor_sync(0xffffffffu, mh, o));
    }
    ull* mx = (ull*)(g_na_scratch + kOffMax);
    if ((threadIdx.x & 31) == 0) {
        if (mg > 0.0) atomicMax(&mx[0], (ull)__double_as_longlong(mg));
        if (mh > 0.0) atomicMax(&mx[1], (ull)__double_as_longlong(mh));
    }
}

// The session's score-channel scale rule: max |v| * 2^s < 2^kPackBits.
__device__ __forceinline__ double na_scale(int c, bool inverse) {
    const double m = __longlong_as_double((long long)((ull*)(g_na_scratch + kOffMax))[c]);
    int s = 0;
    if (m > 0.0) {
        int e;
        frexp(m, &e);
        s = kPackBits - e;
    }
    return ldexp(1.0, inverse ? -s : s);
}

__global__ void na_pack_kernel(int64_t n, const double* __restrict__ g, const double* __restrict__ h) {
    const double sg = na_scale(0, false), sh = na_scale(1, false);
    uint4* qs = (uint4*)(g_na_scratch + kOffQstats);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const long long qg = __double2ll_rn(__dmul_rn(g[i], sg));
        const long long qh = __double2ll_rn(__dmul_rn(h[i], sh));
        qs[i] = make_uint4((uint32_t)(qg & ((1ll << kPackSplit) - 1)), (uint32_t)(int32_t)(qg >> kPackSplit),
                           (uint32_t)(qh & ((1ll << kPackSplit) - 1)), (uint32_t)(int32_t)(qh >> kPackSplit));
    }
}

__global__ void na_convert_kernel(int64_t cells, double* __restrict__ out) {
    const double ig = na_scale(0, true), ih = na_scale(1, true);
    const ull* acc = (const ull*)(g_na_scratch + kOffAcc);
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < 2 * cells;
         k += (int64_t)gridDim.x * blockDim.x)
        out[k] = __dmul_rn((double)(long long)acc[k], (k & 1) ? ih : ig);
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
    return CBGPU_OK;
}

}  // extern "C"
