// apply.cu -- raw predictions of a float-only oblivious ensemble on the device.
//
// The reference's GPU apply (cb_backend::gpu_runtime::launch_apply_oblivious_f64
// over the CSR lowering of cb_model::flatten_oblivious_f64,
// crates/cb-model/src/gpu_apply.rs:83-193, kernel crates/cb-backend/src/
// kernels.rs:629-690) evaluates every tree for one object per thread, reading
// each split's feature from the feature-major matrix in HBM.  Here a block
// first stages its objects' whole feature rows in shared memory (one coalesced
// pass over the feature-major input, rows padded to an odd stride so the
// per-object reads are bank-conflict free), then each thread walks the trees
// from shared memory with the model's split and leaf arrays broadcast through
// the read-only cache.  HBM traffic is the feature matrix once plus the
// output, whatever the number of trees.
//
// Results follow the CPU apply (crates/cb-model/src/apply.rs:150-173, 374-410)
// bit for bit: a split passes iff (double)x > border, NaN takes the feature's
// nan_mode=Max rule (above every border) and otherwise fails, a feature index
// beyond the batch never passes, an out-of-range leaf contributes 0, and the
// prediction is bias + the per-tree values summed in tree order.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <vector>

#include "../../include/cbgpu.h"
#include "cbgpu_common.cuh"

namespace cbgpu {
int record_error(int code, const char* msg);  // session.cu: sets cbgpu_last_error()
}

namespace {

constexpr int kApplyMaxDepth = 16;             // tree.rs MAX_DEPTH
constexpr size_t kApplySmemBudget = 100 * 1024; // two staged blocks per SM
constexpr int64_t kApplyChunkBytes = 1ll << 30;  // feature bytes staged per chunk

int afail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    return cbgpu::record_error(code, buf);
}

#define ACU(call)                                                                            \
    do {                                                                                     \
        cudaError_t _e = (call);                                                             \
        if (_e != cudaSuccess) {                                                             \
            rc = afail(_e == cudaErrorMemoryAllocation ? CBGPU_ERR_OOM : CBGPU_ERR_CUDA,     \
                       "%s failed: %s", #call, cudaGetErrorString(_e));                      \
            goto done;                                                                       \
        }                                                                                    \
    } while (0)

struct ApplyModel {
    const uint32_t* split_features;
    const double* split_borders;
    const uint32_t* split_offsets;  // [n_trees + 1]
    const double* leaf_values;
    const uint32_t* leaf_offsets;   // [n_trees + 1]
    const uint8_t* nan_above;       // [F] or nullptr
    int32_t n_trees;
    double bias;
};

// kStage: the block's feature rows are staged in shared memory first (rows
// of `stride` floats, stride odd); otherwise every split reads HBM directly.
template <bool kStage>
__global__ void apply_oblivious_kernel(const float* __restrict__ x, int64_t rows, int32_t F, int32_t stride,
                                       ApplyModel m, double* __restrict__ out) {
    extern __shared__ float s_x[];
    const int64_t obj = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (kStage) {
        float* row = s_x + (size_t)threadIdx.x * (size_t)stride;
        if (obj < rows)
            for (int f = 0; f < F; ++f) row[f] = x[(size_t)f * (size_t)rows + (size_t)obj];
        __syncthreads();
    }
    if (obj >= rows) return;
    const float* row = kStage ? s_x + (size_t)threadIdx.x * (size_t)stride : nullptr;
    double acc = 0.0;
    uint32_t s = __ldg(&m.split_offsets[0]);
    uint32_t lo = __ldg(&m.leaf_offsets[0]);
    for (int t = 0; t < m.n_trees; ++t) {
        const uint32_t s1 = __ldg(&m.split_offsets[t + 1]);
        const uint32_t lo1 = __ldg(&m.leaf_offsets[t + 1]);
        uint32_t leaf = 0, bit = 0;
        for (; s < s1; ++s, ++bit) {
            const uint32_t f = __ldg(&m.split_features[s]);
            bool passes = false;
            if (f < (uint32_t)F) {
                const float v = kStage ? row[f] : __ldg(&x[(size_t)f * (size_t)rows + (size_t)obj]);
                passes = isnan(v) ? (m.nan_above != nullptr && __ldg(&m.nan_above[f]) != 0)
                                  : ((double)v > __ldg(&m.split_borders[s]));
            }
            leaf |= (uint32_t)passes << bit;
        }
        const uint64_t li = (uint64_t)lo + leaf;
        acc = __dadd_rn(acc, li < (uint64_t)lo1 ? __ldg(&m.leaf_values[li]) : 0.0);
        lo = lo1;
    }
    // bias + sum(oblivious) + sum(non-symmetric) + sum(region), the latter two empty
    out[obj] = __dadd_rn(__dadd_rn(__dadd_rn(m.bias, acc), 0.0), 0.0);
}

template <typename T>
int upload(T** d, const T* h, size_t count, cudaStream_t st) {
    *d = nullptr;
    cudaError_t e = cudaMalloc((void**)d, sizeof(T) * (count ? count : 1));
    if (e == cudaSuccess && count) e = cudaMemcpyAsync(*d, h, sizeof(T) * count, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess)
        return afail(e == cudaErrorMemoryAllocation ? CBGPU_ERR_OOM : CBGPU_ERR_CUDA, "apply upload: %s",
                     cudaGetErrorString(e));
    return CBGPU_OK;
}

}  // namespace

int cbgpu_apply_oblivious(const float* features_fm, int64_t n, int32_t n_features, const uint32_t* split_features,
                          const double* split_borders, const uint32_t* tree_split_offsets, int32_t n_trees,
                          const double* leaf_values, const uint32_t* tree_leaf_offsets, double bias,
                          const uint8_t* nan_above, int32_t device, double* out) {
    if (n < 0 || n_features < 0 || n_trees < 0 || !out || (n > 0 && n_features > 0 && !features_fm) ||
        (n_trees > 0 && (!tree_split_offsets || !tree_leaf_offsets)))
        return afail(CBGPU_ERR_INVALID, "apply_oblivious: bad arguments");
    // the CSR lowering's invariants (gpu_apply.rs:83-110)
    uint32_t n_splits = 0, n_leaves = 0;
    if (n_trees > 0) {
        if (tree_split_offsets[0] != 0 || tree_leaf_offsets[0] != 0)
            return afail(CBGPU_ERR_INVALID, "apply_oblivious: offsets must start at 0");
        for (int t = 0; t < n_trees; ++t) {
            if (tree_split_offsets[t + 1] < tree_split_offsets[t] || tree_leaf_offsets[t + 1] < tree_leaf_offsets[t])
                return afail(CBGPU_ERR_INVALID, "apply_oblivious: offsets of tree %d decrease", t);
            if (tree_split_offsets[t + 1] - tree_split_offsets[t] > (uint32_t)kApplyMaxDepth)
                return afail(CBGPU_ERR_INVALID, "apply_oblivious: tree %d has more than %d splits", t,
                             kApplyMaxDepth);
        }
        n_splits = tree_split_offsets[n_trees];
        n_leaves = tree_leaf_offsets[n_trees];
        if ((n_splits && (!split_features || !split_borders)) || (n_leaves && !leaf_values))
            return afail(CBGPU_ERR_INVALID, "apply_oblivious: missing split or leaf arrays");
    }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return afail(CBGPU_ERR_NO_DEVICE, "no CUDA device");
    if (device < 0 || device >= ndev) return afail(CBGPU_ERR_INVALID, "apply_oblivious: bad device %d", device);
    if (n == 0) return CBGPU_OK;

    int rc = CBGPU_OK;
    const int F = n_features;
    const int stride = F | 1;  // odd row stride: lanes hit distinct banks
    int threads = 256;
    while (threads > 32 && (size_t)threads * (size_t)stride * sizeof(float) > kApplySmemBudget) threads >>= 1;
    const size_t smem = (size_t)threads * (size_t)stride * sizeof(float);
    const bool stage = F > 0 && smem <= kApplySmemBudget;
    // rows per chunk: about 1 GiB of features, a whole number of blocks
    int64_t chunk = F > 0 ? std::max<int64_t>(threads, kApplyChunkBytes / (4 * (int64_t)F)) : n;
    chunk = std::min<int64_t>(n, chunk / threads * threads);
    if (chunk < 1) chunk = std::min<int64_t>(n, threads);

    cudaStream_t st[2] = {nullptr, nullptr};
    float* d_x[2] = {nullptr, nullptr};
    uint32_t *d_sf = nullptr, *d_so = nullptr, *d_lo = nullptr;
    double *d_sb = nullptr, *d_lv = nullptr, *d_out = nullptr;
    uint8_t* d_na = nullptr;
    cudaEvent_t model_ready = nullptr;
    ApplyModel m{};
    const std::vector<uint32_t> zero_off(1, 0u);

    ACU(cudaSetDevice(device));
    for (int k = 0; k < 2; ++k) ACU(cudaStreamCreateWithFlags(&st[k], cudaStreamNonBlocking));
    ACU(cudaEventCreateWithFlags(&model_ready, cudaEventDisableTiming));
    if ((rc = upload(&d_sf, split_features, n_splits, st[0]))) goto done;
    if ((rc = upload(&d_sb, split_borders, n_splits, st[0]))) goto done;
    if ((rc = upload(&d_so, n_trees ? tree_split_offsets : zero_off.data(), (size_t)n_trees + 1, st[0]))) goto done;
    if ((rc = upload(&d_lv, leaf_values, n_leaves, st[0]))) goto done;
    if ((rc = upload(&d_lo, n_trees ? tree_leaf_offsets : zero_off.data(), (size_t)n_trees + 1, st[0]))) goto done;
    if (nan_above && F > 0 && (rc = upload(&d_na, nan_above, (size_t)F, st[0]))) goto done;
    ACU(cudaEventRecord(model_ready, st[0]));
    ACU(cudaStreamWaitEvent(st[1], model_ready, 0));
    ACU(cudaMalloc((void**)&d_out, sizeof(double) * (size_t)n));
    if (F > 0)
        for (int k = 0; k < 2; ++k) ACU(cudaMalloc((void**)&d_x[k], sizeof(float) * (size_t)chunk * (size_t)F));
    if (stage)
        ACU(cudaFuncSetAttribute(apply_oblivious_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem));
    m = ApplyModel{d_sf, d_sb, d_so, d_lv, d_lo, d_na, n_trees, bias};
    // chunks alternate between two streams and two buffers: chunk i + 1's
    // upload overlaps chunk i's kernel; a buffer is reused only after the
    // kernel that read it (same stream).
    for (int64_t r0 = 0, i = 0; r0 < n; r0 += chunk, ++i) {
        const int k = (int)(i & 1);
        const int64_t rows = std::min<int64_t>(chunk, n - r0);
        if (F > 0)
            ACU(cudaMemcpy2DAsync(d_x[k], sizeof(float) * (size_t)rows, features_fm + r0, sizeof(float) * (size_t)n,
                                  sizeof(float) * (size_t)rows, (size_t)F, cudaMemcpyHostToDevice, st[k]));
        const unsigned blocks = (unsigned)((rows + threads - 1) / threads);
        if (stage)
            apply_oblivious_kernel<true><<<blocks, threads, smem, st[k]>>>(d_x[k], rows, F, stride, m, d_out + r0);
        else
            apply_oblivious_kernel<false><<<blocks, threads, 0, st[k]>>>(d_x[k], rows, F, stride, m, d_out + r0);
        ACU(cudaGetLastError());
        ACU(cudaMemcpyAsync(out + r0, d_out + r0, sizeof(double) * (size_t)rows, cudaMemcpyDeviceToHost, st[k]));
    }
    for (int k = 0; k < 2; ++k) ACU(cudaStreamSynchronize(st[k]));
done:
    for (int k = 0; k < 2; ++k)
        if (st[k]) cudaStreamSynchronize(st[k]);
    for (int k = 0; k < 2; ++k) cudaFree(d_x[k]);
    cudaFree(d_sf);
    cudaFree(d_sb);
    cudaFree(d_so);
    cudaFree(d_lv);
    cudaFree(d_lo);
    cudaFree(d_na);
    cudaFree(d_out);
    if (model_ready) cudaEventDestroy(model_ready);
    for (int k = 0; k < 2; ++k)
        if (st[k]) cudaStreamDestroy(st[k]);
    return rc;
}
