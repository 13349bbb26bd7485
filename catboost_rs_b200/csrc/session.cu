// session.cu -- the C ABI (include/cbgpu.h): a B200 training session behind the
// reference's Runtime seam (crates/cb-compute/src/runtime.rs:1410-1651).
//
// A session owns the quantized rows of this rank in HBM (row-major for the
// histogram gathers, feature-major for routing), the resident approximant and
// per-tree scratch.  grow_tree enqueues the whole tree on one stream with no
// host synchronisation until the small result copy at the end.
#include <cfloat>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstddef>
#include <cstring>
#include <string>
#include <vector>

#include <nccl.h>

#include "../../include/cbgpu.h"
#include "kernels.cuh"

using namespace cbgpu;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

#define CU(call)                                                                      \
    do {                                                                              \
        cudaError_t _e = (call);                                                      \
        if (_e != cudaSuccess) {                                                      \
            return fail(_e == cudaErrorMemoryAllocation ? CBGPU_ERR_OOM : CBGPU_ERR_CUDA, \
                        "%s failed: %s (%s:%d)", #call, cudaGetErrorString(_e),       \
                        __FILE__, __LINE__);                                          \
        }                                                                             \
    } while (0)

#define NC(call)                                                                            \
    do {                                                                                    \
        ncclResult_t _r = (call);                                                           \
        if (_r != ncclSuccess)                                                              \
            return fail(CBGPU_ERR_NCCL, "%s failed: %s", #call, ncclGetErrorString(_r));    \
    } while (0)

// Host replica of the reference's main TFastRng64 stream (rng.rs), with the
// call counter that cb-train's draw accounting is expressed in.
struct HostRng {
    Rng64 r{};
    uint64_t calls = 0;
    void seed(uint64_t s) {
        r = Rng64::from_seed(s);
        calls = 0;
    }
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

inline int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

template <typename T>
int dalloc(T** p, size_t count) {
    *p = nullptr;
    if (count == 0) count = 1;
    cudaError_t e = cudaMalloc((void**)p, sizeof(T) * count);
    if (e != cudaSuccess)
        return fail(e == cudaErrorMemoryAllocation ? CBGPU_ERR_OOM : CBGPU_ERR_CUDA,
                    "cudaMalloc(%zu bytes) failed: %s", sizeof(T) * count, cudaGetErrorString(e));
    return CBGPU_OK;
}

#define DA(p, count)                       \
    do {                                   \
        int _rc = dalloc(&(p), (count));   \
        if (_rc) return _rc;               \
    } while (0)

// Pinned host allocation (device copies into it are asynchronous and graph-capturable).
template <typename T>
int halloc(T** p, size_t count) {
    *p = nullptr;
    if (count == 0) count = 1;
    cudaError_t e = cudaMallocHost((void**)p, sizeof(T) * count);
    if (e != cudaSuccess)
        return fail(CBGPU_ERR_OOM, "cudaMallocHost(%zu bytes) failed: %s", sizeof(T) * count,
                    cudaGetErrorString(e));
    memset((void*)*p, 0, sizeof(T) * count);
    return CBGPU_OK;
}

#define HA(p, count)                       \
    do {                                   \
        int _rc = halloc(&(p), (count));   \
        if (_rc) return _rc;               \
    } while (0)

}  // namespace

namespace cbgpu {
// Sets the thread's cbgpu_last_error() message for entry points defined in
// other translation units; returns `code`.
int record_error(int code, const char* msg) { return fail(code, "%s", msg); }
}  // namespace cbgpu

struct cbgpu_session {
    // configuration
    int device = 0;
    int loss = 0, depth = 0, score_fn = 0, boot = 0, sample_from_host = 0;
    // staged host samples (cbgpu_stage_sample): a FIFO of two device buffers
    // filled on copy_st; a grow call without a sample takes the oldest
    cudaStream_t copy_st = nullptr;
    double* stage_buf[2] = {nullptr, nullptr};
    cudaEvent_t stage_done[2] = {nullptr, nullptr}, stage_free[2] = {nullptr, nullptr};
    int stage_head = 0, stage_count = 0;
    // Exact leaves (MAE / Quantile): quantile_der1's alpha / delta, sort buffers
    int exact = 0;
    double q_alpha = 0.5, q_delta = 1e-6;
    ull *ex_keys = nullptr, *ex_keys_sorted = nullptr;
    double *ex_w = nullptr, *ex_w_sorted = nullptr;
    void* ex_tmp = nullptr;
    size_t ex_tmp_bytes = 0;
    float sample_rate = 1.0f, temp = 1.0f;
    int has_mvs_lambda = 0;
    double mvs_lambda = 0.0;
    double lr = 0.0, l2 = 0.0, bias = 0.0;
    uint64_t seed = 0;
    int64_t n = 0, n_total = 0, row_offset = 0, n_stride = 0;
    int F = 0, F_pad = 0, B = 0;
    int rank = 0, world = 1;
    bool weighted = false;
    std::vector<int32_t> border_counts;

    cudaStream_t st = nullptr;
    ncclComm_t comm = nullptr;
    bool broken = false;  // a multi-rank grow failed: peers may be waiting in a collective

    // device data
    uint8_t* bins_rm = nullptr;   // [n][F_pad]
    uint8_t* bins_fm = nullptr;   // [F][n_stride]
    int32_t* d_border_counts = nullptr;
    double* target = nullptr;
    double* weight = nullptr;
    double* approx = nullptr;
    double* wd1 = nullptr;
    uint4* qstats = nullptr;      // per-row packed fixed-point (g_lo, g_hi, h_lo, h_hi)
    float* sw32 = nullptr;
    double* sw64 = nullptr;
    double* mvs_thr = nullptr;
    uint16_t* leaf = nullptr;     // every row's leaf id (routed level by level; final after the tree)
    uint32_t* list = nullptr;     // the rows of each parent's built child, segment by segment
    // per parent of a partition, two levels ([2][kSegMax], by level parity):
    // write cursor into list, row count, segment start
    uint32_t* cursor = nullptr;
    uint32_t* seg_rows = nullptr;
    uint32_t* seg_base = nullptr;
    uint8_t* small_side = nullptr;  // per parent: 1 = the true child is built
    ull* jump = nullptr;            // LCG jump multipliers (launch_jump_table)
    HistChunk* chunks0 = nullptr;  // level-0 work list (all rows), built at begin
    uint32_t* n_chunks0 = nullptr;
    HistChunk* chunks = nullptr;   // the next level's work list, built by launch_segments
    uint32_t chunk_rows = kChunkRows;  // rows per histogram work item (hist_chunk_rows)
    size_t chunk_cap = 0;
    uint32_t* n_chunks = nullptr;
    ull* built = nullptr;
    ull* hist[2] = {nullptr, nullptr};
    double* feat_score = nullptr;
    int32_t* feat_bin = nullptr;
    ull* leaf_sums = nullptr;
    double* leaf_raw = nullptr;
    double* leaf_lrv = nullptr;
    TreeState* ts = nullptr;
    uint32_t* d_err = nullptr;
    void* leaf_export = nullptr;
    size_t built_cells = 0, hist_cells = 0;
    // Feature slice owned by this rank for derive / score: [f0, f0 + Fs) of the
    // world * Fs padded features (features >= F have no borders).
    int Fs = 0, f0 = 0;
    ull* best_all = nullptr;  // per rank: slice winner record for the all-gather

    // host state
    HostRng rng;
    bool target_ready = false;
    bool pending = false;
    bool has_prev_mean = false;
    double prev_mean = 0.0;
    int64_t trees = 0;
    bool profiling = false;
    // Per-tree CUDA events, two sets: a tree records into one set while the
    // previous tree's times are read from the other, during this tree's
    // device work instead of between trees.
    static constexpr int kEv = 2 + 5 * 16 + 1;
    cudaEvent_t ev[2][kEv] = {};
    int ev_set = 0;                       // set of the tree grown last
    bool ev_pending[2] = {false, false};  // a finished tree whose times are unread
    int ev_depth[2] = {0, 0};
    bool ev_prof[2] = {false, false};
    double ev_host[2][2] = {};            // rows histogrammed, kernels launched
    double timing_sum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    cudaEvent_t uev[4] = {};
    double timing[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    TreeState* h_ts = nullptr;  // pinned: the tree's result state
    double* h_raw = nullptr;     // pinned: the tree's leaf values
    TreeParams* h_tp = nullptr;  // pinned: per-tree scalars, copied to d_tp before each tree
    TreeParams* d_tp = nullptr;
    // Captured tree graphs, one per event set (their event nodes differ), with
    // the launch shape they were captured for and their kernel count.
    bool use_graphs = true;
    cudaGraphExec_t graph[2] = {nullptr, nullptr};
    int graph_key[2] = {-1, -1};
    int graph_launches[2] = {0, 0};
};

namespace {

int check_args(const cbgpu_begin_args* a) {
    if (!a) return fail(CBGPU_ERR_INVALID, "null begin args");
    // Coverage gate (session.rs:1379-1633 / boosting.rs:5789-6010 analogue):
    // anything outside the covered regime declines to the CPU grower.
    if (a->grow_policy != CBGPU_GROW_SYMMETRIC)
        return fail(CBGPU_DECLINED, "grow_policy %d is not SymmetricTree", a->grow_policy);
    if (!a->boosting_type_is_plain) return fail(CBGPU_DECLINED, "Ordered boosting is not covered");
    if (a->fold_count != 1) return fail(CBGPU_DECLINED, "fold_count %d != 1", a->fold_count);
    const bool quantile = a->loss == CBGPU_LOSS_MAE || a->loss == CBGPU_LOSS_QUANTILE;
    if ((a->loss < 0 || a->loss > 2) && !quantile) return fail(CBGPU_DECLINED, "loss %d not covered", a->loss);
    // map_leaf_method (session.rs:1176-1200): MAE / Quantile only with Exact
    // leaves, Exact only for them, and only without draws on one rank
    if (quantile != (a->exact_leaf != 0))
        return fail(CBGPU_DECLINED, a->exact_leaf ? "Exact leaves are covered for MAE / Quantile only"
                                                  : "MAE / Quantile are covered with Exact leaves only");
    if (a->exact_leaf) {
        if (a->bootstrap_type != CBGPU_BOOT_NO || a->sample_from_host || a->has_mvs_lambda)
            return fail(CBGPU_DECLINED, "Exact leaves need bootstrap No");
        if (a->world_size != 1) return fail(CBGPU_DECLINED, "Exact leaves run on one rank");
        if (a->n >= (int64_t)0x7fffffff) return fail(CBGPU_DECLINED, "Exact leaves: n >= 2^31 rows");
        if (a->loss == CBGPU_LOSS_QUANTILE && !(a->quantile_alpha >= 0.0 && a->quantile_alpha <= 1.0 &&
                                                 a->quantile_delta >= 0.0))
            return fail(CBGPU_ERR_INVALID, "Quantile alpha %g / delta %g", a->quantile_alpha, a->quantile_delta);
    }
    if (a->score_function != CBGPU_SCORE_COSINE && a->score_function != CBGPU_SCORE_L2 &&
        a->score_function != CBGPU_SCORE_SOLAR_L2 && a->score_function != CBGPU_SCORE_LOO_L2 &&
        a->score_function != CBGPU_SCORE_SAT_L2)
        return fail(CBGPU_DECLINED, "score function %d not covered", a->score_function);
    if (a->depth < 1 || a->depth > 16) return fail(CBGPU_DECLINED, "depth %d outside 1..16", a->depth);
    if (a->n_bins < 2 || a->n_bins > 256)
        return fail(CBGPU_DECLINED, "n_bins %d outside 2..256", a->n_bins);
    if (a->bootstrap_type == CBGPU_BOOT_POISSON) return fail(CBGPU_DECLINED, "Poisson bootstrap not covered");
    if (a->bootstrap_type < 0 || a->bootstrap_type > 4)
        return fail(CBGPU_ERR_INVALID, "bad bootstrap type %d", a->bootstrap_type);
    if (a->random_strength != 0.0) return fail(CBGPU_DECLINED, "random_strength != 0 is not covered");
    if (a->n < 0 || a->n_features < 1) return fail(CBGPU_ERR_INVALID, "bad shape n=%lld F=%d",
                                                   (long long)a->n, a->n_features);
    if (a->n >= (int64_t)0xfffffff0ll) return fail(CBGPU_DECLINED, "n >= 2^32 rows per rank");
    if (a->world_size < 1 || a->rank < 0 || a->rank >= a->world_size)
        return fail(CBGPU_ERR_INVALID, "bad rank %d / world %d", a->rank, a->world_size);
    if (a->world_size > 1 && !a->nccl_unique_id)
        return fail(CBGPU_ERR_INVALID, "world_size > 1 needs nccl_unique_id");
    if (a->bootstrap_type == CBGPU_BOOT_MVS && (a->row_offset % 8192) != 0)
        return fail(CBGPU_ERR_INVALID, "MVS needs row_offset aligned to 8192 (got %lld)",
                    (long long)a->row_offset);
    return CBGPU_OK;
}

int alloc_session(cbgpu_session* s, const cbgpu_begin_args* a) {
    s->device = a->device;
    CU(cudaSetDevice(s->device));
    CU(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking));
    s->loss = a->loss;
    s->exact = a->exact_leaf ? 1 : 0;
    if (a->loss == CBGPU_LOSS_QUANTILE) {  // MAE keeps the median anchor 0.5 / 1e-6 (loss.rs:186-193)
        s->q_alpha = a->quantile_alpha;
        s->q_delta = a->quantile_delta;
    }
    s->depth = a->depth;
    s->score_fn = a->score_function;
    s->boot = a->bootstrap_type;
    s->sample_from_host = a->sample_from_host;
    s->sample_rate = a->sample_rate;
    s->temp = a->bagging_temperature;
    s->has_mvs_lambda = a->has_mvs_lambda;
    s->mvs_lambda = a->mvs_lambda;
    s->lr = a->learning_rate;
    s->l2 = a->scaled_l2;
    s->bias = a->bias;
    s->seed = a->rng_seed;
    s->n = a->n;
    s->n_total = a->n_total > 0 ? a->n_total : a->n;
    s->row_offset = a->row_offset;
    s->n_stride = round_up(s->n > 0 ? s->n : 1, 16);
    s->F = a->n_features;
    s->F_pad = (int)round_up(s->F, 32);
    s->B = a->n_bins;
    s->rank = a->rank;
    s->world = a->world_size;
    s->weighted = a->weight != nullptr;
    s->rng.seed(a->rng_seed);

    const int64_t n = s->n > 0 ? s->n : 1;
    const int L = 1 << s->depth;
    DA(s->bins_rm, (size_t)n * s->F_pad);
    DA(s->bins_fm, (size_t)s->F * s->n_stride);
    DA(s->d_border_counts, s->F);
    DA(s->target, n);
    if (s->weighted) DA(s->weight, n);
    DA(s->approx, n);
    DA(s->wd1, n);
    DA(s->qstats, n);
    DA(s->sw32, n);
    if (s->sample_from_host) DA(s->sw64, n);
    DA(s->mvs_thr, (n + 8191) / 8192);
    DA(s->leaf, n);
    DA(s->list, n);
    DA(s->cursor, 2 * kSegMax);  // up to 2^15 parents per partition (depth <= 16)
    DA(s->seg_rows, 2 * kSegMax);
    DA(s->seg_base, 2 * kSegMax);
    DA(s->small_side, kSegMax);
    DA(s->jump, 2 * kJumpSteps);
    // full chunks plus one partial chunk per segment
    {
        int sms = 0;
        CU(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, s->device));
        s->chunk_rows = hist_chunk_rows(n, hist_tiles(s->F, s->B), 1, sms);
    }
    s->chunk_cap = (size_t)(n / s->chunk_rows) + (L / 2) + 2;
    DA(s->chunks, s->chunk_cap);
    DA(s->n_chunks, 1);
    DA(s->chunks0, (size_t)(n / s->chunk_rows) + 2);
    DA(s->n_chunks0, 1);
    feature_slice(s->F, s->world, s->rank, &s->f0, &s->Fs);
    s->built_cells = (size_t)(L / 2 > 0 ? L / 2 : 1) * s->world * s->Fs * s->B * 2;
    s->hist_cells = (size_t)(L / 2 > 0 ? L / 2 : 1) * s->Fs * s->B * 2;
    DA(s->built, s->built_cells);
    DA(s->hist[0], s->hist_cells);
    DA(s->hist[1], s->hist_cells);
    DA(s->feat_score, (size_t)s->Fs * 8);  // per (feature, 32-border group) winners of the slice
    DA(s->feat_bin, (size_t)s->Fs * 8);
    DA(s->best_all, (size_t)(2 + L) * s->world);  // per rank: score, key, 2 * 2^level weight sums
    DA(s->leaf_sums, 2 * L);
    DA(s->leaf_raw, L);
    DA(s->leaf_lrv, L);
    if (s->exact) {
        DA(s->ex_keys, s->n);
        DA(s->ex_keys_sorted, s->n);
        DA(s->ex_w, s->n);
        DA(s->ex_w_sorted, s->n);
        s->ex_tmp_bytes = exact_sort_scratch_bytes(s->n);
        DA(*(char**)&s->ex_tmp, s->ex_tmp_bytes);
    }
    DA(s->ts, 1);
    DA(s->d_err, 1);
    DA(s->d_tp, 1);
    HA(s->h_ts, 1);
    HA(s->h_raw, L);
    HA(s->h_tp, 1);
    CU(cudaMemsetAsync(s->ts, 0, sizeof(TreeState), s->st));
    CU(cudaMemsetAsync(s->d_err, 0, sizeof(uint32_t), s->st));
    CU(cudaMemsetAsync(s->leaf, 0, sizeof(uint16_t) * n, s->st));
    if (s->weighted)
        CU(cudaMemcpyAsync(s->weight, a->weight, sizeof(double) * s->n, cudaMemcpyHostToDevice, s->st));
    // resident approximant starts at the bias (DeviceTrainConfig::bias)
    {
        std::vector<double> h((size_t)std::min<int64_t>(n, 1 << 20), s->bias);
        for (int64_t off = 0; off < s->n; off += (int64_t)h.size()) {
            int64_t c = std::min<int64_t>((int64_t)h.size(), s->n - off);
            CU(cudaMemcpyAsync(s->approx + off, h.data(), sizeof(double) * c, cudaMemcpyHostToDevice, s->st));
            CU(cudaStreamSynchronize(s->st));
        }
    }
    for (auto& set : s->ev)
        for (auto& e : set) CU(cudaEventCreate(&e));
    for (auto& e : s->uev) CU(cudaEventCreate(&e));
    if (s->world > 1) {
        ncclUniqueId id;
        memcpy(&id, a->nccl_unique_id, sizeof(id));
        NC(ncclCommInitRank(&s->comm, s->world, id, s->rank));
    }
    return CBGPU_OK;
}

void free_session(cbgpu_session* s) {
    if (!s) return;
    cudaSetDevice(s->device);
    // After a failed multi-rank step this rank's queued collectives may never
    // complete (the peers went their own way), so the communicator is aborted
    // before the stream is drained instead of destroyed after it.
    if (s->broken && s->comm) {
        ncclCommAbort(s->comm);
        s->comm = nullptr;
    }
    if (s->st) cudaStreamSynchronize(s->st);
    if (s->copy_st) cudaStreamSynchronize(s->copy_st);  // staged copies still read the caller's buffers
    // graphs hold NCCL work: released before the communicator
    for (auto& g : s->graph)
        if (g) cudaGraphExecDestroy(g);
    void* ptrs[] = {s->bins_rm, s->bins_fm, s->d_border_counts, s->target, s->weight, s->approx,
                    s->wd1, s->qstats, s->sw32, s->sw64, s->mvs_thr, s->leaf, s->list, s->cursor,
                    s->seg_rows, s->seg_base, s->small_side, s->jump, s->chunks0, s->n_chunks0, s->chunks, s->n_chunks, s->built,
                    s->hist[0], s->hist[1], s->feat_score, s->feat_bin, s->best_all, s->leaf_sums, s->leaf_raw,
                    s->leaf_lrv, s->ts, s->d_err, s->leaf_export, s->d_tp, s->ex_keys, s->ex_keys_sorted,
                    s->ex_w, s->ex_w_sorted, s->ex_tmp};
    for (void* p : ptrs)
        if (p) cudaFree(p);
    void* hptrs[] = {s->h_ts, s->h_raw, s->h_tp};
    for (void* p : hptrs)
        if (p) cudaFreeHost(p);
    for (auto& set : s->ev)
        for (auto& e : set)
            if (e) cudaEventDestroy(e);
    for (auto& e : s->uev)
        if (e) cudaEventDestroy(e);
    for (int k = 0; k < 2; ++k) {
        if (s->stage_buf[k]) cudaFree(s->stage_buf[k]);
        if (s->stage_done[k]) cudaEventDestroy(s->stage_done[k]);
        if (s->stage_free[k]) cudaEventDestroy(s->stage_free[k]);
    }
    if (s->comm) ncclCommDestroy(s->comm);
    if (s->copy_st) cudaStreamDestroy(s->copy_st);
    if (s->st) cudaStreamDestroy(s->st);
    delete s;
}

int finish_begin(cbgpu_session* s) {
    for (int f = 0; f < s->F; ++f)
        if (s->border_counts[f] > s->B - 1)
            return fail(CBGPU_ERR_INVALID, "feature %d has %d borders > n_bins - 1 = %d", f,
                        s->border_counts[f], s->B - 1);
    bool any = false;
    for (int f = 0; f < s->F; ++f) any |= s->border_counts[f] > 0;
    if (!any) return fail(CBGPU_DECLINED, "no feature has a border: nothing to split on");
    CU(cudaMemcpyAsync(s->d_border_counts, s->border_counts.data(), sizeof(int32_t) * s->F,
                       cudaMemcpyHostToDevice, s->st));
    if (s->n > 0) launch_transpose_fm_to_rm(s->bins_fm, s->n, s->n_stride, s->F, s->bins_rm, s->F_pad, s->st);
    launch_jump_table(s->jump, s->st);
    launch_level0_chunks(s->n, s->chunks0, (uint32_t)(s->n / s->chunk_rows) + 2, s->n_chunks0, s->d_err,
                         s->chunk_rows, s->st);
    uint32_t herr = 0;
    CU(cudaMemcpyAsync(&herr, s->d_err, sizeof(uint32_t), cudaMemcpyDeviceToHost, s->st));
    CU(cudaStreamSynchronize(s->st));
    CU(cudaGetLastError());
    if (herr & kErrBinRange) return fail(CBGPU_ERR_INVALID, "a bin index >= n_bins was passed");
    return CBGPU_OK;
}

template <typename T>
int allreduce(cbgpu_session* s, T* buf, size_t count, ncclDataType_t dt, ncclRedOp_t op) {
    if (s->world <= 1 || count == 0) return CBGPU_OK;
    NC(ncclAllReduce(buf, buf, count, dt, op, s->comm, s->st));
    return CBGPU_OK;
}

// In place: buf holds world equal pieces of `per_rank` elements; afterwards
// piece `rank` holds the sum over ranks of that piece.
int reduce_scatter_u64(cbgpu_session* s, ull* buf, size_t per_rank) {
    if (s->world <= 1 || per_rank == 0) return CBGPU_OK;
    NC(ncclReduceScatter(buf, buf + (size_t)s->rank * per_rank, per_rank, ncclUint64, ncclSum, s->comm, s->st));
    return CBGPU_OK;
}

// In place: piece `rank` of buf (per_rank elements) is sent to every rank.
int all_gather_u64(cbgpu_session* s, ull* buf, size_t per_rank) {
    if (s->world <= 1 || per_rank == 0) return CBGPU_OK;
    NC(ncclAllGather(buf + (size_t)s->rank * per_rank, buf, per_rank, ncclUint64, s->comm, s->st));
    return CBGPU_OK;
}

float ev_ms(cbgpu_session* s, int set, int a, int b) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, s->ev[set][a], s->ev[set][b]);
    return ms;
}

// Reads a finished tree's event times into timing (that tree) and timing_sum.
void collect_timing(cbgpu_session* s, int set) {
    if (!s->ev_pending[set]) return;
    s->ev_pending[set] = false;
    const int D = s->ev_depth[set];
    double t[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    t[0] = ev_ms(s, set, 0, 2 + 5 * D);
    if (s->ev_prof[set]) {
        for (int l = 0; l < D; ++l) {
            const int e = 2 + 5 * l;
            t[1] += ev_ms(s, set, e, e + 1);
            t[5] += ev_ms(s, set, e + 1, e + 2);
            t[2] += ev_ms(s, set, e + 2, e + 3);
            t[3] += ev_ms(s, set, e + 3, e + 4);
        }
        t[4] = ev_ms(s, set, 0, 1);
    }
    t[6] = s->ev_host[set][0];
    t[7] = s->ev_host[set][1];
    for (int k = 0; k < 8; ++k) {
        s->timing[k] = t[k];
        s->timing_sum[k] += t[k];
    }
}

}  // namespace

namespace cbgpu {
// One rank's link of the first-tree MVS lambda chain (bootstrap.rs:358-376):
// continues the sequential f64 sum of |w * der1| (der_obj, taken through
// sqrt(v * v) twice as the reference does) over this rank's rows, starting
// from the previous rank's partial sum.  RMSE (loss 0) or Logloss ders at
// approx (NULL = bias everywhere).
double mvs_abs_der_partial(double acc, int loss, int64_t n, const double* approx, double bias, const double* target,
                           const double* weight) {
    for (int64_t i = 0; i < n; ++i) {
        const double a = approx ? approx[i] : bias;
        const double d1 = loss == 0 ? target[i] - a : target[i] - (1.0 - 1.0 / (1.0 + std::exp(a)));
        const double v = d1 * (weight ? weight[i] : 1.0);
        const double dobj = std::sqrt(v * v);
        acc += std::sqrt(dobj * dobj);
    }
    return acc;
}
}  // namespace cbgpu

namespace {

// First-tree MVS lambda (bootstrap.rs:358-376): (sum |w*der1| / n)^2 with a
// sequential f64 sum over all rows; the chain crosses ranks in rank order.
int first_mvs_lambda(cbgpu_session* s, const double* approx_h, const double* target_h, double* out) {
    std::vector<double> w;
    if (s->weighted) {
        w.resize((size_t)s->n);
        CU(cudaMemcpy(w.data(), s->weight, sizeof(double) * s->n, cudaMemcpyDeviceToHost));
    }
    const double* wp = s->weighted ? w.data() : nullptr;
    double acc = 0.0;
    if (s->world > 1) {
        double* d;
        DA(d, 1);
        if (s->rank > 0) {
            ncclResult_t r = ncclRecv(d, 1, ncclFloat64, s->rank - 1, s->comm, s->st);
            if (r != ncclSuccess) { cudaFree(d); return fail(CBGPU_ERR_NCCL, "ncclRecv: %s", ncclGetErrorString(r)); }
            CU(cudaMemcpyAsync(&acc, d, sizeof(double), cudaMemcpyDeviceToHost, s->st));
            CU(cudaStreamSynchronize(s->st));
        }
        acc = mvs_abs_der_partial(acc, s->loss, s->n, approx_h, s->bias, target_h, wp);
        CU(cudaMemcpyAsync(d, &acc, sizeof(double), cudaMemcpyHostToDevice, s->st));
        if (s->rank + 1 < s->world) NC(ncclSend(d, 1, ncclFloat64, s->rank + 1, s->comm, s->st));
        NC(ncclBroadcast(d, d, 1, ncclFloat64, s->world - 1, s->comm, s->st));
        CU(cudaMemcpyAsync(&acc, d, sizeof(double), cudaMemcpyDeviceToHost, s->st));
        CU(cudaStreamSynchronize(s->st));
        cudaFree(d);
    } else {
        acc = mvs_abs_der_partial(acc, s->loss, s->n, approx_h, s->bias, target_h, wp);
    }
    double mean = s->n_total > 0 ? acc / (double)s->n_total : 0.0;
    *out = mean * mean;
    return CBGPU_OK;
}

// The device work of one tree, in stream order on s->st: everything from the
// tree-state reset to the copies of the result into pinned host buffers.  It
// makes no host decisions and no allocations, so it can be captured into a
// graph once and replayed: per-tree scalars come from s->d_tp.
// boot_mode: 0 none, 1 Bayesian, 2 Bernoulli; s_mode as launch_der.
int enqueue_tree(cbgpu_session* s, int set, bool prof, int boot_mode, int s_mode, bool mvs, bool capturing,
                 int* launches_out) {
    cudaStream_t st = s->st;
    const int D = s->depth;
    const int L = 1 << D;
    int launches = 0;
    // event slots: 0 tree start, 1 after derivatives, per level l: 2+5l .. 6+5l, last: 2+5D
    // (under capture they become event-record nodes; the External flag is only
    // valid while capturing)
    auto rec = [&](int k) {
        if (!(prof || k == 0 || k == 2 + 5 * D)) return;
        if (capturing) cudaEventRecordWithFlags(s->ev[set][k], st, cudaEventRecordExternal);
        else cudaEventRecord(s->ev[set][k], st);
    };
    rec(0);
    CU(cudaMemsetAsync(s->ts, 0, sizeof(TreeState), st));
    // the Bayesian / Bernoulli sample is drawn inside the derivative pass
    launch_der(s->n, s->loss, s->approx, s->target, s->weight, s->leaf, s->leaf_lrv, s->d_tp, s_mode, s->sw32,
               s->sw64, s->wd1, s->ts, mvs, boot_mode, s->row_offset, boot_mode == 2 ? (double)s->sample_rate : 0.0,
               boot_mode == 1 ? s->temp : 0.0f, s->jump, st);
    ++launches;
    if (mvs) {
        launch_mvs(s->n, s->row_offset, s->wd1, s->d_tp, (double)s->sample_rate, s->mvs_thr, s->sw32, st);
        launch_max_gh(s->n, s->wd1, s->weight, s->sw32, s->ts, st);
        launches += 3;
    }
    {
        ull* maxbits = (ull*)((char*)s->ts + offsetof(TreeState, maxbits));
        int rc = allreduce(s, maxbits, 4, ncclUint64, ncclMax);
        if (rc) return rc;
    }
    launch_pack_stats(s->n, s->wd1, s->weight, s_mode, s->sw32, s->sw64, s->ts, s->n_total, s->qstats, st);
    launches += 1;
    rec(1);

    // ---- level loop
    int cur = 0;
    for (int l = 0; l < D; ++l) {
        const int e = 2 + 5 * l;
        const size_t built_slots = l == 0 ? 1 : (size_t)1 << (l - 1);
        // built is feature-major [world * Fs][slot][B][2], so each rank's
        // feature slice is one contiguous piece for the reduce-scatter
        const size_t slice_cells = (size_t)s->Fs * built_slots * s->B * 2;
        CU(cudaMemsetAsync(s->built, 0, sizeof(ull) * slice_cells * s->world, st));
        const uint32_t max_chunks =
            (uint32_t)(s->n / s->chunk_rows + (l == 0 ? 1 : (1u << (l - 1))) + 1);
        rec(e);
        launch_hist(s->bins_rm, s->F_pad, s->F, s->B, s->qstats, l == 0 ? nullptr : s->list,
                    l == 0 ? s->chunks0 : s->chunks, l == 0 ? s->n_chunks0 : s->n_chunks, max_chunks, s->built,
                    (int64_t)built_slots * s->B * 2, (int64_t)s->B * 2, st);
        rec(e + 1);
        launches += 1;
        {
            int rc = reduce_scatter_u64(s, s->built, slice_cells);
            if (rc) return rc;
        }
        rec(e + 2);
        const ull* built_slice = s->built + (size_t)s->rank * slice_cells;
        launch_derive_prefix(l, s->Fs, s->B, built_slice, s->hist[cur ^ 1], s->hist[cur], s->small_side, st);
        const int stride = 2 + 2 * (1 << l);  // all-gather record: score, key, (false, true) per leaf
        launch_score(l, s->Fs, s->f0, s->F, s->B, s->hist[cur], s->d_border_counts, s->l2, s->score_fn,
                     s->feat_score, s->feat_bin, s->ts,
                     s->world > 1 ? s->best_all + (size_t)stride * s->rank : nullptr,
                     l + 1 < D ? s->small_side : nullptr, st);
        launches += 2;
        if (s->world > 1) {
            int rc = all_gather_u64(s, s->best_all, (size_t)stride);
            if (rc) return rc;
            // also picks the next level's build side: no child-count all-reduce
            launch_select_split(l, s->world, stride, s->best_all, s->ts, l + 1 < D ? s->small_side : nullptr, st);
            ++launches;
        }
        rec(e + 3);
        if (l + 1 < D) {
            // route every row and list the rows of each parent's built child
            // (the side the score kernel or select_split chose from the
            // split's weights), then the next level's work list and segments
            const int p = l & 1, np = p ^ 1;
            uint32_t* cur_l = l == 0 ? (uint32_t*)((char*)s->ts + offsetof(TreeState, cursor0))
                                     : s->cursor + (size_t)p * kSegMax;
            const bool more = l + 2 < D;  // another partition follows
            launch_partition(l, s->n, s->bins_fm, s->n_stride, s->leaf, s->small_side, cur_l, s->list,
                             (const int32_t*)((char*)s->ts + offsetof(TreeState, split)),
                             (int)(sizeof(SplitRec) / sizeof(int32_t)), 0x7fffffff, st);
            launch_segments(l, s->n, l == 0 ? nullptr : s->seg_rows + (size_t)p * kSegMax,
                            l == 0 ? nullptr : s->seg_base + (size_t)p * kSegMax, cur_l, s->small_side,
                            more ? s->seg_rows + (size_t)np * kSegMax : nullptr,
                            more ? s->seg_base + (size_t)np * kSegMax : nullptr,
                            more ? s->cursor + (size_t)np * kSegMax : nullptr, s->chunks,
                            (uint32_t)s->chunk_cap, s->n_chunks, s->ts, s->chunk_rows, st);
            rec(e + 4);
            launches += 2;
        } else {
            CU(cudaMemsetAsync(s->leaf_sums, 0, sizeof(ull) * 2 * L, st));
            launch_route_leafsum(l, s->n, s->bins_fm, s->n_stride, s->leaf, s->wd1, s->weight, s->ts,
                                 s->leaf_sums, st);
            launches += 1;
            rec(e + 4);
            int rc = allreduce(s, s->leaf_sums, (size_t)2 * L, ncclUint64, ncclSum);
            if (rc) return rc;
        }
        cur ^= 1;
    }
    launch_leaf_values(D, D, s->leaf_sums, s->l2, s->lr, s->ts, s->leaf_raw, s->leaf_lrv, st);
    ++launches;
    if (s->exact) {  // the Exact leaf values replace the Gradient ones (boosting.rs:2561-2606)
        launch_exact_leaves(D, s->n, s->approx, s->target, s->weight, s->leaf, s->ex_keys, s->ex_keys_sorted,
                            s->ex_w, s->ex_w_sorted, s->ex_tmp, s->ex_tmp_bytes, s->q_alpha, s->q_delta, s->lr,
                            s->leaf_raw, s->leaf_lrv, st);
        launches += 2;
    }
    CU(cudaGetLastError());
    CU(cudaMemcpyAsync(s->h_ts, s->ts, sizeof(TreeState), cudaMemcpyDeviceToHost, st));
    CU(cudaMemcpyAsync(s->h_raw, s->leaf_raw, sizeof(double) * L, cudaMemcpyDeviceToHost, st));
    rec(2 + 5 * D);
    *launches_out = launches;
    return CBGPU_OK;
}

// The tree graph for event set `set` and this launch shape, captured from
// enqueue_tree on first use (the stream's own work only: thread-local capture).
int ensure_graph(cbgpu_session* s, int set, bool prof, int boot_mode, int s_mode, bool mvs) {
    const int key = (prof ? 1 : 0) | (boot_mode << 1) | (s_mode << 3) | (mvs ? 1 << 5 : 0);
    if (s->graph[set] && s->graph_key[set] == key) return CBGPU_OK;
    if (s->graph[set]) {
        cudaGraphExecDestroy(s->graph[set]);
        s->graph[set] = nullptr;
    }
    cudaGraph_t g = nullptr;
    CU(cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal));
    int launches = 0;
    const int rc = enqueue_tree(s, set, prof, boot_mode, s_mode, mvs, true, &launches);
    const cudaError_t ce = cudaStreamEndCapture(s->st, &g);
    if (rc != CBGPU_OK || ce != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        if (rc != CBGPU_OK) return rc;
        return fail(CBGPU_ERR_CUDA, "tree graph capture failed: %s", cudaGetErrorString(ce));
    }
    const cudaError_t ie = cudaGraphInstantiate(&s->graph[set], g, 0);
    cudaGraphDestroy(g);
    if (ie != cudaSuccess) {
        s->graph[set] = nullptr;
        return fail(CBGPU_ERR_CUDA, "tree graph instantiation failed: %s", cudaGetErrorString(ie));
    }
    s->graph_key[set] = key;
    s->graph_launches[set] = launches;
    return CBGPU_OK;
}

int grow(cbgpu_session* s, const double* approx_h, const double* target_h, int64_t n,
         const double* sample, int64_t sample_len, int32_t* split_feature, int32_t* split_bin,
         int32_t* n_splits, double* leaf_values, void* leaf_of, int32_t leaf_of_bytes) {
    if (n != s->n) return fail(CBGPU_ERR_INVALID, "LengthMismatch: n=%lld, session has %lld",
                               (long long)n, (long long)s->n);
    // sample validation (session.rs:2405-2428); a staged sample stands in
    // for a passed one
    if (sample_len != 0) {
        if (!s->sample_from_host)
            return fail(CBGPU_ERR_INVALID,
                        "Degenerate: a %lld-element host bootstrap sample was passed to a session opened "
                        "with sample_from_host = false", (long long)sample_len);
        if (sample_len != s->n)
            return fail(CBGPU_ERR_INVALID, "LengthMismatch: sample has %lld elements, expected %lld",
                        (long long)sample_len, (long long)s->n);
        if (!sample) return fail(CBGPU_ERR_INVALID, "null sample pointer");
        if (s->stage_count > 0)
            return fail(CBGPU_ERR_INVALID, "a sample was passed while %d staged sample(s) wait: pass none to "
                                           "take the oldest staged one", s->stage_count);
    } else if (s->sample_from_host && s->stage_count == 0) {
        return fail(CBGPU_ERR_INVALID,
                    "Degenerate: the session was opened with sample_from_host = true but no sample "
                    "was passed or staged");
    }
    if (!s->target_ready && !target_h) return fail(CBGPU_ERR_INVALID, "target required on the first grow");
    if (leaf_of && leaf_of_bytes) {
        if (leaf_of_bytes != 1 && leaf_of_bytes != 2 && leaf_of_bytes != 4)
            return fail(CBGPU_ERR_INVALID, "leaf_of_bytes must be 1, 2 or 4");
        if (leaf_of_bytes == 1 && s->depth > 8) return fail(CBGPU_ERR_INVALID, "u8 leaf ids need depth <= 8");
    }
    CU(cudaSetDevice(s->device));
    cudaStream_t st = s->st;
    const int D = s->depth;
    const int L = 1 << D;
    const bool prof = s->profiling;
    const int set = s->ev_set ^ 1;  // the other set may still hold the previous tree's unread times

    if (!s->target_ready) {
        CU(cudaMemcpyAsync(s->target, target_h, sizeof(double) * s->n, cudaMemcpyHostToDevice, st));
        s->target_ready = true;
    }
    if (approx_h) {
        CU(cudaMemcpyAsync(s->approx, approx_h, sizeof(double) * s->n, cudaMemcpyHostToDevice, st));
        s->pending = false;
    }

    // ---- bootstrap: the host stream replica decides the draws (boosting.rs:6568-6660)
    TreeParams& tp = *s->h_tp;  // pinned; the previous tree's copy finished at its sync
    tp = TreeParams{};
    int s_mode = 0, boot_mode = 0;
    bool mvs = false;
    if (s->sample_from_host && sample_len == 0) {
        // the oldest staged sample: wait for its upload, move it into the
        // buffer the tree reads, and free its slot for the next stage call
        const int k = s->stage_head;
        CU(cudaStreamWaitEvent(st, s->stage_done[k], 0));
        CU(cudaMemcpyAsync(s->sw64, s->stage_buf[k], sizeof(double) * s->n, cudaMemcpyDeviceToDevice, st));
        CU(cudaEventRecord(s->stage_free[k], st));
        s->stage_head ^= 1;
        --s->stage_count;
        s_mode = 2;
    } else if (s->sample_from_host) {
        CU(cudaMemcpyAsync(s->sw64, sample, sizeof(double) * s->n, cudaMemcpyHostToDevice, st));
        s_mode = 2;
    } else if (s->boot != CBGPU_BOOT_NO) {
        s->rng.gen();  // PRE_TREE_DRAWS = 2 (boosting.rs:59)
        s->rng.gen();
        if (s->boot == CBGPU_BOOT_BAYESIAN) {
            if (s->temp != 0.0f) {
                tp.boot_seed = s->rng.gen();
                boot_mode = 1;
                s_mode = 1;
            }
        } else if (s->boot == CBGPU_BOOT_BERNOULLI) {
            if ((double)s->sample_rate < 1.0) {
                tp.boot_base = s->rng.r;
                s->rng.advance((uint64_t)s->n_total);
                boot_mode = 2;
                s_mode = 1;
            }
        } else if (s->boot == CBGPU_BOOT_MVS) {
            if ((double)s->sample_rate < 1.0) {
                double lam = 0.0;
                if (s->has_mvs_lambda) lam = s->mvs_lambda;
                else if (s->has_prev_mean) lam = s->prev_mean * s->prev_mean;
                else {
                    int rc = first_mvs_lambda(s, approx_h, target_h, &lam);
                    if (rc) return rc;
                }
                tp.mvs_lambda = lam;
                tp.boot_seed = s->rng.gen();
                mvs = true;
                s_mode = 1;
            }
        }
    }
    tp.pending = s->pending ? 1 : 0;
    tp.q_alpha = s->q_alpha;
    tp.q_delta = s->q_delta;
    CU(cudaMemcpyAsync(s->d_tp, s->h_tp, sizeof(TreeParams), cudaMemcpyHostToDevice, st));
    s->pending = false;

    // The first tree of a session is enqueued directly (it also sets the
    // kernels' launch attributes); later trees replay one captured graph of
    // the same work, so a tree costs one launch instead of ~90.
    int launches = 0;
    if (s->use_graphs && s->trees > 0) {
        int rc = ensure_graph(s, set, prof, boot_mode, s_mode, mvs);
        if (rc) return rc;
        CU(cudaGraphLaunch(s->graph[set], st));
        launches = s->graph_launches[set];
    } else {
        int rc = enqueue_tree(s, set, prof, boot_mode, s_mode, mvs, false, &launches);
        if (rc) return rc;
    }
    if (leaf_of && leaf_of_bytes) {
        if (!s->leaf_export) DA(*(uint32_t**)&s->leaf_export, s->n);
        launch_leaf_export(s->n, s->leaf, s->leaf_export, leaf_of_bytes, st);
        ++launches;
        CU(cudaMemcpyAsync(leaf_of, s->leaf_export, (size_t)leaf_of_bytes * s->n, cudaMemcpyDeviceToHost, st));
    }
    // Host work that needs no device result runs while the tree executes: the
    // previous tree's event times, and the RNG phase after the tree
    // (boosting.rs:7267-7300 + device_draw_replay.rs), which depends only on
    // the depth and the feature count.
    collect_timing(s, set ^ 1);
    if (!s->sample_from_host && s->boot != CBGPU_BOOT_NO) {
        for (int l = 0; l < D; ++l) {
            for (int f = 0; f < s->F; ++f) (void)s->rng.real1();
            (void)s->rng.gen();
            for (int f = 0; f < s->F; ++f) (void)s->rng.std_normal();
        }
        s->rng.gen();  // POST_TREE_EXTRA_DRAWS = 2
        s->rng.gen();
    }
    CU(cudaStreamSynchronize(st));
    CU(cudaGetLastError());
    const TreeState& hts = *s->h_ts;
    s->ev_set = set;
    s->ev_pending[set] = true;
    s->ev_depth[set] = D;
    s->ev_prof[set] = prof;
    {
        double rows = 0;
        for (int l = 0; l < D; ++l) rows += (double)hts.hist_rows[l];
        s->ev_host[set][0] = rows;
        s->ev_host[set][1] = (double)launches;
    }
    if (hts.err) {
        if (hts.err & kErrNoCandidate)
            return fail(CBGPU_ERR_DEVICE, "Degenerate: no split candidate available");
        return fail(CBGPU_ERR_DEVICE, "device error word 0x%x (non-finite derivative or range error)", hts.err);
    }
    for (int l = 0; l < D; ++l) {
        if (split_feature) split_feature[l] = hts.split[l].feature;
        if (split_bin) split_bin[l] = hts.split[l].bin;
    }
    if (n_splits) *n_splits = D;
    const double* raw = s->h_raw;
    if (leaf_values) memcpy(leaf_values, raw, sizeof(double) * L);
    s->pending = true;
    // last_iter_mean_leaf_value over the learning-rate-scaled leaves (bootstrap.rs:382-389)
    double acc = 0.0;
    for (int k = 0; k < L; ++k) {
        double v = raw[k] * s->lr;
        acc += std::sqrt(v * v);
    }
    s->prev_mean = acc / (double)L;
    s->has_prev_mean = true;
    s->trees++;
    return CBGPU_OK;
}

}  // namespace

extern "C" {

const char* cbgpu_last_error(void) { return g_last_error.c_str(); }

const char* cbgpu_version(void) { return "cbgpu 0.1.0 (sm_100a)"; }

int cbgpu_nccl_unique_id(uint8_t* out128) {
    if (!out128) return fail(CBGPU_ERR_INVALID, "null output");
    ncclUniqueId id;
    NC(ncclGetUniqueId(&id));
    static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
    memcpy(out128, &id, sizeof(id));
    return CBGPU_OK;
}

int cbgpu_begin(const cbgpu_begin_args* a, const uint32_t* bins_feature_major, cbgpu_session** out) {
    if (!out) return fail(CBGPU_ERR_INVALID, "null out");
    *out = nullptr;
    int rc = check_args(a);
    if (rc) return rc;
    if (!bins_feature_major && a->n > 0) return fail(CBGPU_ERR_INVALID, "null bins");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
        return fail(CBGPU_ERR_NO_DEVICE, "no CUDA device");
    cbgpu_session* s = new cbgpu_session();
    rc = alloc_session(s, a);
    if (rc) { free_session(s); return rc; }
    s->border_counts.assign((size_t)s->F, s->B - 1);
    if (a->border_counts)
        for (int f = 0; f < s->F; ++f) s->border_counts[(size_t)f] = a->border_counts[f];
    // per-feature column upload + range-checked narrowing to u8
    uint32_t* tmp = nullptr;
    if (s->n > 0) {
        rc = dalloc(&tmp, (size_t)s->n);
        if (rc) { free_session(s); return rc; }
        for (int f = 0; f < s->F && !rc; ++f) {
            cudaError_t e = cudaMemcpyAsync(tmp, bins_feature_major + (size_t)f * s->n,
                                            sizeof(uint32_t) * s->n, cudaMemcpyHostToDevice, s->st);
            if (e != cudaSuccess) rc = fail(CBGPU_ERR_CUDA, "bins upload: %s", cudaGetErrorString(e));
            launch_u32_to_u8_column(tmp, s->n, s->B, s->bins_fm + (size_t)f * s->n_stride, s->d_err, s->st);
        }
        cudaStreamSynchronize(s->st);
        cudaFree(tmp);
    }
    if (!rc) rc = finish_begin(s);
    if (rc) { free_session(s); return rc; }
    *out = s;
    return CBGPU_OK;
}

int cbgpu_begin_raw(const cbgpu_begin_args* a, const float* const* cols, const double* borders_flat,
                    const int32_t* border_counts, cbgpu_session** out) {
    if (!out) return fail(CBGPU_ERR_INVALID, "null out");
    *out = nullptr;
    int rc = check_args(a);
    if (rc) return rc;
    if (!border_counts || (!cols && a->n > 0)) return fail(CBGPU_ERR_INVALID, "null columns / borders");
    int maxb = 0;
    int64_t off = 0;
    for (int f = 0; f < a->n_features; ++f) {
        if (border_counts[f] < 0 || border_counts[f] > 255)
            return fail(CBGPU_DECLINED, "feature %d has %d borders (> 255)", f, border_counts[f]);
        for (int k = 1; k < border_counts[f]; ++k)
            if (!(borders_flat[off + k - 1] <= borders_flat[off + k]))
                return fail(CBGPU_ERR_INVALID, "feature %d borders are not ascending", f);
        off += border_counts[f];
        maxb = std::max(maxb, border_counts[f]);
    }
    if (maxb + 1 > a->n_bins) return fail(CBGPU_ERR_INVALID, "n_bins %d < max borders + 1 = %d", a->n_bins, maxb + 1);
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
        return fail(CBGPU_ERR_NO_DEVICE, "no CUDA device");
    cbgpu_session* s = new cbgpu_session();
    rc = alloc_session(s, a);
    if (rc) { free_session(s); return rc; }
    s->border_counts.assign(border_counts, border_counts + a->n_features);
    float* col = nullptr;
    double* bord = nullptr;
    if (s->n > 0) {
        rc = dalloc(&col, (size_t)s->n);
        if (!rc) rc = dalloc(&bord, (size_t)(off > 0 ? off : 1));
        if (!rc && off > 0) {
            cudaError_t e = cudaMemcpy(bord, borders_flat, sizeof(double) * off, cudaMemcpyHostToDevice);
            if (e != cudaSuccess) rc = fail(CBGPU_ERR_CUDA, "borders upload: %s", cudaGetErrorString(e));
        }
        int64_t boff = 0;
        for (int f = 0; f < s->F && !rc; ++f) {
            cudaError_t e = cudaMemcpyAsync(col, cols[f], sizeof(float) * s->n, cudaMemcpyHostToDevice, s->st);
            if (e != cudaSuccess) rc = fail(CBGPU_ERR_CUDA, "column upload: %s", cudaGetErrorString(e));
            launch_quantize_column(col, s->n, bord + boff, border_counts[f],
                                   s->bins_fm + (size_t)f * s->n_stride, s->d_err, s->st);
            boff += border_counts[f];
        }
        cudaStreamSynchronize(s->st);
        if (col) cudaFree(col);
        if (bord) cudaFree(bord);
    }
    if (!rc) rc = finish_begin(s);
    if (rc) { free_session(s); return rc; }
    *out = s;
    return CBGPU_OK;
}

int cbgpu_grow_tree(cbgpu_session* s, const double* approx, const double* target, int64_t n,
                    const double* sample, int64_t sample_len, int32_t* split_feature, int32_t* split_bin,
                    int32_t* n_splits, double* leaf_values, void* leaf_of, int32_t leaf_of_bytes) {
    if (!s) return fail(CBGPU_ERR_INVALID, "null session");
    const int rc = grow(s, approx, target, n, sample, sample_len, split_feature, split_bin, n_splits,
                        leaf_values, leaf_of, leaf_of_bytes);
    if (rc != CBGPU_OK && s->world > 1) s->broken = true;
    return rc;
}

int cbgpu_end(cbgpu_session* s) {
    free_session(s);
    return CBGPU_OK;
}

int cbgpu_stage_sample(cbgpu_session* s, const double* sample, int64_t sample_len) {
    if (!s) return fail(CBGPU_ERR_INVALID, "null session");
    if (!s->sample_from_host)
        return fail(CBGPU_ERR_INVALID, "Degenerate: staging a host sample needs a session opened with "
                                       "sample_from_host = true");
    if (sample_len != s->n)
        return fail(CBGPU_ERR_INVALID, "LengthMismatch: sample has %lld elements, expected %lld",
                    (long long)sample_len, (long long)s->n);
    if (!sample) return fail(CBGPU_ERR_INVALID, "null sample pointer");
    if (s->stage_count >= 2)
        return fail(CBGPU_ERR_INVALID, "two staged samples already wait for their grow calls");
    CU(cudaSetDevice(s->device));
    if (!s->copy_st) {
        // all or nothing: a failed setup leaves no half-built staging state
        cudaStream_t cs = nullptr;
        double* buf[2] = {nullptr, nullptr};
        cudaEvent_t done[2] = {nullptr, nullptr}, fr[2] = {nullptr, nullptr};
        cudaError_t e = cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking);
        for (int k = 0; k < 2 && e == cudaSuccess; ++k) {
            e = cudaMalloc(&buf[k], sizeof(double) * std::max<int64_t>(s->n, 1));
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done[k], cudaEventDisableTiming);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&fr[k], cudaEventDisableTiming);
        }
        if (e != cudaSuccess) {
            for (int k = 0; k < 2; ++k) {
                if (buf[k]) cudaFree(buf[k]);
                if (done[k]) cudaEventDestroy(done[k]);
                if (fr[k]) cudaEventDestroy(fr[k]);
            }
            if (cs) cudaStreamDestroy(cs);
            return fail(e == cudaErrorMemoryAllocation ? CBGPU_ERR_OOM : CBGPU_ERR_CUDA,
                        "sample staging setup failed: %s", cudaGetErrorString(e));
        }
        s->copy_st = cs;
        for (int k = 0; k < 2; ++k) {
            s->stage_buf[k] = buf[k];
            s->stage_done[k] = done[k];
            s->stage_free[k] = fr[k];
        }
    }
    const int k = (s->stage_head + s->stage_count) & 1;
    // the slot's previous sample was moved out by a grow call on the session
    // stream (an event never recorded is already complete)
    CU(cudaStreamWaitEvent(s->copy_st, s->stage_free[k], 0));
    CU(cudaMemcpyAsync(s->stage_buf[k], sample, sizeof(double) * s->n, cudaMemcpyHostToDevice, s->copy_st));
    CU(cudaEventRecord(s->stage_done[k], s->copy_st));
    ++s->stage_count;
    return CBGPU_OK;
}

int cbgpu_session_approx(cbgpu_session* s, double* out, int64_t n) {
    if (!s || !out || n != s->n) return fail(CBGPU_ERR_INVALID, "bad arguments");
    CU(cudaSetDevice(s->device));
    if (s->pending) {
        launch_apply(s->n, s->approx, s->leaf, s->leaf_lrv, s->st);
        s->pending = false;
    }
    CU(cudaMemcpyAsync(out, s->approx, sizeof(double) * n, cudaMemcpyDeviceToHost, s->st));
    CU(cudaStreamSynchronize(s->st));
    return CBGPU_OK;
}

int cbgpu_session_bins(cbgpu_session* s, uint8_t* out, int64_t n, int32_t F) {
    if (!s || !out || n != s->n || F != s->F) return fail(CBGPU_ERR_INVALID, "bad arguments");
    CU(cudaSetDevice(s->device));
    for (int f = 0; f < F; ++f)
        CU(cudaMemcpyAsync(out + (size_t)f * n, s->bins_fm + (size_t)f * s->n_stride, n,
                           cudaMemcpyDeviceToHost, s->st));
    CU(cudaStreamSynchronize(s->st));
    return CBGPU_OK;
}

int cbgpu_session_last_sample(cbgpu_session* s, double* out, int64_t n) {
    if (!s || !out || n != s->n) return fail(CBGPU_ERR_INVALID, "bad arguments");
    CU(cudaSetDevice(s->device));
    CU(cudaStreamSynchronize(s->st));
    if (s->sample_from_host) {
        CU(cudaMemcpy(out, s->sw64, sizeof(double) * n, cudaMemcpyDeviceToHost));
        return CBGPU_OK;
    }
    std::vector<float> sw((size_t)n);
    CU(cudaMemcpy(sw.data(), s->sw32, sizeof(float) * n, cudaMemcpyDeviceToHost));
    for (int64_t i = 0; i < n; ++i) out[i] = (double)sw[(size_t)i];
    return CBGPU_OK;
}

int cbgpu_session_timing(cbgpu_session* s, double* out8) {
    if (!s || !out8) return fail(CBGPU_ERR_INVALID, "bad arguments");
    CU(cudaSetDevice(s->device));
    collect_timing(s, s->ev_set);  // the last tree's events completed when its grow returned
    for (int k = 0; k < 8; ++k) out8[k] = s->timing[k];
    return CBGPU_OK;
}

int cbgpu_session_timing_sum(cbgpu_session* s, double* out8, int32_t reset) {
    if (!s || !out8) return fail(CBGPU_ERR_INVALID, "bad arguments");
    CU(cudaSetDevice(s->device));
    collect_timing(s, s->ev_set ^ 1);
    collect_timing(s, s->ev_set);
    for (int k = 0; k < 8; ++k) {
        out8[k] = s->timing_sum[k];
        if (reset) s->timing_sum[k] = 0.0;
    }
    return CBGPU_OK;
}

int cbgpu_session_mark(cbgpu_session* s, int32_t slot) {
    if (!s || slot < 0 || slot > 3) return fail(CBGPU_ERR_INVALID, "bad arguments");
    CU(cudaSetDevice(s->device));
    CU(cudaEventRecord(s->uev[slot], s->st));
    return CBGPU_OK;
}

int cbgpu_session_elapsed_ms(cbgpu_session* s, int32_t a, int32_t b, double* out) {
    if (!s || !out || a < 0 || a > 3 || b < 0 || b > 3) return fail(CBGPU_ERR_INVALID, "bad arguments");
    CU(cudaSetDevice(s->device));
    CU(cudaEventSynchronize(s->uev[b]));
    float ms = 0.f;
    CU(cudaEventElapsedTime(&ms, s->uev[a], s->uev[b]));
    *out = ms;
    return CBGPU_OK;
}

int cbgpu_session_set_profiling(cbgpu_session* s, int32_t enabled) {
    if (!s) return fail(CBGPU_ERR_INVALID, "null session");
    s->profiling = enabled != 0;
    return CBGPU_OK;
}

int cbgpu_session_set_graphs(cbgpu_session* s, int32_t enabled) {
    if (!s) return fail(CBGPU_ERR_INVALID, "null session");
    s->use_graphs = enabled != 0;
    return CBGPU_OK;
}

int cbgpu_session_rng_state(cbgpu_session* s, uint64_t* out5) {
    if (!s || !out5) return fail(CBGPU_ERR_INVALID, "bad arguments");
    out5[0] = s->rng.r.x1;
    out5[1] = s->rng.r.c1;
    out5[2] = s->rng.r.x2;
    out5[3] = s->rng.r.c2;
    out5[4] = s->rng.calls;
    return CBGPU_OK;
}

int cbgpu_compute_gradients(int32_t loss, const double* approx, const double* target, int64_t n,
                            double* der1, double* der2) {
    if (loss < 0 || loss > 2) return fail(CBGPU_DECLINED, "loss %d not covered", loss);
    if (n < 0 || (n > 0 && (!approx || !target || !der1)))
        return fail(CBGPU_ERR_INVALID, "bad arguments");
    if (n == 0) return CBGPU_OK;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
        return fail(CBGPU_ERR_NO_DEVICE, "no CUDA device");
    double *a, *t, *d1, *d2 = nullptr;
    DA(a, n);
    DA(t, n);
    DA(d1, n);
    if (der2) DA(d2, n);
    CU(cudaMemcpy(a, approx, sizeof(double) * n, cudaMemcpyHostToDevice));
    CU(cudaMemcpy(t, target, sizeof(double) * n, cudaMemcpyHostToDevice));
    launch_gradients(n, loss, a, t, d1, d2, 0);
    CU(cudaMemcpy(der1, d1, sizeof(double) * n, cudaMemcpyDeviceToHost));
    if (der2) CU(cudaMemcpy(der2, d2, sizeof(double) * n, cudaMemcpyDeviceToHost));
    cudaFree(a);
    cudaFree(t);
    cudaFree(d1);
    if (d2) cudaFree(d2);
    return CBGPU_OK;
}

int cbgpu_histogram(const uint8_t* bins_rm_h, int64_t n, int32_t F, int32_t B, const double* g,
                    const double* h, const int32_t* leaf_of, int32_t n_leaves, double* out_hist) {
    if (n < 0 || F < 1 || B < 1 || B > 256 || n_leaves < 1 || !out_hist ||
        (n > 0 && (!bins_rm_h || !g || !h)))
        return fail(CBGPU_ERR_INVALID, "bad arguments");
    for (int64_t i = 0; i < n; ++i)
        for (int f = 0; f < F; ++f)
            if (bins_rm_h[(size_t)i * F + f] >= B)
                return fail(CBGPU_ERR_INVALID, "bin %d >= n_bins %d at row %lld feature %d",
                            bins_rm_h[(size_t)i * F + f], B, (long long)i, f);
    for (int64_t i = 0; i < n; ++i)
        if (!std::isfinite(g[i]) || !std::isfinite(h[i]))
            return fail(CBGPU_ERR_INVALID, "non-finite g or h at row %lld", (long long)i);
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
        return fail(CBGPU_ERR_NO_DEVICE, "no CUDA device");
    const int F_pad = (int)round_up(F, 32);
    // stable counting sort of rows by leaf -> one contiguous segment per leaf
    std::vector<uint32_t> perm;
    std::vector<HistChunk> chunks;
    {
        std::vector<int64_t> cnt((size_t)n_leaves + 1, 0);
        for (int64_t i = 0; i < n; ++i) {
            int32_t q = leaf_of ? leaf_of[i] : 0;
            if (q >= 0 && q < n_leaves) cnt[(size_t)q + 1]++;
        }
        for (int q = 0; q < n_leaves; ++q) cnt[(size_t)q + 1] += cnt[(size_t)q];
        perm.resize((size_t)cnt[(size_t)n_leaves]);
        std::vector<int64_t> pos(cnt.begin(), cnt.end() - 1);
        for (int64_t i = 0; i < n; ++i) {
            int32_t q = leaf_of ? leaf_of[i] : 0;
            if (q >= 0 && q < n_leaves) perm[(size_t)pos[(size_t)q]++] = (uint32_t)i;
        }
        for (int q = 0; q < n_leaves; ++q)
            for (int64_t st0 = cnt[(size_t)q]; st0 < cnt[(size_t)q + 1]; st0 += kChunkRows)
                chunks.push_back(HistChunk{(uint32_t)q, (uint32_t)st0,
                                           (uint32_t)std::min<int64_t>(kChunkRows, cnt[(size_t)q + 1] - st0), 0u});
    }
    std::vector<uint8_t> rm((size_t)std::max<int64_t>(n, 1) * F_pad, 0);
    for (int64_t i = 0; i < n; ++i) memcpy(&rm[(size_t)i * F_pad], bins_rm_h + (size_t)i * F, (size_t)F);
    // the session's scale rule for the score channels (max |v| * 2^s < 2^kPackBits)
    Pow2 scale[2], inv[2];
    {
        double mx[2] = {0.0, 0.0};
        for (int64_t i = 0; i < n; ++i) {
            mx[0] = std::max(mx[0], std::fabs(g[i]));
            mx[1] = std::max(mx[1], std::fabs(h[i]));
        }
        for (int c = 0; c < 2; ++c) {
            const int sx = fixed_shift(mx[c], kPackBits);
            scale[c] = pow2_of(sx);
            inv[c] = pow2_of(-sx);
        }
    }
    std::vector<uint4> qs((size_t)std::max<int64_t>(n, 1));
    for (int64_t i = 0; i < n; ++i) qs[(size_t)i] = pack_gh(g[i], h[i], scale[0], scale[1]);
    uint8_t* d_rm;
    uint4* d_qs;
    uint32_t *d_perm, *d_nch;
    HistChunk* d_ch;
    ull* d_out;
    const size_t cells = (size_t)n_leaves * F * B * 2;
    DA(d_rm, rm.size());
    DA(d_qs, qs.size());
    DA(d_perm, std::max<size_t>(perm.size(), 1));
    DA(d_ch, std::max<size_t>(chunks.size(), 1));
    DA(d_nch, 1);
    DA(d_out, cells);
    const uint32_t nch = (uint32_t)chunks.size();
    CU(cudaMemcpy(d_rm, rm.data(), rm.size(), cudaMemcpyHostToDevice));
    CU(cudaMemcpy(d_qs, qs.data(), sizeof(uint4) * qs.size(), cudaMemcpyHostToDevice));
    if (!perm.empty()) CU(cudaMemcpy(d_perm, perm.data(), sizeof(uint32_t) * perm.size(), cudaMemcpyHostToDevice));
    if (!chunks.empty()) CU(cudaMemcpy(d_ch, chunks.data(), sizeof(HistChunk) * chunks.size(), cudaMemcpyHostToDevice));
    CU(cudaMemcpy(d_nch, &nch, sizeof(uint32_t), cudaMemcpyHostToDevice));
    CU(cudaMemset(d_out, 0, sizeof(ull) * cells));
    launch_hist(d_rm, F_pad, F, B, d_qs, d_perm, d_ch, d_nch, std::max<uint32_t>(nch, 1), d_out, (int64_t)B * 2,
                (int64_t)F * B * 2, 0);
    CU(cudaGetLastError());
    std::vector<ull> hout(cells);
    CU(cudaMemcpy(hout.data(), d_out, sizeof(ull) * cells, cudaMemcpyDeviceToHost));
    for (size_t k = 0; k < cells; ++k) out_hist[k] = from_fixed((long long)hout[k], inv[k & 1]);
    cudaFree(d_rm); cudaFree(d_qs); cudaFree(d_perm); cudaFree(d_ch); cudaFree(d_nch); cudaFree(d_out);
    return CBGPU_OK;
}

int cbgpu_rank_feature_slice(int32_t n_features, int32_t world, int32_t rank, int32_t* f0, int32_t* fs) {
    if (n_features < 1 || world < 1 || rank < 0 || rank >= world || !f0 || !fs)
        return fail(CBGPU_ERR_INVALID, "rank_feature_slice: bad arguments");
    int a = 0, b = 0;
    feature_slice(n_features, world, rank, &a, &b);
    *f0 = a;
    *fs = b;
    return CBGPU_OK;
}

int cbgpu_rank_select_split(int32_t level, int32_t world, int32_t stride, const uint64_t* all_best,
                            int32_t* feature, int32_t* bin, double* score, int32_t* winner_rank,
                            uint8_t* small_side) {
    if (level < 0 || level > 15 || world < 1 || stride < 2 + 2 * (1 << level) || !all_best || !feature || !bin ||
        !score || !winner_rank)
        return fail(CBGPU_ERR_INVALID, "rank_select_split: bad arguments");
    double sc = 0.0;
    int key = 0;
    const int r = pick_split((const unsigned long long*)all_best, world, stride, &sc, &key);
    *winner_rank = r;
    *feature = r < 0 ? -1 : key >> 8;
    *bin = r < 0 ? -1 : key & 255;
    *score = r < 0 ? -INFINITY : sc;
    if (small_side) {
        const unsigned long long* rec = r >= 0 ? (const unsigned long long*)all_best + (size_t)r * stride : nullptr;
        for (int q = 0; q < (1 << level); ++q) small_side[q] = build_true_side(rec, q);
    }
    return CBGPU_OK;
}

int cbgpu_rank_mvs_partial(int32_t loss, int64_t n, const double* approx, double bias, const double* target,
                           const double* weight, double acc_in, double* acc_out) {
    if (n < 0 || (n > 0 && !target) || !acc_out) return fail(CBGPU_ERR_INVALID, "rank_mvs_partial: bad arguments");
    *acc_out = mvs_abs_der_partial(acc_in, loss == CBGPU_LOSS_RMSE ? 0 : 1, n, approx, bias, target, weight);
    return CBGPU_OK;
}

int cbgpu_bootstrap_weights(int32_t type, int64_t n, int64_t row_offset, uint64_t rand_seed,
                            const uint64_t* rng_raw4, float sample_rate, float temp,
                            const double* der_obj, double lambda, double* out) {
    if (n < 0 || (n > 0 && !out)) return fail(CBGPU_ERR_INVALID, "bad arguments");
    if (n == 0) return CBGPU_OK;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
        return fail(CBGPU_ERR_NO_DEVICE, "no CUDA device");
    float* d_sw;
    DA(d_sw, n);
    double* d_der = nullptr;
    double* d_thr = nullptr;
    TreeParams tp{};
    tp.boot_seed = rand_seed;
    tp.mvs_lambda = lambda;
    if (rng_raw4) tp.boot_base = Rng64{rng_raw4[0], rng_raw4[1], rng_raw4[2], rng_raw4[3]};
    TreeParams* d_tp;
    DA(d_tp, 1);
    CU(cudaMemcpy(d_tp, &tp, sizeof(tp), cudaMemcpyHostToDevice));
    if (type == CBGPU_BOOT_BAYESIAN) {
        launch_bootstrap(1, n, row_offset, d_tp, 0.0, temp, d_sw, 0);
    } else if (type == CBGPU_BOOT_BERNOULLI) {
        if (!rng_raw4) { cudaFree(d_sw); cudaFree(d_tp); return fail(CBGPU_ERR_INVALID, "Bernoulli needs rng_raw4"); }
        launch_bootstrap(2, n, row_offset, d_tp, (double)sample_rate, 0.0f, d_sw, 0);
    } else if (type == CBGPU_BOOT_MVS) {
        if (!der_obj || row_offset % 8192) {
            cudaFree(d_sw);
            cudaFree(d_tp);
            return fail(CBGPU_ERR_INVALID, "MVS needs der_obj, aligned row_offset");
        }
        DA(d_der, n);
        DA(d_thr, (n + 8191) / 8192);
        CU(cudaMemcpy(d_der, der_obj, sizeof(double) * n, cudaMemcpyHostToDevice));
        launch_mvs(n, row_offset, d_der, d_tp, (double)sample_rate, d_thr, d_sw, 0);
    } else {
        cudaFree(d_sw);
        cudaFree(d_tp);
        return fail(CBGPU_ERR_INVALID, "bootstrap type %d has no device weights", type);
    }
    CU(cudaGetLastError());
    std::vector<float> h((size_t)n);
    CU(cudaMemcpy(h.data(), d_sw, sizeof(float) * n, cudaMemcpyDeviceToHost));
    for (int64_t i = 0; i < n; ++i) out[i] = (double)h[(size_t)i];
    cudaFree(d_sw);
    cudaFree(d_tp);
    if (d_der) cudaFree(d_der);
    if (d_thr) cudaFree(d_thr);
    return CBGPU_OK;
}

}  // extern "C"
