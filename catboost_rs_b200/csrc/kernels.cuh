// kernels.cuh -- device kernels of the B200 oblivious-tree path and their launchers.
#pragma once

#include <cstdint>
#include <utility>
#include <cuda_runtime.h>

#include "cbgpu_common.cuh"

namespace cbgpu {

using ull = unsigned long long;

// Fixed-point scales for the four int64 accumulation channels:
// 0 = score der (g), 1 = score weight (h), 2 = leaf der (w*der1), 3 = leaf weight (w).
struct Scales {
    double scale[4];
    double inv[4];
};

// One histogram work item: rows [start, start+len) of the (leaf-sorted) order
// go into built-histogram slot `slot`.
struct HistChunk {
    uint32_t slot;
    uint32_t start;
    uint32_t len;
    uint32_t pad;
};

// The split chosen at one level.
struct SplitRec {
    int32_t feature;
    int32_t bin;
    double score;
};

// Per-tree device-side results (one D2H per tree).
// Per-tree scalars the host decides (from its RNG stream replica) and the
// kernels read from device memory, so a captured tree graph replays with new
// values: copied host -> device before every tree.
struct TreeParams {
    uint64_t boot_seed;  // Bayesian rand_seed / MVS seed
    Rng64 boot_base;     // Bernoulli: the main stream at the tree's first row
    double mvs_lambda;
    int32_t pending;     // apply the previous tree's leaf values before the derivatives
    int32_t pad;
    double q_alpha;      // MAE / Quantile: quantile_der1's alpha and delta
    double q_delta;
};

struct TreeState {
    SplitRec split[16];
    uint32_t err;
    uint32_t score_done;   // last-block-done counter of the score kernel
    uint32_t pad[2];
    uint32_t hist_rows[16];  // rows histogrammed at each level (the smaller children)
    ull maxbits[4];        // bit patterns of max |channel| (non-negative doubles)
    Scales sc;
};

constexpr int kTile = 32;          // features per histogram tile (one per lane)
constexpr int kHistSmemMax = 227 * 1024;  // dynamic shared memory opt-in limit per block
constexpr int kChunkRows = 16384;  // rows per histogram work item
// Score-channel fixed point: |row value| <= 2^kPackBits, split at bit kPackSplit
// into (lo, hi) u32 parts whose sums over kChunkRows rows stay below 2^31.
constexpr int kPackBits = 33;
constexpr int kPackSplit = 17;
static_assert((long long)kChunkRows << kPackSplit <= (1ll << 31), "lo sums must fit 31 bits");
static_assert((long long)kChunkRows << (kPackBits - kPackSplit) <= (1ll << 31), "hi sums must fit 31 bits");
constexpr int kPartThreads = 256;
constexpr int kPartItems = 16;     // positions per thread in the partition kernels
constexpr int kPartTile = kPartThreads * kPartItems;
constexpr int kBootRun = 8;        // consecutive rows per thread in the bootstrap kernel

// Leaf segments of the leaf-sorted row order: by leaf id (off, cnt) and in
// position order (mem_start, mem_leaf); *_next are written by the partition
// and swapped in afterwards.  start/end_* and t_start/f_cnt are P1/P2 scratch.
struct SegTables {
    uint32_t *seg_off, *seg_cnt, *mem_start, *mem_leaf;
    uint32_t *seg_off_next, *seg_cnt_next, *mem_start_next, *mem_leaf_next;
    uint32_t *start_blk, *start_part, *end_blk, *end_part, *t_start, *f_cnt;
    void swap() {
        std::swap(seg_off, seg_off_next);
        std::swap(seg_cnt, seg_cnt_next);
        std::swap(mem_start, mem_start_next);
        std::swap(mem_leaf, mem_leaf_next);
    }
};

// ---- begin: quantization / layout ------------------------------------------
void launch_quantize_column(const float* col, int64_t n, const double* borders, int32_t nb,
                            uint8_t* out_fm_row, uint32_t* err, cudaStream_t st);
void launch_u32_to_u8_column(const uint32_t* col, int64_t n, int32_t n_bins, uint8_t* out_fm_row,
                             uint32_t* err, cudaStream_t st);
void launch_transpose_fm_to_rm(const uint8_t* fm, int64_t n, int64_t n_stride, int32_t F,
                               uint8_t* rm, int32_t F_pad, cudaStream_t st);
void launch_transpose_rm_to_fm(const uint8_t* rm, int64_t n, int32_t F, int32_t F_src,
                               uint8_t* fm, int64_t n_stride, cudaStream_t st);

// ---- per tree: bootstrap, derivatives, scales -------------------------------
// mode: 1 = Bayesian (tp->boot_seed, temp), 2 = Bernoulli (tp->boot_base, rate)
void launch_bootstrap(int mode, int64_t n, int64_t row_offset, const TreeParams* tp, double rate, float temp,
                      float* out_sw, cudaStream_t st);
// MVS with lambda tp->mvs_lambda and seed tp->boot_seed
void launch_mvs(int64_t n, int64_t row_offset, const double* wd1, const TreeParams* tp, double rate,
                double* thresholds, float* out_sw, cudaStream_t st);
// s_mode: 0 = none (weights 1), 1 = f32 device sample, 2 = f64 host sample.
// approx += lrv[leaf] first when tp->pending.
void launch_der(int64_t n, int loss, double* approx, const double* target, const double* weight,
                const uint16_t* leaf, const double* lrv, const TreeParams* tp, int s_mode, const float* sw32,
                const double* sw64, double* wd1, TreeState* ts, bool defer_gh, cudaStream_t st);
void launch_max_gh(int64_t n, const double* wd1, const double* weight, const float* sw32, TreeState* ts,
                   cudaStream_t st);
void launch_scales(TreeState* ts, int64_t n_total, cudaStream_t st);
void launch_pack_stats(int64_t n, const double* wd1, const double* weight, int s_mode, const float* sw32,
                       const double* sw64, const TreeState* ts, uint4* qstats, cudaStream_t st);
void launch_apply(int64_t n, double* approx, const uint16_t* leaf, const double* lrv,
                  cudaStream_t st);

// ---- per level ---------------------------------------------------------------
void launch_zero(void* p, size_t bytes, cudaStream_t st);
int hist_tiles(int32_t F, int32_t B);  // feature tiles (grid x) of the histogram launch
// n_chunks: device chunk count; max_chunks bounds it.  Cell (slot, f, bin, c)
// of the output is built[slot * slot_stride + f * feat_stride + bin * 2 + c].
void launch_hist(const uint8_t* bins_rm, int32_t F_pad, int32_t F, int32_t B, const uint4* qstats,
                 const uint32_t* perm, const HistChunk* chunks, const uint32_t* n_chunks, uint32_t max_chunks,
                 ull* built, int64_t feat_stride, int64_t slot_stride, cudaStream_t st);
// level 0 also initialises the segment tables to the single all-rows segment.
// cap = entries of `chunks`: at most n / kChunkRows + 2^(level-1) + 1 are written.
void launch_make_chunks(int level, uint32_t* seg_off, uint32_t* seg_cnt, uint32_t* mem_start,
                        uint32_t* mem_leaf, const uint8_t* small_side, int64_t n_level0,
                        HistChunk* chunks, uint32_t cap, uint32_t* n_chunks, TreeState* ts, cudaStream_t st);
// Derive and score work on this rank's feature slice [f0, f0 + Fs) in
// feature-major layouts (see derive_prefix_kernel).  With rank_best null the
// winner goes to ts->split[level]; otherwise the slice winner's record goes to
// rank_best (score bits, key, then 2^level (false, true) weight sums) for
// launch_select_split after an all-gather (records of `stride` words; a null
// small_side skips the next level's build-side choice).
void launch_derive_prefix(int level, int32_t Fs, int32_t B, const ull* built, const ull* prev,
                          ull* cur, const uint8_t* small_side, cudaStream_t st);
void launch_score(int level, int32_t Fs, int32_t f0, int32_t F, int32_t B, const ull* cur,
                  const int32_t* border_counts, double l2, int score_fn, double* grp_score, int32_t* grp_bin,
                  TreeState* ts, ull* rank_best, cudaStream_t st);
void launch_select_split(int level, int world, int stride, const ull* all_best, TreeState* ts,
                         uint8_t* small_side, cudaStream_t st);
// flags: 2 * (ceil(n / 32) + 1) words (the split outcome bits, natural then position order); blk_true: ceil(n / kPartTile) + 1; child_cnt: 2^(level+1) (false counts, then true).
void launch_partition(int level, int64_t n, const uint8_t* bins_fm, int64_t n_stride,
                      const uint32_t* perm, uint32_t* perm_next, SegTables& sg, uint32_t* blk_true,
                      uint32_t* flags, uint32_t* child_cnt, TreeState* ts, cudaStream_t st);
void launch_small_side(int level_next, const uint32_t* child_cnt_global, uint8_t* small_side,
                       cudaStream_t st);
void launch_route_leafsum(int depth, int64_t n, const uint8_t* bins_fm, int64_t n_stride, uint16_t* leaf,
                          const double* wd1, const double* weight, TreeState* ts, ull* leaf_sums,
                          cudaStream_t st);
// Exact leaves (MAE / Quantile): keys[i] = leaf << 32 | total-order bits of
// the f32 residual, sorted with the weights, then one block per leaf takes
// the weighted alpha-quantile into leaf_raw / leaf_lrv.  tmp / tmp_bytes is
// the radix sort's scratch (exact_sort_scratch_bytes).
size_t exact_sort_scratch_bytes(int64_t n);
void launch_exact_leaves(int depth, int64_t n, const double* approx, const double* target, const double* weight,
                         const uint16_t* leaf, ull* keys, ull* keys_sorted, double* w, double* w_sorted, void* tmp,
                         size_t tmp_bytes, double alpha, double delta, double lr, double* leaf_raw,
                         double* leaf_lrv, cudaStream_t st);

void launch_leaf_values(int depth, int n_splits_expected, const ull* leaf_sums, double l2, double lr,
                        TreeState* ts, double* leaf_raw, double* leaf_lrv, cudaStream_t st);
void launch_leaf_export(int64_t n, const uint16_t* leaf, void* out, int bytes, cudaStream_t st);
void launch_gradients(int64_t n, int loss, const double* approx, const double* target, double* d1,
                      double* d2, cudaStream_t st);

}  // namespace cbgpu
