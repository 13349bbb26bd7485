// kernels.cuh -- device kernels of the B200 oblivious-tree path and their launchers.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>
#include <utility>
#include <cuda_runtime.h>

#include "cbgpu_common.cuh"

namespace cbgpu {

using ull = unsigned long long;

// A power of two 2^s held as two factors 2^(s/2) and 2^(s - s/2): both stay
// normal doubles for |s| <= 2044, and (v * a) * b rounds exactly as v * 2^s
// does whenever the result is not subnormal, so a fixed-point scale can
// follow any finite magnitude (a channel whose largest |v| is 1e-300 still
// gets a 2^-33-relative grid).
struct Pow2 {
    double a, b;
};
CBGPU_HD Pow2 pow2_of(int s) {
    const int h = s / 2;
#ifdef __CUDA_ARCH__
    return Pow2{ldexp(1.0, h), ldexp(1.0, s - h)};
#else
    return Pow2{std::ldexp(1.0, h), std::ldexp(1.0, s - h)};
#endif
}
// Fixed-point exponent for a channel whose largest magnitude is m: the s with
// m * 2^s < 2^bits (0 for m == 0), clamped to +-2000 (every finite m is inside).
CBGPU_HD int fixed_shift(double m, int bits) {
    if (!(m > 0.0)) return 0;
    int e = 0;
#ifdef __CUDA_ARCH__
    frexp(m, &e);
#else
    std::frexp(m, &e);
#endif
    int s = bits - e;
    if (s > 2000) s = 2000;
    if (s < -2000) s = -2000;
    return s;
}
// round(v * 2^s) and q * 2^-s, both through the two factors.
CBGPU_HD long long to_fixed(double v, Pow2 f) {
#ifdef __CUDA_ARCH__
    return __double2ll_rn(__dmul_rn(__dmul_rn(v, f.a), f.b));
#else
    return std::llrint((v * f.a) * f.b);
#endif
}
CBGPU_HD double from_fixed(long long q, Pow2 inv) {
#ifdef __CUDA_ARCH__
    return __dmul_rn(__dmul_rn((double)q, inv.a), inv.b);
#else
    return ((double)q * inv.a) * inv.b;
#endif
}

// Fixed-point scales for the four int64 accumulation channels:
// 0 = score der (g), 1 = score weight (h), 2 = leaf der (w*der1), 3 = leaf weight (w).
struct Scales {
    Pow2 scale[4];
    Pow2 inv[4];
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
    uint32_t cursor0;      // write cursor of the first partition's one segment
    uint32_t pad;
    uint32_t hist_rows[16];  // rows histogrammed at each level (the smaller children)
    ull maxbits[4];        // bit patterns of max |channel| (non-negative doubles)
    Scales sc;
};

constexpr int kTile = 32;          // features per histogram tile (one per lane)
constexpr int kHistSmemMax = 227 * 1024;  // dynamic shared memory opt-in limit per block
constexpr int kChunkRows = 16384;  // rows per histogram work item
constexpr int kSegMax = 1 << 15;   // parents or children of one partition (depth <= 16)
// Score-channel fixed point: |row value| <= 2^kPackBits, split at bit kPackSplit
// into (lo, hi) u32 parts whose sums over kChunkRows rows stay below 2^31.
constexpr int kPackBits = 33;
constexpr int kPackSplit = 17;
static_assert((long long)kChunkRows << kPackSplit <= (1ll << 31), "lo sums must fit 31 bits");
static_assert((long long)kChunkRows << (kPackBits - kPackSplit) <= (1ll << 31), "hi sums must fit 31 bits");

// One row's packed score channels {g_lo, g_hi, h_lo, h_hi}: g and h rounded
// once to the channel's fixed point and split at bit kPackSplit.
CBGPU_HD uint4 pack_gh(double g, double h, Pow2 sg, Pow2 sh) {
    const long long qg = to_fixed(g, sg), qh = to_fixed(h, sh);
    uint4 o;
    o.x = (uint32_t)(qg & ((1ll << kPackSplit) - 1));
    o.y = (uint32_t)(int32_t)(qg >> kPackSplit);
    o.z = (uint32_t)(qh & ((1ll << kPackSplit) - 1));
    o.w = (uint32_t)(int32_t)(qh >> kPackSplit);
    return o;
}
constexpr int kBootRun = 8;        // consecutive rows per thread in the bootstrap and derivative kernels
constexpr int kJumpSteps = 1010;   // LCG jump table: Bayesian jumps are 10 + (row mod 1000) steps

// ---- multi-rank decisions (host and device share this code) ----------------
//
// Rank r of `world` derives and scores the features [f0, f0 + fs) of the
// world * fs padded feature range (features >= F have no candidates).
CBGPU_HD void feature_slice(int F, int world, int rank, int* f0, int* fs) {
    *fs = (F + world - 1) / world;
    *f0 = rank * *fs;
}
constexpr int kNoSplitKey = 0x7fffffff;  // a slice record without a candidate
// (score, key) better than (bs, bk)?  Strict > with the lowest key on ties --
// key = feature << 8 | border, so this is the CPU's first-wins strict-> scan
// over (feature asc, border asc) (tree.rs:355-366).
CBGPU_HD bool better_split(double s, int k, double bs, int bk) { return s > bs || (s == bs && k < bk); }
CBGPU_HD double bits_as_double(unsigned long long b) {
#ifdef __CUDA_ARCH__
    return __longlong_as_double((long long)b);
#else
    double d;
    memcpy(&d, &b, sizeof d);
    return d;
#endif
}
// The global split over the ranks' all-gathered slice records (`stride`
// words each: score bits, key, then 2^level (false, true) weight sums):
// returns the winning rank (-1 when no rank has a candidate) and its score
// and key.  Every rank runs it on the same records, so all agree.
CBGPU_HD int pick_split(const unsigned long long* all_best, int world, int stride, double* score, int* key) {
    double fb = -INFINITY;
    int fk = kNoSplitKey, fr = -1;
    for (int r = 0; r < world; ++r) {
        const double sc = bits_as_double(all_best[(size_t)r * stride]);
        const int k = (int)(uint32_t)all_best[(size_t)r * stride + 1];
        if (k == kNoSplitKey) continue;
        if (better_split(sc, k, fb, fk)) {
            fb = sc;
            fk = k;
            fr = r;
        }
    }
    if (fk == kNoSplitKey || fb == -INFINITY) fr = -1;
    *score = fb;
    *key = fk;
    return fr;
}
// The next level's build side of parent q from the winner's record: 1 (build
// the true child) when the true child carries no more weight than the false
// one.  Which child is built changes no result -- the sums are exact -- so
// every rank only needs the same answer.
CBGPU_HD uint8_t true_child_built(unsigned long long false_w, unsigned long long true_w) {
    return true_w <= false_w ? 1 : 0;
}
CBGPU_HD uint8_t build_true_side(const unsigned long long* winner_rec, int q) {
    if (!winner_rec) return 1;
    const unsigned long long* m = winner_rec + 2;
    return true_child_built(m[2 * q], m[2 * q + 1]);
}

#ifdef __CUDACC__
// Exact 64-bit add into a (lo, hi) pair of 32-bit words (shared memory, where
// 64-bit atomics are slow): the lo add's wrap carries into hi, so
// hi * 2^32 + lo is the sum mod 2^64 (exact whenever the true sum fits an int64).
__device__ __forceinline__ void add_split64(uint32_t* lo, uint32_t* hi, long long v) {
    const uint32_t l = (uint32_t)(unsigned long long)v;
    const uint32_t old = atomicAdd(lo, l);
    atomicAdd(hi, (uint32_t)(v >> 32) + (old + l < old ? 1u : 0u));
}
#endif

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device)
// and size, thread-safe; returns the cudaError_t of the setting (0 = ok).
int ensure_dyn_smem(const void* kernel, int bytes);

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
// The jump multipliers of 0 .. kJumpSteps - 1 LCG steps (2 * kJumpSteps words).
void launch_jump_table(ull* jump, cudaStream_t st);
// s_mode: 0 = none (weights 1), 1 = f32 device sample, 2 = f64 host sample.
// approx += lrv[leaf] first when tp->pending.  boot_mode 1 / 2 draws the
// Bayesian (temp) / Bernoulli (rate) sample in the same pass (as
// launch_bootstrap, using the jump table when not null) into sw32 and uses
// it (s_mode 1).
void launch_der(int64_t n, int loss, double* approx, const double* target, const double* weight,
                const uint16_t* leaf, const double* lrv, const TreeParams* tp, int s_mode, float* sw32,
                const double* sw64, double* wd1, TreeState* ts, bool defer_gh, int boot_mode, int64_t row_offset,
                double rate, float temp, const ull* jump, cudaStream_t st);
void launch_max_gh(int64_t n, const double* wd1, const double* weight, const float* sw32, TreeState* ts,
                   cudaStream_t st);
// Packs every row's score channels; derives the fixed-point scales of all
// four channels from the tree's maxima itself and records them in ts->sc for
// the later kernels, with this rank's level-0 row count in ts->hist_rows[0].
void launch_pack_stats(int64_t n, const double* wd1, const double* weight, int s_mode, const float* sw32,
                       const double* sw64, TreeState* ts, int64_t n_total, uint4* qstats, cudaStream_t st);
void launch_apply(int64_t n, double* approx, const uint16_t* leaf, const double* lrv,
                  cudaStream_t st);

// ---- per level ---------------------------------------------------------------
void launch_zero(void* p, size_t bytes, cudaStream_t st);
int hist_tiles(int32_t F, int32_t B);  // feature tiles (grid x) of the histogram launch
int hist_lane_features(int32_t B);  // features each lane owns in the histogram launch (1 or 2)
// n_chunks: device chunk count; max_chunks bounds it.  Cell (slot, f, bin, c)
// of the output is built[slot * slot_stride + f * feat_stride + bin * 2 + c].
void launch_hist(const uint8_t* bins_rm, int32_t F_pad, int32_t F, int32_t B, const uint4* qstats,
                 const uint32_t* perm, const HistChunk* chunks, const uint32_t* n_chunks, uint32_t max_chunks,
                 ull* built, int64_t feat_stride, int64_t slot_stride, cudaStream_t st);
// n_sets stat sets over the same rows in one launch (grid z): set k reads
// qstats + k * set_qstride and adds into built + k * set_built_stride.
void launch_hist_sets(const uint8_t* bins_rm, int32_t F_pad, int32_t F, int32_t B, const uint4* qstats,
                      const uint32_t* perm, const HistChunk* chunks, const uint32_t* n_chunks, uint32_t max_chunks,
                      ull* built, int64_t feat_stride, int64_t slot_stride, int32_t n_sets, int64_t set_qstride,
                      int64_t set_built_stride, cudaStream_t st);
// The level-0 histogram work list (all rows), built once per session.
void launch_level0_chunks(int64_t n, HistChunk* chunks, uint32_t cap, uint32_t* n_chunks, uint32_t* err,
                          uint32_t chunk_rows, cudaStream_t st);
// Rows per histogram work item for a session of n rows whose level-0 launch
// has `tiles` feature tiles and `sets` stat sets on a device of `sms` SMs:
// kChunkRows, or kChunkRows / 2 when the launch would fill fewer than 8
// blocks per SM.  The sums do not depend on it.
uint32_t hist_chunk_rows(int64_t n, int tiles, int sets, int sms);
// Derive and score work on this rank's feature slice [f0, f0 + Fs) in
// feature-major layouts (see derive_prefix_kernel).  With rank_best null the
// winner goes to ts->split[level] and, with small_side not null, each leaf's
// build side for the next level (the winner's child with no more weight);
// otherwise the slice winner's record goes to rank_best (score bits, key, then
// 2^level (false, true) weight sums) for launch_select_split after an
// all-gather (records of `stride` words; a null small_side skips the next
// level's build-side choice).
void launch_derive_prefix(int level, int32_t Fs, int32_t B, const ull* built, const ull* prev,
                          ull* cur, const uint8_t* small_side, cudaStream_t st);
// n_sets stat sets in one launch (grid y): set k reads built + k *
// set_built_stride and prev + k * set_cur_stride, writes cur + k * set_cur_stride.
void launch_derive_prefix_sets(int level, int32_t Fs, int32_t B, const ull* built, const ull* prev, ull* cur,
                               const uint8_t* small_side, int32_t n_sets, int64_t set_built_stride,
                               int64_t set_cur_stride, cudaStream_t st);
void launch_score(int level, int32_t Fs, int32_t f0, int32_t F, int32_t B, const ull* cur,
                  const int32_t* border_counts, double l2, int score_fn, double* grp_score, int32_t* grp_bin,
                  TreeState* ts, ull* rank_best, uint8_t* small_side, cudaStream_t st);
void launch_select_split(int level, int world, int stride, const ull* all_best, TreeState* ts,
                         uint8_t* small_side, cudaStream_t st);
// Routing by split `level` (leaf[] is not read at level 0) and, for each
// parent q < 2^level, the rows of its built child (new bit == small_side[q])
// written to list from cursor[q] on (cursor[q] advances past them).  The
// split of level l is (splits[l * split_stride], splits[l * split_stride + 1])
// = (feature, bin); features >= f_eq are one-hot (bit = bin == value), the
// others take bit = bin > border.
void launch_partition(int level, int64_t n, const uint8_t* bins_fm, int64_t n_stride, uint16_t* leaf,
                      const uint8_t* small_side, uint32_t* cursor, uint32_t* list, const int32_t* splits,
                      int split_stride, int f_eq, cudaStream_t st);
// After launch_partition(level): the next level's histogram work list from
// the built segments [base_in[q], cursor[q]) (ts->hist_rows[level + 1]); with
// rows_out not null, the 2^(level+1) children's row counts and segment starts
// (rows_out, base_out, cursor_out = base_out) for the next partition.
// rows_in / base_in null: level 0's single parent of n rows at base 0.
void launch_segments(int level, int64_t n, const uint32_t* rows_in, const uint32_t* base_in, const uint32_t* cursor,
                     const uint8_t* small_side, uint32_t* rows_out, uint32_t* base_out, uint32_t* cursor_out,
                     HistChunk* chunks, uint32_t cap, uint32_t* n_chunks, TreeState* ts, uint32_t chunk_rows,
                     cudaStream_t st);
// The last split (`level`): leaf[i] |= (bin > border) << level, and the exact
// int64 sums of the unsampled w * der1 and w per final leaf added into
// leaf_sums[2 << level][2].
void launch_route_leafsum(int level, int64_t n, const uint8_t* bins_fm, int64_t n_stride, uint16_t* leaf,
                          const double* wd1, const double* weight, TreeState* ts, ull* leaf_sums, cudaStream_t st);
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
