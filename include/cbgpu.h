/*
 * cbgpu.h -- C ABI of the B200-native oblivious-tree training path.
 *
 * This library replaces the device half of catboost_rs's compute seam: the
 * `cb_compute::Runtime` trait methods that `cb_train`'s boosting loop calls
 * (crates/cb-compute/src/runtime.rs:1410-1651).  A thin Rust shim implements
 * `Runtime` on top of these entry points; everything
 * above the seam (cb-train's loop, cb-data's pool, the fit/predict APIs)
 * stays unchanged.
 *
 * Conventions (mirroring the seam, runtime.rs:899-906, 1410-1651):
 *  - plain pointers and sizes; inputs are borrowed for the call only;
 *  - every entry point returns a cbgpu_status; CBGPU_DECLINED means "decline
 *    to the CPU grower" (the trait's Ok(false) / Ok(None));
 *  - on any other non-zero status cbgpu_last_error() returns a message
 *    (thread-local), the analogue of the trait's CbError;
 *  - sessions are not thread-safe; the caller serializes calls per session
 *    (the reference wraps its session in a Mutex, gpu_backend.rs:47-67).
 */
#ifndef CBGPU_H
#define CBGPU_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CBGPU_API __attribute__((visibility("default")))
#else
#define CBGPU_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    CBGPU_OK = 0,
    CBGPU_DECLINED = 1,       /* outside the covered regime: use the CPU grower */
    CBGPU_ERR_INVALID = 2,    /* LengthMismatch / Degenerate / OutOfRange */
    CBGPU_ERR_CUDA = 3,       /* CUDA runtime error */
    CBGPU_ERR_OOM = 4,        /* device allocation failed */
    CBGPU_ERR_NCCL = 5,       /* collective failed or timed out */
    CBGPU_ERR_DEVICE = 6,     /* a kernel raised its device error word */
    CBGPU_ERR_NO_DEVICE = 7   /* no CUDA device / library built without one */
} cbgpu_status;

/* Loss (runtime.rs:57-70, 186-260): only the device-covered subset.  The
 * multi-output losses (MultiClass, MultiClassOneVsAll, MultiLogloss,
 * MultiCrossEntropy) are served by the multi-output session
 * (cbgpu_multi_begin_raw), the grouped losses by its ranking mode
 * (cbgpu_rank_begin_raw); the scalar session declines them. */
typedef enum {
    CBGPU_LOSS_RMSE = 0, CBGPU_LOSS_LOGLOSS = 1, CBGPU_LOSS_CROSSENTROPY = 2, CBGPU_LOSS_MULTICLASS = 3,
    CBGPU_LOSS_QUERYRMSE = 4, CBGPU_LOSS_PAIRLOGIT = 5, CBGPU_LOSS_PAIRLOGIT_PAIRWISE = 6,
    CBGPU_LOSS_QUERYSOFTMAX = 7, CBGPU_LOSS_LAMBDAMART = 8, CBGPU_LOSS_YETIRANK = 9,
    CBGPU_LOSS_STOCHASTICRANK = 10, CBGPU_LOSS_YETIRANK_PAIRWISE = 11,
    CBGPU_LOSS_MULTICLASS_ONE_VS_ALL = 12, CBGPU_LOSS_MULTILOGLOSS = 13, CBGPU_LOSS_MULTICROSSENTROPY = 14,
    CBGPU_LOSS_MAE = 15, CBGPU_LOSS_QUANTILE = 16, /* the scalar session, Exact leaves only */
    CBGPU_LOSS_RMSE_WITH_UNCERTAINTY = 17          /* the multi-output session, approx_dim 2 */
} cbgpu_loss;

/* EScoreFunction (runtime.rs:834-864); Cosine is the default. */
typedef enum {
    CBGPU_SCORE_COSINE = 0, CBGPU_SCORE_L2 = 1, CBGPU_SCORE_SOLAR_L2 = 2, CBGPU_SCORE_NEWTON_L2 = 3,
    CBGPU_SCORE_NEWTON_COSINE = 4, CBGPU_SCORE_LOO_L2 = 5, CBGPU_SCORE_SAT_L2 = 6
} cbgpu_score_fn;

/* DeviceBootstrapType (runtime.rs:1085-1097). */
typedef enum {
    CBGPU_BOOT_NO = 0, CBGPU_BOOT_BAYESIAN = 1, CBGPU_BOOT_BERNOULLI = 2, CBGPU_BOOT_MVS = 3,
    CBGPU_BOOT_POISSON = 4
} cbgpu_bootstrap;

/* DeviceGrowPolicy (runtime.rs DeviceTrainConfig::grow_policy). */
typedef enum { CBGPU_GROW_SYMMETRIC = 0, CBGPU_GROW_DEPTHWISE = 1, CBGPU_GROW_LOSSGUIDE = 2,
               CBGPU_GROW_REGION = 3 } cbgpu_grow_policy;

/* The scalar arguments of Runtime::begin_device_training{,_raw}
 * (runtime.rs:1497, :1546) plus DeviceTrainConfig (runtime.rs:1259-1372)
 * and the document-sharding placement of this rank. */
typedef struct {
    int32_t loss;                    /* cbgpu_loss */
    int32_t depth;                   /* 1..16 (tree.rs MAX_DEPTH) */
    int32_t boosting_type_is_plain;  /* must be 1 */
    int32_t fold_count;              /* must be 1 */
    int32_t score_function;          /* cbgpu_score_fn: Cosine or L2 are covered */
    int64_t n;                       /* rows held by THIS rank */
    int32_t n_features;
    int32_t n_bins;                  /* max(border count) + 1; <= 256 */
    double learning_rate;
    double scaled_l2;                /* l2_leaf_reg * sum(weights) / n_total (leaf.rs:177) */
    const double* weight;            /* [n] per-object weights, or NULL for unit weights */
    /* DeviceTrainConfig */
    int32_t grow_policy;             /* cbgpu_grow_policy: only SymmetricTree is covered */
    int32_t bootstrap_type;          /* cbgpu_bootstrap */
    float sample_rate;               /* Bernoulli / MVS subsample */
    float bagging_temperature;       /* Bayesian temperature */
    int32_t has_mvs_lambda;          /* 1: use mvs_lambda for every tree */
    double mvs_lambda;
    uint64_t rng_seed;               /* the fit's random_seed (main TFastRng64 stream) */
    double bias;                     /* starting approximant for the resident approx */
    int32_t sample_from_host;        /* 1: grow_tree receives the bootstrap multiplier */
    double random_strength;          /* must be 0 (the device gate, boosting.rs:5789-6010) */
    /* placement (1 GPU: rank 0 of 1, row_offset 0, n_total == n) */
    int32_t device;                  /* CUDA ordinal for this rank */
    int32_t rank;
    int32_t world_size;
    int64_t row_offset;              /* global index of this rank's first row */
    int64_t n_total;                 /* rows over all ranks */
    const uint8_t* nccl_unique_id;   /* 128 bytes from cbgpu_nccl_unique_id when world_size > 1 */
    /* [n_features] border count per feature for cbgpu_begin (split candidates
     * are borders 0..count-1), or NULL: n_bins - 1 candidates for every
     * feature, as the reference device scorer does (kernels.rs:4687-4712).
     * cbgpu_begin_raw takes the counts from its border lists. */
    const int32_t* border_counts;
    /* DeviceTrainConfig::exact_leaf / quantile_alpha / quantile_delta
     * (session.rs:1176-1200): 1 takes each leaf's weighted alpha-quantile of
     * the f32 residuals t - a (leaf.rs:445-520) for CBGPU_LOSS_MAE (alpha 0.5,
     * delta 1e-6) or CBGPU_LOSS_QUANTILE (these alpha / delta); the structure
     * comes from quantile_der1 (loss.rs:166-175).  Needs bootstrap No and one
     * rank; 0 with MAE / Quantile, or 1 with another loss, declines.  A zeroed
     * tail (callers built before these fields) means 0. */
    int32_t exact_leaf;
    double quantile_alpha;
    double quantile_delta;
} cbgpu_begin_args;

typedef struct cbgpu_session cbgpu_session;

/* Runtime::begin_device_training (runtime.rs:1497): host-quantized bins,
 * FEATURE-major u32 `bins_feature_major[f * n + i]`.  `*out` is NULL when
 * the call declines. */
CBGPU_API int cbgpu_begin(const cbgpu_begin_args* args, const uint32_t* bins_feature_major,
                cbgpu_session** out);

/* Runtime::begin_device_training_raw (runtime.rs:1546): raw f32 columns
 * (`float_columns[f]` points at n values) and per-feature ascending f64
 * borders, quantized on the device with the reference's bin_of rule
 * (histogram.rs:159-165; NaN -> bin 0, or the top bin under the f32::MAX
 * nan_mode=Max sentinel). */
CBGPU_API int cbgpu_begin_raw(const cbgpu_begin_args* args, const float* const* float_columns,
                    const double* borders_flat, const int32_t* border_counts,
                    cbgpu_session** out);

/* Runtime::grow_tree_on_device (runtime.rs:1629) for the SymmetricTree arm.
 *  approx  [n] the caller's raw approximant, or NULL to use the session's
 *          resident approximant (initialised to args.bias, advanced by
 *          learning_rate * leaf value after every tree, as the reference
 *          session does, session.rs:2560-2760);
 *  target  [n] uploaded on the first call only;
 *  sample  [sample_len] per-object bootstrap multiplier (control ? w : 0);
 *          sample_len must be n when the session was opened with
 *          sample_from_host, else 0 (session.rs:2405-2428); NULL / 0 on a
 *          sample_from_host session takes the oldest cbgpu_stage_sample;
 * Outputs (DeviceGrownTree, runtime.rs:989-1059):
 *  split_feature / split_bin  [depth] feature and border index per level
 *          (level l is leaf bit l); the split passes iff bin > split_bin;
 *  n_splits                   splits written;
 *  leaf_values [2^depth]      raw leaf deltas, NOT scaled by learning_rate;
 *  leaf_of / leaf_of_bytes    optional per-object leaf ids (1 = u8, 2 = u16,
 *                             4 = u32; 0 / NULL = not requested). */
CBGPU_API int cbgpu_grow_tree(cbgpu_session* s, const double* approx, const double* target, int64_t n,
                    const double* sample, int64_t sample_len, int32_t* split_feature,
                    int32_t* split_bin, int32_t* n_splits, double* leaf_values, void* leaf_of,
                    int32_t leaf_of_bytes);

/* Upload a host bootstrap sample ahead of the grow call that uses it.  The
 * copy runs on a session-owned copy stream and this call returns at once; a
 * later cbgpu_grow_tree on this session with sample = NULL, sample_len = 0
 * takes the oldest staged sample (at most two wait at a time).  Calling
 * stage(t + 1) before grow(t) overlaps tree t + 1's upload with tree t's
 * device work.  The caller keeps `sample` unchanged until the grow call that
 * takes it returns; pinned (page-locked) memory is needed for the copy to
 * overlap.  Only for sessions opened with sample_from_host; a grow call that
 * passes a sample while staged ones wait is an error.  No counterpart in the
 * reference: Runtime::grow_tree_on_device (runtime.rs:1629) takes the sample
 * with the call, which this splits in two. */
CBGPU_API int cbgpu_stage_sample(cbgpu_session* s, const double* sample, int64_t sample_len);

/* Runtime::end_device_training (runtime.rs:1648): frees the session. */
CBGPU_API int cbgpu_end(cbgpu_session* s);

/* Runtime::compute_gradients (runtime.rs:1431) for RMSE / Logloss /
 * CrossEntropy at approx_dimension 1 (loss.rs:35-80), on the device. */
CBGPU_API int cbgpu_compute_gradients(int32_t loss, const double* approx, const double* target, int64_t n,
                            double* der1, double* der2);

/* Thread-local message for the last non-OK status (CbError analogue). */
CBGPU_API const char* cbgpu_last_error(void);

/* ---- session introspection (tests / drivers) ------------------------- */

/* Copy the session's resident approximant to the host (flushes the pending
 * learning_rate * leaf update first). */
CBGPU_API int cbgpu_session_approx(cbgpu_session* s, double* out, int64_t n);

/* Copy the device-quantized bins back, feature-major u8 [F][n]. */
CBGPU_API int cbgpu_session_bins(cbgpu_session* s, uint8_t* out_feature_major, int64_t n, int32_t n_features);

/* Copy the per-object score-channel bootstrap weights of the last tree
 * (control ? sample_weight : 0) to the host. */
CBGPU_API int cbgpu_session_last_sample(cbgpu_session* s, double* out, int64_t n);

/* Last tree: [0] device ms of the whole tree (always measured); with
 * profiling on, device ms of [1] histogram kernels, [2] derive + score,
 * [3] partition / route, [4] derivative + bootstrap, [5] collectives; always
 * [6] rows histogrammed over all levels and [7] kernels launched. */
CBGPU_API int cbgpu_session_timing(cbgpu_session* s, double* out8);

/* The same eight figures summed over every tree since the last reset (reset
 * != 0 zeroes the sums after reading).  Reading a tree's event times happens
 * during the next tree's device work, so a loop that only reads the sum at
 * its end adds no host time between trees.  No counterpart in the reference
 * (the reference reports stage times through its own profiler). */
CBGPU_API int cbgpu_session_timing_sum(cbgpu_session* s, double* out8, int32_t reset);

/* Record user event `slot` (0..3) on the session's stream, and read the
 * device milliseconds between two recorded slots (synchronizes on `b`). */
CBGPU_API int cbgpu_session_mark(cbgpu_session* s, int32_t slot);
CBGPU_API int cbgpu_session_elapsed_ms(cbgpu_session* s, int32_t a, int32_t b, double* out);

/* Enable (1) / disable (0) per-stage CUDA-event timing (off by default). */
CBGPU_API int cbgpu_session_set_profiling(cbgpu_session* s, int32_t enabled);

/* From the second tree on, a session replays each tree's device work as one
 * captured CUDA graph (on by default); 0 enqueues every kernel and collective
 * of every tree instead.  Results are identical either way.  No counterpart
 * in the reference. */
CBGPU_API int cbgpu_session_set_graphs(cbgpu_session* s, int32_t enabled);

/* Host TFastRng64 replica of the session's main stream (raw state + calls),
 * so a driver can check it stays in lockstep with cb-train's RNG. */
CBGPU_API int cbgpu_session_rng_state(cbgpu_session* s, uint64_t* out5);

/* ---- building blocks (each is a standalone device computation) ------- */

/* One level histogram over `n` rows: bins row-major u8 [n][n_features]
 * (each < n_bins), g/h [n] finite f64 score channels, leaf_of [n] (or NULL =
 * all leaf 0).  Output hist[leaf][feature][bin][2] f64 (channel 0 = sum g,
 * 1 = sum h), computed with exact int64 fixed-point accumulation
 * (crates/cb-compute/src/histogram.rs:239-294 semantics). */
CBGPU_API int cbgpu_histogram(const uint8_t* bins_row_major, int64_t n, int32_t n_features, int32_t n_bins,
                    const double* g, const double* h, const int32_t* leaf_of, int32_t n_leaves,
                    double* out_hist);

/* Bootstrap weights exactly as crates/cb-train/src/bootstrap.rs produces them
 * for global rows [row_offset, row_offset + n):
 *  Bayesian: rand_seed = the main-stream draw; out = sample weight.
 *  Bernoulli: rng_raw4 = main-stream raw state before the n_total draws;
 *             out = 1.0 / 0.0 control mask.
 *  MVS: der_obj [n] (|w * der1|), lambda, rand_seed; out = sample weight
 *       (row_offset must be a multiple of 8192). */
CBGPU_API int cbgpu_bootstrap_weights(int32_t type, int64_t n, int64_t row_offset, uint64_t rand_seed,
                            const uint64_t* rng_raw4, float sample_rate, float bagging_temperature,
                            const double* der_obj, double lambda, double* out);

/* ---- multi-rank decisions, run on the host ------------------------------
 * The document-sharded session (world > 1) makes three decisions every rank
 * must take identically; these entry points run the very code the session
 * and its kernels use, so a host-only harness (for example gloo ranks on
 * CPUs) can check them.  No counterpart in the reference, which trains on
 * one device per process (crates/cb-backend/src/gpu_runtime/mod.rs:2711).
 *
 * cbgpu_rank_feature_slice: the features [f0, f0 + fs) of the world * fs
 * padded range that `rank` derives and scores (features >= n_features have
 * no candidates).
 *
 * cbgpu_rank_select_split: the global split of one level from the ranks'
 * all-gathered slice records, `stride` u64 words each: the slice winner's
 * score (f64 bits), its key (feature << 8 | border; 0x7fffffff = no
 * candidate), then 2^level pairs of (false, true) child weight sums (u64
 * fixed point).  The winner is the highest score, the lowest key on equal
 * scores -- the CPU's first-wins scan over (feature, border)
 * (crates/cb-train/src/tree.rs:355-366).  Outputs its feature / border /
 * score and rank (-1, -1, -inf, -1 when no rank has a candidate), and, when
 * small_side is not NULL, the next level's build side per parent [2^level]
 * (1 = build the true child: it carries no more weight).
 *
 * cbgpu_rank_mvs_partial: one rank's link of the first-tree MVS lambda
 * (crates/cb-train/src/bootstrap.rs:358-376): continues the sequential f64
 * sum of |w * der1| over this rank's n rows from acc_in (the previous rank's
 * result; 0 on rank 0).  loss: CBGPU_LOSS_RMSE, else the Logloss der;
 * approx NULL = bias for every row; weight NULL = unit weights.  Chained in
 * rank order, the last rank's sum is bit-identical to one rank's over all
 * rows; lambda = (sum / n_total)^2. */
CBGPU_API int cbgpu_rank_feature_slice(int32_t n_features, int32_t world, int32_t rank, int32_t* f0, int32_t* fs);
CBGPU_API int cbgpu_rank_select_split(int32_t level, int32_t world, int32_t stride, const uint64_t* all_best,
                                      int32_t* feature, int32_t* bin, double* score, int32_t* winner_rank,
                                      uint8_t* small_side);
CBGPU_API int cbgpu_rank_mvs_partial(int32_t loss, int64_t n, const double* approx, double bias,
                                     const double* target, const double* weight, double acc_in, double* acc_out);

/* Allocation-free level histogram.  No counterpart in the reference: it exists
 * for callers that cannot call cudaMalloc when they need a histogram
 * (processes whose device memory belongs to their own pool allocator, hosts
 * that forbid allocation on their hot path, latency-bound loops that cannot
 * afford an allocator call or its failure).  Inputs and output are DEVICE
 * pointers owned by the caller: bins row-major u8 [n][row_stride] (16-byte
 * aligned; row_stride a multiple of 32 and at least n_features rounded up to
 * 32), g/h f64 [n]; out f64 [n_features][n_bins][2] (channel 0 = sum g,
 * 1 = sum h), the one-leaf histogram cbgpu_histogram computes.
 * Preconditions checked on the device: every bin of the first n_features
 * columns is < n_bins, and every g and h is finite; otherwise no histogram
 * is built, the output is all NaN and the call returns CBGPU_ERR_DEVICE.
 * Work is enqueued on `stream` (a cudaStream_t; NULL = the legacy default
 * stream) and the call waits for it (it reads the checks' verdict back).
 * Intermediate state lives in one fixed device array of about 5.1 MiB that
 * every GPU loading the library holds until exit; limits per call:
 * n <= 262144 rows, n_features * n_bins <= 65536, n_bins <= 256; larger sizes
 * return CBGPU_ERR_INVALID.  The first call on a device looks up the array's
 * device address (once per device), so make that first call before any
 * stream capture.  All calls share the array, which keeps the previous call's
 * contents (each call clears what must start at zero): calls that overlap on
 * the GPU, on different streams or from different threads, race. */
CBGPU_API int cbgpu_histogram_noalloc(const uint8_t* d_bins_row_major, int64_t n, int32_t n_features,
                                      int32_t row_stride, int32_t n_bins, const double* d_g,
                                      const double* d_h, double* d_out_hist, void* stream);

/* ---- multi-output (MultiClass) arm ------------------------------------- */

/* The seam's FamilyTreeArgs::MultiOutput family (runtime.rs:935-948) for
 * MultiClass (softmax, Newton leaves): one oblivious tree per iteration, a
 * K-vector per leaf.  The reference's device session declines every
 * multi-output fit (crates/cb-backend/src/gpu_runtime/session.rs:1401-1467)
 * and cb-train grows these trees on the CPU
 * (crates/cb-train/src/boosting.rs:7400-8930 at approx_dimension K); this arm
 * reproduces that CPU branch on one GPU.
 *
 * The diagonal losses MultiClassOneVsAll, MultiLogloss and MultiCrossEntropy
 * (loss.rs:501-560) share the arm: per dimension p = sigmoid(a_d),
 * der1 = t_d - p, der2 = -p (1 - p), and each dimension's Newton leaf is
 * solved on its own (boosting.rs:8323-8420) instead of the coupled softmax
 * solve.  RMSEWithUncertainty (loss.rs:680-720; approx_dim 2, bootstrap No)
 * takes the same per-dimension leaf with der1 = w [diff, diff^2 prec - 1],
 * der2 = w [-1, -2 diff^2 prec], diff = t - a0, prec = exp(-2 a1).
 *
 * cbgpu_multi_begin_raw: begin_device_training_raw's arguments (loss one of
 * CBGPU_LOSS_MULTICLASS, _MULTICLASS_ONE_VS_ALL, _MULTILOGLOSS,
 * _MULTICROSSENTROPY; world_size 1) plus approx_dim = K (2..16; 1..16 for the
 * two label losses).  Declines (CBGPU_DECLINED) outside SymmetricTree / Plain /
 * one fold / Cosine-L2-Solar-LOO-Sat / bootstrap No-Bayesian-Bernoulli /
 * depth <= 10 / <= 255 borders.  The approximant starts at 0 (no
 * boost_from_average on this family). */
typedef struct cbgpu_multi_session cbgpu_multi_session;
CBGPU_API int cbgpu_multi_begin_raw(const cbgpu_begin_args* args, int32_t approx_dim,
                                    const float* const* float_columns, const double* borders_flat,
                                    const int32_t* border_counts, cbgpu_multi_session** out);

/* cbgpu_multi_begin_raw plus one-hot categorical features (the reference's
 * CPU grower: equality candidates on each learn-set bin after every float
 * candidate, TRUE = the bin, crates/cb-compute/src/histogram.rs:1160-1290,
 * crates/cb-train/src/tree.rs:1290-1380; the reference's device session
 * declines them).  cat_columns[c] holds the n perfect-hash bins (first-seen
 * order, <= 255) of categorical feature c; it becomes split feature
 * n_features + c, whose split passes iff bin == split_bin.  Declines with any
 * bootstrap, as upstream does. */
CBGPU_API int cbgpu_multi_begin_cat_raw(const cbgpu_begin_args* args, int32_t approx_dim,
                                        const float* const* float_columns, const double* borders_flat,
                                        const int32_t* border_counts, int32_t n_cat,
                                        const uint32_t* const* cat_columns, cbgpu_multi_session** out);

/* grow_tree_on_device with FamilyTreeArgs::MultiOutput (runtime.rs:1629):
 *  approx_k  [K * n] DIM-major approximant (approx_k[d * n + i]) or NULL for
 *            the resident approximant (advanced by learning_rate * leaf);
 *  target    read on the first call: [n] class index per object as a double
 *            (0..K-1) for MultiClass and MultiClassOneVsAll; for MultiLogloss
 *            ({0, 1}) and MultiCrossEntropy ([0, 1]) the [K * n] DIM-major
 *            label matrix target[d * n + i], the reference's multilabel
 *            layout; for RMSEWithUncertainty the [n] targets, and the
 *            approximant then starts at [f32 mean, 0.5 ln f32 variance]
 *            (boosting.rs:1895-1914);
 *  sample    the host bootstrap multiplier, as for cbgpu_grow_tree;
 *  leaf_values [2^depth * K] LEAF-major raw deltas (DeviceGrownTree's
 *            leaf_count x approx_dim block, runtime.rs:1008-1024), not scaled
 *            by learning_rate; the rest as cbgpu_grow_tree. */
CBGPU_API int cbgpu_multi_grow_tree(cbgpu_multi_session* s, const double* approx_k, const double* target,
                                    int64_t n, const double* sample, int64_t sample_len, int32_t* split_feature,
                                    int32_t* split_bin, int32_t* n_splits, double* leaf_values, void* leaf_of,
                                    int32_t leaf_of_bytes);

/* Loss parameters of the grouped families; NULL takes the defaults. */
typedef struct {
    double l2_leaf_reg;     /* the unscaled l2 of PairLogitPairwise's scorer and leaves
                               (boosting.rs:8270-8300); < 0: use args->scaled_l2 */
    double softmax_lambda;  /* QuerySoftMax lambda (runtime.rs:541, default 0.01) */
    double softmax_beta;    /* QuerySoftMax beta (runtime.rs:545, default 1.0) */
    double lambdamart_sigma;   /* LambdaMart sigma (runtime.rs:374-388, default 1.0) */
    int64_t lambdamart_top;    /* LambdaMart top; -1 = the whole group (default) */
    int32_t lambdamart_norm;   /* LambdaMart norm (default 1) */
    int32_t lambdamart_metric; /* 0 = NDCG (default), 1 = DCG, 2 = MRR, 3 = ERR, 4 = MAP; the last
                                  three give zero ders, as the reference's no-op arms
                                  (ranking_der.rs:574-581) */
    int32_t yeti_permutations; /* YetiRank permutations (default 10) */
    double yeti_decay;         /* YetiRank decay (default 0.85) */
    int32_t srank_metric;      /* StochasticRank metric: 0 = NDCG, 1 = DCG; others decline */
    int32_t srank_num_estimations; /* StochasticRank num_estimations (default 1) */
    double srank_sigma;        /* StochasticRank sigma (default 1.0) */
    double srank_mu;           /* StochasticRank mu (default 0.0) */
    const double* pair_weight; /* [n_pairs] per-pair weight (Competitor::weight, query_info.rs:205-250)
                                  for PairLogit; NULL = 1.0 each.  PairLogitPairwise declines
                                  weights other than 1 */
} cbgpu_rank_params;

/* The seam's grouped families (FamilyTreeArgs::Ranking / ::Pairwise,
 * runtime.rs:918-934) for QueryRMSE, QuerySoftMax, LambdaMart, YetiRank,
 * StochasticRank, PairLogit and PairLogitPairwise: the reference's device
 * session declines them
 * (crates/cb-backend/src/gpu_runtime/session.rs:1401-1444); this mode
 * reproduces cb-train's grouped CPU branch (grouped ders,
 * crates/cb-compute/src/ranking_der.rs:139-440; PairLogit's pairwise
 * histogram weights, boosting.rs:1761-1780; Newton leaves, Gradient leaves for
 * QuerySoftMax, boosting.rs:8330-8400) on one GPU.
 * YetiRank resamples its pairs on the device every tree from the per-tree
 * query seeds of YetiRankTreeSeeder (crates/cb-train/src/yetirank.rs), keeps
 * the learning-fold approximant beside the model's, and takes Newton leaves
 * (boosting.rs:7347-7420, 8070-8200, 8787-8880); explicit pairs are not used.
 * YetiRankPairwise takes the same resamples through the pairwise scorer and
 * Cholesky pairwise leaves, for the stored leaves and the learning fold.
 * StochasticRank draws each group's Monte-Carlo noise on the device from the
 * same seeder's recalc bases (boosting.rs:5065-5100) and takes Gradient
 * leaves.
 * PairLogitPairwise scores splits with the pairwise scorer
 * (crates/cb-compute/src/pairwise_scoring.rs:101-580) and takes Cholesky
 * pairwise leaves (crates/cb-train/src/pairwise_leaves.rs:51-242), both with
 * the raw l2_leaf_reg and the PairwiseNonDiagReg prior 0.1; depth 1..8.
 *  group_offsets [n_groups + 1] contiguous groups over object order, 0..n;
 *  pair_winner / pair_loser [n_pairs] global object ids of the pairs
 *                (both in one group; weights in params->pair_weight, else 1),
 *                ignored for QueryRMSE;
 *  params        cbgpu_rank_params or NULL (defaults).
 * The session is grown with cbgpu_multi_grow_tree at approx_dim 1 (target =
 * the relevance per object); its leaf_values are the raw deltas, and the
 * resident approximant advances by the pair-loss-centred deltas x lr, as
 * normalize_leaf_values does (boosting.rs:2844-2880).  Declines bootstrap,
 * random_strength and more than one GPU. */
CBGPU_API int cbgpu_rank_begin_raw(const cbgpu_begin_args* args, const int64_t* group_offsets, int32_t n_groups,
                                   const int64_t* pair_winner, const int64_t* pair_loser, int64_t n_pairs,
                                   const cbgpu_rank_params* params, const float* const* float_columns, const double* borders_flat,
                                   const int32_t* border_counts, cbgpu_multi_session** out);

/* The resident approximant, DIM-major [K * n] (flushes the pending update).
 * No counterpart in the reference. */
CBGPU_API int cbgpu_multi_approx(cbgpu_multi_session* s, double* out_dim_major, int64_t n);

/* end_device_training for a multi-output session. */
CBGPU_API int cbgpu_multi_end(cbgpu_multi_session* s);

/* ---- fit preparation -------------------------------------------------- */

/* EBorderSelectionType (crates/cb-data/src/border_types.rs:52-70), in the
 * reference's listing order. */
typedef enum {
    CBGPU_BORDER_MEDIAN = 0, CBGPU_BORDER_GREEDY_LOGSUM = 1, CBGPU_BORDER_UNIFORM_AND_QUANTILES = 2,
    CBGPU_BORDER_MIN_ENTROPY = 3, CBGPU_BORDER_MAX_LOGSUM = 4, CBGPU_BORDER_UNIFORM = 5,
    CBGPU_BORDER_GREEDY_MIN_ENTROPY = 6
} cbgpu_border_type;

/* NanMode (crates/cb-data/src/nan_mode.rs). */
typedef enum { CBGPU_NAN_MIN = 0, CBGPU_NAN_MAX = 1, CBGPU_NAN_FORBIDDEN = 2 } cbgpu_nan_mode;

/* Quantization borders of every float column, selected on the device.
 * Replaces the builder's per-column border derivation
 * (crates/catboost-rs/src/builder.rs:1677-1720 -> cb_data::select_borders_f32,
 * crates/cb-data/src/border_types.rs:134-236 and borders.rs:272-345): columns
 * longer than 200,000 rows select from the reference's fixed-seed 200,000-row
 * sample (borders.rs:504-520); NaNs are dropped; a column holding a NaN spends
 * one of its border_count borders on the nan_mode sentinel (f32::MIN first
 * under Min, f32::MAX last under Max); Forbidden with a NaN column returns
 * CBGPU_ERR_INVALID with the builder's message.
 *  float_columns[f]  host pointer to n f32 values of feature f;
 *  border_count      1..1024 borders per feature, sentinel included;
 *  border_type       GreedyLogSum (the default), GreedyMinEntropy, Median,
 *                    Uniform or UniformAndQuantiles; the exact binarizers
 *                    (MinEntropy, MaxLogSum) return CBGPU_DECLINED;
 *  borders_out       [n_features][border_count] f64: feature f's ascending
 *                    borders in its first counts_out[f] slots. */
CBGPU_API int cbgpu_select_borders(const float* const* float_columns, int64_t n, int32_t n_features,
                                   int32_t border_count, int32_t border_type, int32_t nan_mode,
                                   int32_t device, double* borders_out, int32_t* counts_out);

/* ---- apply ------------------------------------------------------------- */

/* Raw predictions (RawFormulaVal) of a float-only oblivious ensemble on the
 * device: replaces cb_backend::gpu_runtime::launch_apply_oblivious_f64, the
 * launcher behind Model::predict_raw_on_device
 * (crates/catboost-rs/src/model.rs:360-384), over the same CSR lowering
 * (cb_model::flatten_oblivious_f64, crates/cb-model/src/gpu_apply.rs:83-193).
 * Results equal the CPU apply (crates/cb-model/src/apply.rs:150-173, 374-410)
 * bit for bit.
 *  features_fm        host, feature-major f32 [n_features][n];
 *  split_features/_borders  [tree_split_offsets[n_trees]] per split; split s of
 *                     tree t is leaf bit s - tree_split_offsets[t] and passes
 *                     iff (double)x > border; a feature >= n_features never
 *                     passes; at most 16 splits per tree;
 *  leaf_values        [tree_leaf_offsets[n_trees]] learning-rate scaled;
 *  nan_above          [n_features] 1 where NaN passes every split (the
 *                     nan_mode=Max rule: the feature's last border is
 *                     f32::MAX), or NULL; otherwise NaN never passes;
 *  out                [n] host, bias + the per-tree values in tree order. */
CBGPU_API int cbgpu_apply_oblivious(const float* features_fm, int64_t n, int32_t n_features,
                                    const uint32_t* split_features, const double* split_borders,
                                    const uint32_t* tree_split_offsets, int32_t n_trees,
                                    const double* leaf_values, const uint32_t* tree_leaf_offsets, double bias,
                                    const uint8_t* nan_above, int32_t device, double* out);

/* NCCL unique id (128 bytes) for world_size > 1 sessions. */
CBGPU_API int cbgpu_nccl_unique_id(uint8_t* out128);

/* Library version string. */
CBGPU_API const char* cbgpu_version(void);

#ifdef __cplusplus
}
#endif
#endif /* CBGPU_H */
