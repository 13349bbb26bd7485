/*
 * cb_oracle.h -- CPU restatement of catboost_rs's oblivious-tree training path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * implementation in catboost_rs_b200/csrc and the CPU baseline timed by
 * bench.py.  Nothing in the product path links, loads or calls it.
 *
 * Every routine restates the reference's CPU algorithm in plain C with the
 * same floating-point operation order (strict left-to-right f64 sums, no FMA
 * contraction: build with -ffp-contract=off).  Citations are file:line inside
 * the reference project (BectorVoom/catboost_rs).
 *
 * Parity status: pinned.  tests/test_oracle_golden.py checks this library
 * against the reference's committed golden vectors (TFastRng64 / std_normal /
 * FastLogf vectors) and against the upstream CatBoost 1.2.10 end-to-end
 * fixtures the reference's own oracle tests use (tests/golden/).
 */
#ifndef CB_ORACLE_H
#define CB_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- TFastRng64 (crates/cb-core/src/rng.rs) ---------------------------- */
typedef struct {
    uint64_t x1, c1, x2, c2; /* two PCG-XSH-RR LCG streams: state, addend */
    uint64_t calls;          /* primitive gen_rand draws consumed */
} orc_rng;

void     orc_rng_new(orc_rng* r, uint64_t seed1, uint32_t seq1, uint64_t seed2, uint32_t seq2);
void     orc_rng_from_seed(orc_rng* r, uint64_t seed);
uint64_t orc_rng_gen(orc_rng* r);
double   orc_rng_real1(orc_rng* r);
void     orc_rng_advance(orc_rng* r, uint64_t delta);
uint64_t orc_rng_uniform(orc_rng* r, uint64_t bound);
double   orc_std_normal(orc_rng* r);

/* ---- FastLogf (crates/cb-train/src/fast_approx.rs) --------------------- */
float orc_fast_log2f(float v);
float orc_fast_logf(float v);

/* ---- ordered reduction (crates/cb-core/src/reduction.rs) --------------- */
double orc_sum_f64(const double* v, int64_t n);

/* ---- quantization (crates/cb-compute/src/histogram.rs:159-165) --------- */
/* cols: feature-major f32 [F][n]; borders_flat: per-feature ascending f64
 * borders concatenated, border_counts[f] entries each; out: bins [F][n]. */
void orc_quantize(const float* cols, int64_t n, int32_t F, const double* borders_flat,
                  const int32_t* border_counts, uint8_t* out_bins_fm);

/* ---- border selection (crates/cb-data/src/borders.rs, border_types.rs) - */
/* EBorderSelectionType in the reference's listing order (border_types.rs:112-124). */
enum {
    ORC_BORDER_MEDIAN = 0, ORC_BORDER_GREEDY_LOGSUM = 1, ORC_BORDER_UNIFORM_AND_QUANTILES = 2,
    ORC_BORDER_MIN_ENTROPY = 3, ORC_BORDER_MAX_LOGSUM = 4, ORC_BORDER_UNIFORM = 5,
    ORC_BORDER_GREEDY_MIN_ENTROPY = 6
};
enum { ORC_PENALTY_MAXSUMLOG = 0, ORC_PENALTY_MIN_ENTROPY = 1 };
enum { ORC_NAN_MIN = 0, ORC_NAN_MAX = 1, ORC_NAN_FORBIDDEN = 2 };

/* Borders of one f32 column as catboost-rs's builder derives them
 * (builder.rs:1677-1720 -> select_borders_f32, border_types.rs:134-236):
 * columns over 200,000 rows use the fixed-seed 200k object sample, NaNs are
 * dropped, a NaN-bearing column spends one border on the nan_mode sentinel
 * (f32::MIN prepended under Min, f32::MAX appended under Max).  Returns the
 * number of borders written (ascending f64), or < 0 on error.  MaxLogSum and
 * MinEntropy (the exact DP binarizers) return -2. */
int64_t orc_select_borders(const float* col, int64_t n, int32_t border_count, int32_t border_type,
                           int32_t nan_mode, double* out, int64_t out_cap);

/* sample_indices_for_build_borders (borders.rs:504-520): the sorted object
 * sample (malloc'd; the caller frees it). */
int64_t* orc_border_sample_indices(int64_t n, int64_t sample_size, int64_t* out_len);

/* ---- apply (crates/cb-model/src/apply.rs:150-173, 264-271, 374-410) ---- */
/* Raw prediction of a float-only oblivious ensemble in the flat CSR layout of
 * cb_model::flatten_oblivious_f64 (crates/cb-model/src/gpu_apply.rs:83-110):
 * x_fm feature-major f32 [F][n]; split s of tree t in [tree_split_offsets[t],
 * tree_split_offsets[t+1]) is leaf bit s - tree_split_offsets[t] and passes iff
 * (double)x > border (NaN: nan_above[f], the nan_mode=Max rule; a feature
 * index >= F never passes); leaf_values already learning-rate scaled; the
 * prediction is bias + the ordered sum over trees. */
void orc_apply_oblivious(const float* x_fm, int64_t n, int32_t F, const uint32_t* split_features,
                         const double* split_borders, const uint32_t* tree_split_offsets, int32_t n_trees,
                         const double* leaf_values, const uint32_t* tree_leaf_offsets, double bias,
                         const uint8_t* nan_above, double* out);

/* ---- derivatives (crates/cb-compute/src/loss.rs:35-80) ----------------- */
enum { ORC_LOSS_RMSE = 0, ORC_LOSS_LOGLOSS = 1, ORC_LOSS_CROSSENTROPY = 2, ORC_LOSS_MAE = 3, ORC_LOSS_QUANTILE = 4 };

/* exact_leaf_delta (crates/cb-compute/src/leaf.rs:445-520): the weighted
 * alpha-quantile of one leaf's f32 residuals with the delta adjustment. */
double orc_exact_leaf_delta(const float* residuals, const double* weights, int64_t n, double alpha, double delta);
void orc_compute_gradients(int32_t loss, const double* approx, const double* target, int64_t n,
                           double* der1, double* der2);

/* ---- bootstrap (crates/cb-train/src/bootstrap.rs) ---------------------- */
enum { ORC_BOOT_NO = 0, ORC_BOOT_BAYESIAN = 1, ORC_BOOT_BERNOULLI = 2, ORC_BOOT_MVS = 3 };
int orc_bootstrap(int32_t type, const double* der_obj, int64_t n, double subsample,
                  float bagging_temperature, int32_t has_prev_leaf_mean, double prev_leaf_mean,
                  orc_rng* rng, double* out_sample_weights, uint8_t* out_control);

/* ---- one histogram (crates/cb-compute/src/histogram.rs:239-294) -------- */
/* Sequential object-order f64 scatter: hist[leaf][feature][bin][2] with channel 0
 * = sum g, channel 1 = sum h.  Objects with leaf >= n_leaves are skipped. */
void orc_build_histogram(const uint8_t* bins_fm, int64_t n, int32_t F, int32_t n_bins,
                         const double* g, const double* h, const int32_t* leaf_of,
                         int32_t n_leaves, double* out_hist);

/* ---- the boosting loop (crates/cb-train/src/boosting.rs CPU branch) ---- */
enum { ORC_SCORE_COSINE = 0, ORC_SCORE_L2 = 1, ORC_SCORE_SOLAR_L2 = 2, ORC_SCORE_LOO_L2 = 5, ORC_SCORE_SAT_L2 = 6 };

/* The per-leaf terms of SolarL2 / LOOL2 / SatL2 (score.rs:266-330): the
 * score is their sum in dimension-then-leaf order, without l2. */
double orc_score_term(int32_t score_fn, double sum, double weight);

typedef struct {
    int64_t n;
    int32_t n_features;
    const uint8_t* bins_fm;        /* [F][n] bin indices (bin_of) */
    const int32_t* border_counts;  /* [F] number of borders per feature */
    const double* target;          /* [n] */
    const double* weights;         /* [n] or NULL (unit weights) */
    int32_t loss;
    int32_t depth;
    int32_t iterations;
    double learning_rate;
    double l2_leaf_reg;
    int32_t score_function;
    int32_t bootstrap_type;
    double subsample;
    float bagging_temperature;
    double random_strength;
    uint64_t random_seed;
    int32_t boost_from_average;
    int32_t n_threads;             /* 0 = OpenMP default */
    /* one-hot categorical features (plain search only): perfect-hash bins
     * (first-seen order) [n_cat][n]; split candidates are bin == value */
    int32_t n_cat;
    const uint8_t* cat_bins_fm;
    /* MAE / Quantile: der1 = quantile_der1 (loss.rs:166-175); exact_leaf 1 takes
     * the Exact leaf method (boosting.rs:2561-2606) instead of Gradient */
    int32_t exact_leaf;
    double quantile_alpha;
    double quantile_delta;
} orc_train_args;

/* CalcCatFeatureHash (crates/cb-data/src/cat_hash.rs): CityHash64 (v1.0) of the
 * category's string form, low 32 bits. */
uint32_t orc_cat_hash(const char* s, size_t len);
uint64_t orc_city_hash64(const char* s, size_t len);

typedef struct {
    int32_t* split_feature;  /* [iterations * depth] (-1 past an early stop); >= n_features: one-hot
                                cat feature split_feature - n_features */
    int32_t* split_bin;      /* [iterations * depth] border index: passes iff bin > split_bin;
                                one-hot: passes iff cat bin == split_bin */
    int32_t* tree_depth;     /* [iterations] splits actually taken */
    double* leaf_values;     /* [iterations * 2^depth] learning-rate scaled */
    double* staged;          /* [iterations * n] or NULL */
    double* final_approx;    /* [n] */
    double* bias;            /* [1] starting approx */
    uint64_t* rng_calls;     /* [iterations] main-RNG call count after each tree, or NULL */
    double* level_top2;      /* [iterations * depth * 2] best and runner-up raw candidate score per
                                level (-inf past an early stop), or NULL */
} orc_train_out;

int orc_train(const orc_train_args* a, orc_train_out* o);

/* ---- MultiClass (softmax) loop (boosting.rs multi-output CPU branch) --- */
typedef struct {
    int64_t n;
    int32_t n_features;
    const uint8_t* bins_fm;        /* [F][n] */
    const int32_t* border_counts;  /* [F] */
    const int32_t* target_class;   /* [n] class index in 0..n_classes-1 */
    const double* weights;         /* [n] or NULL */
    int32_t n_classes;             /* approx_dimension K */
    int32_t depth;
    int32_t iterations;
    double learning_rate;
    double l2_leaf_reg;
    int32_t score_function;
    int32_t bootstrap_type;
    double subsample;
    float bagging_temperature;
    uint64_t random_seed;
    int32_t n_threads;
    int32_t n_cat;                 /* one-hot cat features (plain search only) */
    const uint8_t* cat_bins_fm;    /* [n_cat][n] first-seen perfect-hash bins */
    int32_t loss_kind;             /* 0: MultiClass softmax; 1: diagonal logistic
                                      (MultiClassOneVsAll / MultiLogloss / MultiCrossEntropy);
                                      2: RMSEWithUncertainty (K = 2, [mean, log-scale]) */
    const double* target_matrix;   /* [K][n] per-dimension targets for loss_kind 1; [n] for 2 */
} orc_multi_args;

typedef struct {
    int32_t* split_feature;  /* [iterations * depth]; >= n_features: one-hot cat feature - n_features */
    int32_t* split_bin;      /* [iterations * depth]; one-hot: passes iff cat bin == split_bin */
    int32_t* tree_depth;     /* [iterations] */
    double* leaf_values;     /* [iterations * 2^depth * K] LEAF-major, learning-rate scaled */
    double* staged;          /* [iterations * n * K] object-major, or NULL */
    double* final_approx;    /* [n * K] object-major, or NULL */
} orc_multi_out;

int orc_train_multiclass(const orc_multi_args* a, orc_multi_out* o);

/* cholesky_solve (crates/cb-compute/src/leaf.rs:360-420): A (k x k,
 * row-major, symmetric) x = b with scratch L (k x k) and y (k); returns 0 on
 * a non-positive pivot. */
int orc_cholesky_solve(const double* A, const double* b, int32_t k, double* L, double* y, double* x);

/* solve_symmetric_newton (crates/cb-compute/src/leaf.rs:281-340). */
void orc_solve_symmetric_newton(const double* sum_der, const double* sum_der2_packed, int32_t k,
                                double scaled_l2, double* out);

/* ---- grouped (ranking) losses, pointwise histograms -------------------- */
enum { ORC_RANK_QUERYRMSE = 0, ORC_RANK_PAIRLOGIT = 1, ORC_RANK_PAIRLOGIT_PAIRWISE = 2, ORC_RANK_QUERYSOFTMAX = 3,
       ORC_RANK_LAMBDAMART = 4, ORC_RANK_YETIRANK = 5, ORC_RANK_STOCHASTICRANK = 6,
       ORC_RANK_YETIRANK_PAIRWISE = 7 };

/* The greedy oblivious search of the scalar loop, exported for the grouped
 * loop: returns the splits taken; leaf_of gets the final leaf ids. */
int orc_search_tree(int64_t n, int32_t F, int32_t n_bins, int32_t depth, int32_t score_fn, const uint8_t* bins,
                    const int32_t* border_counts, const double* g, const double* h, double l2, int32_t draws,
                    orc_rng* rng, int32_t* feat, int32_t* sbin, int32_t* leaf_of, int32_t* err);

typedef struct {
    int64_t n;
    int32_t n_features;
    const uint8_t* bins_fm;        /* [F][n] */
    const int32_t* border_counts;  /* [F] */
    const double* target;          /* [n] */
    const double* weights;         /* [n] or NULL */
    int32_t loss;                  /* ORC_RANK_* */
    int32_t n_groups;
    const int64_t* group_offsets;  /* [n_groups + 1] contiguous groups over object order */
    int64_t n_pairs;
    const int64_t* pair_winner;    /* [n_pairs] global object ids (PairLogit) */
    const int64_t* pair_loser;
    int32_t depth;
    int32_t iterations;
    double learning_rate;
    double l2_leaf_reg;
    int32_t score_function;
    uint64_t random_seed;
    double softmax_lambda;         /* QuerySoftMax lambda (default 0.01) */
    double softmax_beta;           /* QuerySoftMax beta (default 1.0) */
    double lambdamart_sigma;       /* LambdaMart sigma (default 1.0) */
    int64_t lambdamart_top;        /* LambdaMart top (-1: the whole group) */
    int32_t lambdamart_norm;       /* LambdaMart norm (default 1) */
    int32_t yeti_permutations;     /* YetiRank permutations (default 10) */
    double yeti_decay;             /* YetiRank decay (default 0.85) */
    int32_t srank_ndcg;            /* StochasticRank metric: 1 NDCG, 0 DCG */
    double srank_sigma;            /* StochasticRank sigma (default 1.0) */
    double srank_mu;               /* StochasticRank mu (default 0.0) */
    int32_t srank_num_estimations; /* StochasticRank num_estimations (default 1) */
    int32_t lambdamart_no_op;      /* LambdaMart metric MRR / ERR / MAP: zero ders (ranking_der.rs:574-581) */
    const double* pair_weight;     /* [n_pairs] Competitor::weight per pair (PairLogit); NULL = 1 */
} orc_rank_args;

/* YetiRank's sampler for one group (sample_pairs, crates/cb-train/src/
 * yetirank.rs:75-171): out[w * g + l] = the sampled pair weight winner w over
 * loser l (0: no pair). */
void orc_yeti_sample_pairs(const double* raw_approx, const double* relevs, int64_t g, double query_weight,
                           int32_t permutations, double decay, uint64_t query_seed, double* out);
/* derive_query_seeds (yetirank.rs:173-184): the single-block query seeds. */
void orc_yeti_query_seeds(uint64_t random_seed, int32_t n_groups, uint64_t* out);
/* YetiRankTreeSeeder (yetirank.rs:262-430): for each of `trees` trees the
 * recalc seeds (deriv, learning fold, leaf values) -> out[3 * tree + k]. */
void orc_yeti_recalc_seeds(uint64_t random_seed, int32_t n_groups, int32_t n_features, int32_t depth, int32_t trees,
                           uint64_t* out);

typedef struct {
    int32_t* split_feature;  /* [iterations * depth] */
    int32_t* split_bin;
    double* leaf_values;     /* [iterations * 2^depth] centred (PairLogit) and learning-rate scaled */
    double* raw_leaf_values; /* [iterations * 2^depth] the Newton deltas before normalisation, or NULL */
    double* staged;          /* [iterations * n] or NULL */
} orc_rank_out;

int orc_train_ranking(const orc_rank_args* a, orc_rank_out* o);

#ifdef __cplusplus
}
#endif
#endif
