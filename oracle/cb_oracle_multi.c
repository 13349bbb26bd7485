/*
 * cb_oracle_multi.c -- CPU restatement of catboost_rs's MultiClass (softmax)
 * oblivious-tree loop: the multi-output CPU branch of crates/cb-train/src/
 * boosting.rs with approx_dimension = K.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for the device multi-output
 * arm.  The product path never calls it.  Build with -ffp-contract=off so
 * every f64 operation rounds as the reference's Rust code does.
 *
 * Per iteration (boosting.rs:7400-8930 with approx_dimension = K):
 *  1. softmax derivatives per object (crates/cb-compute/src/loss.rs:424-515):
 *     der1[d] = [d == y] - p[d], packed symmetric Hessian; weighted der1;
 *  2. PRE draws, der_obj = sqrt(sum_d wd1[d]^2) (boosting.rs:7604-7614),
 *     bootstrap, score channels control ? v * sw : 0 per dimension;
 *  3. greedy oblivious search over K + 1 histogram channels (K der, 1 weight)
 *     scored by multi_dim_split_score_into (score.rs:192-265) in
 *     dimension-then-leaf order, subtraction trick on the smaller side;
 *  4. softmax Newton leaves (boosting.rs:2610-2700, leaf.rs:250-420): ordered
 *     per-leaf sums of wd1 and w-weighted packed der2, then the trace-regularised
 *     Cholesky solve; x lr (f32-narrowed, boosting.rs:4958);
 *  5. dim-major approx update, POST draws, MVS lambda from the mean |leaf|.
 */
#include "cb_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline double mc_calc_average(double sum_delta, double count, double l2) {
    return count > 0.0 ? sum_delta / (count + l2) : 0.0;
}

/* calc_softmax + softmax_ders (loss.rs:424-515) for one object. */
static void softmax_ders(const double* a, int32_t K, int32_t y, double* p, double* d1, double* d2p) {
    double mx = -INFINITY;
    for (int32_t d = 0; d < K; ++d)
        if (a[d] > mx) mx = a[d];
    double s = 0.0;
    for (int32_t d = 0; d < K; ++d) {
        p[d] = exp(a[d] - mx);
        s += p[d];
    }
    for (int32_t d = 0; d < K; ++d) p[d] = p[d] / s;
    int32_t j = 0;
    for (int32_t dy = 0; dy < K; ++dy) {
        d2p[j++] = p[dy] * (p[dy] - 1.0);
        for (int32_t dx = dy + 1; dx < K; ++dx) d2p[j++] = p[dy] * p[dx];
    }
    for (int32_t d = 0; d < K; ++d) d1[d] = -p[d];
    if (y >= 0 && y < K) d1[y] += 1.0;
}

/* cholesky_solve (leaf.rs:360-420); returns 0 on a non-positive pivot. */
int orc_cholesky_solve(const double* A, const double* b, int32_t k, double* L, double* y, double* x) {
    for (int32_t i = 0; i < k * k; ++i) L[i] = 0.0;
    for (int32_t i = 0; i < k; ++i) {
        for (int32_t j = 0; j <= i; ++j) {
            double sum = A[i * k + j];
            for (int32_t p = 0; p < j; ++p) sum -= L[i * k + p] * L[j * k + p];
            if (i == j) {
                if (sum <= 0.0) return 0;
                L[i * k + j] = sqrt(sum);
            } else {
                double ljj = L[j * k + j];
                if (ljj == 0.0) return 0;
                L[i * k + j] = sum / ljj;
            }
        }
    }
    for (int32_t i = 0; i < k; ++i) {
        double sum = b[i];
        for (int32_t p = 0; p < i; ++p) sum -= L[i * k + p] * y[p];
        if (L[i * k + i] == 0.0) return 0;
        y[i] = sum / L[i * k + i];
    }
    for (int32_t i = k - 1; i >= 0; --i) {
        double sum = y[i];
        for (int32_t p = i + 1; p < k; ++p) sum -= L[p * k + i] * x[p];
        if (L[i * k + i] == 0.0) return 0;
        x[i] = sum / L[i * k + i];
    }
    return 1;
}

static inline float f32_max(float a, float b) {
    /* Rust f32::max: the non-NaN operand when one is NaN */
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    return a > b ? a : b;
}

/* solve_symmetric_newton (leaf.rs:281-340): out[k] = leaf delta per dimension. */
void orc_solve_symmetric_newton(const double* sum_der, const double* sum_der2_packed, int32_t k,
                                double scaled_l2, double* out) {
    double* H = (double*)calloc((size_t)k * k * 3 + (size_t)k * 3, sizeof(double));
    double* L = H + (size_t)k * k;
    double* y = L + (size_t)k * k;
    double* x = y + k;
    double* nd = x + k;
    int32_t idx = 0;
    for (int32_t i = 0; i < k; ++i)
        for (int32_t j = i; j < k; ++j) {
            double v = sum_der2_packed[idx++];
            H[i * k + j] = v;
            H[j * k + i] = v;
        }
    float max_trace = (float)scaled_l2;
    for (int32_t d = 0; d < k; ++d) max_trace = f32_max(max_trace, (float)(-H[d * k + d]));
    double adjusted = (double)f32_max((float)scaled_l2, max_trace * FLT_EPSILON);
    for (int32_t d = 0; d < k; ++d) H[d * k + d] -= adjusted;
    for (int32_t i = 0; i < k * k; ++i) H[i] = -H[i];
    for (int32_t d = 0; d < k; ++d) nd[d] = -sum_der[d];
    if (orc_cholesky_solve(H, nd, k, L, y, x)) {
        for (int32_t d = 0; d < k; ++d) out[d] = -x[d];
    } else {
        for (int32_t d = 0; d < k; ++d) out[d] = 0.0;
    }
    free(H);
}

/* multi_dim_split_score_into (score.rs:192-265): ld[d * nl + leaf], lw[leaf]. */
static double mc_split_score(int32_t score_fn, const double* ld, const double* lw, int32_t K, int32_t nl,
                             double l2) {
    if (score_fn > ORC_SCORE_L2) { /* SolarL2 / LOOL2 / SatL2 */
        double acc = 0.0;
        for (int32_t d = 0; d < K; ++d)
            for (int32_t q = 0; q < nl; ++q) acc += orc_score_term(score_fn, ld[d * nl + q], lw[q]);
        return acc;
    }
    double num = 0.0;
    for (int32_t d = 0; d < K; ++d)
        for (int32_t q = 0; q < nl; ++q) {
            double s = ld[d * nl + q];
            num += mc_calc_average(s, lw[q], l2) * s;
        }
    if (score_fn == ORC_SCORE_L2) return num;
    double den = 0.0;
    den += 1e-100;
    for (int32_t d = 0; d < K; ++d)
        for (int32_t q = 0; q < nl; ++q) {
            double avg = mc_calc_average(ld[d * nl + q], lw[q], l2);
            den += avg * avg * lw[q];
        }
    return num / sqrt(den);
}

/* scan_and_score_borders_into (histogram.rs:1007-1171) over C = K + 1
 * channels: hist[parent][bin][C], channel K = weight. */
static void mc_scan_and_score(const double* hist, int32_t n_parent, int32_t NB, int32_t K, int32_t n_borders,
                              int32_t score_fn, double l2, double* scores) {
    const int32_t C = K + 1, nl = 2 * n_parent;
    double* tot_w = (double*)calloc((size_t)n_parent * (2 + 2 * K) + (size_t)nl * (K + 1), sizeof(double));
    double* acc_w = tot_w + n_parent;
    double* tot_d = acc_w + n_parent;                 /* [parent][K] */
    double* acc_d = tot_d + (size_t)n_parent * K;     /* [parent][K] */
    double* ld = acc_d + (size_t)n_parent * K;        /* [K][nl] */
    double* lw = ld + (size_t)K * nl;                 /* [nl] */
    for (int32_t q = 0; q < n_parent; ++q) {
        const double* row = hist + (size_t)q * NB * C;
        double s = 0.0;
        for (int32_t b = 0; b < NB; ++b) s += row[(size_t)b * C + K];
        tot_w[q] = s;
        for (int32_t d = 0; d < K; ++d) {
            double sd = 0.0;
            for (int32_t b = 0; b < NB; ++b) sd += row[(size_t)b * C + d];
            tot_d[(size_t)q * K + d] = sd;
        }
    }
    for (int32_t b = 0; b < n_borders; ++b) {
        for (int32_t q = 0; q < n_parent; ++q) {
            const double* cell = hist + ((size_t)q * NB + b) * C;
            acc_w[q] += cell[K];
            double wf = acc_w[q];
            double wt = tot_w[q] - wf;
            lw[q] = wf;
            lw[q + n_parent] = wt;
            for (int32_t d = 0; d < K; ++d) {
                acc_d[(size_t)q * K + d] += cell[d];
                double df = acc_d[(size_t)q * K + d];
                ld[(size_t)d * nl + q] = df;
                ld[(size_t)d * nl + q + n_parent] = tot_d[(size_t)q * K + d] - df;
            }
        }
        scores[b] = mc_split_score(score_fn, ld, lw, K, nl, l2);
    }
    free(tot_w);
}

/* scan_and_score_one_hot_bins_into (histogram.rs:1160-1290) over C = K + 1
 * channels: per present bin v the TRUE children are the bin's cells, the
 * FALSE children the parent totals minus them. */
static void mc_scan_one_hot(const double* hist, int32_t n_parent, int32_t NB, int32_t K, const uint8_t* present,
                            int32_t score_fn, double l2, double* scores) {
    const int32_t C = K + 1, nl = 2 * n_parent;
    double* tot_w = (double*)calloc((size_t)n_parent * (1 + K) + (size_t)nl * (K + 1), sizeof(double));
    double* tot_d = tot_w + n_parent;              /* [parent][K] */
    double* ld = tot_d + (size_t)n_parent * K;     /* [K][nl] */
    double* lw = ld + (size_t)K * nl;              /* [nl] */
    for (int32_t q = 0; q < n_parent; ++q) {
        const double* row = hist + (size_t)q * NB * C;
        double s = 0.0;
        for (int32_t b = 0; b < NB; ++b) s += row[(size_t)b * C + K];
        tot_w[q] = s;
        for (int32_t d = 0; d < K; ++d) {
            double sd = 0.0;
            for (int32_t b = 0; b < NB; ++b) sd += row[(size_t)b * C + d];
            tot_d[(size_t)q * K + d] = sd;
        }
    }
    for (int32_t v = 0; v < NB; ++v) {
        if (!present[v]) {
            scores[v] = -INFINITY;
            continue;
        }
        for (int32_t q = 0; q < n_parent; ++q) {
            const double* cell = hist + ((size_t)q * NB + v) * C;
            lw[q] = tot_w[q] - cell[K];
            lw[q + n_parent] = cell[K];
            for (int32_t d = 0; d < K; ++d) {
                ld[(size_t)d * nl + q] = tot_d[(size_t)q * K + d] - cell[d];
                ld[(size_t)d * nl + q + n_parent] = cell[d];
            }
        }
        scores[v] = mc_split_score(score_fn, ld, lw, K, nl, l2);
    }
    free(tot_w);
}

typedef struct {
    int64_t n;
    int32_t F, NB, K, depth, score_fn;
    const uint8_t* bins;
    const int32_t* bc;
    const double* sg; /* [K][n] */
    const double* sh; /* [n] */
    double l2;
    int draws;
    orc_rng* rng;
    int32_t C;                /* one-hot cat features, candidates after the floats */
    const uint8_t* cat_bins;  /* [C][n] */
} mc_ctx;

/* the greedy oblivious search (tree.rs:704-1131, 1403-1606 at std_dev 0) over
 * K + 1 channels.  Returns the splits taken. */
static int mc_search(const mc_ctx* c, int32_t* feat, int32_t* sbin, int32_t* leaf_of, int* err) {
    const int64_t n = c->n;
    const int32_t F0 = c->F, F = c->F + c->C, NB = c->NB, K = c->K, C = K + 1;
    *err = 0;
    if (c->C > 0 && c->draws) { /* upstream rejects one-hot with draws active (tree.rs:1403-1420) */
        *err = 2;
        return 0;
    }
    uint8_t* present = (uint8_t*)calloc((size_t)(c->C > 0 ? c->C : 1) * (size_t)NB, 1);
    for (int32_t k = 0; k < c->C; ++k)
        for (int64_t o = 0; o < n; ++o)
            if (c->cat_bins[(int64_t)k * n + o] < NB) present[(size_t)k * NB + c->cat_bins[(int64_t)k * n + o]] = 1;
    double** cur = (double**)calloc((size_t)F, sizeof(double*));
    double* scores_all = (double*)malloc(sizeof(double) * (size_t)F * (size_t)NB);
    for (int64_t o = 0; o < n; ++o) leaf_of[o] = 0;
    int taken = 0;
    for (int32_t level = 0; level < c->depth; ++level) {
        int32_t n_leaves = 1 << level;
        if (c->draws)
            for (int32_t f = 0; f < F; ++f) (void)orc_rng_real1(c->rng); /* RSM draws */
        int32_t n_par = level == 0 ? 1 : (1 << (level - 1));
        int64_t n_true = 0;
        if (level > 0)
            for (int64_t o = 0; o < n; ++o) n_true += (leaf_of[o] & n_par) != 0;
        int build_true = (n_true <= n - n_true);
        double** next = (double**)calloc((size_t)F, sizeof(double*));
#pragma omp parallel for schedule(dynamic, 1)
        for (int32_t f = 0; f < F; ++f) {
            const int cat = f >= F0;
            int32_t nb = cat ? NB : c->bc[f];
            if (nb == 0) continue;
            const uint8_t* col = cat ? c->cat_bins + (int64_t)(f - F0) * n : c->bins + (int64_t)f * n;
            size_t pc = (size_t)NB * C;
            double* hist = (double*)calloc((size_t)n_leaves * pc, sizeof(double));
            if (level == 0) {
                for (int64_t o = 0; o < n; ++o) {
                    int32_t b = col[o];
                    if (b >= NB) continue;
                    double* cell = hist + (size_t)b * C;
                    for (int32_t d = 0; d < K; ++d) cell[d] += c->sg[(size_t)d * n + o];
                    cell[K] += c->sh[o];
                }
            } else {
                double* built = (double*)calloc((size_t)n_par * pc, sizeof(double));
                for (int64_t o = 0; o < n; ++o) {
                    int32_t l = leaf_of[o];
                    if (((l & n_par) != 0) != build_true) continue;
                    int32_t b = col[o];
                    if (b >= NB) continue;
                    double* cell = built + ((size_t)(l & (n_par - 1)) * NB + b) * C;
                    for (int32_t d = 0; d < K; ++d) cell[d] += c->sg[(size_t)d * n + o];
                    cell[K] += c->sh[o];
                }
                for (int32_t p = 0; p < n_par; ++p) {
                    double* fl = hist + (size_t)p * pc;
                    double* tr = hist + (size_t)(p + n_par) * pc;
                    const double* par = cur[f] + (size_t)p * pc;
                    const double* bt = built + (size_t)p * pc;
                    for (size_t k = 0; k < pc; ++k) {
                        if (build_true) {
                            tr[k] = bt[k];
                            fl[k] = par[k] - bt[k];
                        } else {
                            fl[k] = bt[k];
                            tr[k] = par[k] - bt[k];
                        }
                    }
                }
                free(built);
            }
            if (cat)
                mc_scan_one_hot(hist, n_leaves, NB, K, present + (size_t)(f - F0) * NB, c->score_fn, c->l2,
                                scores_all + (size_t)f * NB);
            else
                mc_scan_and_score(hist, n_leaves, NB, K, nb, c->score_fn, c->l2, scores_all + (size_t)f * NB);
            next[f] = hist;
        }
        for (int32_t f = 0; f < F; ++f) free(cur[f]);
        free(cur);
        cur = next;
        int32_t best_f = -1, best_b = -1;
        if (!c->draws) {
            double best = -INFINITY;
            for (int32_t f = 0; f < F; ++f) {
                const int32_t nc = f >= F0 ? NB : c->bc[f];
                for (int32_t b = 0; b < nc; ++b) {
                    if (f >= F0 && !present[(size_t)(f - F0) * NB + b]) continue;
                    double s = scores_all[(size_t)f * NB + b];
                    if (s > best) { best = s; best_f = f; best_b = b; }
                }
            }
            if (best_f < 0) { *err = 1; break; }
        } else {
            /* perturbed selection at std_dev 0 (tree.rs:1498-1606) */
            (void)orc_rng_gen(c->rng);
            double best_gain = -INFINITY;
            for (int32_t f = 0; f < F; ++f) {
                int32_t nb = c->bc[f];
                if (nb == 0) {
                    (void)orc_std_normal(c->rng);
                    continue;
                }
                double braw = -INFINITY;
                int32_t bb = 0;
                for (int32_t b = 0; b < nb; ++b) {
                    double raw = scores_all[(size_t)f * NB + b];
                    if (raw > braw) { braw = raw; bb = b; }
                }
                double inst = braw + orc_std_normal(c->rng) * 0.0;
                if (inst > best_gain) { best_gain = inst; best_f = f; best_b = bb; }
            }
            if (best_f < 0) break;
        }
        feat[level] = best_f;
        sbin[level] = best_b;
        taken = level + 1;
        if (best_f >= F0) { /* one-hot: passes on bin == value */
            const uint8_t* col = c->cat_bins + (int64_t)(best_f - F0) * n;
            for (int64_t o = 0; o < n; ++o)
                if ((int32_t)col[o] == best_b) leaf_of[o] += n_leaves;
        } else {
            const uint8_t* col = c->bins + (int64_t)best_f * n;
            for (int64_t o = 0; o < n; ++o)
                if ((int32_t)col[o] > best_b) leaf_of[o] += n_leaves;
        }
    }
    for (int32_t f = 0; f < F; ++f) free(cur[f]);
    free(cur);
    free(scores_all);
    free(present);
    return taken;
}

int orc_train_multiclass(const orc_multi_args* a, orc_multi_out* o) {
#ifdef _OPENMP
    if (a->n_threads > 0) omp_set_num_threads(a->n_threads);
#endif
    const int64_t n = a->n;
    const int32_t F = a->n_features, K = a->n_classes, D = a->depth, L = 1 << D;
    const int32_t pk = K * (K + 1) / 2;
    if (K < 1 || D < 1 || D > 16) return -1;
    int32_t NB = 1;
    for (int32_t f = 0; f < F; ++f)
        if (a->border_counts[f] + 1 > NB) NB = a->border_counts[f] + 1;
    for (int64_t k = 0; k < (int64_t)a->n_cat * n; ++k)
        if (a->cat_bins_fm[k] + 1 > NB) NB = a->cat_bins_fm[k] + 1;
    double* w = (double*)malloc(sizeof(double) * (size_t)(n > 0 ? n : 1));
    for (int64_t i = 0; i < n; ++i) w[i] = a->weights ? a->weights[i] : 1.0;
    double sum_w = orc_sum_f64(w, n);
    double scaled_l2 = n == 0 ? a->l2_leaf_reg : a->l2_leaf_reg * (sum_w / (double)n);
    const double lr = (double)(float)a->learning_rate;

    size_t nk = (size_t)n * K;
    double* approx = (double*)calloc(nk + 1, sizeof(double)); /* [K][n], bias 0 */
    if (a->loss_kind == 2 && n > 0) {
        /* RMSEWithUncertainty starts at [mean, 0.5 ln var] (boosting.rs:1895-1914,
         * 5190-5208): the f32 mean, the population variance about it in f32 */
        const double mean = (double)(float)(orc_sum_f64(a->target_matrix, n) / (double)n);
        double* sq = (double*)malloc(sizeof(double) * (size_t)n);
        for (int64_t i = 0; i < n; ++i) sq[i] = (a->target_matrix[i] - mean) * (a->target_matrix[i] - mean);
        const float var = (float)(orc_sum_f64(sq, n) / (double)n);
        free(sq);
        const double log_scale = 0.5 * log((double)var);
        for (int64_t i = 0; i < n; ++i) {
            approx[i] = mean;
            approx[(size_t)n + i] = log_scale;
        }
    }
    double* wd1 = (double*)malloc(sizeof(double) * (nk + 1));  /* [K][n] */
    double* d2p = (double*)malloc(sizeof(double) * ((size_t)n * pk + 1));
    const int diag = a->loss_kind == 1 || a->loss_kind == 2;
    double* sg = (double*)malloc(sizeof(double) * (nk + 1));
    double* sh = (double*)malloc(sizeof(double) * ((size_t)n + 1));
    double* dobj = (double*)malloc(sizeof(double) * ((size_t)n + 1));
    double* sw = (double*)malloc(sizeof(double) * ((size_t)n + 1));
    uint8_t* ctl = (uint8_t*)malloc((size_t)n + 1);
    int32_t* leaf = (int32_t*)malloc(sizeof(int32_t) * ((size_t)n + 1));
    double* lvd = (double*)malloc(sizeof(double) * (size_t)K * L); /* [K][L] */
    double* ls = (double*)malloc(sizeof(double) * (size_t)L * (K + pk));
    double *pa = (double*)malloc(sizeof(double) * (size_t)K * 4 + sizeof(double) * pk);
    double *pp = pa + K, *p1 = pp + K, *sq = p1 + K, *p2 = sq + K;

    orc_rng rng;
    orc_rng_from_seed(&rng, a->random_seed);
    const int draws = a->bootstrap_type != ORC_BOOT_NO;
    int has_prev = 0;
    double prev_mean = 0.0;
    int rc = 0;
    for (int32_t it = 0; it < a->iterations; ++it) {
        for (int64_t i = 0; i < n; ++i) {
            if (a->loss_kind == 2) {
                /* rmse_with_uncertainty_ders (loss.rs:680-720): diff = t - a0,
                 * prec = exp(-2 a1); der1 = [diff, diff^2 prec - 1],
                 * der2 = [-1, -2 diff^2 prec], the weight folded in once below */
                const double t = a->target_matrix[i];
                const double diff = t - approx[i];
                const double prec = exp(-2.0 * approx[(size_t)n + i]);
                const double dsp = diff * diff * prec;
                wd1[i] = w[i] * diff;
                wd1[(size_t)n + i] = w[i] * (dsp - 1.0);
                d2p[(size_t)i * pk] = -1.0;
                d2p[(size_t)i * pk + 1] = -2.0 * dsp;
                for (int32_t j = 2; j < pk; ++j) d2p[(size_t)i * pk + j] = 0.0;
                continue;
            }
            if (diag) {
                /* multiclass_onevsall_ders / multi_crossentropy_ders (loss.rs:501-560):
                 * per dimension p = sigmoid(a_d), der1 = t_d - p, der2 = -p (1 - p) */
                for (int32_t d = 0; d < K; ++d) {
                    const double av = approx[(size_t)d * n + i];
                    const double p = 1.0 - 1.0 / (1.0 + exp(av));
                    const double t = a->target_matrix[(size_t)d * n + i];
                    wd1[(size_t)d * n + i] = (t - p) * w[i];
                    d2p[(size_t)i * pk + d] = -p * (1.0 - p);
                }
                for (int32_t j = K; j < pk; ++j) d2p[(size_t)i * pk + j] = 0.0;
                continue;
            }
            for (int32_t d = 0; d < K; ++d) pa[d] = approx[(size_t)d * n + i];
            softmax_ders(pa, K, a->target_class[i], pp, p1, p2);
            for (int32_t d = 0; d < K; ++d) wd1[(size_t)d * n + i] = p1[d] * w[i];
            memcpy(d2p + (size_t)i * pk, p2, sizeof(double) * pk);
        }
        if (draws) {
            (void)orc_rng_gen(&rng); /* PRE_TREE_DRAWS */
            (void)orc_rng_gen(&rng);
        }
        for (int64_t i = 0; i < n; ++i) {
            for (int32_t d = 0; d < K; ++d) {
                double v = wd1[(size_t)d * n + i];
                sq[d] = v * v;
            }
            dobj[i] = sqrt(orc_sum_f64(sq, K));
        }
        if (orc_bootstrap(a->bootstrap_type, dobj, n, a->subsample, a->bagging_temperature, has_prev,
                          prev_mean, &rng, sw, ctl) != 0) {
            rc = -2;
            break;
        }
        for (int64_t i = 0; i < n; ++i) {
            for (int32_t d = 0; d < K; ++d)
                sg[(size_t)d * n + i] = ctl[i] ? wd1[(size_t)d * n + i] * sw[i] : 0.0;
            sh[i] = ctl[i] ? w[i] * sw[i] : 0.0;
        }
        mc_ctx c = {n, F, NB, K, D, a->score_function, a->bins_fm, a->border_counts, sg, sh, scaled_l2, draws, &rng,
                    a->n_cat, a->cat_bins_fm};
        int32_t* tf = o->split_feature + (size_t)it * D;
        int32_t* tb = o->split_bin + (size_t)it * D;
        for (int32_t l = 0; l < D; ++l) { tf[l] = -1; tb[l] = -1; }
        int err = 0;
        int taken = mc_search(&c, tf, tb, leaf, &err);
        if (err) { rc = -3; break; }
        o->tree_depth[it] = taken;
        const int32_t nl = 1 << taken;
        /* compute_softmax_leaf_deltas: ordered per-leaf sums over members in
         * object order, then the symmetric Newton solve per leaf */
        for (int32_t k = 0; k < L * (K + pk); ++k) ls[k] = 0.0;
        for (int64_t i = 0; i < n; ++i) {
            double* s = ls + (size_t)leaf[i] * (K + pk);
            for (int32_t d = 0; d < K; ++d) s[d] += wd1[(size_t)d * n + i];
            for (int32_t j = 0; j < pk; ++j) s[K + j] += d2p[(size_t)i * pk + j] * w[i];
        }
        for (int32_t k = 0; k < K * L; ++k) lvd[k] = 0.0;
        for (int32_t q = 0; q < nl; ++q) {
            const double* s = ls + (size_t)q * (K + pk);
            if (diag) { /* newton_leaf_delta per dimension (leaf.rs:196-232) */
                for (int32_t d = 0; d < K; ++d) {
                    const double den = -s[K + d] + scaled_l2;
                    pp[d] = den == 0.0 ? 0.0 : s[d] / den;
                }
            } else {
                orc_solve_symmetric_newton(s, s + K, K, scaled_l2, pp);
            }
            for (int32_t d = 0; d < K; ++d) lvd[(size_t)d * L + q] = pp[d] * lr; /* normalize_leaf_values */
        }
        double* out_lv = o->leaf_values + (size_t)it * L * K; /* leaf-major */
        for (int32_t q = 0; q < L; ++q)
            for (int32_t d = 0; d < K; ++d) out_lv[(size_t)q * K + d] = lvd[(size_t)d * L + q];
        for (int32_t d = 0; d < K; ++d)
            for (int64_t i = 0; i < n; ++i) approx[(size_t)d * n + i] += lvd[(size_t)d * L + leaf[i]];
        if (o->staged) {
            double* st = o->staged + (size_t)it * nk; /* object-major [n][K] */
            for (int64_t i = 0; i < n; ++i)
                for (int32_t d = 0; d < K; ++d) st[(size_t)i * K + d] = approx[(size_t)d * n + i];
        }
        if (draws) {
            (void)orc_rng_gen(&rng); /* POST_TREE_EXTRA_DRAWS */
            (void)orc_rng_gen(&rng);
        }
        /* last_iter_mean_leaf_value over the dim-major leaf block (bootstrap.rs:382-389) */
        double acc = 0.0;
        for (int32_t d = 0; d < K; ++d)
            for (int32_t q = 0; q < nl; ++q) {
                double v = lvd[(size_t)d * L + q];
                acc += sqrt(v * v);
            }
        prev_mean = acc / (double)(K * nl);
        has_prev = 1;
    }
    if (o->final_approx)
        for (int64_t i = 0; i < n; ++i)
            for (int32_t d = 0; d < K; ++d) o->final_approx[(size_t)i * K + d] = approx[(size_t)d * n + i];
    free(w); free(approx); free(wd1); free(d2p); free(sg); free(sh); free(dobj); free(sw); free(ctl);
    free(leaf); free(lvd); free(ls); free(pa);
    return rc;
}
