/*
 * cb_oracle_rank.c -- CPU restatement of catboost_rs's grouped (ranking)
 * losses on the pointwise-histogram oblivious loop: QueryRMSE and PairLogit
 * (crates/cb-compute/src/ranking_der.rs, crates/cb-train/src/boosting.rs
 * grouped branch, crates/cb-train/src/query_info.rs).
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for the device ranking arm.
 * The product path never calls it.  Build with -ffp-contract=off.
 *
 * Per iteration:
 *  1. grouped derivatives (calc_ders_for_queries, ranking_der.rs:139-400):
 *     QueryRMSE der1 = ((t - a) - queryAvrg) * w, der2 = -w with
 *     queryAvrg = sum((t - a) * w) / sum(w) per group; PairLogit scatters
 *     w_pair * p (p = e^loser / (e^loser + e^winner)) doc-ascending,
 *     competitor-order;  the ders already carry the weights;
 *  2. the histogram weight channel: PairLogit uses the pairwise weights
 *     (calc_pairwise_weights, boosting.rs:1761-1780), QueryRMSE the object
 *     weights;
 *  3. the scalar greedy search;
 *  4. Newton leaves sum(der1) / (-sum(der2) + scaled_l2) over unit leaf
 *     weights (boosting.rs:8330-8400, leaf.rs:223-232), scaled_l2 from the
 *     object-weight sum;
 *  5. normalize_leaf_values (boosting.rs:2844-2880): PairLogit subtracts the
 *     document-weighted mean leaf value, then x lr (f32-narrowed).
 */
#include "cb_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* pairlogit_pair_prob (loss.rs:640-652) */
static double pair_prob(double winner, double loser) {
    double el = exp(loser), ew = exp(winner);
    double den = el + ew;
    return den > 0.0 ? el / den : 0.5;
}

typedef struct {
    int64_t* start; /* [n + 1] CSR over winners (global object ids) */
    int64_t* loser; /* [n_pairs] in pair order per winner */
} competitors;

/* build_query_info step 3 (query_info.rs:205-250): pairs in input order,
 * pushed to their winner's row, weight 1.0. */
static int build_competitors(const orc_rank_args* a, competitors* c) {
    const int64_t n = a->n;
    c->start = (int64_t*)calloc((size_t)n + 1, sizeof(int64_t));
    c->loser = (int64_t*)malloc(sizeof(int64_t) * (size_t)(a->n_pairs > 0 ? a->n_pairs : 1));
    if (!c->start || !c->loser) return -1;
    for (int64_t k = 0; k < a->n_pairs; ++k) {
        if (a->pair_winner[k] < 0 || a->pair_winner[k] >= n || a->pair_loser[k] < 0 || a->pair_loser[k] >= n)
            return -1;
        c->start[a->pair_winner[k] + 1]++;
    }
    for (int64_t i = 0; i < n; ++i) c->start[i + 1] += c->start[i];
    int64_t* fill = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n > 0 ? n : 1));
    if (!fill) return -1;
    for (int64_t i = 0; i < n; ++i) fill[i] = c->start[i];
    for (int64_t k = 0; k < a->n_pairs; ++k) c->loser[fill[a->pair_winner[k]]++] = a->pair_loser[k];
    free(fill);
    return 0;
}

int orc_train_ranking(const orc_rank_args* a, orc_rank_out* o) {
    const int64_t n = a->n;
    const int32_t F = a->n_features, D = a->depth, L = 1 << D;
    if (D < 1 || D > 16 || a->n_groups < 0) return -1;
    if (a->n_groups > 0 && (a->group_offsets[0] != 0 || a->group_offsets[a->n_groups] != n)) return -1;
    int32_t NB = 1;
    for (int32_t f = 0; f < F; ++f)
        if (a->border_counts[f] + 1 > NB) NB = a->border_counts[f] + 1;
    competitors cp = {NULL, NULL};
    if (a->loss == ORC_RANK_PAIRLOGIT && build_competitors(a, &cp) != 0) {
        free(cp.start);
        free(cp.loser);
        return -2;
    }
    double* w = (double*)calloc((size_t)(n > 0 ? n : 1), sizeof(double));
    for (int64_t i = 0; i < n; ++i) w[i] = a->weights ? a->weights[i] : 1.0;
    const double sum_w = orc_sum_f64(w, n);
    const double scaled_l2 = n == 0 ? a->l2_leaf_reg : a->l2_leaf_reg * (sum_w / (double)n);
    const double lr = (double)(float)a->learning_rate;

    double* approx = (double*)calloc((size_t)n + 1, sizeof(double)); /* boost_from_average off */
    double* d1 = (double*)malloc(sizeof(double) * ((size_t)n + 1));
    double* d2 = (double*)malloc(sizeof(double) * ((size_t)n + 1));
    double* eff = (double*)malloc(sizeof(double) * ((size_t)n + 1));
    double* sh = (double*)malloc(sizeof(double) * ((size_t)n + 1));
    double* tmp = (double*)malloc(sizeof(double) * ((size_t)(n > L ? n : L) + 1));
    int32_t* leaf = (int32_t*)malloc(sizeof(int32_t) * ((size_t)n + 1));
    double* lv = (double*)malloc(sizeof(double) * L);
    double* lw = (double*)malloc(sizeof(double) * L);

    /* histogram weights: pairwise weights for PairLogit, object weights otherwise */
    if (a->loss == ORC_RANK_PAIRLOGIT) {
        for (int64_t i = 0; i < n; ++i) eff[i] = 0.0;
        for (int32_t g = 0; g < a->n_groups; ++g)
            for (int64_t wi = a->group_offsets[g]; wi < a->group_offsets[g + 1]; ++wi)
                for (int64_t k = cp.start[wi]; k < cp.start[wi + 1]; ++k) {
                    eff[wi] += 1.0;
                    eff[cp.loser[k]] += 1.0;
                }
    } else {
        for (int64_t i = 0; i < n; ++i) eff[i] = w[i];
    }
    for (int64_t i = 0; i < n; ++i) sh[i] = eff[i]; /* no bootstrap: control 1, sample weight 1 */

    orc_rng rng;
    orc_rng_from_seed(&rng, a->random_seed);
    int rc = 0;
    for (int32_t it = 0; it < a->iterations; ++it) {
        /* 1. grouped derivatives */
        for (int64_t i = 0; i < n; ++i) {
            d1[i] = 0.0;
            d2[i] = 0.0;
        }
        for (int32_t g = 0; g < a->n_groups; ++g) {
            const int64_t b = a->group_offsets[g], e = a->group_offsets[g + 1];
            if (e <= b) continue;
            if (a->loss == ORC_RANK_QUERYRMSE) {
                for (int64_t i = b; i < e; ++i) tmp[i - b] = (a->target[i] - approx[i]) * w[i];
                double num = orc_sum_f64(tmp, e - b);
                double den = orc_sum_f64(w + b, e - b);
                double avg = den > 0.0 ? num / den : 0.0;
                for (int64_t i = b; i < e; ++i) {
                    d1[i] = (a->target[i] - approx[i] - avg) * w[i];
                    d2[i] = -1.0 * w[i];
                }
            } else {
                for (int64_t wi = b; wi < e; ++wi) {
                    double wd = 0.0, wd2 = 0.0;
                    for (int64_t k = cp.start[wi]; k < cp.start[wi + 1]; ++k) {
                        const int64_t li = cp.loser[k];
                        const double p = pair_prob(approx[wi], approx[li]);
                        const double pw = 1.0;
                        wd += pw * p;
                        wd2 += pw * p * (p - 1.0);
                        d1[li] -= pw * p;
                        d2[li] += pw * p * (p - 1.0);
                    }
                    d1[wi] += wd;
                    d2[wi] += wd2;
                }
            }
        }
        /* 2-3. score channels (control 1, sample weight 1) and the search */
        int32_t* tf = o->split_feature + (size_t)it * D;
        int32_t* tb = o->split_bin + (size_t)it * D;
        for (int32_t l = 0; l < D; ++l) {
            tf[l] = -1;
            tb[l] = -1;
        }
        int32_t err = 0;
        int taken = orc_search_tree(n, F, NB, D, a->score_function, a->bins_fm, a->border_counts, d1, sh, scaled_l2,
                                    0, &rng, tf, tb, leaf, &err);
        if (err) {
            rc = -3;
            break;
        }
        const int32_t nl = 1 << taken;
        /* 4. Newton leaves over unit leaf weights, ordered per-leaf sums */
        double* sd = (double*)calloc((size_t)nl * 3, sizeof(double));
        for (int64_t i = 0; i < n; ++i) {
            sd[3 * leaf[i]] += d1[i];
            sd[3 * leaf[i] + 1] += d2[i] * 1.0;
            sd[3 * leaf[i] + 2] += w[i];
        }
        for (int32_t q = 0; q < L; ++q) {
            lv[q] = 0.0;
            lw[q] = 0.0;
        }
        for (int32_t q = 0; q < nl; ++q) {
            const double den = -sd[3 * q + 1] + scaled_l2;
            lv[q] = den == 0.0 ? 0.0 : sd[3 * q] / den;
            lw[q] = sd[3 * q + 2];
        }
        free(sd);
        if (o->raw_leaf_values) memcpy(o->raw_leaf_values + (size_t)it * L, lv, sizeof(double) * L);
        /* 5. normalize_leaf_values */
        if (a->loss == ORC_RANK_PAIRLOGIT) {
            const double total = orc_sum_f64(lw, nl);
            if (fabs(total) > 1e-9) {
                for (int32_t q = 0; q < nl; ++q) tmp[q] = lv[q] * lw[q];
                const double avg = orc_sum_f64(tmp, nl) / total;
                for (int32_t q = 0; q < nl; ++q) lv[q] = fabs(lw[q]) > 1e-9 ? lv[q] - avg : 0.0;
            }
        }
        for (int32_t q = 0; q < nl; ++q) lv[q] *= lr;
        memcpy(o->leaf_values + (size_t)it * L, lv, sizeof(double) * L);
        for (int64_t i = 0; i < n; ++i) approx[i] += lv[leaf[i]];
        if (o->staged) memcpy(o->staged + (size_t)it * n, approx, sizeof(double) * (size_t)n);
    }
    free(cp.start);
    free(cp.loser);
    free(w); free(approx); free(d1); free(d2); free(eff); free(sh); free(tmp); free(leaf); free(lv); free(lw);
    return rc;
}
