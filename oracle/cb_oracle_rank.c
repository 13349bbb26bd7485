/*
 * cb_oracle_rank.c -- CPU restatement of catboost_rs's grouped (ranking)
 * losses on the oblivious loop: QueryRMSE, QuerySoftMax, LambdaMart (NDCG /
 * DCG), StochasticRank (DCG / NDCG), PairLogit and YetiRank on pointwise
 * histograms, and PairLogitPairwise with the pairwise split scoring and
 * Cholesky leaves (crates/cb-compute/src/ranking_der.rs, pairwise_scoring.rs,
 * crates/cb-train/src/boosting.rs grouped branch, pairwise_leaves.rs,
 * tree.rs:3740-3960, query_info.rs).
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for the device ranking arm.
 * The product path never calls it.  Build with -ffp-contract=off.
 *
 * Per iteration:
 *  1. grouped derivatives (calc_ders_for_queries, ranking_der.rs:139-400):
 *     QueryRMSE der1 = ((t - a) - queryAvrg) * w, der2 = -w with
 *     queryAvrg = sum((t - a) * w) / sum(w) per group; PairLogit scatters
 *     w_pair * p (p = e^loser / (e^loser + e^winner)) doc-ascending,
 *     competitor-order; QuerySoftMax (ranking_der.rs:247-320, loss.rs:608-619)
 *     takes p = e^(beta (a - max)) w / sum over the group (max over w > 0),
 *     der1 = beta (-sumWT p + w t), der2 = beta sumWT (beta p (p - 1) - lambda)
 *     with sumWT = sum(w t) over w > 0, t > 0 (ders 0 when sumWT <= 0 or
 *     w <= 0); LambdaMart (ranking_der.rs:440-630, loss.rs:660-680) stable-sorts
 *     the group by approx descending and scatters each ordered pair's lambda
 *     (first target > second target; the second position bounded by top)
 *     with delta = (t1 - t2) |1/log2(2 + p1) - 1/log2(2 + p2)| / idealDCG,
 *     / (0.01 + |a1 - a2|) under norm, then rescales the group by
 *     log2(1 + sumDer1) / sumDer1 under norm;  the ders already carry the
 *     weights;
 *  2. the histogram weight channel: PairLogit uses the pairwise weights
 *     (calc_pairwise_weights, boosting.rs:1761-1780), QueryRMSE the object
 *     weights;
 *  3. the scalar greedy search;
 *  4. Newton leaves sum(der1) / (-sum(der2) + scaled_l2) over unit leaf
 *     weights (boosting.rs:8330-8400, leaf.rs:223-232), scaled_l2 from the
 *     object-weight sum; QuerySoftMax takes Gradient leaves over the same unit
 *     weights, sum(der1) / (count + scaled_l2) (leaf.rs:161-194);
 *  5. normalize_leaf_values (boosting.rs:2844-2880): PairLogit subtracts the
 *     document-weighted mean leaf value, then x lr (f32-narrowed).
 * PairLogitPairwise replaces 3-4: per level and feature the der sums
 * [leaf][bucket] and pair statistics [leaf][leaf][bucket], a running
 * 2P x 2P weight system per border with a Cholesky leaf solve and score
 * (pairwise_scoring.rs:101-580); leaves from the leaf pair-weight system with
 * the raw l2 (pairwise_leaves.rs:51-242); the same centring and x lr.
 */
#include "cb_oracle.h"

#include <float.h>
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
    int64_t* start;  /* [n + 1] CSR over winners (global object ids) */
    int64_t* loser;  /* [n_pairs] in pair order per winner */
    double* weight;  /* [n_pairs] the pair's Competitor::weight, same order */
} competitors;

/* build_query_info step 3 (query_info.rs:205-250): pairs in input order,
 * pushed to their winner's row with their weight (1.0 when none is given). */
static int build_competitors(const orc_rank_args* a, competitors* c) {
    const int64_t n = a->n;
    c->start = (int64_t*)calloc((size_t)n + 1, sizeof(int64_t));
    c->loser = (int64_t*)malloc(sizeof(int64_t) * (size_t)(a->n_pairs > 0 ? a->n_pairs : 1));
    c->weight = (double*)malloc(sizeof(double) * (size_t)(a->n_pairs > 0 ? a->n_pairs : 1));
    if (!c->start || !c->loser || !c->weight) return -1;
    for (int64_t k = 0; k < a->n_pairs; ++k) {
        if (a->pair_winner[k] < 0 || a->pair_winner[k] >= n || a->pair_loser[k] < 0 || a->pair_loser[k] >= n)
            return -1;
        c->start[a->pair_winner[k] + 1]++;
    }
    for (int64_t i = 0; i < n; ++i) c->start[i + 1] += c->start[i];
    int64_t* fill = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n > 0 ? n : 1));
    if (!fill) return -1;
    for (int64_t i = 0; i < n; ++i) fill[i] = c->start[i];
    for (int64_t k = 0; k < a->n_pairs; ++k) {
        const int64_t at = fill[a->pair_winner[k]]++;
        c->loser[at] = a->pair_loser[k];
        c->weight[at] = a->pair_weight ? a->pair_weight[k] : 1.0;
    }
    free(fill);
    return 0;
}

/* ndcg_denominator (ranking_der.rs:456-467): log2(2 + pos) as log(x) * log2(e) */
static double lm_den(int64_t pos) { return log(2.0 + (double)pos) * 1.4426950408889634; }

/* LambdaMart ders of one group (lambdamart_group_der, ranking_der.rs:482-606;
 * lambdamart_pair_grad, loss.rs:673-679), NDCG / DCG; order and ts are
 * group-sized scratch. */
static void lambdamart_group(const double* ap, const double* tg, int64_t cnt, double sigma, int64_t top, int norm,
                             int64_t* order, double* ts, double* d1, double* d2) {
    for (int64_t i = 0; i < cnt; ++i) {
        d1[i] = 0.0;
        d2[i] = 0.0;
    }
    if (cnt <= 1) return;
    for (int64_t i = 0; i < cnt; ++i) order[i] = i;
    for (int64_t i = 1; i < cnt; ++i) { /* stable insertion sort, approx descending */
        const int64_t key = order[i];
        int64_t j = i - 1;
        while (j >= 0 && ap[order[j]] < ap[key]) {
            order[j + 1] = order[j];
            --j;
        }
        order[j + 1] = key;
    }
    const int same = fabs(ap[order[0]] - ap[order[cnt - 1]]) == 0.0;
    const int64_t top_size = (top == -1 || top > cnt) ? cnt : top;
    /* lambdamart_ideal_ndcg (ranking_der.rs:616-628) */
    for (int64_t i = 0; i < cnt; ++i) ts[i] = tg[i];
    for (int64_t i = 1; i < cnt; ++i) {
        const double key = ts[i];
        int64_t j = i - 1;
        while (j >= 0 && ts[j] < key) {
            ts[j + 1] = ts[j];
            --j;
        }
        ts[j + 1] = key;
    }
    double ideal = 0.0;
    for (int64_t p = 0; p < top_size; ++p) ideal += ts[p] / lm_den(p);
    double sum_der1 = 0.0;
    for (int64_t fi = 0; fi < cnt; ++fi) {
        const int64_t bound = fi < top_size ? cnt : top_size;
        for (int64_t si = 0; si < bound; ++si) {
            const double ft = tg[order[fi]], st = tg[order[si]];
            if (ft <= st) continue;
            const double adiff = ap[order[fi]] - ap[order[si]];
            const double dnum = ft - st;
            const double dden = fabs(1.0 / lm_den(fi) - 1.0 / lm_den(si));
            double delta = ideal != 0.0 ? dnum * dden / ideal : 0.0;
            if (norm && !same) delta /= 0.01 + fabs(adiff);
            const double sig = 1.0 / (1.0 + exp(sigma * adiff));
            double hess = sig * (1.0 - sig);
            const double anti = -sigma * delta * sig;
            hess *= sigma * sigma * delta;
            d1[order[fi]] += anti;
            d2[order[fi]] += hess;
            d1[order[si]] -= anti;
            d2[order[si]] += hess;
            sum_der1 -= 2.0 * anti;
        }
    }
    if (norm && sum_der1 > 0.0) {
        const double norma = log2(1.0 + sum_der1) / sum_der1;
        for (int64_t i = 0; i < cnt; ++i) {
            d1[i] *= norma;
            d2[i] *= norma;
        }
    }
}

/* ---- StochasticRank (ranking_der.rs:640-1000) --------------------------- */

/* normal_density (ranking_der.rs:640-655) */
static double srank_density(double x, double mean, double sigma) {
    const double t = (x - mean) / sigma;
    const double z = t * t;
    return exp(-z / 2.0) * 0.398942280401432677939946 / sigma;
}

/* calc_dcg_metric_diff (ranking_der.rs:920-965) */
static double srank_metric_diff(int64_t old_pos, int64_t new_pos, const double* tg, const int64_t* order,
                                const double* pw, const double* cs, const double* csu, const double* csl) {
    const double gain = tg[order[old_pos]];
    const double doc_diff = gain * (pw[new_pos] - pw[old_pos]);
    double mid;
    if (new_pos < old_pos) {
        const double old_mid = cs[old_pos] - cs[new_pos];
        const double new_mid = csl[old_pos] - csl[new_pos];
        mid = new_mid - old_mid;
    } else {
        const double old_mid = cs[new_pos + 1] - cs[old_pos + 1];
        const double new_mid = csu[new_pos + 1] - csu[old_pos + 1];
        mid = new_mid - old_mid;
    }
    return doc_diff + mid;
}

/* stochastic_rank_group_der (ranking_der.rs:710-910), DCG / NDCG, the whole
 * group as the top; der2 = 0.  ws: 9 * cnt + 3 doubles, order: cnt. */
static void stochastic_rank_group(const double* ap_raw, const double* tg, int64_t cnt, int is_ndcg, double sigma_p,
                                  double mu, int32_t num_est, uint64_t seed, double* ws, int64_t* order, double* d1,
                                  double* d2) {
    for (int64_t i = 0; i < cnt; ++i) {
        d1[i] = 0.0;
        d2[i] = 0.0;
    }
    if (cnt <= 1) return;
    if (num_est < 1) num_est = 1;
    double* ap = ws;
    double* sh = ap + cnt;
    double* pw = sh + cnt;
    double* noise = pw + cnt;
    double* sc = noise + cnt;
    double* cs = sc + cnt;
    double* csu = cs + cnt + 1;
    double* csl = csu + cnt + 1;
    double* tmp = csl + cnt + 1;
    const double am = orc_sum_f64(ap_raw, cnt) / (double)cnt; /* group-mean centring */
    for (int64_t i = 0; i < cnt; ++i) ap[i] = ap_raw[i] - am;
    for (int64_t i = 0; i < cnt; ++i) sh[i] = ap[i] - sigma_p * mu * tg[i];
    const double avs = orc_sum_f64(sh, cnt) / (double)cnt;
    for (int64_t i = 0; i < cnt; ++i) sh[i] -= avs;
    /* compute_dcg_pos_weights (ranking_der.rs:659-690) */
    for (int64_t p = 0; p < cnt; ++p) pw[p] = 1.0 / lm_den(p);
    if (is_ndcg) {
        for (int64_t i = 0; i < cnt; ++i) tmp[i] = tg[i];
        for (int64_t i = 1; i < cnt; ++i) {
            const double key = tmp[i];
            int64_t j = i - 1;
            while (j >= 0 && tmp[j] < key) {
                tmp[j + 1] = tmp[j];
                --j;
            }
            tmp[j + 1] = key;
        }
        double ideal = 0.0;
        for (int64_t p = 0; p < cnt; ++p) ideal += tmp[p] * pw[p];
        if (ideal > DBL_EPSILON)
            for (int64_t p = 0; p < cnt; ++p) pw[p] /= ideal;
    }
    orc_rng rng;
    orc_rng_from_seed(&rng, seed);
    const double sigma = sigma_p * sqrt((double)cnt / ((double)cnt - 1.0));
    for (int32_t s = 0; s < num_est; ++s) {
        for (int64_t d = 0; d < cnt; ++d) {
            noise[d] = orc_std_normal(&rng);
            sc[d] = sh[d] + sigma_p * noise[d];
        }
        const double noise_sum = orc_sum_f64(noise, cnt);
        for (int64_t i = 0; i < cnt; ++i) order[i] = i;
        for (int64_t i = 1; i < cnt; ++i) { /* stable, descending by score */
            const int64_t key = order[i];
            int64_t j = i - 1;
            while (j >= 0 && sc[order[j]] < sc[key]) {
                order[j + 1] = order[j];
                --j;
            }
            order[j + 1] = key;
        }
        /* CalcDCGCumulativeStatistics */
        for (int64_t p = 0; p <= cnt; ++p) {
            cs[p] = 0.0;
            csu[p] = 0.0;
            csl[p] = 0.0;
        }
        for (int64_t p = 0; p < cnt; ++p) {
            const double gain = tg[order[p]];
            cs[p + 1] = cs[p] + gain * pw[p];
            if (p + 1 < cnt) csl[p + 1] = csl[p] + gain * pw[p + 1];
            if (p > 0) csu[p + 1] = csu[p] + gain * pw[p - 1];
        }
        csl[cnt] = csl[cnt - 1];
        for (int64_t p = 0; p < cnt; ++p) {
            const int64_t doc = order[p];
            const double score = sc[doc], a = ap[doc];
            const double mean = a + (noise_sum - (score - a)) / ((double)cnt - 1.0);
            double der_sum = 0.0;
            for (int64_t np = 0; np < cnt; ++np) {
                if (np == p) continue;
                const double md = srank_metric_diff(p, np, tg, order, pw, cs, csu, csl);
                double dd;
                if (np == 0) dd = srank_density(sc[order[0]], mean, sigma);
                else if (np + 1 == cnt) dd = -srank_density(sc[order[cnt - 1]], mean, sigma);
                else if (np < p) dd = srank_density(sc[order[np]], mean, sigma) - srank_density(sc[order[np - 1]], mean, sigma);
                else dd = srank_density(sc[order[np + 1]], mean, sigma) - srank_density(sc[order[np]], mean, sigma);
                der_sum += md * dd;
            }
            d1[doc] += der_sum / (double)num_est;
        }
    }
    /* SFA: remove the mean der, then project out the approx direction */
    const double avg_der = orc_sum_f64(d1, cnt) / (double)cnt;
    for (int64_t i = 0; i < cnt; ++i) d1[i] -= avg_der;
    if (cnt > 2) {
        const double aa = orc_sum_f64(ap, cnt) / (double)cnt;
        for (int64_t i = 0; i < cnt; ++i) {
            sh[i] = ap[i] - aa; /* zero-mean approx */
            tmp[i] = sh[i] * sh[i];
        }
        const double nr = sqrt(orc_sum_f64(tmp, cnt)) + 0.01;
        const double norm_sqr = nr * nr;
        for (int64_t i = 0; i < cnt; ++i) tmp[i] = d1[i] * sh[i];
        const double dot = orc_sum_f64(tmp, cnt);
        if (norm_sqr > 0.0) {
            const double k = 1.0 * dot / norm_sqr;
            for (int64_t i = 0; i < cnt; ++i) d1[i] -= k * sh[i];
        }
    }
}

/* ---- YetiRank (crates/cb-train/src/yetirank.rs) ------------------------- */

void orc_yeti_sample_pairs(const double* raw_approx, const double* relevs, int64_t g, double query_weight,
                           int32_t permutations, double decay, uint64_t query_seed, double* out) {
    for (int64_t k = 0; k < g * g; ++k) out[k] = 0.0;
    if (g == 0 || permutations <= 0) return;
    float* cw = (float*)calloc((size_t)(g * g), sizeof(float));
    double* ea = (double*)malloc(sizeof(double) * (size_t)g);
    double* boot = (double*)malloc(sizeof(double) * (size_t)g);
    int64_t* idx = (int64_t*)malloc(sizeof(int64_t) * (size_t)g);
    for (int64_t i = 0; i < g; ++i) ea[i] = exp(raw_approx[i]);
    orc_rng r;
    orc_rng_from_seed(&r, query_seed);
    for (int32_t perm = 0; perm < permutations; ++perm) {
        for (int64_t i = 0; i < g; ++i) {
            idx[i] = i;
            boot[i] = ea[i];
        }
        /* Gumbel noise, f32 draw and ratio (yetirank.rs:106-121) */
        for (int64_t i = 0; i < g; ++i) {
            const float u = (float)orc_rng_real1(&r);
            const float ratio = u / (1.000001f - u);
            boot[i] *= (double)ratio;
        }
        for (int64_t i = 1; i < g; ++i) { /* stable sort, descending */
            const int64_t key = idx[i];
            int64_t j = i - 1;
            while (j >= 0 && boot[idx[j]] < boot[key]) {
                idx[j + 1] = idx[j];
                --j;
            }
            idx[j + 1] = key;
        }
        /* calc_weights_classic + add_weight (yetirank.rs:450-514), f32 storage */
        double dc = 1.0;
        for (int64_t d = 1; d < g; ++d) {
            const int64_t first = idx[d - 1], second = idx[d];
            const float rf = (float)relevs[first], rs = (float)relevs[second];
            const float pw = (float)(0.15 * dc * (double)fabsf(rf - rs));
            if (rf > rs) cw[first * g + second] += pw;
            else if (rf < rs) cw[second * g + first] += pw;
            dc *= decay;
        }
    }
    const float qw = (float)query_weight, den = (float)permutations;
    for (int64_t k = 0; k < g * g; ++k) {
        const float wf = qw * cw[k] / den;
        out[k] = (double)wf;
    }
    free(cw);
    free(ea);
    free(boot);
    free(idx);
}

static uint64_t first_gen(uint64_t seed) {
    orc_rng t;
    orc_rng_from_seed(&t, seed);
    return orc_rng_gen(&t);
}

void orc_yeti_query_seeds(uint64_t random_seed, int32_t n_groups, uint64_t* out) {
    orc_rng b;
    orc_rng_from_seed(&b, first_gen(random_seed));
    for (int32_t g = 0; g < n_groups; ++g) out[g] = orc_rng_gen(&b);
}

/* derive_per_tree_query_seeds (yetirank.rs:215-221) */
static void per_tree_query_seeds(uint64_t recalc, int32_t n_groups, uint64_t* out) {
    orc_rng t;
    orc_rng_from_seed(&t, recalc);
    for (int32_t g = 0; g < n_groups; ++g) out[g] = first_gen(orc_rng_gen(&t));
}

/* YetiRankTreeSeeder::next_tree (yetirank.rs:340-430) */
static void yeti_next_tree(orc_rng* r, int32_t G, int32_t F, int32_t depth, uint64_t* deriv, uint64_t* learnfold,
                           uint64_t* leafval, uint64_t* recalc) {
    (void)orc_rng_gen(r); /* structure-fold selection */
    const uint64_t drs = first_gen(orc_rng_gen(r));
    for (int32_t level = 0; level < depth; ++level) {
        for (int32_t f = 0; f < F; ++f) (void)orc_rng_real1(r);
        (void)orc_rng_gen(r);
        for (int32_t f = 0; f < F; ++f) (void)orc_std_normal(r);
    }
    const uint64_t lrs = first_gen(first_gen(orc_rng_gen(r)));
    const uint64_t vb = orc_rng_gen(r);
    if (deriv) per_tree_query_seeds(drs, G, deriv);
    if (learnfold) per_tree_query_seeds(lrs, G, learnfold);
    if (leafval) per_tree_query_seeds(vb, G, leafval);
    if (recalc) {
        recalc[0] = drs;
        recalc[1] = lrs;
        recalc[2] = vb;
    }
}

void orc_yeti_recalc_seeds(uint64_t random_seed, int32_t n_groups, int32_t n_features, int32_t depth, int32_t trees,
                           uint64_t* out) {
    orc_rng r;
    orc_rng_from_seed(&r, random_seed);
    for (int32_t t = 0; t < trees; ++t) yeti_next_tree(&r, n_groups, n_features, depth, NULL, NULL, NULL, out + 3 * t);
}

/* One YetiRank phase's ders: per group the sampled pairs from `ap` with the
 * phase's query seeds, then the PairLogit der over them (pairlogit_group_der,
 * ranking_der.rs:400-440) and, when eff != NULL, the pairwise weights
 * (calc_pairwise_weights, boosting.rs:1761-1780), winner-ascending,
 * loser-ascending. */
static void yeti_phase_ders(const orc_rank_args* a, const double* ap, const double* gw, const uint64_t* seeds,
                            double* cwbuf, double* d1, double* d2, double* eff, int64_t* pw_out, int64_t* pl_out,
                            double* pwt_out, int64_t* n_out) {
    const int64_t n = a->n;
    if (n_out) *n_out = 0;
    for (int64_t i = 0; i < n; ++i) {
        d1[i] = 0.0;
        d2[i] = 0.0;
        if (eff) eff[i] = 0.0;
    }
    for (int32_t gi = 0; gi < a->n_groups; ++gi) {
        const int64_t b = a->group_offsets[gi], e = a->group_offsets[gi + 1], g = e - b;
        orc_yeti_sample_pairs(ap + b, a->target + b, g, gw[gi], a->yeti_permutations, a->yeti_decay, seeds[gi],
                              cwbuf);
        for (int64_t wl = 0; wl < g; ++wl) {
            double wd = 0.0, wd2 = 0.0;
            for (int64_t ll = 0; ll < g; ++ll) {
                const double cw = cwbuf[wl * g + ll];
                if (cw == 0.0) continue;
                const double p = pair_prob(ap[b + wl], ap[b + ll]);
                wd += cw * p;
                wd2 += cw * p * (p - 1.0);
                d1[b + ll] -= cw * p;
                d2[b + ll] += cw * p * (p - 1.0);
                if (eff) {
                    eff[b + wl] += cw;
                    eff[b + ll] += cw;
                }
                if (n_out) { /* flatten_global_pairs order (tree.rs:3747-3760) */
                    pw_out[*n_out] = b + wl;
                    pl_out[*n_out] = b + ll;
                    pwt_out[*n_out] = cw;
                    ++*n_out;
                }
            }
            d1[b + wl] += wd;
            d2[b + wl] += wd2;
        }
    }
}

static int pairwise_search(const orc_rank_args* a, const double* der1, const int64_t* pw, const int64_t* pl,
                           const double* pwt, int64_t n_pairs, int32_t* feat, int32_t* sbin, int32_t* leaf_of);
static void pairwise_leaf_deltas(const int64_t* pw, const int64_t* pl, const double* pwt, int64_t n_pairs,
                                 const int32_t* leaf, const double* d1, int64_t n, int32_t nl, double l2, double* lv);

/* Newton deltas over unit leaf weights (ordered per-leaf sums) */
static void newton_unit(const double* d1, const double* d2, const int32_t* leaf, int64_t n, int32_t nl, double l2,
                        double* out) {
    double* sd = (double*)calloc((size_t)nl * 2, sizeof(double));
    for (int64_t i = 0; i < n; ++i) {
        sd[2 * leaf[i]] += d1[i];
        sd[2 * leaf[i] + 1] += d2[i] * 1.0;
    }
    for (int32_t q = 0; q < nl; ++q) {
        const double den = -sd[2 * q + 1] + l2;
        out[q] = den == 0.0 ? 0.0 : sd[2 * q] / den;
    }
    free(sd);
}

/* The YetiRank loop (boosting.rs:4997-5060, 7347-7420, 8070-8200, 8787-8880):
 * per tree the seeder's three per-group seed sets; the gradient / split ders
 * and the histogram's pairwise weights from pairs sampled off the learning-fold
 * approximant; the stored leaves (Newton, unit weights, pairwise centring,
 * x lr) from pairs sampled off the model approximant; the learning-fold
 * approximant advanced by its own resample's Newton deltas x lr.
 * YetiRankPairwise scores the splits with the pairwise scorer over the
 * sampled, weighted pairs and takes Cholesky pairwise leaves (raw l2) for both
 * the stored leaves and the learning fold (boosting.rs:8270-8300, 8840-8860). */
static int train_yetirank(const orc_rank_args* a, orc_rank_out* o, int32_t NB) {
    const int pairwise = a->loss == ORC_RANK_YETIRANK_PAIRWISE;
    const int64_t n = a->n;
    const int32_t F = a->n_features, D = a->depth, L = 1 << D, G = a->n_groups;
    double* w = (double*)calloc((size_t)n + 1, sizeof(double));
    for (int64_t i = 0; i < n; ++i) w[i] = a->weights ? a->weights[i] : 1.0;
    const double sum_w = orc_sum_f64(w, n);
    const double scaled_l2 = n == 0 ? a->l2_leaf_reg : a->l2_leaf_reg * (sum_w / (double)n);
    const double lr = (double)(float)a->learning_rate;
    int64_t maxg = 1;
    double* gw = (double*)malloc(sizeof(double) * (size_t)(G > 0 ? G : 1));
    for (int32_t gi = 0; gi < G; ++gi) { /* group weight: mean member weight (query_info.rs:180-187) */
        const int64_t b = a->group_offsets[gi], e = a->group_offsets[gi + 1];
        gw[gi] = e > b ? orc_sum_f64(w + b, e - b) / (double)(e - b) : 1.0;
        if (e - b > maxg) maxg = e - b;
    }
    double* cwbuf = (double*)malloc(sizeof(double) * (size_t)(maxg * maxg));
    double* approx = (double*)calloc((size_t)n + 1, sizeof(double));
    double* lapprox = (double*)calloc((size_t)n + 1, sizeof(double));
    double* d1 = (double*)malloc(sizeof(double) * ((size_t)n + 1));
    double* d2 = (double*)malloc(sizeof(double) * ((size_t)n + 1));
    double* eff = (double*)malloc(sizeof(double) * ((size_t)n + 1));
    double* tmp = (double*)malloc(sizeof(double) * ((size_t)L + 1));
    int32_t* leaf = (int32_t*)malloc(sizeof(int32_t) * ((size_t)n + 1));
    double* lv = (double*)malloc(sizeof(double) * L);
    double* lw = (double*)malloc(sizeof(double) * L);
    uint64_t* seeds = (uint64_t*)malloc(sizeof(uint64_t) * 3 * (size_t)(G > 0 ? G : 1));
    int64_t cells = 1, n_flat = 0;
    for (int32_t gi = 0; gi < G; ++gi) {
        const int64_t g = a->group_offsets[gi + 1] - a->group_offsets[gi];
        cells += g * g;
    }
    int64_t* fw = pairwise ? (int64_t*)malloc(sizeof(int64_t) * (size_t)cells) : NULL;
    int64_t* fl = pairwise ? (int64_t*)malloc(sizeof(int64_t) * (size_t)cells) : NULL;
    double* fwt = pairwise ? (double*)malloc(sizeof(double) * (size_t)cells) : NULL;
    int64_t* nf = pairwise ? &n_flat : NULL;
    uint64_t* sd = seeds;
    uint64_t* sl = seeds + G;
    uint64_t* sv = seeds + 2 * G;
    orc_rng seeder, unused;
    orc_rng_from_seed(&seeder, a->random_seed);
    orc_rng_from_seed(&unused, a->random_seed);
    int rc = 0;
    for (int32_t it = 0; it < a->iterations; ++it) {
        yeti_next_tree(&seeder, G, F, D, sd, sl, sv, NULL);
        /* gradient / split: the learning fold */
        yeti_phase_ders(a, lapprox, gw, sd, cwbuf, d1, d2, eff, fw, fl, fwt, nf);
        int32_t* tf = o->split_feature + (size_t)it * D;
        int32_t* tb = o->split_bin + (size_t)it * D;
        int32_t err = 0;
        const int taken = pairwise ? pairwise_search(a, d1, fw, fl, fwt, n_flat, tf, tb, leaf)
                                   : orc_search_tree(n, F, NB, D, a->score_function, a->bins_fm, a->border_counts,
                                                     d1, eff, scaled_l2, 0, &unused, tf, tb, leaf, &err);
        if (err || taken < 0) {
            rc = -3;
            break;
        }
        const int32_t nl = 1 << taken;
        /* stored leaves: the model approximant's resample */
        yeti_phase_ders(a, approx, gw, sv, cwbuf, d1, d2, NULL, fw, fl, fwt, nf);
        for (int32_t q = 0; q < L; ++q) {
            lv[q] = 0.0;
            lw[q] = 0.0;
        }
        if (pairwise) pairwise_leaf_deltas(fw, fl, fwt, n_flat, leaf, d1, n, nl, a->l2_leaf_reg, lv);
        else newton_unit(d1, d2, leaf, n, nl, scaled_l2, lv);
        for (int64_t i = 0; i < n; ++i) lw[leaf[i]] += w[i];
        if (o->raw_leaf_values) memcpy(o->raw_leaf_values + (size_t)it * L, lv, sizeof(double) * L);
        const double total = orc_sum_f64(lw, nl);
        if (fabs(total) > 1e-9) {
            for (int32_t q = 0; q < nl; ++q) tmp[q] = lv[q] * lw[q];
            const double avg = orc_sum_f64(tmp, nl) / total;
            for (int32_t q = 0; q < nl; ++q) lv[q] = fabs(lw[q]) > 1e-9 ? lv[q] - avg : 0.0;
        }
        for (int32_t q = 0; q < nl; ++q) lv[q] *= lr;
        memcpy(o->leaf_values + (size_t)it * L, lv, sizeof(double) * L);
        for (int64_t i = 0; i < n; ++i) approx[i] += lv[leaf[i]];
        /* the learning fold's own resample, Newton (or Cholesky) deltas x lr (no centring) */
        yeti_phase_ders(a, lapprox, gw, sl, cwbuf, d1, d2, NULL, fw, fl, fwt, nf);
        if (pairwise) pairwise_leaf_deltas(fw, fl, fwt, n_flat, leaf, d1, n, nl, a->l2_leaf_reg, lv);
        else newton_unit(d1, d2, leaf, n, nl, scaled_l2, lv);
        for (int64_t i = 0; i < n; ++i) lapprox[i] += lv[leaf[i]] * lr;
        if (o->staged) memcpy(o->staged + (size_t)it * n, approx, sizeof(double) * (size_t)n);
    }
    free(w); free(gw); free(cwbuf); free(approx); free(lapprox); free(d1); free(d2); free(eff); free(tmp);
    free(leaf); free(lv); free(lw); free(seeds); free(fw); free(fl); free(fwt);
    return rc;
}

/* The StochasticRank loop: the YetiRank seeder's derivative and leaf-value
 * recalc seeds per tree (boosting.rs:5065-5100, 7331-7345, 8135-8170), each
 * group's noise seeded with base + group index; one approximant; Gradient
 * leaves over unit weights; no centring. */
static int train_stochasticrank(const orc_rank_args* a, orc_rank_out* o, int32_t NB) {
    const int64_t n = a->n;
    const int32_t F = a->n_features, D = a->depth, L = 1 << D, G = a->n_groups;
    double* w = (double*)calloc((size_t)n + 1, sizeof(double));
    for (int64_t i = 0; i < n; ++i) w[i] = a->weights ? a->weights[i] : 1.0;
    const double sum_w = orc_sum_f64(w, n);
    const double scaled_l2 = n == 0 ? a->l2_leaf_reg : a->l2_leaf_reg * (sum_w / (double)n);
    const double lr = (double)(float)a->learning_rate;
    int64_t maxg = 1;
    for (int32_t gi = 0; gi < G; ++gi)
        if (a->group_offsets[gi + 1] - a->group_offsets[gi] > maxg) maxg = a->group_offsets[gi + 1] - a->group_offsets[gi];
    double* ws = (double*)malloc(sizeof(double) * (size_t)(9 * maxg + 3));
    int64_t* order = (int64_t*)malloc(sizeof(int64_t) * (size_t)maxg);
    double* approx = (double*)calloc((size_t)n + 1, sizeof(double));
    double* d1 = (double*)malloc(sizeof(double) * ((size_t)n + 1));
    double* d2 = (double*)malloc(sizeof(double) * ((size_t)n + 1));
    int32_t* leaf = (int32_t*)malloc(sizeof(int32_t) * ((size_t)n + 1));
    double* lv = (double*)malloc(sizeof(double) * L);
    double* cnt = (double*)malloc(sizeof(double) * L);
    orc_rng seeder, unused;
    orc_rng_from_seed(&seeder, a->random_seed);
    orc_rng_from_seed(&unused, a->random_seed);
    int rc = 0;
    for (int32_t it = 0; it < a->iterations; ++it) {
        uint64_t rs[3];
        yeti_next_tree(&seeder, G, F, D, NULL, NULL, NULL, rs);
        for (int32_t phase = 0; phase < 2; ++phase) {
            const uint64_t base = phase == 0 ? rs[0] : rs[2];
            for (int32_t gi = 0; gi < G; ++gi) {
                const int64_t b = a->group_offsets[gi], e = a->group_offsets[gi + 1];
                stochastic_rank_group(approx + b, a->target + b, e - b, a->srank_ndcg, a->srank_sigma, a->srank_mu,
                                      a->srank_num_estimations, base + (uint64_t)gi, ws, order, d1 + b, d2 + b);
            }
            if (phase == 0) {
                int32_t* tf = o->split_feature + (size_t)it * D;
                int32_t* tb = o->split_bin + (size_t)it * D;
                int32_t err = 0;
                orc_search_tree(n, F, NB, D, a->score_function, a->bins_fm, a->border_counts, d1, w, scaled_l2, 0,
                                &unused, tf, tb, leaf, &err);
                if (err) {
                    rc = -3;
                    break;
                }
            }
        }
        if (rc) break;
        for (int32_t q = 0; q < L; ++q) {
            lv[q] = 0.0;
            cnt[q] = 0.0;
        }
        for (int64_t i = 0; i < n; ++i) {
            lv[leaf[i]] += d1[i];
            cnt[leaf[i]] += 1.0;
        }
        for (int32_t q = 0; q < L; ++q) lv[q] = cnt[q] > 0.0 ? lv[q] / (cnt[q] + scaled_l2) : 0.0;
        if (o->raw_leaf_values) memcpy(o->raw_leaf_values + (size_t)it * L, lv, sizeof(double) * L);
        for (int32_t q = 0; q < L; ++q) lv[q] *= lr;
        memcpy(o->leaf_values + (size_t)it * L, lv, sizeof(double) * L);
        for (int64_t i = 0; i < n; ++i) approx[i] += lv[leaf[i]];
        if (o->staged) memcpy(o->staged + (size_t)it * n, approx, sizeof(double) * (size_t)n);
    }
    free(w); free(ws); free(order); free(approx); free(d1); free(d2); free(leaf); free(lv); free(cnt);
    return rc;
}

/* ---- pairwise scoring (crates/cb-compute/src/pairwise_scoring.rs) ------- */

/* make_zero_average (pairwise_leaves.rs:202-212) */
static void make_zero_average(double* v, int32_t n) {
    if (n == 0) return;
    const double avg = orc_sum_f64(v, n) / (double)n;
    for (int32_t i = 0; i < n; ++i) v[i] -= avg;
}

/* calculate_pairwise_leaf_values (pairwise_leaves.rs:113-200): the n x n
 * weight matrix w (row-major) and der vector -> n zero-averaged values. */
static void pairwise_leaf_values(const double* w, const double* der, int32_t n, double l2, double prior,
                                 double* out) {
    if (n == 0) return;
    if (n == 1) {
        out[0] = 0.0;
        return;
    }
    const double cell_prior = 1.0 / (double)n;
    const double non_diag = -prior * cell_prior;
    const double diag = prior * (1.0 - cell_prior) + l2;
    if (n == 2) {
        const double den = w[0] + diag;
        out[0] = den != 0.0 ? der[0] / den : 0.0;
        out[1] = 0.0;
        make_zero_average(out, 2);
        return;
    }
    const int32_t m = n - 1;
    double* A = (double*)calloc((size_t)m * m * 2 + (size_t)m * 2, sizeof(double));
    double* L = A + (size_t)m * m;
    double* y = L + (size_t)m * m;
    double* x = y + m;
    for (int32_t r = 0; r < m; ++r) {
        for (int32_t c = 0; c < r; ++c) {
            const double v = w[(size_t)r * n + c] + non_diag;
            A[(size_t)r * m + c] = v;
            A[(size_t)c * m + r] = v;
        }
        A[(size_t)r * m + r] = w[(size_t)r * n + r] + diag;
    }
    if (orc_cholesky_solve(A, der, m, L, y, x)) {
        for (int32_t i = 0; i < m; ++i) out[i] = x[i];
    } else {
        for (int32_t i = 0; i < m; ++i) out[i] = 0.0;
    }
    out[m] = 0.0;
    make_zero_average(out, n);
    free(A);
}

/* calculate_score (pairwise_scoring.rs:367-391) */
static double pairwise_score(const double* avrg, const double* der, const double* w, int32_t n, double* tmp) {
    double outer = 0.0;
    for (int32_t x = 0; x < n; ++x) {
        for (int32_t y = 0; y < n; ++y) tmp[y] = avrg[y] * w[(size_t)x * n + y];
        const double sub = orc_sum_f64(tmp, n);
        outer += avrg[x] * (der[x] - 0.5 * sub);
    }
    return outer;
}

#define WS(r, c) ws[(size_t)(r) * n2 + (c)]

/* One feature's pairwise scores over its B - 1 borders at a level with P
 * leaves (compute_der_sums + compute_pair_weight_statistics +
 * calculate_pairwise_score, pairwise_scoring.rs:101-580): the bucket of a
 * row is its bin. */
static void pairwise_feature_scores(const uint8_t* col, int64_t n, int32_t B, const int32_t* leaf_of, int32_t P,
                                    const double* der1, const int64_t* pw, const int64_t* pl, const double* pwt,
                                    int64_t n_pairs, double l2, double prior, double* scores) {
    const int32_t n2 = 2 * P;
    double* ds = (double*)calloc((size_t)P * B, sizeof(double));        /* [P][B] */
    double* sm = (double*)calloc((size_t)P * P * B, sizeof(double));    /* smaller [P][P][B] */
    double* gr = (double*)calloc((size_t)P * P * B, sizeof(double));    /* greater-right [P][P][B] */
    double* ws = (double*)calloc((size_t)n2 * n2, sizeof(double));
    double* dsum = (double*)calloc((size_t)n2, sizeof(double));
    double* lv = (double*)malloc(sizeof(double) * (size_t)n2);
    double* tmp = (double*)malloc(sizeof(double) * (size_t)(n2 > 2 * B ? n2 : 2 * B));
    for (int64_t i = 0; i < n; ++i) ds[(size_t)leaf_of[i] * B + col[i]] += der1[i];
    for (int64_t k = 0; k < n_pairs; ++k) {
        const int64_t wv = pw[k], lo = pl[k];
        if (wv == lo) continue;
        const int32_t wb = col[wv], wl = leaf_of[wv], lb = col[lo], ll = leaf_of[lo];
        const double wt = pwt ? pwt[k] : 1.0;
        if (wb > lb) {
            sm[((size_t)ll * P + wl) * B + lb] -= wt;
            gr[((size_t)ll * P + wl) * B + wb] -= wt;
        } else {
            sm[((size_t)wl * P + ll) * B + wb] -= wt;
            gr[((size_t)wl * P + ll) * B + lb] -= wt;
        }
    }
    for (int32_t q = 0; q < P; ++q) dsum[2 * q + 1] += orc_sum_f64(ds + (size_t)q * B, B);
    for (int32_t y = 0; y < P; ++y)
        for (int32_t x = y + 1; x < P; ++x) {
            for (int32_t b = 0; b < B; ++b) {
                tmp[2 * b] = sm[((size_t)x * P + y) * B + b];
                tmp[2 * b + 1] = sm[((size_t)y * P + x) * B + b];
            }
            const double t = orc_sum_f64(tmp, 2 * B);
            WS(2 * y + 1, 2 * x + 1) += t;
            WS(2 * x + 1, 2 * y + 1) += t;
            WS(2 * x + 1, 2 * x + 1) += -t;
            WS(2 * y + 1, 2 * y + 1) += -t;
        }
    for (int32_t b = 0; b < B - 1; ++b) {
        for (int32_t y = 0; y < P; ++y) {
            const double dd = ds[(size_t)y * B + b];
            dsum[2 * y] += dd;
            dsum[2 * y + 1] += -dd;
            const double wd = sm[((size_t)y * P + y) * B + b] - gr[((size_t)y * P + y) * B + b];
            WS(2 * y, 2 * y + 1) += wd;
            WS(2 * y + 1, 2 * y) += wd;
            WS(2 * y, 2 * y) += -wd;
            WS(2 * y + 1, 2 * y + 1) += -wd;
            for (int32_t x = y + 1; x < P; ++x) {
                const size_t ixy = ((size_t)x * P + y) * B + b, iyx = ((size_t)y * P + x) * B + b;
                const double w00 = gr[ixy] + gr[iyx];
                const double w01 = sm[ixy] - gr[ixy];
                const double w10 = sm[iyx] - gr[iyx];
                const double w11 = -(sm[ixy] + sm[iyx]);
                WS(2 * x, 2 * y) += w00;
                WS(2 * y, 2 * x) += w00;
                WS(2 * x, 2 * y + 1) += w01;
                WS(2 * y + 1, 2 * x) += w01;
                WS(2 * x + 1, 2 * y) += w10;
                WS(2 * y, 2 * x + 1) += w10;
                WS(2 * x + 1, 2 * y + 1) += w11;
                WS(2 * y + 1, 2 * x + 1) += w11;
                WS(2 * y, 2 * y) += -(w00 + w10);
                WS(2 * x, 2 * x) += -(w00 + w01);
                WS(2 * x + 1, 2 * x + 1) += -(w10 + w11);
                WS(2 * y + 1, 2 * y + 1) += -(w01 + w11);
            }
        }
        pairwise_leaf_values(ws, dsum, n2, l2, prior, lv);
        scores[b] = pairwise_score(lv, dsum, ws, n2, tmp);
    }
    free(ds);
    free(sm);
    free(gr);
    free(ws);
    free(dsum);
    free(lv);
    free(tmp);
}
#undef WS

/* compute_pairwise_leaf_deltas (pairwise_leaves.rs:219-242): the leaf
 * pair-weight matrix in the pairs' order, the ordered leaf der sums, the
 * Cholesky system with the raw l2 and the 0.1 prior. */
static void pairwise_leaf_deltas(const int64_t* pw, const int64_t* pl, const double* pwt, int64_t n_pairs,
                                 const int32_t* leaf, const double* d1, int64_t n, int32_t nl, double l2, double* lv) {
    double* wsum = (double*)calloc((size_t)nl * nl, sizeof(double));
    double* dsl = (double*)calloc((size_t)nl, sizeof(double));
    for (int64_t k = 0; k < n_pairs; ++k) {
        const int32_t wl = leaf[pw[k]], ll = leaf[pl[k]];
        if (wl == ll) continue;
        const double wt = pwt ? pwt[k] : 1.0;
        wsum[(size_t)wl * nl + ll] -= wt;
        wsum[(size_t)ll * nl + wl] -= wt;
        wsum[(size_t)wl * nl + wl] += wt;
        wsum[(size_t)ll * nl + ll] += wt;
    }
    for (int64_t i = 0; i < n; ++i) dsl[leaf[i]] += d1[i];
    pairwise_leaf_values(wsum, dsl, nl, l2, 0.1, lv);
    free(wsum);
    free(dsl);
}

/* the pairwise greedy search (tree.rs:3861-3960): per level, every feature's
 * pairwise scores, strict first-wins over (feature, border). */
static int pairwise_search(const orc_rank_args* a, const double* der1, const int64_t* pw, const int64_t* pl,
                           const double* pwt, int64_t n_pairs, int32_t* feat, int32_t* sbin, int32_t* leaf_of) {
    const int64_t n = a->n;
    double* sc = (double*)malloc(sizeof(double) * 256);
    for (int64_t i = 0; i < n; ++i) leaf_of[i] = 0;
    for (int32_t level = 0; level < a->depth; ++level) {
        const int32_t P = 1 << level;
        double best = -INFINITY;
        int32_t bf = -1, bb = -1;
        for (int32_t f = 0; f < a->n_features; ++f) {
            const int32_t nb = a->border_counts[f];
            if (nb == 0) continue;
            pairwise_feature_scores(a->bins_fm + (size_t)f * n, n, nb + 1, leaf_of, P, der1, pw, pl, pwt, n_pairs,
                                    a->l2_leaf_reg, 0.1, sc);
            for (int32_t b = 0; b < nb; ++b)
                if (sc[b] > best) {
                    best = sc[b];
                    bf = f;
                    bb = b;
                }
        }
        if (bf < 0) {
            free(sc);
            return -1;
        }
        feat[level] = bf;
        sbin[level] = bb;
        const uint8_t* col = a->bins_fm + (size_t)bf * n;
        for (int64_t i = 0; i < n; ++i)
            if ((int32_t)col[i] > bb) leaf_of[i] += P;
    }
    free(sc);
    return a->depth;
}

int orc_train_ranking(const orc_rank_args* a, orc_rank_out* o) {
    const int64_t n = a->n;
    const int32_t F = a->n_features, D = a->depth, L = 1 << D;
    if (D < 1 || D > 16 || a->n_groups < 0) return -1;
    if (a->n_groups > 0 && (a->group_offsets[0] != 0 || a->group_offsets[a->n_groups] != n)) return -1;
    int32_t NB = 1;
    for (int32_t f = 0; f < F; ++f)
        if (a->border_counts[f] + 1 > NB) NB = a->border_counts[f] + 1;
    if (a->loss == ORC_RANK_YETIRANK || a->loss == ORC_RANK_YETIRANK_PAIRWISE) return train_yetirank(a, o, NB);
    if (a->loss == ORC_RANK_STOCHASTICRANK) return train_stochasticrank(a, o, NB);
    competitors cp = {NULL, NULL, NULL};
    const int pairlogit = a->loss == ORC_RANK_PAIRLOGIT || a->loss == ORC_RANK_PAIRLOGIT_PAIRWISE;
    if (pairlogit && build_competitors(a, &cp) != 0) {
        free(cp.start);
        free(cp.loser);
        free(cp.weight);
        return -2;
    }
    if (a->loss == ORC_RANK_PAIRLOGIT_PAIRWISE && a->pair_weight) {
        /* the pairwise statistics here take unit pair weights */
        for (int64_t k = 0; k < a->n_pairs; ++k)
            if (a->pair_weight[k] != 1.0) {
                free(cp.start);
                free(cp.loser);
                free(cp.weight);
                return -3;
            }
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
    int64_t* lm_order = (int64_t*)malloc(sizeof(int64_t) * ((size_t)n + 1));
    double* lv = (double*)malloc(sizeof(double) * L);
    double* lw = (double*)malloc(sizeof(double) * L);

    /* histogram weights: pairwise weights for PairLogit, object weights otherwise */
    if (pairlogit) {
        for (int64_t i = 0; i < n; ++i) eff[i] = 0.0;
        for (int32_t g = 0; g < a->n_groups; ++g)
            for (int64_t wi = a->group_offsets[g]; wi < a->group_offsets[g + 1]; ++wi)
                for (int64_t k = cp.start[wi]; k < cp.start[wi + 1]; ++k) {
                    eff[wi] += cp.weight[k];
                    eff[cp.loser[k]] += cp.weight[k];
                }
    } else {
        for (int64_t i = 0; i < n; ++i) eff[i] = w[i];
    }
    for (int64_t i = 0; i < n; ++i) sh[i] = eff[i]; /* no bootstrap: control 1, sample weight 1 */

    /* flatten_global_pairs (tree.rs:3747-3760): group, winner, competitor order */
    int64_t n_flat = 0;
    int64_t* pairs_w = (int64_t*)malloc(sizeof(int64_t) * (size_t)(a->n_pairs > 0 ? a->n_pairs : 1));
    int64_t* pairs_l = (int64_t*)malloc(sizeof(int64_t) * (size_t)(a->n_pairs > 0 ? a->n_pairs : 1));
    if (pairlogit)
        for (int32_t g = 0; g < a->n_groups; ++g)
            for (int64_t wi = a->group_offsets[g]; wi < a->group_offsets[g + 1]; ++wi)
                for (int64_t k = cp.start[wi]; k < cp.start[wi + 1]; ++k) {
                    pairs_w[n_flat] = wi;
                    pairs_l[n_flat] = cp.loser[k];
                    ++n_flat;
                }

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
            if (a->loss == ORC_RANK_LAMBDAMART) {
                /* MRR / ERR / MAP: the reference accepts the metric and leaves
                 * the group's ders at zero (ranking_der.rs:574-581) */
                if (!a->lambdamart_no_op)
                    lambdamart_group(approx + b, a->target + b, e - b, a->lambdamart_sigma, a->lambdamart_top,
                                     a->lambdamart_norm, lm_order, tmp, d1 + b, d2 + b);
            } else if (a->loss == ORC_RANK_QUERYSOFTMAX) {
                const double beta = a->softmax_beta, lambda = a->softmax_lambda;
                double max_a = -DBL_MAX;
                int64_t nt = 0;
                for (int64_t i = b; i < e; ++i)
                    if (w[i] > 0.0) {
                        if (approx[i] > max_a) max_a = approx[i];
                        if (a->target[i] > 0.0) tmp[nt++] = w[i] * a->target[i];
                    }
                const double swt = orc_sum_f64(tmp, nt);
                if (swt > 0.0) {
                    for (int64_t i = b; i < e; ++i) tmp[i - b] = exp(beta * (approx[i] - max_a)) * w[i];
                    const double sum_exp = orc_sum_f64(tmp, e - b);
                    for (int64_t i = b; i < e; ++i) {
                        if (w[i] > 0.0 && sum_exp > 0.0) {
                            const double p = tmp[i - b] / sum_exp;
                            d2[i] = beta * swt * (beta * p * (p - 1.0) - lambda);
                            d1[i] = beta * (-swt * p + w[i] * a->target[i]);
                        }
                    }
                }
            } else if (a->loss == ORC_RANK_QUERYRMSE) {
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
                        const double pw = cp.weight[k];
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
        int taken;
        if (a->loss == ORC_RANK_PAIRLOGIT_PAIRWISE) {
            /* pairwise scoring over the flattened competitor pairs (tree.rs:3747-3760) */
            taken = pairwise_search(a, d1, pairs_w, pairs_l, NULL, n_flat, tf, tb, leaf);
            if (taken < 0) {
                rc = -3;
                break;
            }
        } else {
            int32_t err = 0;
            taken = orc_search_tree(n, F, NB, D, a->score_function, a->bins_fm, a->border_counts, d1, sh, scaled_l2,
                                    0, &rng, tf, tb, leaf, &err);
            if (err) {
                rc = -3;
                break;
            }
        }
        const int32_t nl = 1 << taken;
        /* 4. Newton leaves over unit leaf weights, ordered per-leaf sums */
        double* sd = (double*)calloc((size_t)nl * 4, sizeof(double));
        for (int64_t i = 0; i < n; ++i) {
            sd[4 * leaf[i]] += d1[i];
            sd[4 * leaf[i] + 1] += d2[i] * 1.0;
            sd[4 * leaf[i] + 2] += w[i];
            sd[4 * leaf[i] + 3] += 1.0;
        }
        for (int32_t q = 0; q < L; ++q) {
            lv[q] = 0.0;
            lw[q] = 0.0;
        }
        for (int32_t q = 0; q < nl; ++q) {
            if (a->loss == ORC_RANK_QUERYSOFTMAX) {
                const double cnt = sd[4 * q + 3];
                lv[q] = cnt > 0.0 ? sd[4 * q] / (cnt + scaled_l2) : 0.0;
            } else {
                const double den = -sd[4 * q + 1] + scaled_l2;
                lv[q] = den == 0.0 ? 0.0 : sd[4 * q] / den;
            }
            lw[q] = sd[4 * q + 2];
        }
        free(sd);
        if (a->loss == ORC_RANK_PAIRLOGIT_PAIRWISE) {
            /* compute_pairwise_leaf_deltas (pairwise_leaves.rs:219-242): the
             * leaf pair-weight matrix in group / winner / competitor order, the
             * ordered leaf der sums, the Cholesky system with the raw l2 */
            pairwise_leaf_deltas(pairs_w, pairs_l, NULL, n_flat, leaf, d1, n, nl, a->l2_leaf_reg, lv);
        }
        if (o->raw_leaf_values) memcpy(o->raw_leaf_values + (size_t)it * L, lv, sizeof(double) * L);
        /* 5. normalize_leaf_values */
        if (pairlogit) {
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
    free(cp.weight);
    free(pairs_w);
    free(pairs_l);
    free(w); free(approx); free(d1); free(d2); free(eff); free(sh); free(tmp); free(leaf); free(lv); free(lw);
    free(lm_order);
    return rc;
}
