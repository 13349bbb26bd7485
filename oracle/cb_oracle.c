/*
 * cb_oracle.c -- CPU restatement of catboost_rs's oblivious-tree training path.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA implementation and
 * the CPU baseline that bench.py times.  The product path never calls it.
 *
 * Build: gcc -O2 -ffp-contract=off -fopenmp -shared -fPIC (no FMA contraction so
 * every f64/f32 operation rounds exactly as the reference's Rust code does).
 * Citations are file:line inside the reference project.
 */
#include "cb_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ======================================================================== */
/* TFastRng64 -- crates/cb-core/src/rng.rs:26-292                           */
/* ======================================================================== */

#define LCG_A 6364136223846793005ULL /* rng.rs:26 */

/* PCG XSH-RR output mix (rng.rs:31-38). */
static inline uint32_t pcg_mix(uint64_t x) {
    uint32_t xs = (uint32_t)(((x >> 18) ^ x) >> 27);
    uint32_t rot = (uint32_t)(x >> 59);
    return (xs >> rot) | (xs << ((32u - rot) & 31u));
}

/* O(log delta) LCG jump: x_n = A^n x_0 + (A^n - 1)/(A - 1) c (rng.rs:45-69). */
static uint64_t lcg_advance(uint64_t seed, uint64_t a, uint64_t c, uint64_t delta) {
    uint64_t mask = 1;
    while (mask != (1ULL << 63) && (mask << 1) <= delta) mask <<= 1;
    uint64_t apow = 1, adiv = 0;
    while (mask != 0) {
        adiv = adiv * (apow + 1);
        apow = apow * apow;
        if (delta & mask) {
            adiv = adiv + apow;
            apow = apow * a;
        }
        mask >>= 1;
    }
    return seed * apow + c * adiv;
}

static inline uint32_t lcg_gen32(uint64_t* x, uint64_t c) {
    *x = *x * LCG_A + c;
    return pcg_mix(*x);
}

/* FixSeq (rng.rs:128-136). */
static uint32_t fix_seq(uint32_t s1, uint32_t s2) {
    const uint32_t m = 0x7fffffffu;
    return ((s1 & m) == (s2 & m)) ? ~s2 : s2;
}

void orc_rng_new(orc_rng* r, uint64_t seed1, uint32_t seq1, uint64_t seed2, uint32_t seq2) {
    r->x1 = seed1;
    r->c1 = ((uint64_t)seq1 << 1) | 1u;
    r->x2 = seed2;
    r->c2 = ((uint64_t)fix_seq(seq1, seq2) << 1) | 1u;
    r->calls = 0;
}

/* One-seed constructor: parameters drawn from TReallyFastRng32(seed)
 * (rng.rs:171-179): Seed1 = GenRand64, Seq1 = GenRand, Seed2, Seq2. */
void orc_rng_from_seed(orc_rng* r, uint64_t seed) {
    uint64_t x = seed;
    uint64_t lo, hi;
    lo = lcg_gen32(&x, 1);
    hi = lcg_gen32(&x, 1);
    uint64_t seed1 = lo | (hi << 32);
    uint32_t seq1 = lcg_gen32(&x, 1);
    lo = lcg_gen32(&x, 1);
    hi = lcg_gen32(&x, 1);
    uint64_t seed2 = lo | (hi << 32);
    uint32_t seq2 = lcg_gen32(&x, 1);
    orc_rng_new(r, seed1, seq1, seed2, seq2);
}

/* Stream 1 gives the high word, stream 2 the low word (rng.rs:183-189). */
uint64_t orc_rng_gen(orc_rng* r) {
    uint64_t hi = lcg_gen32(&r->x1, r->c1);
    uint64_t lo = lcg_gen32(&r->x2, r->c2);
    r->calls++;
    return (hi << 32) | lo;
}

/* (GenRand() >> 11) * (1 / (2^53 - 1)) (rng.rs:256-259). */
double orc_rng_real1(orc_rng* r) {
    return (double)(orc_rng_gen(r) >> 11) * (1.0 / 9007199254740991.0);
}

void orc_rng_advance(orc_rng* r, uint64_t delta) {
    r->x1 = lcg_advance(r->x1, LCG_A, r->c1, delta);
    r->x2 = lcg_advance(r->x2, LCG_A, r->c2, delta);
    r->calls += delta;
}

/* Rejection-sampled Uniform (rng.rs:269-292). */
uint64_t orc_rng_uniform(orc_rng* r, uint64_t bound) {
    if (bound == 0) return 0;
    uint64_t randmax = UINT64_MAX - (UINT64_MAX % bound);
    for (;;) {
        uint64_t v = orc_rng_gen(r);
        if (v < randmax) return v % bound;
    }
}

/* Marsaglia polar StdNormalDistribution (crates/cb-core/src/normal.rs). */
double orc_std_normal(orc_rng* r) {
    for (;;) {
        double x = orc_rng_real1(r) * 2.0 - 1.0;
        double y = orc_rng_real1(r) * 2.0 - 1.0;
        double rr = x * x + y * y;
        if (!(rr > 1.0 || rr <= 0.0)) return x * sqrt(-2.0 * log(rr) / rr);
    }
}

/* ======================================================================== */
/* FastLog2f / FastLogf -- crates/cb-train/src/fast_approx.rs:154-188        */
/* ======================================================================== */

float orc_fast_log2f(float value) {
    uint32_t vx;
    memcpy(&vx, &value, 4);
    uint32_t mxi = (vx & 0x007FFFFFu) | 0x3f000000u;
    float mx;
    memcpy(&mx, &mxi, 4);
    float y = (float)vx;
    y *= 1.1920928955078125e-7f;
    return y - 124.22551499f - 1.498030302f * mx - 1.72587999f / (0.3520887068f + mx);
}

float orc_fast_logf(float value) { return 0.69314718f * orc_fast_log2f(value); }

/* ======================================================================== */
/* reductions -- crates/cb-core/src/reduction.rs (strict left-to-right)     */
/* ======================================================================== */

double orc_sum_f64(const double* v, int64_t n) {
    double acc = 0.0;
    for (int64_t i = 0; i < n; ++i) acc += v[i];
    return acc;
}

/* ======================================================================== */
/* quantization -- crates/cb-compute/src/histogram.rs:159-165               */
/* bin = #{k : borders[k] < value}; NaN -> top bin when the last border is   */
/* the f32::MAX sentinel (nan_mode=Max), else bin 0 (nan_mode=Min).          */
/* ======================================================================== */

static inline uint32_t bin_of(const double* borders, int32_t nb, float value) {
    if (isnan(value) && nb > 0 && borders[nb - 1] == (double)FLT_MAX) return (uint32_t)nb;
    double v = (double)value;
    uint32_t c = 0;
    for (int32_t k = 0; k < nb; ++k) c += (borders[k] < v) ? 1u : 0u;
    return c;
}

void orc_quantize(const float* cols, int64_t n, int32_t F, const double* borders_flat,
                  const int32_t* border_counts, uint8_t* out) {
    int64_t* off = (int64_t*)malloc(sizeof(int64_t) * (size_t)(F + 1));
    off[0] = 0;
    for (int32_t f = 0; f < F; ++f) off[f + 1] = off[f] + border_counts[f];
#pragma omp parallel for schedule(static)
    for (int32_t f = 0; f < F; ++f) {
        const double* b = borders_flat + off[f];
        for (int64_t i = 0; i < n; ++i)
            out[(int64_t)f * n + i] = (uint8_t)bin_of(b, border_counts[f], cols[(int64_t)f * n + i]);
    }
    free(off);
}

/* ======================================================================== */
/* derivatives -- crates/cb-compute/src/loss.rs:35-80                        */
/* ======================================================================== */

void orc_compute_gradients(int32_t loss, const double* approx, const double* target, int64_t n,
                           double* der1, double* der2) {
    for (int64_t i = 0; i < n; ++i) {
        if (loss == ORC_LOSS_RMSE) {
            der1[i] = target[i] - approx[i];
            if (der2) der2[i] = -1.0;
        } else {
            double e = exp(approx[i]);
            double p = 1.0 - 1.0 / (1.0 + e);
            der1[i] = target[i] - p;
            if (der2) der2[i] = -p * (1.0 - p);
        }
    }
}

/* ======================================================================== */
/* bootstrap -- crates/cb-train/src/bootstrap.rs                            */
/* ======================================================================== */

#define BAYESIAN_BLOCK 1000 /* bootstrap.rs BAYESIAN_BLOCK_SIZE */
#define MVS_BLOCK 8192      /* bootstrap.rs MVS_BLOCK_SIZE */

/* bayesian_weight: w = powf(-FastLogf((f32)u + 1e-100f), T).  The 1e-100
 * literal rounds to 0.0f in f32, so the addend is +0.0f. */
static double bayesian_weight(float temp, orc_rng* r) {
    double u = orc_rng_real1(r);
    float w = -orc_fast_logf((float)u + 0.0f);
    return (double)powf(w, temp);
}

static void generate_random_weights(int64_t n, float temp, orc_rng* r, double* w) {
    if (temp == 0.0f) {
        for (int64_t i = 0; i < n; ++i) w[i] = 1.0;
        return;
    }
    uint64_t rand_seed = orc_rng_gen(r);
    int64_t blocks = (n + BAYESIAN_BLOCK - 1) / BAYESIAN_BLOCK;
    for (int64_t b = 0; b < blocks; ++b) {
        orc_rng br;
        orc_rng_from_seed(&br, rand_seed + (uint64_t)b);
        orc_rng_advance(&br, 10);
        int64_t beg = b * BAYESIAN_BLOCK, end = beg + BAYESIAN_BLOCK < n ? beg + BAYESIAN_BLOCK : n;
        for (int64_t i = beg; i < end; ++i) w[i] = bayesian_weight(temp, &br);
    }
}

static double single_probability(double d, double thr) {
    if (d > thr) return 1.0;
    if (thr > 0.0) return d / thr;
    return 0.0;
}

/* calculate_threshold (bootstrap.rs:205-269): quickselect-style recursion on
 * the first element with sequential f64 partial sums.  `buf` has room for the
 * recursion's stable partitions. */
static double calculate_threshold(double* cand, int64_t len, double sum_small_cur,
                                  double n_large_cur, double sample_size, double* scratch) {
    for (;;) {
        if (len == 0) return 0.0;
        double thr = cand[0];
        /* stable 3-way partition: small first, then large into scratch */
        int64_t ns = 0, nm = 0, nl = 0;
        double sum_small_upd = 0.0;
        for (int64_t i = 0; i < len; ++i) {
            double c = cand[i];
            if (c < thr) {
                sum_small_upd += c;
                scratch[ns++] = c;
            } else if (c <= thr) {
                nm++;
            }
        }
        double* large = scratch + ns;
        for (int64_t i = 0; i < len; ++i) {
            double c = cand[i];
            if (!(c < thr) && !(c <= thr)) large[nl++] = c;
        }
        double n_large_upd = (double)nl;
        double n_middle = (double)nm;
        double sum_middle = n_middle * thr;
        double est;
        if (thr != 0.0)
            est = (sum_small_cur + sum_small_upd) / thr + n_large_cur + n_large_upd + n_middle;
        else
            est = INFINITY;
        if (est > sample_size) {
            if (nl > 0) {
                double next_small = sum_small_cur + sum_middle + sum_small_upd;
                memmove(cand, large, sizeof(double) * (size_t)nl);
                len = nl;
                sum_small_cur = next_small;
                continue;
            }
            double denom = sample_size - n_large_cur;
            return denom != 0.0 ? (sum_small_cur + sum_small_upd + sum_middle) / denom : thr;
        } else if (ns > 0) {
            double next_large = n_large_cur + n_large_upd + n_middle;
            memmove(cand, scratch, sizeof(double) * (size_t)ns);
            len = ns;
            n_large_cur = next_large;
            continue;
        } else {
            double denom = sample_size - n_large_cur - n_middle - n_large_upd;
            return denom != 0.0 ? sum_small_cur / denom : thr;
        }
    }
}

static void mvs_sample_weights(const double* der, int64_t n, double lambda, double rate_in,
                               orc_rng* r, double* w) {
    if (rate_in >= 1.0) {
        for (int64_t i = 0; i < n; ++i) w[i] = 1.0;
        return;
    }
    double rate = (double)(float)rate_in;
    uint64_t rand_seed = orc_rng_gen(r);
    int64_t blocks = (n + MVS_BLOCK - 1) / MVS_BLOCK;
    double* cand = (double*)malloc(sizeof(double) * MVS_BLOCK);
    double* scratch = (double*)malloc(sizeof(double) * MVS_BLOCK);
    for (int64_t b = 0; b < blocks; ++b) {
        orc_rng br;
        orc_rng_from_seed(&br, rand_seed + (uint64_t)b);
        orc_rng_advance(&br, 10);
        int64_t beg = b * MVS_BLOCK, end = beg + MVS_BLOCK < n ? beg + MVS_BLOCK : n;
        int64_t bs = end - beg;
        for (int64_t k = 0; k < bs; ++k) {
            double d = der[beg + k];
            cand[k] = sqrt(lambda + d * d);
        }
        double sample_size = (double)((float)rate * (float)bs);
        double thr = calculate_threshold(cand, bs, 0.0, 0.0, sample_size, scratch);
        for (int64_t k = 0; k < bs; ++k) {
            double d = der[beg + k];
            double g2 = d * d;
            double p = single_probability(sqrt(g2 + lambda), thr);
            if (p > DBL_EPSILON) {
                double weight = 1.0 / p;
                double u = orc_rng_real1(&br);
                w[beg + k] = (double)(float)(weight * (double)(u < p));
            } else {
                w[beg + k] = 0.0;
            }
        }
    }
    free(cand);
    free(scratch);
}

int orc_bootstrap(int32_t type, const double* der_obj, int64_t n, double subsample, float temp,
                  int32_t has_prev, double prev_leaf_mean, orc_rng* r, double* sw, uint8_t* ctl) {
    switch (type) {
    case ORC_BOOT_NO:
        for (int64_t i = 0; i < n; ++i) { sw[i] = 1.0; ctl[i] = 1; }
        return 0;
    case ORC_BOOT_BAYESIAN:
        generate_random_weights(n, temp, r, sw);
        for (int64_t i = 0; i < n; ++i) ctl[i] = 1;
        return 0;
    case ORC_BOOT_BERNOULLI: {
        for (int64_t i = 0; i < n; ++i) sw[i] = 1.0;
        if (subsample >= 1.0) {
            for (int64_t i = 0; i < n; ++i) ctl[i] = 1;
        } else {
            double rate = (double)(float)subsample;
            for (int64_t i = 0; i < n; ++i) ctl[i] = orc_rng_real1(r) < rate;
        }
        return 0;
    }
    case ORC_BOOT_MVS: {
        double lambda;
        if (has_prev) {
            lambda = prev_leaf_mean * prev_leaf_mean;
        } else {
            double mean = 0.0;
            if (n > 0) {
                double acc = 0.0;
                for (int64_t i = 0; i < n; ++i) acc += sqrt(der_obj[i] * der_obj[i]);
                mean = acc / (double)n;
            }
            lambda = mean * mean;
        }
        mvs_sample_weights(der_obj, n, lambda, subsample, r, sw);
        for (int64_t i = 0; i < n; ++i) ctl[i] = sw[i] > (double)FLT_EPSILON;
        return 0;
    }
    default:
        return -1;
    }
}

/* ======================================================================== */
/* histogram -- crates/cb-compute/src/histogram.rs:239-294                  */
/* ======================================================================== */

void orc_build_histogram(const uint8_t* bins_fm, int64_t n, int32_t F, int32_t n_bins,
                         const double* g, const double* h, const int32_t* leaf_of,
                         int32_t n_leaves, double* out) {
    memset(out, 0, sizeof(double) * (size_t)n_leaves * F * n_bins * 2);
#pragma omp parallel for schedule(static)
    for (int32_t f = 0; f < F; ++f) {
        const uint8_t* col = bins_fm + (int64_t)f * n;
        for (int64_t o = 0; o < n; ++o) {
            int32_t leaf = leaf_of ? leaf_of[o] : 0;
            if (leaf < 0 || leaf >= n_leaves) continue;
            int32_t b = col[o];
            if (b >= n_bins) continue;
            double* cell = out + (((int64_t)leaf * F + f) * n_bins + b) * 2;
            cell[0] += g[o];
            cell[1] += h[o];
        }
    }
}

/* ======================================================================== */
/* split scoring -- crates/cb-compute/src/score.rs:39-135, leaf.rs:161-180   */
/* ======================================================================== */

static inline double calc_average(double sum_delta, double count, double l2) {
    return count > 0.0 ? sum_delta / (count + l2) : 0.0;
}

double orc_score_term(int32_t score_fn, double sum, double weight) {
    if (score_fn == ORC_SCORE_SOLAR_L2)
        return weight > 1e-20 ? (-sum * sum) * (1.0 + 2.0 * log(weight + 1.0)) / weight : 0.0;
    double adjust;
    if (score_fn == ORC_SCORE_LOO_L2) {
        adjust = weight > 1.0 ? weight / (weight - 1.0) : 0.0;
        adjust *= adjust;
    } else {
        adjust = weight > 2.0 ? weight * (weight - 2.0) / (weight * weight - 3.0 * weight + 1.0) : 0.0;
    }
    return weight > 0.0 ? adjust * (-sum * sum) / weight : 0.0;
}

/* multi_dim_split_score_into at dim 1 (score.rs:192-265): `ld`/`lw` hold the
 * 2P canonical-order leaves (false children 0..P-1, then true children). */
static double split_score(int32_t score_fn, const double* ld, const double* lw, int32_t nleaves,
                          double l2) {
    if (score_fn > ORC_SCORE_L2) {
        double acc = 0.0;
        for (int32_t k = 0; k < nleaves; ++k) acc += orc_score_term(score_fn, ld[k], lw[k]);
        return acc;
    }
    double num = 0.0;
    for (int32_t k = 0; k < nleaves; ++k) {
        double avg = calc_average(ld[k], lw[k], l2);
        num += avg * ld[k];
    }
    if (score_fn == ORC_SCORE_L2) return num;
    double den = 0.0;
    den += 1e-100;
    for (int32_t k = 0; k < nleaves; ++k) {
        double avg = calc_average(ld[k], lw[k], l2);
        den += avg * avg * lw[k];
    }
    return num / sqrt(den);
}

/* scan_and_score_borders_into (histogram.rs:1007-1171) for one feature whose
 * histogram is hist[leaf][bin][2] over n_parent leaves, n_bins wide. */
static void scan_and_score(const double* hist, int32_t n_parent, int32_t n_bins, int32_t n_borders,
                           int32_t score_fn, double l2, double* scores, double* work) {
    double* tot_w = work;
    double* tot_d = tot_w + n_parent;
    double* acc_w = tot_d + n_parent;
    double* acc_d = acc_w + n_parent;
    double* ld = acc_d + n_parent;
    double* lw = ld + 2 * n_parent;
    for (int32_t q = 0; q < n_parent; ++q) {
        const double* row = hist + (int64_t)q * n_bins * 2;
        double sw = 0.0, sd = 0.0;
        for (int32_t b = 0; b < n_bins; ++b) sw += row[2 * b + 1];
        for (int32_t b = 0; b < n_bins; ++b) sd += row[2 * b + 0];
        tot_w[q] = sw;
        tot_d[q] = sd;
        acc_w[q] = 0.0;
        acc_d[q] = 0.0;
    }
    for (int32_t b = 0; b < n_borders; ++b) {
        for (int32_t q = 0; q < n_parent; ++q) {
            const double* cell = hist + ((int64_t)q * n_bins + b) * 2;
            acc_w[q] += cell[1];
            double w_false = acc_w[q];
            double w_true = tot_w[q] - w_false;
            acc_d[q] += cell[0];
            double d_false = acc_d[q];
            double d_true = tot_d[q] - d_false;
            ld[q] = d_false;
            lw[q] = w_false;
            ld[q + n_parent] = d_true;
            lw[q + n_parent] = w_true;
        }
        scores[b] = split_score(score_fn, ld, lw, 2 * n_parent, l2);
    }
}

/* ======================================================================== */
/* greedy oblivious tree search -- crates/cb-train/src/tree.rs:704-1131,     */
/* 1158-1300 (plain), 1403-1680 (perturbed / RNG-drawing)                    */
/* ======================================================================== */

typedef struct {
    int64_t n;
    int32_t F, n_bins, depth, score_fn;
    const uint8_t* bins;
    const int32_t* bc;
    const double *g, *h;
    double l2;
    int draws;        /* perturbed path (draws_active) */
    orc_rng* rng;
    double std_dev;
    int32_t C;                /* one-hot cat features, candidates after the floats */
    const uint8_t* cat_bins;  /* [C][n] */
    double* top2;             /* [depth][2] best and runner-up score per level (plain search), or NULL */
} search_ctx;

/* scan_and_score_one_hot_bins_into (histogram.rs:1160-1290): per parent the
 * totals summed over the bins as the border path does, then per present bin
 * v the TRUE child = the bin's cell, the FALSE child = total - cell. */
static void scan_one_hot(const double* hist, int32_t n_parent, int32_t n_bins, const uint8_t* present,
                         int32_t score_fn, double l2, double* scores, double* work) {
    double* tot_w = work;
    double* tot_d = tot_w + n_parent;
    double* ld = tot_d + n_parent;
    double* lw = ld + 2 * n_parent;
    for (int32_t q = 0; q < n_parent; ++q) {
        const double* row = hist + (int64_t)q * n_bins * 2;
        double sw = 0.0, sd = 0.0;
        for (int32_t b = 0; b < n_bins; ++b) sw += row[2 * b + 1];
        for (int32_t b = 0; b < n_bins; ++b) sd += row[2 * b + 0];
        tot_w[q] = sw;
        tot_d[q] = sd;
    }
    for (int32_t v = 0; v < n_bins; ++v) {
        if (!present[v]) {
            scores[v] = -INFINITY;
            continue;
        }
        for (int32_t q = 0; q < n_parent; ++q) {
            const double* cell = hist + ((int64_t)q * n_bins + v) * 2;
            ld[q] = tot_d[q] - cell[0];
            lw[q] = tot_w[q] - cell[1];
            ld[q + n_parent] = cell[0];
            lw[q + n_parent] = cell[1];
        }
        scores[v] = split_score(score_fn, ld, lw, 2 * n_parent, l2);
    }
}

/* Returns the number of splits taken; fills feat/bin and leaf_of. */
static int search_tree(const search_ctx* c, int32_t* feat, int32_t* sbin, int32_t* leaf_of,
                       int* err) {
    const int64_t n = c->n;
    const int32_t F0 = c->F, C = c->C, F = c->F + c->C, NB = c->n_bins;
    *err = 0;
    if (C > 0 && c->draws) { /* upstream rejects one-hot with draws active (tree.rs:1403-1420) */
        *err = 2;
        return 0;
    }
    /* distinct_bins_ascending (tree.rs:3606-3615): the candidates of each cat column */
    uint8_t* present = (uint8_t*)calloc((size_t)(C > 0 ? C : 1) * (size_t)(NB > 0 ? NB : 1), 1);
    for (int32_t k = 0; k < C; ++k)
        for (int64_t o = 0; o < n; ++o)
            if (c->cat_bins[(int64_t)k * n + o] < NB) present[(size_t)k * NB + c->cat_bins[(int64_t)k * n + o]] = 1;
    double** cur = (double**)calloc((size_t)F, sizeof(double*));
    double* scores_all = (double*)malloc(sizeof(double) * (size_t)F * (size_t)(NB > 0 ? NB : 1));
    for (int64_t o = 0; o < n; ++o) leaf_of[o] = 0;
    int taken = 0;
    for (int32_t level = 0; level < c->depth; ++level) {
        int32_t n_leaves = 1 << level; /* partitions before this split */
        if (c->draws) {
            for (int32_t f = 0; f < F; ++f) (void)orc_rng_real1(c->rng); /* RSM draws */
        }
        int32_t n_par = level == 0 ? 1 : (1 << (level - 1));
        int64_t n_true = 0;
        if (level > 0)
            for (int64_t o = 0; o < n; ++o) n_true += (leaf_of[o] & n_par) != 0;
        int64_t n_false = n - n_true;
        int build_true = (n_true <= n_false);
        double** next = (double**)calloc((size_t)F, sizeof(double*));
#pragma omp parallel for schedule(dynamic, 1)
        for (int32_t f = 0; f < F; ++f) {
            const int cat = f >= F0;
            int32_t nb = cat ? NB : c->bc[f];
            if (nb == 0) continue;
            const uint8_t* col = cat ? c->cat_bins + (int64_t)(f - F0) * n : c->bins + (int64_t)f * n;
            size_t cells = (size_t)n_leaves * NB * 2;
            double* hist = (double*)calloc(cells, sizeof(double));
            if (level == 0) {
                for (int64_t o = 0; o < n; ++o) {
                    int32_t b = col[o];
                    if (b >= NB) continue;
                    hist[2 * b] += c->g[o];
                    hist[2 * b + 1] += c->h[o];
                }
            } else {
                /* derive_feature_level_hist (tree.rs:1075-1131): build the
                 * globally smaller side into the parent's slot, derive the other
                 * side as parent - built. */
                double* built = (double*)calloc((size_t)n_par * NB * 2, sizeof(double));
                for (int64_t o = 0; o < n; ++o) {
                    int32_t l = leaf_of[o];
                    int pass = (l & n_par) != 0;
                    if (pass != build_true) continue;
                    int32_t b = col[o];
                    if (b >= NB) continue;
                    double* cell = built + ((int64_t)(l & (n_par - 1)) * NB + b) * 2;
                    cell[0] += c->g[o];
                    cell[1] += c->h[o];
                }
                const double* parent = cur[f];
                size_t pc = (size_t)NB * 2;
                for (int32_t p = 0; p < n_par; ++p) {
                    double* fl = hist + (size_t)p * pc;           /* false child p */
                    double* tr = hist + (size_t)(p + n_par) * pc; /* true child p */
                    const double* par = parent + (size_t)p * pc;
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
            double* work = (double*)malloc(sizeof(double) * (size_t)n_leaves * 8);
            if (cat)
                scan_one_hot(hist, n_leaves, NB, present + (size_t)(f - F0) * NB, c->score_fn, c->l2,
                             scores_all + (size_t)f * NB, work);
            else
                scan_and_score(hist, n_leaves, NB, nb, c->score_fn, c->l2,
                               scores_all + (size_t)f * NB, work);
            free(work);
            next[f] = hist;
        }
        for (int32_t f = 0; f < F; ++f) free(cur[f]);
        free(cur);
        cur = next;

        if (c->top2) {
            /* the best and runner-up raw candidate scores (a test's near-tie bar) */
            double best = -INFINITY, second = -INFINITY;
            for (int32_t f = 0; f < F; ++f) {
                const int32_t nc = f >= F0 ? NB : c->bc[f];
                for (int32_t b = 0; b < nc; ++b) {
                    if (f >= F0 && !present[(size_t)(f - F0) * NB + b]) continue;
                    const double s = scores_all[(size_t)f * NB + b];
                    if (s > best) { second = best; best = s; }
                    else if (s > second) second = s;
                }
            }
            c->top2[2 * level] = best;
            c->top2[2 * level + 1] = second;
        }
        int32_t best_f = -1, best_b = -1;
        if (!c->draws) {
            /* select_best: strict > over (feature asc, border asc) (tree.rs:355-366) */
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
            /* perturbed selection (tree.rs:1498-1606) */
            uint64_t rand_seed = orc_rng_gen(c->rng);
            uint64_t task = 0;
            double best_gain = -INFINITY;
            for (int32_t f = 0; f < F; ++f) {
                int32_t nb = c->bc[f];
                if (nb == 0) {
                    (void)orc_std_normal(c->rng);
                    continue;
                }
                double binst = -INFINITY, braw = -INFINITY;
                int32_t bb = 0;
                if (c->std_dev != 0.0) {
                    orc_rng fr;
                    orc_rng_from_seed(&fr, rand_seed + task);
                    orc_rng_advance(&fr, 10);
                    for (int32_t b = 0; b < nb; ++b) {
                        double raw = scores_all[(size_t)f * NB + b];
                        double inst = raw + orc_std_normal(&fr) * c->std_dev;
                        if (inst > binst) { binst = inst; bb = b; braw = raw; }
                    }
                } else {
                    /* std_dev == 0: instance == raw, the per-feature stream is
                     * private to this feature, so its draws are skipped. */
                    for (int32_t b = 0; b < nb; ++b) {
                        double raw = scores_all[(size_t)f * NB + b];
                        if (raw > binst) { binst = raw; bb = b; braw = raw; }
                    }
                }
                task++;
                double inst = braw + orc_std_normal(c->rng) * c->std_dev;
                if (inst > best_gain) { best_gain = inst; best_f = f; best_b = bb; }
            }
            if (best_f < 0) break; /* no candidate: the tree ends here */
        }
        feat[level] = best_f;
        sbin[level] = best_b;
        taken = level + 1;
        /* advance_leaf_only (tree.rs:1005-1016): the new split is the high bit;
         * a one-hot split passes on bin == value */
        if (best_f >= F0) {
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

/* The search above for callers outside this file (the grouped-loss loop in
 * cb_oracle_rank.c): score channels g/h, the RNG-drawing path when `draws`. */
int orc_search_tree(int64_t n, int32_t F, int32_t n_bins, int32_t depth, int32_t score_fn, const uint8_t* bins,
                    const int32_t* border_counts, const double* g, const double* h, double l2, int32_t draws,
                    orc_rng* rng, int32_t* feat, int32_t* sbin, int32_t* leaf_of, int32_t* err) {
    search_ctx sc = {n, F, n_bins, depth, score_fn, bins, border_counts, g, h, l2, draws, rng, 0.0, 0, NULL, NULL};
    int e = 0;
    int taken = search_tree(&sc, feat, sbin, leaf_of, &e);
    *err = e;
    return taken;
}

/* ======================================================================== */
/* boosting loop -- crates/cb-train/src/boosting.rs CPU branch               */
/* (:1871 starting approx, :7400-8930 per-iteration body, :55-69 draws)      */
/* ======================================================================== */

int orc_train(const orc_train_args* a, orc_train_out* o) {
#ifdef _OPENMP
    if (a->n_threads > 0) omp_set_num_threads(a->n_threads);
#endif
    const int64_t n = a->n;
    const int32_t F = a->n_features;
    int32_t NB = 1;
    for (int32_t f = 0; f < F; ++f)
        if (a->border_counts[f] + 1 > NB) NB = a->border_counts[f] + 1;
    for (int64_t k = 0; k < (int64_t)a->n_cat * n; ++k)
        if (a->cat_bins_fm[k] + 1 > NB) NB = a->cat_bins_fm[k] + 1;
    const int32_t L = 1 << a->depth;

    double* w = (double*)malloc(sizeof(double) * (size_t)n);
    for (int64_t i = 0; i < n; ++i) w[i] = a->weights ? a->weights[i] : 1.0;
    double sum_w = orc_sum_f64(w, n);
    double scaled_l2 = n == 0 ? a->l2_leaf_reg : a->l2_leaf_reg * (sum_w / (double)n);
    /* upstream stores the learning rate as f32: every use below sees the
     * narrowed value (boosting.rs:4958) */
    const double lr = (double)(float)a->learning_rate;
    double bias = 0.0;
    if (a->boost_from_average && a->loss == ORC_LOSS_RMSE && n > 0)
        bias = orc_sum_f64(a->target, n) / (double)n;
    if (o->bias) o->bias[0] = bias;

    double* approx = (double*)malloc(sizeof(double) * (size_t)n);
    double* der1 = (double*)malloc(sizeof(double) * (size_t)n);
    double* wd1 = (double*)malloc(sizeof(double) * (size_t)n);
    double* dobj = (double*)malloc(sizeof(double) * (size_t)n);
    double* sw = (double*)malloc(sizeof(double) * (size_t)n);
    uint8_t* ctl = (uint8_t*)malloc((size_t)n);
    double* sg = (double*)malloc(sizeof(double) * (size_t)n);
    double* sh = (double*)malloc(sizeof(double) * (size_t)n);
    int32_t* leaf = (int32_t*)malloc(sizeof(int32_t) * (size_t)n);
    double* ls = (double*)malloc(sizeof(double) * (size_t)L * 2);
    for (int64_t i = 0; i < n; ++i) approx[i] = bias;

    orc_rng rng;
    orc_rng_from_seed(&rng, a->random_seed);
    const int draws = a->bootstrap_type != ORC_BOOT_NO || a->random_strength != 0.0;
    int has_prev = 0;
    double prev_mean = 0.0;
    int rc = 0;

    const int quantile = a->loss == ORC_LOSS_MAE || a->loss == ORC_LOSS_QUANTILE;
    /* MAE is Quantile{alpha 0.5, delta 1e-6} (loss.rs:186-193) */
    const double q_alpha = a->loss == ORC_LOSS_MAE ? 0.5 : a->quantile_alpha;
    const double q_delta = a->loss == ORC_LOSS_MAE ? 1e-6 : a->quantile_delta;
    float* res = a->exact_leaf ? (float*)malloc(sizeof(float) * (size_t)(n ? n : 1)) : NULL;
    double* rw = a->exact_leaf ? (double*)malloc(sizeof(double) * (size_t)(n ? n : 1)) : NULL;

    for (int32_t it = 0; it < a->iterations; ++it) {
        if (quantile) {
            for (int64_t i = 0; i < n; ++i) { /* quantile_der1 (loss.rs:166-175) */
                const double v = a->target[i] - approx[i];
                der1[i] = fabs(v) < q_delta ? 0.0 : (v > 0.0 ? q_alpha : -(1.0 - q_alpha));
            }
        } else {
            orc_compute_gradients(a->loss, approx, a->target, n, der1, NULL);
        }
        for (int64_t i = 0; i < n; ++i) wd1[i] = der1[i] * w[i];
        if (draws) {
            (void)orc_rng_gen(&rng); /* PRE_TREE_DRAWS = 2 */
            (void)orc_rng_gen(&rng);
        }
        for (int64_t i = 0; i < n; ++i) dobj[i] = sqrt(wd1[i] * wd1[i]);
        if (orc_bootstrap(a->bootstrap_type, dobj, n, a->subsample, a->bagging_temperature,
                          has_prev, prev_mean, &rng, sw, ctl) != 0) {
            rc = -2;
            break;
        }
        for (int64_t i = 0; i < n; ++i) {
            sg[i] = ctl[i] ? wd1[i] * sw[i] : 0.0;
            sh[i] = ctl[i] ? w[i] * sw[i] : 0.0;
        }
        double std_dev = 0.0;
        if (a->random_strength != 0.0) {
            /* score_st_dev (score.rs:361-399) */
            double acc = 0.0;
            for (int64_t i = 0; i < n; ++i) acc += wd1[i] * wd1[i];
            double dsdz = n == 0 ? 0.0 : sqrt(acc / (double)n);
            double model_length = (double)it * lr;
            double left = exp(log((double)n) - model_length);
            std_dev = a->random_strength * dsdz * (left / (1.0 + left));
        }
        search_ctx sc = {n, F, NB, a->depth, a->score_function, a->bins_fm, a->border_counts,
                         sg, sh, scaled_l2, draws, &rng, std_dev, a->n_cat, a->cat_bins_fm,
                         o->level_top2 ? o->level_top2 + (size_t)it * a->depth * 2 : NULL};
        int32_t* tf = o->split_feature + (size_t)it * a->depth;
        int32_t* tb = o->split_bin + (size_t)it * a->depth;
        for (int32_t l = 0; l < a->depth; ++l) { tf[l] = -1; tb[l] = -1; }
        int err = 0;
        int taken = search_tree(&sc, tf, tb, leaf, &err);
        if (err) { rc = -3; break; }
        o->tree_depth[it] = taken;
        int32_t nl = 1 << taken;
        /* compute_leaf_deltas Gradient over the unsampled channels
         * (boosting.rs:2470-2517) then normalize_leaf_values (x lr). */
        for (int32_t k = 0; k < 2 * nl; ++k) ls[k] = 0.0;
        for (int64_t i = 0; i < n; ++i) {
            ls[2 * leaf[i]] += wd1[i];
            ls[2 * leaf[i] + 1] += w[i];
        }
        double* lv = o->leaf_values + (size_t)it * L;
        for (int32_t k = 0; k < L; ++k) lv[k] = 0.0;
        if (a->exact_leaf) {
            /* Exact: the leaf's members in object order, residual (f32)(t - a)
             * and object weight (collect_leaf_residuals), no l2 */
            for (int32_t k = 0; k < nl; ++k) {
                int64_t m = 0;
                for (int64_t i = 0; i < n; ++i)
                    if (leaf[i] == k) {
                        res[m] = (float)(a->target[i] - approx[i]);
                        rw[m++] = w[i];
                    }
                lv[k] = orc_exact_leaf_delta(res, rw, m, q_alpha, q_delta) * lr;
            }
        } else {
            for (int32_t k = 0; k < nl; ++k)
                lv[k] = calc_average(ls[2 * k], ls[2 * k + 1], scaled_l2) * lr;
        }
        for (int64_t i = 0; i < n; ++i) approx[i] += lv[leaf[i]];
        if (o->staged) memcpy(o->staged + (size_t)it * n, approx, sizeof(double) * (size_t)n);
        if (draws) {
            (void)orc_rng_gen(&rng); /* POST_TREE_EXTRA_DRAWS = 2 */
            (void)orc_rng_gen(&rng);
        }
        /* last_iter_mean_leaf_value (bootstrap.rs:382-389) */
        double acc = 0.0;
        for (int32_t k = 0; k < nl; ++k) acc += sqrt(lv[k] * lv[k]);
        prev_mean = acc / (double)nl;
        has_prev = 1;
        if (o->rng_calls) o->rng_calls[it] = rng.calls;
    }
    if (o->final_approx) memcpy(o->final_approx, approx, sizeof(double) * (size_t)n);
    free(w); free(approx); free(der1); free(wd1); free(dobj); free(sw); free(ctl);
    free(sg); free(sh); free(leaf); free(ls); free(res); free(rw);
    return rc;
}

typedef struct {
    float v;
    double w;
    int64_t pos;
} orc_vw;

static int vw_cmp(const void* x, const void* y) {
    const orc_vw* a = (const orc_vw*)x;
    const orc_vw* b = (const orc_vw*)y;
    /* ascending value, ties by original position: a stable sort */
    if (a->v < b->v) return -1;
    if (a->v > b->v) return 1;
    return a->pos < b->pos ? -1 : (a->pos > b->pos ? 1 : 0);
}

double orc_exact_leaf_delta(const float* residuals, const double* weights, int64_t n, double alpha, double delta) {
    if (n == 0) return 0.0;
    if (alpha <= 0.0) { /* the minimum element */
        double mn = INFINITY;
        for (int64_t i = 0; i < n; ++i)
            if ((double)residuals[i] < mn) mn = (double)residuals[i];
        return mn;
    }
    orc_vw* e = (orc_vw*)malloc(sizeof(orc_vw) * (size_t)n);
    for (int64_t i = 0; i < n; ++i) {
        e[i].v = residuals[i];
        e[i].w = weights ? weights[i] : 1.0;
        e[i].pos = i;
    }
    qsort(e, (size_t)n, sizeof(orc_vw), vw_cmp);
    double total = 0.0;
    for (int64_t i = 0; i < n; ++i) total += e[i].w; /* sum_f64 in sorted order */
    const double need = total * alpha;
    double acc = 0.0;
    double q = (double)e[n - 1].v;
    for (int64_t i = 0; i < n; ++i) {
        acc += e[i].w;
        if (acc >= need - DBL_EPSILON) {
            q = (double)e[i].v;
            break;
        }
    }
    if (delta > 0.0) {
        const float qf = (float)q;
        double less = 0.0, equal = 0.0;
        for (int64_t i = 0; i < n; ++i) {
            if (e[i].v < qf) less += e[i].w;
            else if (e[i].v == qf) equal += e[i].w;
        }
        q = less + equal * alpha >= need - DBL_EPSILON ? q - delta : q + delta;
    }
    free(e);
    return q;
}


/* ======================================================================== */
/* CityHash64 v1.0 (Google's published CityHash, as catboost's               */
/* util/digest/city.cpp) and CalcCatFeatureHash -- cat_hash.rs               */
/* ======================================================================== */

static const uint64_t kCity0 = 0xc3a5c85c97cb3127ULL, kCity1 = 0xb492b66fbe98f273ULL,
                      kCity2 = 0x9ae16a3b2f90404fULL, kCity3 = 0xc949d7c7509e6557ULL;

static uint64_t city_fetch64(const char* p) {
    uint64_t v;
    memcpy(&v, p, 8);
    return v;
}
static uint32_t city_fetch32(const char* p) {
    uint32_t v;
    memcpy(&v, p, 4);
    return v;
}
static uint64_t city_rotate(uint64_t v, int s) { return s == 0 ? v : ((v >> s) | (v << (64 - s))); }
static uint64_t city_rotate1(uint64_t v, int s) { return (v >> s) | (v << (64 - s)); }
static uint64_t city_shift_mix(uint64_t v) { return v ^ (v >> 47); }
static uint64_t city_hash16(uint64_t u, uint64_t v) {
    const uint64_t m = 0x9ddfea08eb382d69ULL;
    uint64_t a = (u ^ v) * m;
    a ^= (a >> 47);
    uint64_t b = (v ^ a) * m;
    b ^= (b >> 47);
    b *= m;
    return b;
}
static uint64_t city_len0to16(const char* s, size_t len) {
    if (len > 8) {
        const uint64_t a = city_fetch64(s), b = city_fetch64(s + len - 8);
        return city_hash16(a, city_rotate1(b + len, (int)len)) ^ b;
    }
    if (len >= 4) {
        const uint64_t a = city_fetch32(s);
        return city_hash16(len + (a << 3), city_fetch32(s + len - 4));
    }
    if (len > 0) {
        const uint8_t a = (uint8_t)s[0], b = (uint8_t)s[len >> 1], c = (uint8_t)s[len - 1];
        const uint32_t y = (uint32_t)a + ((uint32_t)b << 8);
        const uint32_t z = (uint32_t)len + ((uint32_t)c << 2);
        return city_shift_mix(y * kCity2 ^ z * kCity3) * kCity2;
    }
    return kCity2;
}
static uint64_t city_len17to32(const char* s, size_t len) {
    const uint64_t a = city_fetch64(s) * kCity1, b = city_fetch64(s + 8);
    const uint64_t c = city_fetch64(s + len - 8) * kCity2, d = city_fetch64(s + len - 16) * kCity0;
    return city_hash16(city_rotate(a - b, 43) + city_rotate(c, 30) + d, a + city_rotate(b ^ kCity3, 20) - c + len);
}
typedef struct {
    uint64_t first, second;
} city_pair;
static city_pair city_weak32(uint64_t w, uint64_t x, uint64_t y, uint64_t z, uint64_t a, uint64_t b) {
    a += w;
    b = city_rotate(b + a + z, 21);
    const uint64_t c = a;
    a += x;
    a += y;
    b += city_rotate(a, 44);
    city_pair r = {a + z, b + c};
    return r;
}
static city_pair city_weak32s(const char* s, uint64_t a, uint64_t b) {
    return city_weak32(city_fetch64(s), city_fetch64(s + 8), city_fetch64(s + 16), city_fetch64(s + 24), a, b);
}
static uint64_t city_len33to64(const char* s, size_t len) {
    uint64_t z = city_fetch64(s + 24);
    uint64_t a = city_fetch64(s) + (len + city_fetch64(s + len - 16)) * kCity0;
    uint64_t b = city_rotate(a + z, 52);
    uint64_t c = city_rotate(a, 37);
    a += city_fetch64(s + 8);
    c += city_rotate(a, 7);
    a += city_fetch64(s + 16);
    const uint64_t vf = a + z, vs = b + city_rotate(a, 31) + c;
    a = city_fetch64(s + 16) + city_fetch64(s + len - 32);
    z = city_fetch64(s + len - 8);
    b = city_rotate(a + z, 52);
    c = city_rotate(a, 37);
    a += city_fetch64(s + len - 24);
    c += city_rotate(a, 7);
    a += city_fetch64(s + len - 16);
    const uint64_t wf = a + z, ws = b + city_rotate(a, 31) + c;
    const uint64_t r = city_shift_mix((vf + ws) * kCity2 + (wf + vs) * kCity0);
    return city_shift_mix(r * kCity0 + vs) * kCity2;
}

uint64_t orc_city_hash64(const char* s, size_t len) {
    if (len <= 32) return len <= 16 ? city_len0to16(s, len) : city_len17to32(s, len);
    if (len <= 64) return city_len33to64(s, len);
    uint64_t x = city_fetch64(s + len - 40);
    uint64_t y = city_fetch64(s + len - 16) + city_fetch64(s + len - 56);
    uint64_t z = city_hash16(city_fetch64(s + len - 48) + len, city_fetch64(s + len - 24));
    city_pair v = city_weak32s(s + len - 64, len, z);
    city_pair w = city_weak32s(s + len - 32, y + kCity1, x);
    x = x * kCity1 + city_fetch64(s);
    len = (len - 1) & ~(size_t)63;
    do {
        x = city_rotate(x + y + v.first + city_fetch64(s + 8), 37) * kCity1;
        y = city_rotate(y + v.second + city_fetch64(s + 48), 42) * kCity1;
        x ^= w.second;
        y += v.first + city_fetch64(s + 40);
        z = city_rotate(z + w.first, 33) * kCity1;
        v = city_weak32s(s, v.second * kCity1, x + w.first);
        w = city_weak32s(s + 32, z + w.second, y + city_fetch64(s + 16));
        const uint64_t t = z;
        z = x;
        x = t;
        s += 64;
        len -= 64;
    } while (len != 0);
    return city_hash16(city_hash16(v.first, w.first) + city_shift_mix(y) * kCity1 + z,
                       city_hash16(v.second, w.second) + x);
}

uint32_t orc_cat_hash(const char* s, size_t len) { return (uint32_t)(orc_city_hash64(s, len) & 0xffffffffULL); }
