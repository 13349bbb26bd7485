/*
 * cb_oracle_apply.c -- CPU restatement of catboost_rs's float-only oblivious
 * ensemble apply (crates/cb-model/src/apply.rs) over the CSR lowering of
 * crates/cb-model/src/gpu_apply.rs.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for cbgpu_apply_oblivious.
 * The product path never calls it.  Build with -ffp-contract=off.
 */
#include "cb_oracle.h"

#include <math.h>

/* ======================================================================== */
/* oblivious-ensemble apply -- crates/cb-model/src/apply.rs:150-173,        */
/* 264-271, 374-410                                                         */
/* ======================================================================== */

void orc_apply_oblivious(const float* x_fm, int64_t n, int32_t F, const uint32_t* split_features,
                         const double* split_borders, const uint32_t* tree_split_offsets, int32_t n_trees,
                         const double* leaf_values, const uint32_t* tree_leaf_offsets, double bias,
                         const uint8_t* nan_above, double* out) {
    for (int64_t i = 0; i < n; ++i) {
        double sum = 0.0; /* sum_f64 over the per-tree values, tree order */
        for (int32_t t = 0; t < n_trees; ++t) {
            uint64_t leaf = 0;
            for (uint32_t s = tree_split_offsets[t]; s < tree_split_offsets[t + 1]; ++s) {
                uint32_t f = split_features[s];
                int passes = 0;
                if (f < (uint32_t)F) {
                    float v = x_fm[(int64_t)f * n + i];
                    passes = isnan(v) ? (nan_above && nan_above[f]) : ((double)v > split_borders[s]);
                }
                leaf |= (uint64_t)passes << (s - tree_split_offsets[t]);
            }
            uint64_t li = (uint64_t)tree_leaf_offsets[t] + leaf;
            sum += li < (uint64_t)tree_leaf_offsets[t + 1] ? leaf_values[li] : 0.0;
        }
        /* bias + sum(oblivious) + sum(non_symmetric = 0) + sum(region = 0) */
        out[i] = ((bias + sum) + 0.0) + 0.0;
    }
}
