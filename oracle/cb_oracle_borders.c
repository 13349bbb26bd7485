/*
 * cb_oracle_borders.c -- CPU restatement of catboost_rs's float-feature border
 * selection (crates/cb-data/src/borders.rs, border_types.rs) and of the
 * builder's per-column rule (crates/catboost-rs/src/builder.rs:1677-1720).
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for the device border
 * selection in catboost_rs_b200/csrc.  The product path never calls it.
 *
 * Border VALUES are computed in f32 and split scores in f64, exactly as the
 * reference does; build with -ffp-contract=off so no multiply-add is fused.
 * The exact dynamic-programming binarizers (MaxLogSum, MinEntropy,
 * border_types.rs:381-760) are not restated: no path of this build uses them.
 */
#include "cb_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* borders.rs:46 */
#define MAX_SUBSET 200000

/* ---- penalties (borders.rs:51-63) -------------------------------------- */
static double penalty(int32_t kind, double w) {
    return kind == ORC_PENALTY_MIN_ENTROPY ? w * log(w + 1e-8) : -log(w + 1e-8);
}

/* ---- ascending f32 sort by the total-order key (borders.rs:436-502) ---- */
static inline uint32_t f32_key(float v) {
    uint32_t b;
    memcpy(&b, &v, 4);
    return (b & 0x80000000u) ? ~b : (b ^ 0x80000000u);
}

static inline float key_f32(uint32_t k) {
    uint32_t b = (k & 0x80000000u) ? (k ^ 0x80000000u) : ~k;
    float v;
    memcpy(&v, &b, 4);
    return v;
}

/* LSD radix over the key; the sorted VALUE sequence is all any caller reads
 * (the reference's argument, borders.rs:418-434). */
static int sort_f32(float* v, int64_t n) {
    if (n < 2) return 0;
    uint32_t* a = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)n);
    uint32_t* b = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)n);
    if (!a || !b) {
        free(a);
        free(b);
        return -1;
    }
    for (int64_t i = 0; i < n; ++i) a[i] = f32_key(v[i]);
    for (int pass = 0; pass < 4; ++pass) {
        int sh = pass * 8;
        int64_t cnt[257] = {0};
        for (int64_t i = 0; i < n; ++i) cnt[((a[i] >> sh) & 0xFF) + 1]++;
        for (int d = 0; d < 256; ++d) cnt[d + 1] += cnt[d];
        for (int64_t i = 0; i < n; ++i) b[cnt[(a[i] >> sh) & 0xFF]++] = a[i];
        uint32_t* t = a;
        a = b;
        b = t;
    }
    for (int64_t i = 0; i < n; ++i) v[i] = key_f32(a[i]);
    free(a);
    free(b);
    return 0;
}

/* ---- fixed-seed object sample (borders.rs:504-520) ---------------------- */
/* Partial Fisher-Yates with TFastRng64::from_seed(0); returns the sorted
 * index set (the caller frees it). */
int64_t* orc_border_sample_indices(int64_t n, int64_t sample_size, int64_t* out_len) {
    int64_t take = sample_size < n ? sample_size : n;
    int64_t* idx = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n > 0 ? n : 1));
    if (!idx) return NULL;
    for (int64_t i = 0; i < n; ++i) idx[i] = i;
    orc_rng r;
    orc_rng_from_seed(&r, 0);
    for (int64_t i = 0; i < take; ++i) {
        int64_t off = (int64_t)orc_rng_uniform(&r, (uint64_t)(n - i));
        int64_t t = idx[i];
        idx[i] = idx[i + off];
        idx[i + off] = t;
    }
    /* sort the prefix ascending (counting over a bitmap keeps it O(n)) */
    uint8_t* mark = (uint8_t*)calloc((size_t)(n > 0 ? n : 1), 1);
    if (!mark) {
        free(idx);
        return NULL;
    }
    for (int64_t i = 0; i < take; ++i) mark[idx[i]] = 1;
    int64_t k = 0;
    for (int64_t i = 0; i < n; ++i)
        if (mark[i]) idx[k++] = i;
    free(mark);
    *out_len = take;
    return idx;
}

/* ---- greedy binarizer (borders.rs:116-226, 572-640) --------------------- */
typedef struct {
    int64_t start, end, best_split;
    double best_score;
    uint64_t seq;
} gbin;

static double split_score(const gbin* b, int64_t pos, int32_t pen) {
    if (pos == b->start || pos == b->end) return -INFINITY;
    double left = -penalty(pen, (double)(pos - b->start));
    double right = -penalty(pen, (double)(b->end - pos));
    double curr = -penalty(pen, (double)(b->end - b->start));
    return left + right - curr;
}

/* first index in [lo, hi) with v >= t (else hi) */
static int64_t lower_bound_f(const float* v, int64_t lo, int64_t hi, float t) {
    while (lo < hi) {
        int64_t m = lo + (hi - lo) / 2;
        if (v[m] < t) lo = m + 1;
        else hi = m;
    }
    return lo;
}

/* first index in [lo, hi) with v > t (else hi) */
static int64_t upper_bound_f(const float* v, int64_t lo, int64_t hi, float t) {
    while (lo < hi) {
        int64_t m = lo + (hi - lo) / 2;
        if (v[m] <= t) lo = m + 1;
        else hi = m;
    }
    return lo;
}

/* UpdateBestSplitProperties (borders.rs:178-198): probe the lower and upper
 * bound of the middle value, ties to the lower bound. */
static void update_best(gbin* b, const float* v, int32_t pen) {
    int64_t mid = b->start + (b->end - b->start) / 2;
    float mv = v[mid];
    int64_t lb = lower_bound_f(v, b->start, mid, mv);
    int64_t ub = upper_bound_f(v, mid, b->end, mv);
    double sl = split_score(b, lb, pen), sr = split_score(b, ub, pen);
    if (sl >= sr) {
        b->best_split = lb;
        b->best_score = sl;
    } else {
        b->best_split = ub;
        b->best_score = sr;
    }
}

/* heap order: higher score first, then the earlier insertion (borders.rs:640-660) */
static int heap_above(const gbin* a, const gbin* b) {
    if (a->best_score != b->best_score) return a->best_score > b->best_score;
    return a->seq < b->seq;
}

static void heap_push(gbin* h, int64_t* n, gbin x) {
    int64_t i = (*n)++;
    h[i] = x;
    while (i > 0) {
        int64_t p = (i - 1) / 2;
        if (!heap_above(&h[i], &h[p])) break;
        gbin t = h[i];
        h[i] = h[p];
        h[p] = t;
        i = p;
    }
}

static gbin heap_pop(gbin* h, int64_t* n) {
    gbin top = h[0];
    h[0] = h[--(*n)];
    int64_t i = 0;
    for (;;) {
        int64_t l = 2 * i + 1, r = l + 1, m = i;
        if (l < *n && heap_above(&h[l], &h[m])) m = l;
        if (r < *n && heap_above(&h[r], &h[m])) m = r;
        if (m == i) break;
        gbin t = h[i];
        h[i] = h[m];
        h[m] = t;
        i = m;
    }
    return top;
}

/* GreedySplit (borders.rs:572-619): pop the best bin while the queue holds
 * <= max_borders bins and the best can split; emit every non-first bin's
 * left border 0.5f*v[start-1] + 0.5f*v[start] (borders.rs:216-225). */
static int64_t greedy_split(const float* v, int64_t n, int64_t max_borders, int32_t pen, float* out) {
    if (n < 2) return 0;
    gbin* h = (gbin*)malloc(sizeof(gbin) * (size_t)(max_borders + 3));
    if (!h) return -1;
    int64_t hn = 0;
    uint64_t seq = 0;
    gbin root = {0, n, 0, 0.0, seq++};
    update_best(&root, v, pen);
    heap_push(h, &hn, root);
    while (hn <= max_borders) {
        gbin* t = &h[0];
        if (!(t->start != t->best_split && t->end != t->best_split)) break;
        gbin top = heap_pop(h, &hn);
        gbin left = {top.start, top.best_split, top.start, 0.0, 0};
        update_best(&left, v, pen);
        top.start = top.best_split;
        update_best(&top, v, pen);
        left.seq = seq++;
        heap_push(h, &hn, left);
        top.seq = seq++;
        heap_push(h, &hn, top);
    }
    int64_t k = 0;
    for (int64_t i = 0; i < hn; ++i) {
        if (h[i].start == 0) continue;
        float b = 0.5f * v[h[i].start - 1];
        b += 0.5f * v[h[i].start];
        out[k++] = b;
    }
    free(h);
    return k;
}

/* ---- Median / Uniform / UniformAndQuantiles (border_types.rs:238-378) --- */
/* RegularBorder: snap onto the midpoint of the straddling observed pair. */
static float regular_border(float border, const float* s, int64_t n) {
    float front = s[0], back = s[n - 1];
    int64_t idx = lower_bound_f(s, 0, n, border);
    if (idx == n) return fmaxf(2.0f * back, back + 1.0f);
    if (idx == 0) return fminf(0.5f * front, 2.0f * front);
    float hi = s[idx], lo = s[idx - 1];
    float res = (hi + lo) * 0.5f;
    if (res == hi) res = lo;
    return res;
}

static int64_t median_borders(const float* s, int64_t n, int64_t max_borders, float* out) {
    if (n == 0 || s[0] == s[n - 1]) return 0;
    int64_t k = 0;
    for (int64_t i = 0; i < max_borders; ++i) {
        uint64_t i1 = (uint64_t)(i + 1) * (uint64_t)n / (uint64_t)(max_borders + 1);
        if (i1 > (uint64_t)(n - 1)) i1 = (uint64_t)(n - 1);
        float val = s[i1];
        if (val != s[0]) out[k++] = regular_border(val, s, n);
    }
    return k;
}

static int64_t uniform_borders(const float* v, int64_t n, int64_t max_borders, float* out) {
    if (n == 0) return 0;
    float mn = INFINITY, mx = -INFINITY;
    for (int64_t i = 0; i < n; ++i) {
        if (v[i] < mn) mn = v[i];
        if (v[i] > mx) mx = v[i];
    }
    if (mn == mx) return 0;
    for (int64_t i = 0; i < max_borders; ++i) {
        float step = (float)(i + 1) * (mx - mn);
        out[i] = mn + step / (float)(max_borders + 1);
    }
    return max_borders;
}

static int64_t median_plus_uniform(const float* s, int64_t n, int64_t max_borders, float* out) {
    if (n == 0 || s[0] == s[n - 1]) return 0;
    int64_t half = max_borders / 2;
    int64_t k = median_borders(s, n, max_borders - half, out);
    float mn = s[0], mx = s[n - 1];
    for (int64_t i = 0; i < half; ++i) {
        float step = (float)(i + 1) * (mx - mn);
        float val = mn + step / (float)(half + 1);
        out[k++] = regular_border(val, s, n);
    }
    return k;
}

/* ---- finalize (borders.rs:403-424): -0 -> +0, sort, dedup, widen -------- */
static int cmp_f32(const void* a, const void* b) {
    float x = *(const float*)a, y = *(const float*)b;
    return (x > y) - (x < y);
}

static int64_t finalize(float* b, int64_t k, int nan_sentinel, double* out, int64_t cap) {
    for (int64_t i = 0; i < k; ++i)
        if (b[i] == 0.0f) b[i] = 0.0f;
    qsort(b, (size_t)k, sizeof(float), cmp_f32);
    int64_t m = 0;
    if (nan_sentinel) {
        if (m >= cap) return -1;
        out[m++] = (double)(-FLT_MAX);
    }
    for (int64_t i = 0; i < k; ++i) {
        if (i > 0 && b[i] == b[i - 1]) continue;
        if (m >= cap) return -1;
        out[m++] = (double)b[i];
    }
    return m;
}

/* select_borders_from_values (border_types.rs:178-236) over NaN-free values. */
static int64_t borders_from_values(float* vals, int64_t n, int64_t border_count, int32_t type,
                                   int nan_sentinel, double* out, int64_t cap) {
    int64_t max_b = nan_sentinel ? (border_count > 0 ? border_count - 1 : 0) : border_count;
    float* tmp = (float*)malloc(sizeof(float) * (size_t)(max_b + 2));
    if (!tmp) return -1;
    int64_t k = 0;
    switch (type) {
    case ORC_BORDER_GREEDY_LOGSUM:
    case ORC_BORDER_GREEDY_MIN_ENTROPY:
        if (sort_f32(vals, n) != 0) k = -1;
        else k = greedy_split(vals, n, max_b, type == ORC_BORDER_GREEDY_LOGSUM ? ORC_PENALTY_MAXSUMLOG
                                                                               : ORC_PENALTY_MIN_ENTROPY, tmp);
        break;
    case ORC_BORDER_UNIFORM:
        k = uniform_borders(vals, n, max_b, tmp);
        break;
    case ORC_BORDER_MEDIAN:
        k = sort_f32(vals, n) != 0 ? -1 : median_borders(vals, n, max_b, tmp);
        break;
    case ORC_BORDER_UNIFORM_AND_QUANTILES:
        k = sort_f32(vals, n) != 0 ? -1 : median_plus_uniform(vals, n, max_b, tmp);
        break;
    default:
        k = -2;
    }
    int64_t m = k < 0 ? k : finalize(tmp, k, nan_sentinel, out, cap);
    free(tmp);
    return m;
}

/* select_borders_f32 (border_types.rs:134-153) + the builder's per-column
 * NaN rule (builder.rs:1677-1720).  Returns the border count written to
 * out, or a negative value on error (-1 capacity / memory, -2 unknown type,
 * -3 NaN under nan_mode=Forbidden). */
int64_t orc_select_borders(const float* col, int64_t n, int32_t border_count, int32_t border_type,
                           int32_t nan_mode, double* out, int64_t out_cap) {
    int has_nan = 0;
    for (int64_t i = 0; i < n && !has_nan; ++i) has_nan = isnan(col[i]);
    if (has_nan && nan_mode == ORC_NAN_FORBIDDEN) return -3;
    int64_t bc = border_count;
    int sentinel = 0;
    if (has_nan && nan_mode == ORC_NAN_MIN) sentinel = 1;
    if (has_nan && nan_mode == ORC_NAN_MAX) bc = bc > 0 ? bc - 1 : 0;
    float* vals = (float*)malloc(sizeof(float) * (size_t)(n > MAX_SUBSET ? MAX_SUBSET : (n > 0 ? n : 1)));
    if (!vals) return -1;
    int64_t m = 0;
    if (n > MAX_SUBSET) {
        int64_t len = 0;
        int64_t* idx = orc_border_sample_indices(n, MAX_SUBSET, &len);
        if (!idx) {
            free(vals);
            return -1;
        }
        for (int64_t i = 0; i < len; ++i)
            if (!isnan(col[idx[i]])) vals[m++] = col[idx[i]];
        free(idx);
    } else {
        for (int64_t i = 0; i < n; ++i)
            if (!isnan(col[i])) vals[m++] = col[i];
    }
    int64_t k = borders_from_values(vals, m, bc, border_type, sentinel, out, out_cap);
    free(vals);
    if (k >= 0 && has_nan && nan_mode == ORC_NAN_MAX) {
        if (k >= out_cap) return -1;
        out[k++] = (double)FLT_MAX;
    }
    return k;
}
