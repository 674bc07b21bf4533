/*
 * skv_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the SeoulKV4 sparse-decode funnel.  It is the parity
 * checker for the CUDA engine in seoulkv_b200/csrc: only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg load it, and never
 * as the thing that is shipped or measured as the product.
 *
 * It restates, per KV head ("cell"), the arithmetic of the reference
 * (daniel-geon-park/SeoulKV, package src/seoulkv4):
 *
 *   query operands     _kernels/query_prepare/host.py:26-51
 *   coarse intervals   _kernels/codegen/coarse_compute.py:61-119,
 *                      _kernels/stage1_coarse/seoulkv4_coarse_score.py:197-218
 *   coarse threshold   _kernels/stage1_coarse/seoulkv4_coarse_select.py:20-36,
 *                      205-345 (P-th largest lower bound, ordered BF16 compare)
 *   fine scores        _kernels/codegen/fine_postscale_codegen.py:8-70
 *   fine top-P, union  _kernels/stage1_fine/seoulkv4_fine_native_select.py:35-67,
 *                      _kernels/stage1_fine/seoulkv4_fine_parallel.py:135-159
 *   stage-1.5 pool     _kernels/common/seoulkv4_cluster_blocks.py:107-115
 *   stage-1.5 scores   _kernels/codegen/stage15.py:886-905,
 *                      _kernels/stage15/seoulkv4_stage15_matrix.py:10-19
 *   stage-1.5 union    _kernels/stage15/seoulkv4_stage15_union.py:4-25
 *   stage-1.6          _kernels/stage16/seoulkv4_union_matrix.py:49-120,
 *                      _kernels/codegen/refinement.py:2914-3065
 *   stage-II           _kernels/codegen/refinement.py:3090-3152,3860-3880
 *
 * Canonical choices where the reference leaves the arithmetic unpinned
 * (TT FPU accumulation order, TopK-XL tie order):
 *   - every scoring dot product is the EXACT sum of (operand x small integer)
 *     products, rounded once to FP32 (RNE).  Operand rows are first flushed:
 *     an element whose magnitude is below 2^(E-22), E = floor(log2 max|x|)
 *     of that row, becomes zero.  The exact sum is formed here with 64-bit
 *     integers on a 2^(E-31) grid.
 *   - FP32 post-operations are single IEEE operations, each rounded to
 *     nearest even, never contracted into FMA (build with -ffp-contract=off).
 *   - FP32 -> BF16 is round-to-nearest-even.
 *   - query norm and query sum: pairwise (recursive halving) FP64 sums in
 *     dimension order, rounded to FP32.
 *   - selections rank by score (ordered BF16, descending); Fine ties follow
 *     the reference's fused [bf16 | u16 position] IEEE key; every other
 *     selection breaks ties by the lower candidate position.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define D 256
#define G 4

/* Host threads of the per-centroid / per-token scoring loops (1 unless
 * skv_oracle_set_threads raises it).  Each iteration writes only its own
 * outputs, so results do not depend on the thread count. */
static int g_threads = 1;
void skv_oracle_set_threads(int n) { g_threads = n > 0 ? n : 1; }

/* ------------------------------------------------------------------ bits */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

uint16_t skv_oracle_bf16_rne(float f) {
    uint32_t u = f2u(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float bf16f(uint16_t b) { return u2f((uint32_t)b << 16); }

/* Total order of BF16 bit patterns used by every reference selector
 * (_kernels/stage1_coarse/seoulkv4_coarse_select.py:31-36). */
static inline uint16_t ord16(uint16_t b) {
    return (uint16_t)(b ^ (0x8000u | (0u - (uint32_t)(b >> 15))));
}

/* IEEE order of the fused Fine key (bf16 << 16 | u16 position) mapped to an
 * unsigned total order (_kernels/stage1_fine/seoulkv4_fine_native_select.py:70-90). */
static inline uint32_t ord_fused(uint16_t score, uint32_t pos16) {
    uint32_t x = ((uint32_t)score << 16) | (pos16 & 0xffffu);
    return (x & 0x80000000u) ? ~x : (x | 0x80000000u);
}

/* ------------------------------------------------------------ structures */

typedef struct {
    int32_t nc;                  /* live centroids, multiple of 32 */
    int32_t nprobe;              /* P */
    float lam;                   /* interval lambda (FP32) */
    const uint8_t *upper;        /* [nc][64] codes >> 2, 4 per byte LE */
    const uint8_t *lower;        /* [nc][64] codes & 3 */
    const float *coarse_scale4;  /* [nc/32] group scale / 4 */
    const float *fine_scale;     /* [nc/32] FP16 group_fine_scale as FP32 */
    const uint16_t *resid_bf16;  /* [nc] BF16(coarse_residual_norm) */
    const int32_t *offsets;      /* [nc+1] CSR */
    const int32_t *values;       /* [offsets[nc]] token ids */
    int32_t context;             /* T */
    const uint8_t *prefix2;      /* [T][64] code8 >> 6 */
    const uint8_t *residual2;    /* [T][64] (code8 >> 4) & 3 */
    const uint8_t *residual4;    /* [T][128] code8 & 15 */
    const float *key_scale;      /* [256] per-dimension max |k| */
} OracleCell;

typedef struct {
    float qb[G][D];              /* BF16 query as FP32 */
    uint16_t q15[G][D];          /* bf16(q*s/64)  (reference "stage15" /16) */
    uint16_t qs[G][D];           /* bf16(q*s/256) */
    float qn[G];                 /* lambda * ||q|| */
    float qsum[G];               /* sum q */
    /* exact operand rows: value = X * 2^shift */
    int64_t xa[G][D]; int32_t sa[G];   /* q        (coarse, fine)  */
    int64_t xb[G][D]; int32_t sb[G];   /* 16*q15   (stage 1.5)     */
    int64_t xd[G][D]; int32_t sd[G];   /* qs       (stage II); 16*qs for 1.6 */
    /* the same operand rows before the flush (unflushed mode) */
    float ra[G][D], rb[G][D], rd[G][D];
} OracleQuery;

/* Unflushed mode (a measurement of the flush, not the canonical definition):
 * every operand element takes part in the exact sum, however small.  The
 * sum is formed with 128-bit integers on the grid of the row's smallest
 * element and rounded once to FP32.  A row whose elements span more than
 * UNFLUSHED_SPAN bits of exponent (which no query of the tests comes near)
 * drops the elements below that span, and g_unflushed_dropped counts them. */
static int g_unflushed = 0;
static long long g_unflushed_dropped = 0;
#define UNFLUSHED_SPAN 86
void skv_oracle_set_unflushed(int on) { g_unflushed = on != 0; g_unflushed_dropped = 0; }
long long skv_oracle_unflushed_dropped(void) { return g_unflushed_dropped; }

/* ------------------------------------------------------- query operands */

static double pairwise(const double *v, int n) {
    if (n == 1) return v[0];
    return pairwise(v, n / 2) + pairwise(v + n / 2, n - n / 2);
}

/* Flush + fixed point: kept elements are integers on the 2^(E-31) grid. */
static void exact_row(const float *x, int64_t *X, int32_t *shift) {
    int E = INT32_MIN;
    for (int d = 0; d < D; ++d)
        if (x[d] != 0.0f) { int e = ilogbf(x[d]); if (e > E) E = e; }
    if (E == INT32_MIN) { memset(X, 0, sizeof(int64_t) * D); *shift = 0; return; }
    const double floor_mag = ldexp(1.0, E - 22);
    for (int d = 0; d < D; ++d) {
        double v = (double)x[d];
        X[d] = fabs(v) < floor_mag ? 0 : (int64_t)ldexp(v, 31 - E);
    }
    *shift = E - 31;
}

void skv_oracle_prepare_query(const uint16_t *q /* [4][256] bf16 */,
                              const float *key_scale /* [256] */, float lam,
                              OracleQuery *o) {
    for (int h = 0; h < G; ++h) {
        double sq[D], sv[D];
        float b[D], d16[D];
        for (int d = 0; d < D; ++d) {
            float x = bf16f(q[h * D + d]);
            o->qb[h][d] = x;
            sq[d] = (double)x * (double)x;
            sv[d] = (double)x;
            float prod = x * key_scale[d];               /* fl(q*s) */
            o->q15[h][d] = skv_oracle_bf16_rne(prod / 64.0f);
            o->qs[h][d] = skv_oracle_bf16_rne(prod / 256.0f);
            b[d] = bf16f(o->q15[h][d]) * 16.0f;          /* exact */
            d16[d] = bf16f(o->qs[h][d]);
        }
        float norm = (float)sqrt(pairwise(sq, D));
        o->qn[h] = norm * lam;
        o->qsum[h] = (float)pairwise(sv, D);
        exact_row(o->qb[h], o->xa[h], &o->sa[h]);
        exact_row(b, o->xb[h], &o->sb[h]);
        exact_row(d16, o->xd[h], &o->sd[h]);
        memcpy(o->ra[h], o->qb[h], sizeof(float) * D);
        memcpy(o->rb[h], b, sizeof(float) * D);
        memcpy(o->rd[h], d16, sizeof(float) * D);
    }
}

/* sum_d row[d] * 2^e_add * w[d], exact, rounded once to FP32 (RNE); the
 * unflushed mode's dot (see g_unflushed). */
static float unflushed_dot(const float *row, int e_add, const int32_t *w) {
    int kmax = INT32_MIN, kmin = INT32_MAX;
    for (int d = 0; d < D; ++d)
        if (row[d] != 0.0f) {
            const int k = ilogbf(row[d]) - 23;   /* the element's lsb exponent (24-bit significand) */
            if (k > kmax) kmax = k;
            if (k < kmin) kmin = k;
        }
    if (kmax == INT32_MIN) return 0.0f;
    if (kmax - kmin > UNFLUSHED_SPAN) kmin = kmax - UNFLUSHED_SPAN;
    __int128 acc = 0;
    for (int d = 0; d < D; ++d) {
        if (row[d] == 0.0f) continue;
        const int k = ilogbf(row[d]) - 23;
        if (k < kmin) {
#pragma omp atomic
            ++g_unflushed_dropped;
            continue;
        }
        /* row[d] = m * 2^k exactly, |m| < 2^24 */
        const int64_t m = (int64_t)ldexp((double)row[d], -k);
        acc += ((__int128)m << (k - kmin)) * w[d];
    }
    const int neg = acc < 0;
    unsigned __int128 a = neg ? (unsigned __int128)(-acc) : (unsigned __int128)acc;
    if (a == 0) return 0.0f;
    int n = 0;
    for (unsigned __int128 t = a; t; t >>= 1) ++n;
    int e = kmin + e_add;
    uint64_t mant;
    if (n <= 24) {
        mant = (uint64_t)a;
    } else {
        const int sh = n - 24;
        mant = (uint64_t)(a >> sh);
        const unsigned __int128 rem = a & (((unsigned __int128)1 << sh) - 1);
        const unsigned __int128 half = (unsigned __int128)1 << (sh - 1);
        if (rem > half || (rem == half && (mant & 1))) ++mant;
        e += sh;
    }
    const float f = ldexpf((float)mant, e);   /* mant <= 2^24: exact */
    return neg ? -f : f;
}

/* FP32-accumulation mode (a measurement, not the canonical definition): the
 * dot is summed in FP32 in dimension order, rounding after every add, as a
 * float pipeline without exact accumulation would; the products themselves
 * (an 8-bit significand times an integer below 2^9) are exact in FP32. */
static int g_fp32_acc = 0;
void skv_oracle_set_fp32_accumulation(int on) { g_fp32_acc = on != 0; }

static float fp32_dot(const float *row, int e_add, const int32_t *w) {
    const float scale = ldexpf(1.0f, e_add);
    float acc = 0.0f;
    for (int d = 0; d < D; ++d) {
        const float p = row[d] * scale * (float)w[d];
        acc = acc + p;
    }
    return acc;
}

static inline float exact_dot(const int64_t *X, int32_t shift, const float *row, int e_add, const int32_t *w) {
    if (g_fp32_acc) return fp32_dot(row, e_add, w);
    if (g_unflushed) return unflushed_dot(row, e_add, w);
    int64_t acc = 0;
    for (int d = 0; d < D; ++d) acc += X[d] * (int64_t)w[d];
    return (float)ldexp((double)acc, shift);
}

/* ------------------------------------------------------------ selection */

typedef struct { uint64_t key; int32_t idx; } KeyIdx;

static int by_key_desc(const void *a, const void *b) {
    uint64_t x = ((const KeyIdx *)a)->key, y = ((const KeyIdx *)b)->key;
    return x < y ? 1 : x > y ? -1 : 0;
}

/* Rank order of the top-k entries of `keys` (unique 64-bit keys). */
static void top_k(KeyIdx *items, int n, int k, int32_t *out) {
    qsort(items, (size_t)n, sizeof(KeyIdx), by_key_desc);
    for (int i = 0; i < k; ++i) out[i] = items[i].idx;
}

/* Tie order of the Stage-1.5, 1.6 and II selections: equal scores go to the
 * lower position (the canonical rule); with g_tie_high set, to the higher
 * one.  The switch measures how much the unpinned tie order of the
 * reference's TT top-k can move the selected ids and the output; the engine
 * follows the canonical rule. */
static int g_tie_high = 0;
void skv_oracle_set_tie_high(int on) { g_tie_high = on != 0; }

static inline uint64_t rank_key(uint16_t score, int32_t pos) {
    const uint32_t low = g_tie_high ? (uint32_t)pos : 0xffffffffu - (uint32_t)pos;
    return ((uint64_t)ord16(score) << 32) | (uint64_t)low;
}

/* ---------------------------------------------------------------- coarse */

/* Returns the number of survivor tags written (ascending centroid order). */
int skv_oracle_coarse(const OracleCell *c, const OracleQuery *q, uint16_t *lo /* [4][nc] */,
                      uint16_t *hi, uint16_t *thresh /* [4] */, uint32_t *tags /* [nc] */) {
    const int nc = c->nc;
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
    for (int i = 0; i < nc; ++i) {
        int32_t w[D];
        const uint8_t *row = c->upper + (size_t)i * 64;
        for (int d = 0; d < D; ++d) w[d] = (row[d >> 2] >> (2 * (d & 3))) & 3;
        const float sc4 = c->coarse_scale4[i >> 5];
        const float r = bf16f(c->resid_bf16[i]);
        for (int h = 0; h < G; ++h) {
            float dot = exact_dot(q->xa[h], q->sa[h], q->ra[h], 0, w);
            float corr = 3.0f * q->qsum[h];
            float centered = 2.0f * dot - corr;
            float v = centered * sc4;
            float margin = q->qn[h] * r;
            lo[h * nc + i] = skv_oracle_bf16_rne(v - margin);
            hi[h * nc + i] = skv_oracle_bf16_rne(v + margin);
        }
    }
    KeyIdx *items_all = (KeyIdx *)malloc(sizeof(KeyIdx) * (size_t)nc * G);
#pragma omp parallel for schedule(static) num_threads(g_threads < G ? g_threads : G) if (g_threads > 1)
    for (int h = 0; h < G; ++h) {
        KeyIdx *items = items_all + (size_t)h * nc;
        for (int i = 0; i < nc; ++i) { items[i].key = ord16(lo[h * nc + i]); items[i].idx = i; }
        qsort(items, (size_t)nc, sizeof(KeyIdx), by_key_desc);
        thresh[h] = lo[h * nc + items[c->nprobe - 1].idx];
    }
    free(items_all);
    int n = 0;
    for (int i = 0; i < nc; ++i) {
        uint32_t mask = 0;
        for (int h = 0; h < G; ++h)
            mask |= (uint32_t)(ord16(hi[h * nc + i]) >= ord16(thresh[h])) << h;
        if (mask) tags[n++] = (uint32_t)i | (mask << 28);
    }
    return n;
}

/* ------------------------------------------------------------------ fine */

/* scores [4][ntags] (BF16 bits; 0xff80 for ineligible), top [4][P] survivor
 * positions in rank order, selected cluster ids ascending.  Returns the
 * number of selected clusters, or -1 when a head has fewer than P eligible
 * survivors. */
int skv_oracle_fine(const OracleCell *c, const OracleQuery *q, const uint32_t *tags, int ntags,
                    uint16_t *scores, int32_t *top, int32_t *selected) {
    const int P = c->nprobe;
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
    for (int i = 0; i < ntags; ++i) {
        int32_t w[D];
        const uint32_t cid = tags[i] & 0x0fffffffu, mask = tags[i] >> 28;
        const uint8_t *up = c->upper + (size_t)cid * 64, *lw = c->lower + (size_t)cid * 64;
        for (int d = 0; d < D; ++d) {
            int code = (((up[d >> 2] >> (2 * (d & 3))) & 3) << 2) | ((lw[d >> 2] >> (2 * (d & 3))) & 3);
            w[d] = 2 * code - 15;
        }
        const float fs = c->fine_scale[cid >> 5];
        for (int h = 0; h < G; ++h) {
            if (!((mask >> h) & 1)) { scores[h * ntags + i] = 0xff80u; continue; }
            float dot = exact_dot(q->xa[h], q->sa[h], q->ra[h], 0, w);
            scores[h * ntags + i] = skv_oracle_bf16_rne(dot * fs);
        }
    }
    KeyIdx *items = (KeyIdx *)malloc(sizeof(KeyIdx) * (size_t)(ntags > 0 ? ntags : 1));
    uint8_t *chosen = (uint8_t *)calloc((size_t)(ntags > 0 ? ntags : 1), 1);
    int bad = 0;
    for (int h = 0; h < G; ++h) {
        int n = 0;
        for (int i = 0; i < ntags; ++i) {
            if (!((tags[i] >> 28 >> h) & 1)) continue;
            items[n].key = ((uint64_t)ord_fused(scores[h * ntags + i], (uint32_t)i) << 32) |
                           (uint64_t)(0xffffffffu - (uint32_t)i);
            items[n].idx = i;
            ++n;
        }
        if (n < P) { bad = 1; break; }
        top_k(items, n, P, top + h * P);
        for (int j = 0; j < P; ++j) chosen[top[h * P + j]] = 1;
    }
    int nsel = 0;
    if (!bad)
        for (int i = 0; i < ntags; ++i)
            if (chosen[i]) selected[nsel++] = (int32_t)(tags[i] & 0x0fffffffu);
    free(items);
    free(chosen);
    return bad ? -1 : nsel;
}

/* ------------------------------------------------------------------ pool */

/* First-occurrence union of the selected clusters' posting lists
 * (_kernels/common/seoulkv4_cluster_blocks.py:107-115).  Writes at most
 * `limit` tokens and returns the full union size. */
int skv_oracle_pool(const OracleCell *c, const int32_t *selected, int nsel, int32_t *pool, int limit) {
    uint8_t *seen = (uint8_t *)calloc((size_t)c->context, 1);
    int n = 0;
    for (int s = 0; s < nsel; ++s) {
        const int cid = selected[s];
        for (int j = c->offsets[cid]; j < c->offsets[cid + 1]; ++j) {
            const int t = c->values[j];
            if (seen[t]) continue;
            seen[t] = 1;
            if (n < limit) pool[n] = t;
            ++n;
        }
    }
    free(seen);
    return n;
}

/* ----------------------------------------------------------- stage 1.5 */

static inline int p2_at(const uint8_t *row, int d) { return (row[d >> 2] >> (2 * (d & 3))) & 3; }
static inline int r4_at(const uint8_t *row, int d) { return (row[d >> 1] >> (4 * (d & 1))) & 15; }

/* scores [4][npool]; top [4][m] pool positions in rank order; u15 pool
 * positions ascending.  Returns |u15|. */
int skv_oracle_stage15(const OracleCell *c, const OracleQuery *q, const int32_t *pool, int npool,
                       int m, uint16_t *scores, int32_t *top, int32_t *u15) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
    for (int i = 0; i < npool; ++i) {
        int32_t w[D];
        const uint8_t *row = c->prefix2 + (size_t)pool[i] * 64;
        for (int d = 0; d < D; ++d) w[d] = 2 * p2_at(row, d) - 3;
        for (int h = 0; h < G; ++h)
            scores[h * npool + i] = skv_oracle_bf16_rne(exact_dot(q->xb[h], q->sb[h], q->rb[h], 0, w));
    }
    const int k = m < npool ? m : npool;
    KeyIdx *items_all = (KeyIdx *)malloc(sizeof(KeyIdx) * (size_t)npool * G);
#pragma omp parallel for schedule(static) num_threads(g_threads < G ? g_threads : G) if (g_threads > 1)
    for (int h = 0; h < G; ++h) {
        KeyIdx *items = items_all + (size_t)h * npool;
        for (int i = 0; i < npool; ++i) { items[i].key = rank_key(scores[h * npool + i], i); items[i].idx = i; }
        top_k(items, npool, k, top + h * m);
    }
    uint8_t *chosen = (uint8_t *)calloc((size_t)npool, 1);
    for (int h = 0; h < G; ++h)
        for (int j = 0; j < k; ++j) chosen[top[h * m + j]] = 1;
    int n = 0;
    for (int i = 0; i < npool; ++i) if (chosen[i]) u15[n++] = i;
    free(items_all);
    free(chosen);
    return n;
}

/* ----------------------------------------------------------- stage 1.6 */

/* scores [4][nu]; top [4][m] u15 positions in rank order; cand u15
 * positions ascending.  Returns |cand|. */
int skv_oracle_stage16(const OracleCell *c, const OracleQuery *q, const int32_t *pool,
                       const int32_t *u15, int nu, int m, uint16_t *scores, int32_t *top,
                       int32_t *cand) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
    for (int u = 0; u < nu; ++u) {
        int32_t w[D];
        const int t = pool[u15[u]];
        const uint8_t *p = c->prefix2 + (size_t)t * 64, *r = c->residual2 + (size_t)t * 64;
        for (int d = 0; d < D; ++d) w[d] = 2 * ((p2_at(p, d) << 2) | p2_at(r, d)) - 15;
        for (int h = 0; h < G; ++h)   /* operand 16*qs: same integers, shift + 4 */
            scores[h * nu + u] = skv_oracle_bf16_rne(exact_dot(q->xd[h], q->sd[h] + 4, q->rd[h], 4, w));
    }
    const int k = m < nu ? m : nu;
    KeyIdx *items_all = (KeyIdx *)malloc(sizeof(KeyIdx) * (size_t)(nu > 0 ? nu : 1) * G);
#pragma omp parallel for schedule(static) num_threads(g_threads < G ? g_threads : G) if (g_threads > 1)
    for (int h = 0; h < G; ++h) {
        KeyIdx *items = items_all + (size_t)h * nu;
        for (int u = 0; u < nu; ++u) { items[u].key = rank_key(scores[h * nu + u], u); items[u].idx = u; }
        top_k(items, nu, k, top + h * m);
    }
    uint8_t *chosen = (uint8_t *)calloc((size_t)(nu > 0 ? nu : 1), 1);
    for (int h = 0; h < G; ++h)
        for (int j = 0; j < k; ++j) chosen[top[h * m + j]] = 1;
    int n = 0;
    for (int u = 0; u < nu; ++u) if (chosen[u]) cand[n++] = u;
    free(items_all);
    free(chosen);
    return n;
}

/* ------------------------------------------------------------ stage II */

/* scores [4][ncand]; final_pos [4][k] u15 positions in rank order;
 * final_ids [4][k] token ids. */
void skv_oracle_stage2(const OracleCell *c, const OracleQuery *q, const int32_t *pool,
                       const int32_t *u15, const int32_t *cand, int ncand, int k,
                       uint16_t *scores, int32_t *final_pos, int32_t *final_ids) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
    for (int j = 0; j < ncand; ++j) {
        int32_t w[D];
        const int t = pool[u15[cand[j]]];
        const uint8_t *p = c->prefix2 + (size_t)t * 64, *r = c->residual2 + (size_t)t * 64,
                      *r4 = c->residual4 + (size_t)t * 128;
        for (int d = 0; d < D; ++d) {
            int code8 = (p2_at(p, d) << 6) | (p2_at(r, d) << 4) | r4_at(r4, d);
            w[d] = 2 * code8 - 255;
        }
        for (int h = 0; h < G; ++h)
            scores[h * ncand + j] = skv_oracle_bf16_rne(exact_dot(q->xd[h], q->sd[h], q->rd[h], 0, w));
    }
    KeyIdx *items = (KeyIdx *)malloc(sizeof(KeyIdx) * (size_t)ncand);
    for (int h = 0; h < G; ++h) {
        for (int j = 0; j < ncand; ++j) { items[j].key = rank_key(scores[h * ncand + j], cand[j]); items[j].idx = j; }
        int32_t idx[1024];
        top_k(items, ncand, k, idx);
        for (int r = 0; r < k; ++r) {
            final_pos[h * k + r] = cand[idx[r]];
            final_ids[h * k + r] = pool[u15[cand[idx[r]]]];
        }
    }
    free(items);
}

size_t skv_oracle_query_bytes(void) { return sizeof(OracleQuery); }
