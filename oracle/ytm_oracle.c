/*
 * ytm_oracle.c — CPU restatement of the reference Tsetlin Machine path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA engine in
 * ytm_b200/: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg may load it.  The product never links or calls it.
 *
 * It restates Mayur1009/YTM src/cutm/cuda/kernel.cu and src/cutm/base.py on the
 * reference's own data layout (one u32 per TA state, [C][L]), one sample or
 * clause at a time, with no bit-slicing, so that it shares no design with the
 * engine it checks.  Each function cites the reference lines it follows.
 *
 * Where the reference draws from curand XORWOW in a data-dependent order
 * (kernel.cu:298, 425-428, 457-460, 573, 582), the restatement takes its
 * decisions from a counter-based Philox4x32-10 stream instead (Salmon, Moraes,
 * Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC'11).  The
 * decision rules are written once here and once in the engine; the training
 * parity tests compare the two bit for bit.  With s = 1, q = K-1 and class sums
 * at +-T every decision is forced, and the restatement then matches the
 * reference kernels themselves (tests/golden fixtures made by the reference).
 *
 * Mini-batches (the reference trains one sample at a time, base.py:306) are
 * defined as: include counts, clause outputs, patch picks and class sums of all
 * B samples are computed on the state at batch start; then every clause applies
 * its feedback for samples 0..B-1 in order, its weights and states changing as
 * it goes.  With B = 1 this is exactly the reference's per-sample loop.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef struct orc_cfg {
    int32_t clauses_per_class, T;
    double s, q;
    int32_t D0, D1, D2, K, P0, P1;
    int32_t n_states, max_included, append_negated, init_neg_weights, negative_polarity;
    int32_t encode_loc, coalesced;
    uint64_t seed;
    /* derived, base.py:94-121 */
    int32_t banks, C, L, W, P;
    int32_t max_state, half_state, state_top;
    uint32_t s_cdf[32];
    uint64_t q_thr;
    uint32_t q_cdf[32];
    int32_t q_select;
    uint32_t run_cdf16[8][65];
    /* rule variants of the reference's CPU TM, pytm/base.py (0 = cutm rules) */
    int32_t one_negative; /* one uniformly chosen negative class per sample, true class first (base.py:139-143) */
    int32_t count_empty;  /* inference counts clauses without includes (base.py:59-67) */
} orc_cfg;

void orc_cfg_set_modes(orc_cfg *c, int32_t one_negative, int32_t count_empty) {
    c->one_negative = one_negative;
    c->count_empty = count_empty;
}

/* The literal mask's set-literal count among 32 is Binomial(32, p) with
 * p = 1/s (the reference's S_INV, kernel.cu:31, used at 425-428, 457-460):
 * cdf[n] = floor(2^32 * P(count <= n)), saturated at 2^32 - 1, from the pmf
 * recurrence pmf(n+1) = pmf(n) * (32-n)/(n+1) * p/(1-p) in IEEE double. */
static void count_cdf(double s, uint32_t cdf[32]) {
    double p = 1.0 / s;
    if (!(p > 0.0)) p = 0.0;
    if (p > 1.0) p = 1.0;
    const double q = 1.0 - p;
    if (!(q > 0.0)) { /* p = 1: every literal is set */
        for (int n = 0; n < 32; ++n) cdf[n] = 0u;
        return;
    }
    double pmf = 1.0, acc = 0.0;
    for (int i = 0; i < 32; ++i) pmf *= q;
    for (int n = 0; n < 32; ++n) {
        acc += pmf;
        const double v = floor(acc * 4294967296.0);
        cdf[n] = v >= 4294967295.0 ? 0xFFFFFFFFu : (uint32_t)v;
        pmf = pmf * (double)(32 - n) / (double)(n + 1) * p / q;
    }
}

/* Type Ib runs are taken inside windows of 128 samples of the batch (64 when
 * the clause sees more than 256 classes). */
static int run_window(const orc_cfg *c) { return (c->coalesced ? c->K : 1) <= 256 ? 128 : 64; }

/* Type Ib runs (see orc_train_update): for m = 8, 16, ..., 64 events the number
 * of decrements of one literal is Binomial(m, p), p = 1/s; entry d of row mi
 * (m = 8 (mi + 1)) is 65536 * P(count <= d) rounded to nearest, 65536 from
 * d = m on; the same pmf recurrence in IEEE double. */
static const int RUN_SIZES[8] = {8, 16, 24, 32, 40, 48, 56, 64};

static void run_cdf(double s, uint32_t out[8][65]) {
    double p = 1.0 / s;
    if (!(p > 0.0)) p = 0.0;
    if (p > 1.0) p = 1.0;
    const double q = 1.0 - p;
    for (int mi = 0; mi < 8; ++mi) {
        const int m = RUN_SIZES[mi];
        for (int d = 0; d < 65; ++d) out[mi][d] = 65536u;
        if (!(q > 0.0)) { /* p = 1: every event decrements */
            for (int d = 0; d < m; ++d) out[mi][d] = 0u;
            continue;
        }
        double pmf = 1.0, acc = 0.0;
        for (int i = 0; i < m; ++i) pmf *= q;
        for (int d = 0; d < m; ++d) {
            acc += pmf;
            const double v = floor(acc * 65536.0 + 0.5); /* nearest: a tail below 2^-17 is never drawn */
            out[mi][d] = v >= 65536.0 ? 65536u : (uint32_t)v;
            pmf = pmf * (double)(m - d) / (double)(d + 1) * p / q;
        }
    }
}

/* ---------------------------------------------------------------- sizes */

/* base.py:76-121 and the macro preamble base.py:129-152. */
int orc_cfg_init(orc_cfg *c, int32_t clauses_per_class, int32_t T, double s, int32_t D0, int32_t D1,
                 int32_t D2, int32_t K, double q, int32_t P0, int32_t P1, int32_t n_states,
                 int32_t max_included, int32_t append_negated, int32_t init_neg_weights,
                 int32_t negative_polarity, int32_t encode_loc, int32_t coalesced, uint64_t seed) {
    memset(c, 0, sizeof(*c));
    c->clauses_per_class = clauses_per_class;
    c->T = T;
    c->s = s;
    c->q = q < (double)K ? q : (double)K; /* base.py:81 */
    c->D0 = D0; c->D1 = D1; c->D2 = D2; c->K = K; c->P0 = P0; c->P1 = P1;
    c->n_states = n_states;
    c->append_negated = append_negated; c->init_neg_weights = init_neg_weights;
    c->negative_polarity = negative_polarity; c->encode_loc = encode_loc; c->coalesced = coalesced;
    c->seed = seed;
    c->banks = coalesced ? 1 : K;                     /* base.py:94 */
    c->C = c->banks * clauses_per_class;              /* base.py:95 */
    if (encode_loc)                                   /* base.py:108-115 */
        c->L = P0 * P1 * D2 + (D0 - P0) + (D1 - P1);
    else
        c->L = P0 * P1 * D2;
    if (append_negated) c->L *= 2;                    /* base.py:117-118 */
    c->W = (c->L - 1) / 32 + 1;                       /* base.py:120 */
    c->P = (D0 - P0 + 1) * (D1 - P1 + 1);             /* base.py:121 */
    c->max_included = max_included < 0 ? c->L : max_included; /* base.py:141 */
    c->max_state = n_states;                          /* base.py:146 */
    c->half_state = n_states / 2;                     /* kernel.cu:33 */
    /* Type II feedback has no upper check (kernel.cu:481-506); one sample can
     * raise an excluded state by at most K, so half + max(half, K) bounds it. */
    {
        int32_t m = c->max_state - c->half_state;
        if (K > m) m = K;
        int32_t p = 1;
        while (p < m || p < c->half_state + 1) p <<= 1;
        c->state_top = p + c->half_state;
    }
    count_cdf(s, c->s_cdf);
    run_cdf(s, c->run_cdf16);
    {
        double qp = c->q / (double)(K - 1 > 1 ? K - 1 : 1); /* kernel.cu:32 */
        if (qp >= 1.0) c->q_thr = 4294967296ull;
        else if (!(qp > 0.0)) c->q_thr = 0;
        else c->q_thr = (uint64_t)floor(qp * 4294967296.0);
        /* coalesced models of at least 32 classes with K * Q <= 2 draw the selection as a set per
         * (clause, sample); count ~ Binomial(K, Q) */
        if (!(qp > 0.0)) qp = 0.0;
        if (qp > 1.0) qp = 1.0;
        c->q_select = (coalesced && K >= 32 && qp > 0.0 && qp < 1.0 && qp * K <= 2.0) ? 1 : 0;
        for (int n = 0; n < 32; ++n) c->q_cdf[n] = 0xFFFFFFFFu;
        if (c->q_select) {
            const double qq = 1.0 - qp;
            double pmf = 1.0, acc = 0.0;
            for (int i = 0; i < K; ++i) pmf *= qq;
            for (int n = 0; n < 32; ++n) {
                acc += pmf;
                const double v = floor(acc * 4294967296.0);
                c->q_cdf[n] = v >= 4294967295.0 ? 0xFFFFFFFFu : (uint32_t)v;
                pmf = n < K ? pmf * (double)(K - n) / (double)(n + 1) * qp / qq : 0.0;
            }
        }
    }
    if (c->W <= 0 || c->P <= 0 || c->C <= 0 || K <= 0) return 1;
    return 0;
}

void orc_cfg_sizes(const orc_cfg *c, int32_t *out) {
    out[0] = c->C; out[1] = c->K; out[2] = c->L; out[3] = c->W; out[4] = c->P;
    out[5] = c->state_top; out[6] = (int32_t)c->s_cdf[0]; out[7] = c->half_state;
}

void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int orc_get_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* --------------------------------------------------------------- Philox */

/* Philox4x32-R (Salmon et al., SC'11): multipliers 0xD2511F53, 0xCD9E8D57,
 * Weyl key increments 0x9E3779B9, 0xBB67AE85. */
void orc_philox4x32(const uint32_t ctr_in[4], const uint32_t key_in[2], int rounds, uint32_t out[4]) {
    uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
    uint32_t k0 = key_in[0], k1 = key_in[1];
    for (int r = 0; r < rounds; ++r) {
        if (r) { k0 += 0x9E3779B9u; k1 += 0xBB67AE85u; }
        uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
        uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

void orc_philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4]) {
    orc_philox4x32(ctr_in, key_in, 10, out);
}

/* Decision streams.  counter = (global clause, sample counter low 32 bits,
 * sub-index, tag | class << 2); key = (seed low, seed high ^ sample high). */
enum { TAG_PATCH = 0, TAG_CLASS = 1, TAG_SMASK = 2, TAG_INIT = 3 };

static inline void draw_r(const orc_cfg *c, uint32_t clause, uint64_t t, uint32_t sub, uint32_t tag,
                          uint32_t k, int rounds, uint32_t out[4]) {
    uint32_t ctr[4] = {clause, (uint32_t)t, sub, tag | (k << 2)};
    uint32_t key[2] = {(uint32_t)c->seed, (uint32_t)(c->seed >> 32) ^ (uint32_t)(t >> 32)};
    orc_philox4x32(ctr, key, rounds, out);
}

/* The patch pick and pytm's other-class draw use Philox4x32-10; the per-class
 * decision draws and the bulk literal-mask draws use the 7-round variant,
 * which Salmon et al. report as passing BigCrush. */
static inline void draw(const orc_cfg *c, uint32_t clause, uint64_t t, uint32_t sub, uint32_t tag,
                        uint32_t k, uint32_t out[4]) {
    draw_r(c, clause, t, sub, tag, k, 10, out);
}

/* Bernoulli(1/s) for the 32 literals of word w (stands in for the reference's
 * per-literal `curand_uniform(rng) <= S_INV`, kernel.cu:425-428, 439,
 * 457-460, 466), by count and placement: the first Philox4x32-7 word r0 of
 * counter sub-index 4w gives the number n of set literals, the smallest n
 * with r0 < cdf[n] (32 if none), i.e. Binomial(32, 1/s); then n distinct
 * positions (or, when n > 16, the 32 - n unset ones) are drawn uniformly by
 * rejection from 5-bit fields: bits 0-4, 5-9, ..., 25-29 of r1, r2, r3, then
 * of all four words of further draws at sub-indices 4w+1, 4w+2, ...  Given n,
 * every n-subset is equally likely, so the bits are independent
 * Bernoulli(p) up to the 2^-32 resolution of the table. */
static uint64_t g_smask_draws;
static int g_smask_counting;

/* Count the Philox4x32-7 calls of orc_smask_word from now on (on != 0) or
 * stop; returns the count so far and resets it. */
uint64_t orc_smask_count(int on) {
    uint64_t v;
#pragma omp atomic read
    v = g_smask_draws;
#pragma omp atomic write
    g_smask_draws = 0;
    g_smask_counting = on;
    return v;
}

uint32_t orc_smask_word(const orc_cfg *c, uint32_t clause, uint64_t t, uint32_t k, uint32_t w) {
    uint32_t R[4];
    uint32_t sub = w * 4u, calls = 1;
    draw_r(c, clause, t, sub, TAG_SMASK, k, 7, R);
    uint32_t n = 0;
    while (n < 32 && R[0] >= c->s_cdf[n]) ++n;
    const int holes = n > 16;
    uint32_t need = holes ? 32u - n : n, m = 0u;
    int wi = 1, left = 6;
    uint32_t cur = R[1];
    while (need) {
        if (left == 0) {
            if (++wi == 4) {
                draw_r(c, clause, t, ++sub, TAG_SMASK, k, 7, R);
                ++calls;
                wi = 0;
            }
            cur = R[wi];
            left = 6;
        }
        const uint32_t b = 1u << (cur & 31u);
        cur >>= 5;
        --left;
        if (!(m & b)) { m |= b; --need; }
    }
    if (g_smask_counting) {
#pragma omp atomic
        g_smask_draws += calls;
    }
    return holes ? ~m : m;
}

/* floor(p * 2^32) for p = (y - v) / (2y), kernel.cu:508-529 (h and mod unused
 * there, as here). */
uint64_t orc_update_threshold(int32_t y, int32_t v) {
    double p = ((double)y - (double)v) / (2.0 * (double)y);
    if (!(p > 0.0)) return 0;
    if (p >= 1.0) return 4294967296ull;
    return (uint64_t)floor(p * 4294967296.0);
}

/* --------------------------------------------------------------- encode */

/* encode_batch, kernel.cu:76-152, one (sample, patch) at a time.  out is
 * zeroed first as base.py:245 does. */
void orc_encode(const orc_cfg *c, const uint32_t *X, int64_t N, uint32_t *out) {
    const int L = c->L, W = c->W, P = c->P;
    const int D0 = c->D0, D1 = c->D1, D2 = c->D2, P0 = c->P0, P1 = c->P1;
    memset(out, 0, (size_t)N * P * W * sizeof(uint32_t));
#pragma omp parallel for schedule(static)
    for (int64_t ep = 0; ep < N * (int64_t)P; ++ep) {
        int64_t e = ep / P;
        int patch = (int)(ep % P);
        int py = patch / (D0 - P0 + 1);
        int px = patch % (D0 - P0 + 1);
        uint32_t *o = out + ep * W;
        if (c->append_negated)
            for (int l = L / 2; l < L; ++l) o[l / 32] |= 1u << (l % 32);
        for (int l = 0; l < py; ++l) {
            o[l / 32] |= 1u << (l % 32);
            if (c->append_negated) { int n = l + L / 2; o[n / 32] &= ~(1u << (n % 32)); }
        }
        for (int l = 0; l < px; ++l) {
            int b = D1 - P1 + l;
            o[b / 32] |= 1u << (b % 32);
            if (c->append_negated) { int n = b + L / 2; o[n / 32] &= ~(1u << (n % 32)); }
        }
        for (int y = py; y < py + P1; ++y)
            for (int x = px; x < px + P0; ++x)
                for (int z = 0; z < D2; ++z) {
                    int64_t idx = e * (int64_t)(D0 * D1 * D2) + (int64_t)y * (D0 * D2) + x * D2 + z;
                    if (X[idx] > 0) {
                        int ry = y - py, rx = x - px;
                        int pos = ry * P0 * D2 + rx * D2 + z;
                        if (c->encode_loc) pos += (D1 - P1) + (D0 - P0);
                        o[pos / 32] |= 1u << (pos % 32);
                        if (c->append_negated) { int n = pos + L / 2; o[n / 32] &= ~(1u << (n % 32)); }
                    }
                }
    }
}

/* ------------------------------------------------------- pack and match */

/* pack_clauses, kernel.cu:155-204, for clauses [0, nc). */
void orc_pack(const orc_cfg *c, const uint32_t *ta, int32_t nc, uint32_t *packed, int32_t *ninc) {
    const int L = c->L, W = c->W;
#pragma omp parallel for schedule(static)
    for (int32_t cl = 0; cl < nc; ++cl) {
        const uint32_t *t = ta + (int64_t)cl * L;
        int count = 0;
        for (int w = 0; w < W; ++w) {
            uint32_t v = 0;
            int end = (w + 1) * 32 < L ? (w + 1) * 32 : L;
            for (int l = w * 32; l < end; ++l)
                if (t[l] > (uint32_t)c->half_state) { v |= 1u << (l % 32); ++count; }
            packed[(int64_t)cl * W + w] = v;
        }
        ninc[cl] = count;
    }
}

/* clause_match, kernel.cu:207-216. */
static inline int match(const orc_cfg *c, const uint32_t *inc, const uint32_t *x) {
    const int W = c->W;
    for (int w = 0; w < W - 1; ++w)
        if ((inc[w] & x[w]) != inc[w]) return 0;
    uint32_t filt = (c->L % 32) ? ~(0xFFFFFFFFu << (c->L % 32)) : 0xFFFFFFFFu;
    if ((inc[W - 1] & (x[W - 1] & filt)) != (inc[W - 1] & filt)) return 0;
    return 1;
}

static inline int clause_class(const orc_cfg *c, int32_t gclause) {
    return gclause / c->clauses_per_class; /* CLAUSES_PER_BANK, kernel.cu:29, 307 */
}

/* ------------------------------------------------------------ inference */

/* calc_class_sums_infer_batch, kernel.cu:319-343, with the bias tiling of
 * _score_batch (base.py:388-392).  Weights are whole numbers; the reference's
 * float sums of them are exact below 2^24, the int64 sums here everywhere. */
void orc_infer(const orc_cfg *c, const uint32_t *ta, const int32_t *weights, const int32_t *bias,
               const uint32_t *lits, int64_t N, int32_t *cs) {
    const int C = c->C, K = c->K, W = c->W, P = c->P;
    uint32_t *packed = (uint32_t *)malloc((size_t)C * W * 4);
    int32_t *ninc = (int32_t *)malloc((size_t)C * 4);
    orc_pack(c, ta, C, packed, ninc);
#pragma omp parallel for schedule(dynamic, 16)
    for (int64_t e = 0; e < N; ++e) {
        int64_t acc[1024];
        int64_t *a = K <= 1024 ? acc : (int64_t *)malloc((size_t)K * 8);
        for (int k = 0; k < K; ++k) a[k] = bias ? bias[k] : 0;
        for (int cl = 0; cl < C; ++cl) {
            if (ninc[cl] == 0 && !c->count_empty) continue; /* kernel.cu:328 */
            int out = 0;
            for (int p = 0; p < P && !out; ++p)
                out = match(c, packed + (int64_t)cl * W, lits + (e * P + p) * W);
            if (out)
                for (int k = 0; k < K; ++k) a[k] += weights[(int64_t)cl * K + k];
        }
        for (int k = 0; k < K; ++k) cs[e * K + k] = (int32_t)a[k];
        if (a != acc) free(a);
    }
    free(packed);
    free(ninc);
}

/* transform, kernel.cu:346-368: empty clauses give 1. */
void orc_transform(const orc_cfg *c, const uint32_t *ta, const uint32_t *lits, int64_t N,
                   uint32_t *out) {
    const int C = c->C, W = c->W, P = c->P;
    uint32_t *packed = (uint32_t *)malloc((size_t)C * W * 4);
    int32_t *ninc = (int32_t *)malloc((size_t)C * 4);
    orc_pack(c, ta, C, packed, ninc);
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < N; ++e)
        for (int cl = 0; cl < C; ++cl) {
            int o = 0;
            if (ninc[cl] == 0) o = 1;
            else
                for (int p = 0; p < P && !o; ++p)
                    o = match(c, packed + (int64_t)cl * W, lits + (e * P + p) * W);
            out[e * C + cl] = (uint32_t)o;
        }
    free(packed);
    free(ninc);
}

/* transform_patchwise, kernel.cu:370-394. */
void orc_transform_patchwise(const orc_cfg *c, const uint32_t *ta, const uint32_t *lits, int64_t N,
                             uint32_t *out) {
    const int C = c->C, W = c->W, P = c->P;
    uint32_t *packed = (uint32_t *)malloc((size_t)C * W * 4);
    int32_t *ninc = (int32_t *)malloc((size_t)C * 4);
    orc_pack(c, ta, C, packed, ninc);
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < N; ++e)
        for (int cl = 0; cl < C; ++cl)
            for (int p = 0; p < P; ++p)
                out[(e * C + cl) * P + p] =
                    ninc[cl] == 0 ? 1u : (uint32_t)match(c, packed + (int64_t)cl * W, lits + (e * P + p) * W);
    free(packed);
    free(ninc);
}

/* ---------------------------------------------------------- init weights */

/* init_weights, kernel.cu:46-73, for global clauses [lo, lo+nc).  Coalesced
 * +-1 signs come from the TAG_INIT stream instead of curand()%2. */
void orc_init_weights(const orc_cfg *c, int32_t lo, int32_t nc, int32_t *w) {
    const int K = c->K;
    for (int32_t i = 0; i < nc; ++i) {
        int32_t g = lo + i;
        for (int k = 0; k < K; ++k) {
            int32_t v;
            if (c->coalesced) {
                v = 1;
                if (c->init_neg_weights) {
                    uint32_t r[4];
                    draw(c, (uint32_t)g, 0, 0, TAG_INIT, (uint32_t)k, r);
                    v = (r[0] & 1u) ? -1 : 1;
                }
            } else if (k == clause_class(c, g)) {
                v = 1;
                if (c->init_neg_weights && (g % c->clauses_per_class) >= c->clauses_per_class / 2) v = -1;
            } else {
                v = 0;
            }
            w[(int64_t)i * K + k] = v;
        }
    }
}

/* ------------------------------------------------------------- training */

/* Part 1 of a batch, for the global clause range [lo, lo+nc): fast_eval
 * (kernel.cu:255-282) and select_active (kernel.cu:285-316) for each of the B
 * samples on the batch-start state.  Arrays are shard-local: ta [nc][L],
 * w [nc][K], drop [nc] (or NULL), patch_w [nc][P], sel [B][nc], ninc [nc].
 * cs [B][K] receives the shard's class sums (+ bias if add_bias). */
void orc_train_eval(const orc_cfg *c, int32_t lo, int32_t nc, const uint32_t *ta, const int32_t *w,
                    const int32_t *bias, const uint32_t *drop, const uint32_t *lits, int32_t B,
                    uint64_t t0, int32_t add_bias, int32_t *cs, int32_t *patch_w, int32_t *sel,
                    int32_t *ninc) {
    const int K = c->K, W = c->W, P = c->P;
    uint32_t *packed = (uint32_t *)malloc((size_t)nc * W * 4);
    orc_pack(c, ta, nc, packed, ninc);
#pragma omp parallel for schedule(dynamic, 8)
    for (int32_t i = 0; i < nc; ++i) {
        int32_t *act = (int32_t *)malloc((size_t)P * 4);
        for (int32_t b = 0; b < B; ++b) {
            int32_t s_ = -1;
            if (!(drop && drop[i] == 1)) {
                int cnt = 0;
                for (int p = 0; p < P; ++p) {
                    int o = ninc[i] == 0 ? 1 /* kernel.cu:273-276 */
                                         : match(c, packed + (int64_t)i * W,
                                                 lits + ((int64_t)b * P + p) * W);
                    if (o) act[cnt++] = p;
                }
                if (cnt > 0) {
                    uint32_t r[4];
                    draw(c, (uint32_t)(lo + i), t0 + (uint64_t)b, 0, TAG_PATCH, 0, r);
                    s_ = act[((uint64_t)r[0] * (uint64_t)cnt) >> 32];
                    patch_w[(int64_t)i * P + s_] += 1; /* kernel.cu:305 */
                }
            }
            sel[(int64_t)b * nc + i] = s_;
        }
        free(act);
    }
    /* class sums, kernel.cu:304-313, summed in a fixed order */
    for (int32_t b = 0; b < B; ++b)
        for (int k = 0; k < K; ++k) {
            int64_t a = (add_bias && bias) ? bias[k] : 0;
            for (int32_t i = 0; i < nc; ++i) {
                if (sel[(int64_t)b * nc + i] < 0) continue;
                if (!c->coalesced && clause_class(c, lo + i) != k) continue;
                a += w[(int64_t)i * K + k];
            }
            cs[(int64_t)b * K + k] = (int32_t)a;
        }
    free(packed);
}

static inline int32_t clip_cs(const orc_cfg *c, int32_t v) { /* kernel.cu:397 */
    return v > c->T ? c->T : (v < -c->T ? -c->T : v);
}

/* type1a_fb, kernel.cu:410-443 */
static void type1a(const orc_cfg *c, uint32_t *st, const uint32_t *x, uint32_t g, uint64_t t, uint32_t k) {
    const int L = c->L;
    uint32_t mask = 0;
    int mw = -1;
    for (int l = 0; l < L; ++l) {
        uint32_t bit = (x[l / 32] >> (l % 32)) & 1u;
        if (bit == 1u && st[l] < (uint32_t)c->max_state) {
            st[l] += 1;
        } else if (bit == 0u && st[l] > 0) {
            if (mw != l / 32) { mw = l / 32; mask = orc_smask_word(c, g, t, k, (uint32_t)mw); }
            if ((mask >> (l % 32)) & 1u) st[l] -= 1;
        }
    }
}

/* type1b_fb, kernel.cu:453-470 */
static void type1b(const orc_cfg *c, uint32_t *st, uint32_t g, uint64_t t, uint32_t k) {
    const int L = c->L;
    uint32_t mask = 0;
    int mw = -1;
    for (int l = 0; l < L; ++l) {
        if (st[l] > 0) {
            if (mw != l / 32) { mw = l / 32; mask = orc_smask_word(c, g, t, k, (uint32_t)mw); }
            if ((mask >> (l % 32)) & 1u) st[l] -= 1;
        }
    }
}

/* A run of m (8, 16 or 32) consecutive Type Ib events of one clause, which
 * the reference applies one by one (type1b_fb, kernel.cu:453-470: each
 * decrements every literal with st > 0 with probability 1/s).  Decrements
 * with a floor at 0 commute, so the run leaves st - d clamped at 0, d the
 * literal's number of successes, Binomial(m, 1/s): drawn per literal by
 * inverse CDF from a 16-bit uniform.  The uniforms of word w come from four
 * Philox4x32-7 calls at sub-indices 0x40000000 | 4w | i keyed on the run's
 * first event (t, k), as bit planes: bit b of literal j's uniform is bit j of
 * word b & 3 of call b >> 2. */
/* Literal j's 16-bit uniform from the four calls R of a word: bit b is bit j
 * of word b & 3 of call b >> 2. */
static uint32_t run_uniform(const uint32_t R[4][4], int j) {
    uint32_t u = 0;
    for (int b = 0; b < 16; ++b) u |= ((R[b >> 2][b & 3] >> j) & 1u) << b;
    return u;
}

static void type1b_run(const orc_cfg *c, uint32_t *st, uint32_t g, uint64_t t, uint32_t k, int mi) {
    const int L = c->L, m = RUN_SIZES[mi];
    for (int w = 0; w * 32 < L; ++w) {
        uint32_t R[4][4];
        for (uint32_t i = 0; i < 4; ++i)
            draw_r(c, g, t, 0x40000000u | ((uint32_t)w << 2) | i, TAG_SMASK, k, 7, R[i]);
        for (int j = 0; j < 32 && w * 32 + j < L; ++j) {
            const uint32_t u = run_uniform(R, j);
            int d = 0;
            while (d < m && u >= c->run_cdf16[mi][d]) ++d;
            uint32_t *x = &st[w * 32 + j];
            *x = *x > (uint32_t)d ? *x - (uint32_t)d : 0u;
        }
    }
}

/* The per-literal decrement counts type1b_run draws for word w (test hook). */
void orc_run_counts(const orc_cfg *c, uint32_t g, uint64_t t, uint32_t k, uint32_t w, int mi, uint32_t out[32]) {
    const int m = RUN_SIZES[mi];
    uint32_t R[4][4];
    for (uint32_t i = 0; i < 4; ++i) draw_r(c, g, t, 0x40000000u | (w << 2) | i, TAG_SMASK, k, 7, R[i]);
    for (int j = 0; j < 32; ++j) {
        const uint32_t u = run_uniform(R, j);
        int d = 0;
        while (d < m && u >= c->run_cdf16[mi][d]) ++d;
        out[j] = (uint32_t)d;
    }
}

/* type2_fb, kernel.cu:481-506.  The reference has no upper check; state_top
 * lies above every value one sample can reach, so the cap only bounds
 * mini-batches. */
static void type2(const orc_cfg *c, uint32_t *st, const uint32_t *x) {
    const int L = c->L;
    for (int l = 0; l < L; ++l) {
        uint32_t bit = (x[l / 32] >> (l % 32)) & 1u;
        if (bit == 0u && st[l] < (uint32_t)c->state_top) st[l] += 1;
    }
}

/* pytm's sample-level pick (pytm/base.py:139-141): the true class is the one
 * whose target is positive; the other class is drawn uniformly among the rest
 * from the counter (clause 0xFFFFFFFF, t, 1, CLASS). */
static void orc_pair(const orc_cfg *c, const int32_t *Yrow, uint64_t t, int *kt, int *ko) {
    const int K = c->K;
    int y = -1;
    for (int k = 0; k < K; ++k)
        if (Yrow[k] > 0) { y = k; break; }
    uint32_t r[4];
    draw(c, 0xFFFFFFFFu, t, 1, TAG_CLASS, 0, r);
    if (y < 0) {
        *ko = (int)(((uint64_t)r[0] * (uint64_t)K) >> 32);
    } else {
        int idx = K > 1 ? (int)(((uint64_t)r[0] * (uint64_t)(K - 1)) >> 32) : 0;
        *ko = K > 1 ? (idx < y ? idx : idx + 1) : -1;
    }
    *kt = y;
}

/* Part 2 of a batch: clause_update, kernel.cu:531-613, for every clause of the
 * shard and every sample of the batch in order.  cs [B][K] are the summed class
 * sums, Y [B][K] the +-T targets, sel [B][nc] and ninc [nc] from part 1. */
/* The negative-class selection (kernel.cu:573: each class with target -1
 * takes part with probability Q) drawn as a set for clause g at sample t
 * when q_select: the Philox4x32-7 call at sub-index 2 (class field 0) gives
 * in word 0 the count n of selected classes among all K, the smallest n with
 * r0 < q_cdf[n] (min(K, 32) if none), i.e. Binomial(K, Q); then n distinct classes
 * by rejection from b-bit fields (b = bits of K - 1, floor(32 / b) fields per
 * word from bit 0) of words 1-3 and of all words of further calls at
 * sub-indices 3, 4, ...: a value >= K or already drawn is skipped.  Every
 * class is then selected independently with probability Q. */
static void orc_qselect(const orc_cfg *c, uint32_t g, uint64_t t, uint8_t *sel) {
    const int K = c->K;
    memset(sel, 0, (size_t)K);
    uint32_t R[4], sub = 2;
    draw_r(c, g, t, sub, TAG_CLASS, 0, 7, R);
    const uint32_t nmax = K < 32 ? (uint32_t)K : 32u;
    uint32_t n = 0;
    while (n < nmax && R[0] >= c->q_cdf[n]) ++n;
    int b = 1;
    while ((1 << b) < K) ++b;
    const int per = 32 / b;
    int wi = 1, f = 0;
    while (n) {
        if (f == per) {
            f = 0;
            if (++wi == 4) { draw_r(c, g, t, ++sub, TAG_CLASS, 0, 7, R); wi = 0; }
        }
        const uint32_t v = (R[wi] >> (b * f)) & ((1u << b) - 1u);
        ++f;
        if ((int)v < K && !sel[v]) { sel[v] = 1; --n; }
    }
}

/* Test hook: the selected set of clause g at sample t as 0/1 per class
 * (sel [K]); the configuration must have q_select. */
void orc_qselect_set(const orc_cfg *c, uint32_t g, uint64_t t, uint8_t *sel) { orc_qselect(c, g, t, sel); }

/* Feedback of a batch (clause_update, kernel.cu:531-613, per sample in
 * order).  Per clause, the events of each 128-sample window (64 above 256 classes) of the batch are
 * decided first (the decisions read only the batch-start fired bits and
 * include counts, and the weights, which they update), then applied in
 * feedback order; maximal runs of consecutive Type Ib events inside a window
 * are applied in pieces of at most 64 events, each the longest multiple of 8
 * events that the rest of the run holds (greedy, from the run's start),
 * with type1b_run, the rest one by one. */
enum { EV_T1A = 1, EV_T1B = 2, EV_T2 = 3 };
typedef struct { int32_t b, k, type; } orc_event;

void orc_train_update(const orc_cfg *c, int32_t lo, int32_t nc, uint32_t *ta, int32_t *w,
                      const int32_t *cs, const int32_t *Y, const uint32_t *drop, const uint32_t *lits,
                      int32_t B, uint64_t t0, const int32_t *sel, const int32_t *ninc) {
    const int K = c->K, L = c->L, W = c->W, P = c->P;
#pragma omp parallel
    {
    const int win = run_window(c);
    orc_event *ev = (orc_event *)malloc(sizeof(orc_event) * (size_t)win * (size_t)(K > 2 ? K : 2));
    uint8_t *qsel = (uint8_t *)malloc((size_t)K);
    const int use_qsel = c->q_select && !c->one_negative;
#pragma omp for schedule(dynamic, 4)
    for (int32_t i = 0; i < nc; ++i) {
        if (drop && drop[i] == 1) continue; /* kernel.cu:555 */
        uint32_t g = (uint32_t)(lo + i);
        uint32_t *st = ta + (int64_t)i * L;
        for (int32_t b0 = 0; b0 < B; b0 += win) {
            int nev = 0;
            for (int32_t b = b0; b < B && b < b0 + win; ++b) {
                uint64_t t = t0 + (uint64_t)b;
                int32_t sp = sel[(int64_t)b * nc + i];
                int fired = sp > -1; /* kernel.cu:558 */
                int k0 = c->coalesced ? 0 : clause_class(c, (int32_t)g);
                int k1 = c->coalesced ? K : k0 + 1;
                int seq[2], nseq = 0;
                if (c->one_negative) { /* the true class, then one other class */
                    int kt, ko;
                    orc_pair(c, Y + (int64_t)b * K, t, &kt, &ko);
                    if (kt >= k0 && kt < k1) seq[nseq++] = kt;
                    if (ko >= k0 && ko < k1) seq[nseq++] = ko;
                }
                int nk = c->one_negative ? nseq : k1 - k0;
                if (use_qsel) orc_qselect(c, g, t, qsel);
                for (int kq = 0; kq < nk; ++kq) { /* kernel.cu:563-568 */
                    const int k = c->one_negative ? seq[kq] : k0 + kq;
                    int32_t v = clip_cs(c, cs[(int64_t)b * K + k]);
                    int32_t y = Y[(int64_t)b * K + k];
                    int target = 1 - 2 * (v > y); /* kernel.cu:571 */
                    /* decision uniforms: the Philox4x32-7 call of the class
                     * pair k >> 1, words 0-1 for the even class, 2-3 for the odd */
                    uint32_t r[4];
                    draw_r(c, g, t, 0, TAG_CLASS, (uint32_t)k >> 1, 7, r);
                    const uint32_t uq = r[2 * (k & 1)], uu = r[2 * (k & 1) + 1];
                    if (!c->one_negative && target == -1 &&
                        !(use_qsel ? qsel[k] : (uint64_t)uq < c->q_thr)) continue; /* kernel.cu:573 */
                    int upd = (uint64_t)uu < orc_update_threshold(y, v);   /* kernel.cu:582 */
                    int32_t *lw = &w[(int64_t)i * K + k];
                    int sign = (*lw >= 0) - (*lw < 0);
                    int ok = fired && ninc[i] <= c->max_included;
                    int t1a = target * sign > 0 && ok;
                    int t1b = target * sign > 0 && !ok;
                    int t2 = target * sign < 0 && fired;
                    if (!upd) continue;
                    if (t1a) {
                        *lw += sign;
                        ev[nev++] = (orc_event){b, k, EV_T1A};
                    } else if (t1b) {
                        ev[nev++] = (orc_event){b, k, EV_T1B};
                    } else if (t2) {
                        *lw -= sign;
                        if (!c->negative_polarity && *lw < 1) *lw = 1; /* kernel.cu:603-606 */
                        ev[nev++] = (orc_event){b, k, EV_T2};
                    }
                }
            }
            for (int e = 0; e < nev;) {
                const orc_event *E = &ev[e];
                const uint64_t t = t0 + (uint64_t)E->b;
                if (E->type == EV_T1B) {
                    int run = 0;
                    while (e + run < nev && run < 64 && ev[e + run].type == EV_T1B) ++run;
                    const int mi = run / 8 - 1; /* the longest multiple of 8 events */
                    if (mi >= 0) {
                        type1b_run(c, st, g, t, (uint32_t)E->k, mi);
                        e += RUN_SIZES[mi];
                        continue;
                    }
                    type1b(c, st, g, t, (uint32_t)E->k);
                } else {
                    const int32_t sp = sel[(int64_t)E->b * nc + i];
                    const uint32_t *x = lits + ((int64_t)E->b * P + sp) * W;
                    if (E->type == EV_T1A) type1a(c, st, x, g, t, (uint32_t)E->k);
                    else type2(c, st, x);
                }
                ++e;
            }
        }
    }
    free(ev);
    free(qsel);
    }
}

/* One whole batch on one process (all clauses): part 1 then part 2.
 * cs_out [B][K] and sel_out [B][C] may be NULL. */
void orc_train_batch(const orc_cfg *c, uint32_t *ta, int32_t *w, int32_t *patch_w, const uint32_t *drop,
                     const uint32_t *lits, const int32_t *Y, int32_t B, uint64_t t0,
                     const int32_t *sel_override, int32_t *cs_out, int32_t *sel_out) {
    const int C = c->C, K = c->K;
    int32_t *cs = (int32_t *)malloc((size_t)B * K * 4);
    int32_t *sel = (int32_t *)malloc((size_t)B * C * 4);
    int32_t *ninc = (int32_t *)malloc((size_t)C * 4);
    orc_train_eval(c, 0, C, ta, w, NULL, drop, lits, B, t0, 0, cs, patch_w, sel, ninc);
    if (sel_override) memcpy(sel, sel_override, (size_t)B * C * 4);
    orc_train_update(c, 0, C, ta, w, cs, Y, drop, lits, B, t0, sel, ninc);
    if (cs_out) memcpy(cs_out, cs, (size_t)B * K * 4);
    if (sel_out) memcpy(sel_out, sel, (size_t)B * C * 4);
    free(cs);
    free(sel);
    free(ninc);
}
