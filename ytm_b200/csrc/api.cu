// api.cu — configuration, workspace sizing and error reporting of libytm.
#include <math.h>

#include <string>

#include "common.cuh"

namespace ytm {

static thread_local std::string g_err;

void set_error(const std::string &msg) { g_err = msg; }

ytm_status fail(ytm_status code, const std::string &msg) {
    g_err = msg;
    return code;
}

ytm_status cuda_check(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return YTM_OK;
    return fail(YTM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

ytm_status launch_check(const char *what) { return cuda_check(cudaGetLastError(), what); }

int sm_count() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    return n;
}

ytm_status check_cfg(const ytm_config *cfg) {
    if (!cfg) return fail(YTM_ERR_ARG, "config is NULL");
    if (cfg->clauses <= 0 || cfg->n_classes <= 0 || cfg->literals <= 0 || cfg->words <= 0 || cfg->patches <= 0)
        return fail(YTM_ERR_ARG, "config has non-positive sizes (was it made by ytm_config_init?)");
    if (cfg->clause_count <= 0 || cfg->clause_lo < 0 || cfg->clause_lo + cfg->clause_count > cfg->clauses)
        return fail(YTM_ERR_ARG, "config clause shard out of range");
    if (cfg->planes < 2 || cfg->planes > 16) return fail(YTM_ERR_UNSUPPORTED, "unsupported plane count");
    if (cfg->input_images) {
        if (cfg->patches <= 1)
            return fail(YTM_ERR_UNSUPPORTED, "bit-image input is for models with several patches (use ytm_encode)");
        if (cfg->image_words != (int32_t)cdiv((uint64_t)cfg->dim0 * cfg->dim1 * cfg->dim2, 32) + 1)
            return fail(YTM_ERR_ARG, "config image_words does not match its dims");
    }
    return YTM_OK;
}

TrainWs train_ws_layout(const ytm_config *cfg, int64_t B) {
    TrainWs l;
    const uint64_t C = cfg->clause_count, P = cfg->patches, K = cfg->n_classes;
    const uint64_t PW = cdiv(P, 32), CW = cdiv(C, 32);
    uint64_t o = 0;
    l.ninc = o;  o = align_up(o + C * 4, 256);
    l.mbits = o; o = align_up(o + (uint64_t)B * C * PW * 4, 256);
    l.fired = o; o = align_up(o + (uint64_t)B * CW * 4, 256);  // right after mbits: one memset clears both
    l.sel = o;   o = align_up(o + (uint64_t)B * C * 4, 256);
    l.fcm = o;   o = align_up(o + C * cdiv(B, 32) * 4, 256);  // single patch: clause-major fired bits
    l.thr = o;   o = align_up(o + (uint64_t)B * K * 8, 256);
    // (sample, class) pairs that can update: bits per sample, bits per class,
    // and the list in feedback order with each sample's offset into it
    l.amask = o; o = align_up(o + (uint64_t)B * cdiv(K, 32) * 4, 256);
    l.colm = o;  o = align_up(o + K * cdiv(B, 32) * 4, 256);
    l.row_off = o; o = align_up(o + ((uint64_t)B + 1) * 4, 256);
    l.npos = o;  o = align_up(o + (uint64_t)B * 4, 256);  // target +1 pairs per sample (q_select)
    l.alist = o; o = align_up(o + (uint64_t)B * K * 8, 256);
    l.pair = o;  o = align_up(o + (uint64_t)B * 2 * 4, 256);
    l.sparse = o; o = align_up(o + sparse_ws_bytes(cfg), 256);  // compacted include words (sparse patch match)
    l.pwords = o; o += batch_words_bytes(cfg, B);  // bit-image input: the batch's patch literal words
    l.total = o;
    return l;
}

InferWs infer_ws_layout(const ytm_config *cfg, int64_t N) {
    InferWs l;
    const uint64_t C = cfg->clause_count, CW = cdiv(C, 32);
    uint64_t o = 0;
    l.ninc = o;  o = align_up(o + C * 4, 256);
    l.fired = o; o = align_up(o + (uint64_t)N * CW * 4, 256);
    l.total = o;
    return l;
}

}  // namespace ytm

using namespace ytm;

extern "C" {

ytm_status ytm_config_init(ytm_config *cfg, int32_t clauses_per_class, int32_t T, double s, int32_t dim0,
                           int32_t dim1, int32_t dim2, int32_t n_classes, double q, int32_t patch_dim0,
                           int32_t patch_dim1, int32_t number_of_ta_states, int32_t max_included_literals,
                           int32_t append_negated, int32_t init_neg_weights, int32_t negative_polarity,
                           int32_t encode_loc, int32_t coalesced, uint64_t seed) {
    if (!cfg) return fail(YTM_ERR_ARG, "config is NULL");
    *cfg = ytm_config{};
    if (clauses_per_class <= 0 || T <= 0 || !(s > 0.0) || n_classes <= 0)
        return fail(YTM_ERR_ARG, "clauses_per_class, T, s and n_classes must be positive");
    if (dim0 <= 0 || dim1 <= 0 || dim2 <= 0 || patch_dim0 <= 0 || patch_dim1 <= 0 || patch_dim0 > dim0 ||
        patch_dim1 > dim1)
        return fail(YTM_ERR_ARG, "dim / patch_dim out of range");
    if (number_of_ta_states < 2) return fail(YTM_ERR_ARG, "number_of_ta_states must be >= 2");
    cfg->clauses_per_class = clauses_per_class;
    cfg->T = T;
    cfg->s = s;
    cfg->q = q < (double)n_classes ? q : (double)n_classes;  // base.py:81
    cfg->dim0 = dim0; cfg->dim1 = dim1; cfg->dim2 = dim2;
    cfg->n_classes = n_classes;
    cfg->patch_dim0 = patch_dim0; cfg->patch_dim1 = patch_dim1;
    cfg->number_of_ta_states = number_of_ta_states;
    cfg->append_negated = append_negated ? 1 : 0;
    cfg->init_neg_weights = init_neg_weights ? 1 : 0;
    cfg->negative_polarity = negative_polarity ? 1 : 0;
    cfg->encode_loc = encode_loc ? 1 : 0;
    cfg->coalesced = coalesced ? 1 : 0;
    cfg->seed = seed;
    // base.py:94-121
    cfg->clause_banks = coalesced ? 1 : n_classes;
    int64_t C = (int64_t)cfg->clause_banks * clauses_per_class;
    cfg->loc_literals = (dim1 - patch_dim1) + (dim0 - patch_dim0);
    int64_t half = (int64_t)patch_dim0 * patch_dim1 * dim2 + (encode_loc ? cfg->loc_literals : 0);
    int64_t L = append_negated ? 2 * half : half;
    if (C > (1ll << 30) || L > (1ll << 28)) return fail(YTM_ERR_UNSUPPORTED, "model too large");
    cfg->clauses = (int32_t)C;
    cfg->literals = (int32_t)L;
    cfg->half_literals = (int32_t)half;
    cfg->words = (int32_t)((L - 1) / 32 + 1);
    cfg->patches = (dim0 - patch_dim0 + 1) * (dim1 - patch_dim1 + 1);
    cfg->input_images = 0;
    cfg->image_words = (int32_t)(((int64_t)dim0 * dim1 * dim2 + 31) / 32 + 1);
    cfg->max_included_literals = max_included_literals < 0 ? (int32_t)L : max_included_literals;
    // The reference sets its location thermometer bits even without
    // encode_loc (kernel.cu:101-121); they must land inside the literal vector.
    if (cfg->loc_literals > half)
        return fail(YTM_ERR_UNSUPPORTED, "patch location literals do not fit the literal vector");
    // Bit-sliced states: include iff state > half (kernel.cu:33); stored
    // value = state + offset puts the include bit in the top plane.  One
    // sample raises an excluded state by at most n_classes (type II has no
    // upper check, kernel.cu:481-506), so the top must reach
    // half + max(max - half, n_classes).
    cfg->max_state = number_of_ta_states;
    cfg->half_state = number_of_ta_states / 2;
    {
        int64_t m = cfg->max_state - cfg->half_state;
        if (n_classes > m) m = n_classes;
        int64_t p = 1;
        int nb = 1;
        while (p < m || p < cfg->half_state + 1) { p <<= 1; ++nb; }
        cfg->planes = nb;
        cfg->state_offset = (int32_t)(p - (cfg->half_state + 1));
        cfg->state_top = (int32_t)(p + cfg->half_state);
        if (nb > 16) return fail(YTM_ERR_UNSUPPORTED, "number_of_ta_states needs more than 16 bit planes");
    }
    // literal-mask count table: Binomial(32, p), p = 1/s (S_INV, kernel.cu:31);
    // cdf[n] = floor(2^32 * P(count <= n)) saturated at 2^32 - 1, from the pmf
    // recurrence pmf(n+1) = pmf(n) * (32-n)/(n+1) * p/(1-p) in IEEE double
    {
        double p = 1.0 / s;
        if (!(p > 0.0)) p = 0.0;
        if (p > 1.0) p = 1.0;
        const double qq = 1.0 - p;
        if (!(qq > 0.0)) {
            for (int n = 0; n < 32; ++n) cfg->s_count_cdf[n] = 0u;
        } else {
            double pmf = 1.0, acc = 0.0;
            for (int i = 0; i < 32; ++i) pmf *= qq;
            for (int n = 0; n < 32; ++n) {
                acc += pmf;
                const double v = floor(acc * 4294967296.0);
                cfg->s_count_cdf[n] = v >= 4294967295.0 ? 0xFFFFFFFFu : (uint32_t)v;
                pmf = pmf * (double)(32 - n) / (double)(n + 1) * p / qq;
            }
        }
    }
    // Type Ib run tables: per literal Binomial(m, p) decrement counts for runs
    // of m = 8, 16, ..., 64 events; entry d = P(count <= d) * 65536 rounded to
    // the nearest integer, 65536 from d = m on, from the same pmf recurrence;
    // run_range: entries below lo are 0 (those counts are certain), entries
    // from hi on are 65536 (never exceeded)
    {
        double p = 1.0 / s;
        if (!(p > 0.0)) p = 0.0;
        if (p > 1.0) p = 1.0;
        const double qq = 1.0 - p;
        for (int mi = 0; mi < 8; ++mi) {
            const int m = 8 * (mi + 1);
            for (int d = 0; d < 65; ++d) cfg->run_cdf16[mi][d] = 65536u;
            if (!(qq > 0.0)) {
                for (int d = 0; d < m; ++d) cfg->run_cdf16[mi][d] = 0u;
                continue;
            }
            double pmf = 1.0, acc = 0.0;
            for (int i = 0; i < m; ++i) pmf *= qq;
            for (int d = 0; d < m; ++d) {
                acc += pmf;
                const double v = floor(acc * 65536.0 + 0.5);  // nearest: a tail below 2^-17 is never drawn
                cfg->run_cdf16[mi][d] = v >= 65536.0 ? 65536u : (uint32_t)v;
                pmf = pmf * (double)(m - d) / (double)(d + 1) * p / qq;
            }
        }
        for (int mi = 0; mi < 8; ++mi) {
            uint32_t lo = 0, hi = 0;
            while (lo < 64 && cfg->run_cdf16[mi][lo] == 0u) ++lo;
            while (hi < 64 && cfg->run_cdf16[mi][hi] < 65536u) ++hi;
            cfg->run_range[mi] = lo | (hi << 16);
        }
    }
    {
        double qp = cfg->q / (double)(n_classes - 1 > 1 ? n_classes - 1 : 1);  // kernel.cu:32
        if (qp >= 1.0) cfg->q_threshold = 4294967296ull;
        else if (!(qp > 0.0)) cfg->q_threshold = 0;
        else cfg->q_threshold = (uint64_t)floor(qp * 4294967296.0);
        // the negative-class selection as a set per (clause, sample) for
        // coalesced models of at least 32 classes whose expected selections
        // K * Q are at most 2 (below 32 classes one draw per class pair is as cheap):
        // count ~ Binomial(K, Q) (this table, IEEE double pmf recurrence)
        if (!(qp > 0.0)) qp = 0.0;
        if (qp > 1.0) qp = 1.0;
        cfg->q_select = (coalesced && n_classes >= 32 && qp > 0.0 && qp < 1.0 && qp * n_classes <= 2.0) ? 1 : 0;
        for (int n = 0; n < 32; ++n) cfg->q_count_cdf[n] = 0xFFFFFFFFu;
        if (cfg->q_select) {
            const double qq = 1.0 - qp;
            double pmf = 1.0, acc = 0.0;
            for (int i = 0; i < n_classes; ++i) pmf *= qq;
            for (int n = 0; n < 32; ++n) {
                acc += pmf;
                const double v = floor(acc * 4294967296.0);
                cfg->q_count_cdf[n] = v >= 4294967295.0 ? 0xFFFFFFFFu : (uint32_t)v;
                pmf = n < n_classes ? pmf * (double)(n_classes - n) / (double)(n + 1) * qp / qq : 0.0;
            }
        }
    }
    cfg->clause_lo = 0;
    cfg->clause_count = cfg->clauses;
    return YTM_OK;
}

ytm_status ytm_config_shard(ytm_config *cfg, int32_t rank, int32_t world) {
    if (!cfg || world <= 0 || rank < 0 || rank >= world) return fail(YTM_ERR_ARG, "bad rank/world");
    int64_t C = cfg->clauses;
    if (C < world) return fail(YTM_ERR_ARG, "fewer clauses than ranks");
    int64_t lo = C * rank / world, hi = C * (rank + 1) / world;
    cfg->clause_lo = (int32_t)lo;
    cfg->clause_count = (int32_t)(hi - lo);
    return YTM_OK;
}

uint64_t ytm_workspace_bytes(const ytm_config *cfg, int32_t op, int64_t n) {
    if (!cfg || n < 0) return 0;
    switch (op) {
        case YTM_OP_ENCODE: {
            uint64_t D = (uint64_t)cfg->dim0 * cfg->dim1 * cfg->dim2;
            return align_up((uint64_t)n * (cdiv(D, 32) + 1) * 4, 256);
        }
        case YTM_OP_ENCODE_THERMO: {
            uint64_t D = (uint64_t)cfg->dim0 * cfg->dim1 * cfg->dim2;
            return align_up((uint64_t)n * (cdiv(D, 32) + 1) * 4 + 256 * 4, 256);
        }
        case YTM_OP_INFER:
        case YTM_OP_TRANSFORM:
            return infer_ws_layout(cfg, n).total + cs_planes_bytes(cfg) + sparse_ws_bytes(cfg);
        case YTM_OP_TRAIN:
            return train_ws_layout(cfg, n).total + cs_planes_bytes(cfg);
        case YTM_OP_TRAIN_B1:
            return b1_ws_layout(cfg).total;
        case YTM_OP_TRAIN_LOOP:
            return align_up((uint64_t)n * cfg->n_classes * 4, 256) + train_ws_layout(cfg, n).total +
                   cs_planes_bytes(cfg);
        default:
            return 0;
    }
}

const char *ytm_last_error(void) { return g_err.c_str(); }

const char *ytm_version(void) { return "ytm-b200 0.1.0 (sm_100a)"; }

int32_t ytm_config_size(void) { return (int32_t)sizeof(ytm_config); }

}  // extern "C"
