// state.cu — bit-sliced TA-state planes: initialisation, conversion to and
// from the reference's flat u32 layout, include masks, and clause weights.
#include "common.cuh"

namespace ytm {

// Plane layout: state[(b * C + c) * W + w], C = clause_count.

__global__ void k_state_fill(uint32_t *__restrict__ state, int64_t CW, int NB, uint32_t value) {
    int64_t total = CW * NB;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int b = (int)(i / CW);
        state[i] = ((value >> b) & 1u) ? 0xFFFFFFFFu : 0u;
    }
}

// One warp per (clause, word): lane j carries literal 32w+j.
__global__ void k_state_from_u32(ytm_config cfg, const uint32_t *__restrict__ ta, uint32_t *__restrict__ state) {
    const int C = cfg.clause_count, W = cfg.words, L = cfg.literals, NB = cfg.planes;
    const int lane = threadIdx.x & 31;
    const int64_t units = (int64_t)C * W;
    const int64_t wid0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t wstride = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const uint32_t top = (uint32_t)cfg.state_top, off = (uint32_t)cfg.state_offset;
    for (int64_t u = wid0; u < units; u += wstride) {
        int64_t c = u / W;
        int w = (int)(u % W);
        int l = w * 32 + lane;
        uint32_t s = (l < L) ? ta[c * L + l] : (uint32_t)cfg.half_state;
        if (s > top) s = top;
        s += off;
        for (int b = 0; b < NB; ++b) {
            uint32_t m = __ballot_sync(0xFFFFFFFFu, (s >> b) & 1u);
            if (lane == 0) state[((int64_t)b * C + c) * W + w] = m;
        }
    }
}

__global__ void k_state_to_u32(ytm_config cfg, const uint32_t *__restrict__ state, uint32_t *__restrict__ ta) {
    const int C = cfg.clause_count, W = cfg.words, L = cfg.literals, NB = cfg.planes;
    const int lane = threadIdx.x & 31;
    const int64_t units = (int64_t)C * W;
    const int64_t wid0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t wstride = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t u = wid0; u < units; u += wstride) {
        int64_t c = u / W;
        int w = (int)(u % W);
        int l = w * 32 + lane;
        uint32_t s = 0;
        for (int b = 0; b < NB; ++b) s |= ((state[((int64_t)b * C + c) * W + w] >> lane) & 1u) << b;
        if (l < L) ta[c * L + l] = s - (uint32_t)cfg.state_offset;
    }
}

// One warp per clause: include count = popcount of the top plane.
__global__ void k_ninc(int C, int W, const uint32_t *__restrict__ inc, int32_t *__restrict__ ninc,
                       uint32_t *__restrict__ inc_out) {
    const int lane = threadIdx.x & 31;
    const int64_t wid0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t wstride = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t c = wid0; c < C; c += wstride) {
        int cnt = 0;
        for (int w = lane; w < W; w += 32) {
            uint32_t v = inc[c * W + w];
            cnt += __popc(v);
            if (inc_out) inc_out[c * W + w] = v;
        }
        for (int o = 16; o; o >>= 1) cnt += __shfl_xor_sync(0xFFFFFFFFu, cnt, o);
        if (lane == 0) ninc[c] = cnt;
    }
}

// init_weights, kernel.cu:46-73.  Coalesced signs come from the TAG_INIT
// Philox stream (the reference draws curand()%2).
__global__ void k_weights_init(ytm_config cfg, int32_t *__restrict__ w) {
    const int K = cfg.n_classes;
    const int64_t total = (int64_t)cfg.clause_count * K;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t c = i / K;
        int k = (int)(i % K);
        int64_t g = cfg.clause_lo + c;
        int32_t v;
        if (cfg.coalesced) {
            v = 1;
            if (cfg.init_neg_weights) v = (draw(cfg.seed, (uint32_t)g, 0, 0, TAG_INIT, (uint32_t)k).x & 1u) ? -1 : 1;
        } else if (k == (int)(g / cfg.clauses_per_class)) {
            v = 1;
            if (cfg.init_neg_weights && (g % cfg.clauses_per_class) >= cfg.clauses_per_class / 2) v = -1;
        } else {
            v = 0;
        }
        w[i] = v;
    }
}

static unsigned grid_for(int64_t threads, int bs) {
    int64_t b = (int64_t)cdiv((uint64_t)threads, bs);
    int64_t cap = (int64_t)sm_count() * 32;
    if (b > cap) b = cap;
    if (b < 1) b = 1;
    return (unsigned)b;
}

ytm_status launch_ninc(const ytm_config *cfg, const uint32_t *state, int32_t *ninc, cudaStream_t st) {
    const int C = cfg->clause_count, W = cfg->words;
    const uint32_t *inc = state + (int64_t)(cfg->planes - 1) * C * W;
    k_ninc<<<grid_for((int64_t)C * 32, 256), 256, 0, st>>>(C, W, inc, ninc, nullptr);
    return launch_check("include counts");
}

}  // namespace ytm

using namespace ytm;

extern "C" {

ytm_status ytm_state_init(const ytm_config *cfg, uint32_t *state, void *stream) {
    ytm_status rc = check_cfg(cfg);
    if (rc) return rc;
    if (!state) return fail(YTM_ERR_ARG, "null pointer");
    int64_t CW = (int64_t)cfg->clause_count * cfg->words;
    uint32_t v = (uint32_t)(cfg->number_of_ta_states / 2 + cfg->state_offset);  // base.py:209
    k_state_fill<<<grid_for(CW * cfg->planes, 256), 256, 0, as_stream(stream)>>>(state, CW, cfg->planes, v);
    return launch_check("state init");
}

ytm_status ytm_state_from_u32(const ytm_config *cfg, const uint32_t *ta, uint32_t *state, void *stream) {
    ytm_status rc = check_cfg(cfg);
    if (rc) return rc;
    if (!ta || !state) return fail(YTM_ERR_ARG, "null pointer");
    int64_t units = (int64_t)cfg->clause_count * cfg->words;
    k_state_from_u32<<<grid_for(units * 32, 256), 256, 0, as_stream(stream)>>>(*cfg, ta, state);
    return launch_check("state from u32");
}

ytm_status ytm_state_to_u32(const ytm_config *cfg, const uint32_t *state, uint32_t *ta, void *stream) {
    ytm_status rc = check_cfg(cfg);
    if (rc) return rc;
    if (!ta || !state) return fail(YTM_ERR_ARG, "null pointer");
    int64_t units = (int64_t)cfg->clause_count * cfg->words;
    k_state_to_u32<<<grid_for(units * 32, 256), 256, 0, as_stream(stream)>>>(*cfg, state, ta);
    return launch_check("state to u32");
}

ytm_status ytm_include_mask(const ytm_config *cfg, const uint32_t *state, uint32_t *inc, int32_t *num_includes,
                            void *stream) {
    ytm_status rc = check_cfg(cfg);
    if (rc) return rc;
    if (!state || !num_includes) return fail(YTM_ERR_ARG, "null pointer");
    const int C = cfg->clause_count, W = cfg->words;
    const uint32_t *top = state + (int64_t)(cfg->planes - 1) * C * W;
    k_ninc<<<grid_for((int64_t)C * 32, 256), 256, 0, as_stream(stream)>>>(C, W, top, num_includes, inc);
    return launch_check("include mask");
}

ytm_status ytm_weights_init(const ytm_config *cfg, int32_t *weights, void *stream) {
    ytm_status rc = check_cfg(cfg);
    if (rc) return rc;
    if (!weights) return fail(YTM_ERR_ARG, "null pointer");
    int64_t total = (int64_t)cfg->clause_count * cfg->n_classes;
    k_weights_init<<<grid_for(total, 256), 256, 0, as_stream(stream)>>>(*cfg, weights);
    return launch_check("weights init");
}

}  // extern "C"
