// fused_b1.cu — the reference's per-sample training loop (base.py:305-357),
// one kernel launch per sample, issued from C++ (no host round trip).
//
// The reference runs 4 kernels and 4 host syncs per sample.  Here launch i
// does, for every clause (one warp each):
//   1. the feedback of sample i (clause_update, kernel.cu:531-613) with the
//      class sums and picks that launch i-1 produced, and
//   2. the evaluation of sample i+1 on the just-updated state (fast_eval +
//      select_active, kernel.cu:255-316): include count, fired bit, patch
//      weight, and the clause's weight row added to the class sums of i+1,
// so the bit planes are read and written once per sample.  Launch boundaries
// are the grid-wide barrier between "all class sums of i+1 are complete" and
// "feedback of i+1 starts".  A prologue launch evaluates the first sample.
//
// Class sums live in a ring of three [K] slots: launch i reads slot i%3,
// accumulates slot (i+1)%3 and clears slot (i+2)%3, which launch i-1 finished
// reading and launch i+1 will fill.  Results are bit-identical to
// ytm_train_eval + ytm_train_update with B = 1.  Convolutional models test,
// per clause, only its non-zero include words against each patch.
#include "common.cuh"

namespace ytm {

// warps per block; clauses per block (CPB) is a template parameter:
// YTM_B1_CPB for single-patch models (measured on configuration 1: 48 clauses
// 10.6 us per sample, 64 13.3, 32 13.2, 128 23.5 — 48 keeps the 417 blocks
// of 20,000 clauses resident in one wave), 16 for convolutional ones, whose
// per-clause patch scan wants more blocks in flight (measured: config 3 17k ->
// 31k samples/s)
constexpr int FB_WARPS = 8;
#ifndef YTM_B1_CPB
#define YTM_B1_CPB 48  // a multiple of FB_WARPS
#endif
// resident blocks per SM the register budget is sized for: 3 (at most 80
// registers) for single-patch models; 4 (64) for convolutional ones, whose
// per-sample work is short and latency-bound (measured on configuration 3:
// 28.6k -> 34.5k samples/s); above 14 planes 64 registers would spill
#ifndef YTM_B1_MINB
#define YTM_B1_MINB 3
#endif
#ifndef YTM_B1_MINB_CONV
#define YTM_B1_MINB_CONV 4
#endif
#ifndef YTM_B1_CPB_CONV
#define YTM_B1_CPB_CONV 16  // a multiple of FB_WARPS
#endif


B1Ws b1_ws_layout(const ytm_config *cfg) {
    B1Ws l;
    const uint64_t C = cfg->clause_count, K = cfg->n_classes;
    uint64_t o = 0;
    l.cs = o;    o = align_up(o + 3 * K * 4, 256);
    l.fired = o; o = align_up(o + 2 * C * 4, 256);
    l.ninc = o;  o = align_up(o + C * 4, 256);
    // bit-image input: the patch literal words of three samples (ring)
    l.ring = o;
    if (cfg->input_images) o = align_up(o + 3ull * cfg->patches * cfg->words * 4, 256);
    l.total = o;
    return l;
}

// Patch literal words u32 [P][W] of sample n of the bit images into out.
__global__ void k_patch_words(const LitSrc src, int64_t n, uint32_t *__restrict__ out) {
    const int64_t total = (int64_t)src.P * src.g.W;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int p = (int)(idx / src.g.W);
        out[idx] = src.word<true>(n, p, (int)(idx - (int64_t)p * src.g.W));
    }
}

// Block = 8 warps owning CPB clauses.  Thresholds of sample i
// are computed once per block; decisions run one clause per thread (the
// Philox class draws of 32 clauses share each warp instruction); then each
// warp streams the words of its clauses (8 per warp), applying the events and
// evaluating sample i+1.
template <int NB, int CPB, bool IMG>
__global__ void __launch_bounds__(FB_WARPS * 32, (CPB == YTM_B1_CPB_CONV && NB <= 14) ? YTM_B1_MINB_CONV : YTM_B1_MINB) k_fused_b1(
    ytm_config cfg, uint32_t *__restrict__ state, int32_t *__restrict__ weights, const int32_t *__restrict__ bias,
    const uint32_t *__restrict__ drop, const uint32_t *__restrict__ lits, const int32_t *__restrict__ Y, int64_t i,
    int64_t N, uint64_t t0, int do_update, int32_t *__restrict__ cs_ring, int32_t *__restrict__ sel_pp,
    int32_t *__restrict__ ninc_ws, int32_t *__restrict__ patch_w, const RoundKeys rk, uint32_t *__restrict__ ring,
    int stage) {
    extern __shared__ __align__(16) unsigned char smraw[];
    // Programmatic dependent launch: let launch i+1 be scheduled now, and
    // wait here until launch i-1 has completed and its writes are visible.
    // Everything below reads what the previous launch wrote.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int C = cfg.clause_count, W = cfg.words, K = cfg.n_classes, L = cfg.literals;
    // Bit-image input (convolutional models): the patch literal words of a
    // sample are formed two launches ahead into a ring of three samples
    // (slot = sample % 3); this launch forms sample e_next + 1's words, which
    // no launch reads before this one has completed.
    const int64_t PWW = (int64_t)cfg.patches * W;
    const uint32_t *lits_of = lits;  // base of the per-sample [P][W] words (lits or the ring)
    int64_t lits_stride = PWW;
    if (IMG) {
        const int64_t e_nx = do_update ? i + 1 : 0;
        if (e_nx + 1 < N) {
            const LitSrc src = lit_src_dev(cfg, lits);
            uint32_t *dst = ring + ((e_nx + 1) % 3) * PWW;
            for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < PWW;
                 idx += (int64_t)gridDim.x * blockDim.x) {
                const int p = (int)(idx / W);
                dst[idx] = src.word<true>(e_nx + 1, p, (int)(idx - (int64_t)p * W));
            }
        }
        lits_of = ring;
        lits_stride = 0;  // slot chosen per sample below
    }
    const int nk = cfg.coalesced ? K : 1;
    const int KB = (nk + 31) >> 5;                       // 32-class chunks per clause
    uint64_t *thr_s = (uint64_t *)smraw;                 // [K]  threshold | target bit
    int32_t *cs_blk = (int32_t *)(thr_s + K);            // [K]
    uint32_t *ev_s = (uint32_t *)(cs_blk + K);           // [CPB][KB][3]: any, type Ia, type II
    uint32_t *lw_s = ev_s + CPB * KB * 3;              // [FB_WARPS][W] non-zero include words (P > 1)
    uint32_t *li_s = lw_s + FB_WARPS * W;                 // [FB_WARPS][W] their include masks
    uint32_t *mb_s = li_s + FB_WARPS * W;                 // [FB_WARPS][PW] patch match bits
    // P > 1 and stage: the patch words of sample i+1, [P][SW] with an odd row
    // stride (lane p reads row p: 32 distinct banks); without stage (too
    // large for shared memory) they are read where they lie, stride W
    const int SW = W | 1;
    uint32_t *xs_s = mb_s + FB_WARPS * ((cfg.patches + 31) >> 5);
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int do_eval = (i + 1 < N) || !do_update;       // the prologue evaluates sample 0
    const int64_t e_next = do_update ? i + 1 : 0;        // sample evaluated by this launch
    const int32_t *cs_cur = cs_ring + (i % 3) * K;
    int32_t *cs_next = cs_ring + (e_next % 3) * K;
    const int32_t *sel_cur = sel_pp + (i & 1) * (int64_t)C;     // picks of sample i (-1: not fired)
    int32_t *sel_next = sel_pp + (e_next & 1) * (int64_t)C;     // picks of sample i+1
    const int P = cfg.patches, PW = (P + 31) >> 5;
    const uint64_t t = t0 + (uint64_t)i;
    if (P > 1 && do_eval && stage) {
        // stage sample i+1's patch words (written by the previous launch or
        // the prologue's k_patch_words when they come from bit images): the
        // per-patch include tests then wait on shared memory, not on L2
        const uint32_t *src = lits_of + (IMG ? e_next % 3 : e_next) * PWW;
        for (int idx = threadIdx.x; idx < P * W; idx += blockDim.x) {
            const int p = idx / W;
            xs_s[p * SW + (idx - p * W)] = src[idx];
        }
    }
    // Block b owns clauses b, b + G, b + 2G, ... (G = grid size): every block
    // gets an even share of every clause bank, so the bank of the true class,
    // where most feedback lands, does not pile up on a few blocks.
    const int G = gridDim.x;

    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        cs_blk[k] = 0;
        if (do_update) {
            int32_t v = cs_cur[k] + (bias ? bias[k] : 0);
            v = v > cfg.T ? cfg.T : (v < -cfg.T ? -cfg.T : v);  // clip_cs, kernel.cu:397
            const int32_t y = Y[i * K + k];
            uint64_t th = update_threshold(y, v);
            if (v > y) th |= 1ull << 63;                          // target -1, kernel.cu:571
            thr_s[k] = th;
        }
    }
    if (blockIdx.x == 0 && do_update)
        for (int k = threadIdx.x; k < K; k += blockDim.x) cs_ring[((i + 2) % 3) * K + k] = 0;
    __shared__ int pair_s[2];  // one_negative: the true class and the other class of sample i
    if (threadIdx.x == 0 && do_update && cfg.one_negative)
        true_other_pair(cfg.seed, Y + i * K, K, t, &pair_s[0], &pair_s[1]);
    __syncthreads();

    // ---- 1. decisions of sample i: one clause per thread
    if (do_update && threadIdx.x < CPB) {
        const int c = (int)threadIdx.x * G + blockIdx.x;
        uint32_t *ev = ev_s + threadIdx.x * KB * 3;
        for (int q = 0; q < KB * 3; ++q) ev[q] = 0u;
        if (c < C && !(drop && drop[c] == 1u)) {  // kernel.cu:555
            const uint32_t g = (uint32_t)(cfg.clause_lo + c);
            const int k0 = cfg.coalesced ? 0 : (int)(g / (uint32_t)cfg.clauses_per_class);
            const bool fired = sel_cur[c] >= 0;
            const bool ok_inc = ninc_ws[c] <= cfg.max_included_literals;
            u32x4 rp{};
            int rp_pair = -1;  // the class pair whose decision call rp holds
            // q_select: the negative classes selected for this clause and sample
            const bool use_qsel = cfg.coalesced && cfg.q_select && !cfg.one_negative;
            uint16_t qs[32];
            int nq = 0;
            if (use_qsel)
                qselect(cfg, [&](uint32_t sub) { return draw_rk<7>(rk, g, t, sub, TAG_CLASS, 0); }, [&](int v) {
                    for (int j = 0; j < nq; ++j)
                        if (qs[j] == (uint16_t)v) return false;
                    qs[nq++] = (uint16_t)v;
                    return true;
                });
            for (int kk = 0; kk < nk; ++kk) {
                const int k = k0 + kk;
                uint64_t th = thr_s[k];
                const int target = (th >> 63) ? -1 : 1;
                th &= ~(1ull << 63);
                if (!th) continue;  // inactive pair: no update whatever the draws (kernel.cu:582)
                bool sel = true;
                if (use_qsel && target == -1) {
                    sel = false;
                    for (int j = 0; j < nq; ++j) sel |= qs[j] == (uint16_t)k;
                    if (!sel) continue;  // kernel.cu:573
                }
                if ((k >> 1) != rp_pair) {
                    rp = class_pair_draw_rk(rk, g, t, (uint32_t)k);
                    rp_pair = k >> 1;
                }
                const uint2 r = class_words(rp, (uint32_t)k);
                if (cfg.one_negative ? (k != pair_s[0] && k != pair_s[1])
                                     : (!use_qsel && target == -1 && !((uint64_t)r.x < cfg.q_threshold)))
                    continue;  // kernel.cu:573
                if (!((uint64_t)r.y < th)) continue;                                // kernel.cu:582
                int32_t *lw = &weights[(int64_t)c * K + k];
                int32_t wv = *lw;
                const int sign = (wv >= 0) - (wv < 0);
                const int ts = target * sign;
                const uint32_t bit = 1u << (kk & 31);
                uint32_t *e3 = ev + (kk >> 5) * 3;
                if (ts > 0 && fired && ok_inc) {
                    e3[0] |= bit;
                    e3[1] |= bit;
                    *lw = wv + sign;
                } else if (ts > 0) {
                    e3[0] |= bit;
                } else if (ts < 0 && fired) {
                    e3[0] |= bit;
                    e3[2] |= bit;
                    wv -= sign;
                    if (!cfg.negative_polarity && wv < 1) wv = 1;  // kernel.cu:603-606
                    *lw = wv;
                }
            }
        }
    }
    __syncthreads();

    // ---- 2. per clause: feedback over the words, then evaluation of sample i+1
    const uint32_t max_s = (uint32_t)(cfg.max_state + cfg.state_offset);
    const uint32_t zero_s = (uint32_t)cfg.state_offset;
    const bool top2 = NB >= 2 && (uint32_t)cfg.state_offset + 1u == (1u << (NB >= 2 ? NB - 2 : 0));
    // the stored maximum is 2^(NB-1) + 2^(NB-2) - 1 (power-of-two state counts)
    const bool max_pow2 = NB >= 3 && max_s == (1u << (NB - 1)) + (1u << (NB >= 2 ? NB - 2 : 0)) - 1u;
    // [P][W] literal words of a sample
    auto words_of = [&](int64_t smp) { return lits_of + (IMG ? (smp % 3) * PWW : smp * lits_stride); };
    const uint32_t *x_next = words_of(e_next);  // patch 0 of sample i+1 (single-patch eval)
    constexpr int CPW = CPB / FB_WARPS;  // clauses per warp
    bool has_ev[CPW];
#pragma unroll
    for (int q = 0; q < CPW; ++q) {
        const int j = wib + q * FB_WARPS;
        bool a = false;
        if (do_update)
            for (int kb = 0; kb < KB; ++kb) a |= ev_s[(j * KB + kb) * 3] != 0u;
        has_ev[q] = a;
    }
    // 2a. clauses without events: only the evaluation of sample i+1, with the
    //     loads of all of this warp's clauses in flight together
    uint32_t viol[CPW];
    int cnt[CPW];
#pragma unroll
    for (int q = 0; q < CPW; ++q) { viol[q] = 0u; cnt[q] = 0; }
    if (do_eval && P == 1) {
        for (int w = lane; w < W; w += 32) {
            const uint32_t xn = x_next[w];
#pragma unroll
            for (int q = 0; q < CPW; ++q) {
                const int c = (wib + q * FB_WARPS) * G + blockIdx.x;
                if (!has_ev[q] && c < C) {
                    const uint32_t top = state[((int64_t)(NB - 1) * C + c) * W + w];
                    viol[q] |= top & ~xn;
                    cnt[q] += __popc(top);
                }
            }
        }
    }
    // 2b. clauses with events: feedback of sample i, then the evaluation
    uint32_t n_calls = 0;  // literal-mask Philox calls (not reported by this kernel)
#pragma unroll 1
    for (int q = 0; q < CPW; ++q) {
        if (!has_ev[q]) continue;
        const int j = wib + q * FB_WARPS;
        const int c = j * G + blockIdx.x;
        const uint32_t g = (uint32_t)(cfg.clause_lo + c);
        const int k0 = cfg.coalesced ? 0 : (int)(g / (uint32_t)cfg.clauses_per_class);
        const uint32_t *ev = ev_s + j * KB * 3;
        const int32_t sc = sel_cur[c];
        const uint32_t *x_cur = words_of(i) + (int64_t)(sc > 0 ? sc : 0) * W;  // the picked patch of sample i
        uint32_t vq = 0u;
        int cq = 0;
        for (int w = lane; w < W; w += 32) {
            const uint32_t vm = valid_mask(w, W, L);
            Counter<NB> ctr;
#pragma unroll
            for (int b = 0; b < NB; ++b) ctr.p[b] = state[((int64_t)b * C + c) * W + w];
            const uint32_t x = sc >= 0 ? x_cur[w] : 0u;
            int skip = 0;  // events of a Type Ib run piece already applied
            for (int kb = 0; kb < KB; ++kb) {
                uint32_t m = ev[kb * 3];
                const uint32_t m1a = ev[kb * 3 + 1], m2 = ev[kb * 3 + 2];
                // one_negative: the true class's event first, then the other's
                const int first = cfg.one_negative ? pair_s[0] - k0 - kb * 32 : -1;
                while (m) {
                    int b = __ffs(m) - 1;
                    if (first >= 0 && first < 32 && ((m >> first) & 1u)) b = first;
                    m &= ~(1u << b);
                    if (skip) {
                        --skip;
                        continue;
                    }
                    if (!cfg.one_negative && !(((m1a | m2) >> b) & 1u)) {
                        // Type Ib: the run of consecutive Type Ib events from
                        // here (classes in order; one sample is one window)
                        int run = 1;
                        {
                            uint32_t rem = m;
                            uint32_t stop = (m1a | m2) & rem;
                            for (int kb2 = kb;;) {
                                run += __popc(stop ? (rem & ((stop & (0u - stop)) - 1u)) : rem);
                                if (stop || run >= 64 || ++kb2 >= KB) break;
                                rem = ev[kb2 * 3];
                                stop = (ev[kb2 * 3 + 1] | ev[kb2 * 3 + 2]) & rem;
                            }
                        }
                        if (run >= 8) {
                            const int mi = min(run, 64) / 8 - 1;
                            const uint32_t kk = (uint32_t)(k0 + kb * 32 + b);
                            uint32_t D[7];
                            run_counts(cfg, mi, [&](uint32_t ii) {
                                return draw_rk<7>(rk, g, t, 0x40000000u | ((uint32_t)w << 2) | ii, TAG_SMASK, kk);
                            }, D, n_calls, n_calls, nullptr);
#pragma unroll
                            for (int ii = 0; ii < 7; ++ii) D[ii] &= vm;
                            ctr.sub_floor(D, zero_s, top2);
                            skip = 8 * (mi + 1) - 1;
                            continue;
                        }
                    }
                    if ((m2 >> b) & 1u) {  // type2_fb, kernel.cu:481-506
                        ctr.inc(~x & vm & ctr.below_top());
                    } else {
                        uint32_t cand;
                        if ((m1a >> b) & 1u) {  // type1a_fb, kernel.cu:410-443
                            ctr.inc(x & vm & ctr.lt_max(max_s, max_pow2));
                            cand = ~x & vm & ctr.nonzero(zero_s, top2);
                        } else {  // type1b_fb, kernel.cu:453-470
                            cand = vm & ctr.nonzero(zero_s, top2);
                        }
                        if (cand)
                            ctr.dec(cand & smask_word_rk(cfg, rk, g, t, (uint32_t)(k0 + kb * 32 + b), (uint32_t)w,
                                                         n_calls));
                    }
                }
            }
#pragma unroll
            for (int b = 0; b < NB; ++b) state[((int64_t)b * C + c) * W + w] = ctr.p[b];
            if (do_eval && P == 1) {
                vq |= ctr.p[NB - 1] & ~x_next[w];
                cq += __popc(ctr.p[NB - 1]);
            }
        }
#pragma unroll
        for (int r = 0; r < CPW; ++r)
            if (r == q) { viol[r] = vq; cnt[r] = cq; }
    }
    // 2c. single patch: fired bits, include counts, patch weights, class sums of i+1
    if (do_eval && P == 1) {
#pragma unroll
        for (int q = 0; q < CPW; ++q) {
            const int c = (wib + q * FB_WARPS) * G + blockIdx.x;
            if (c >= C) break;
            const uint32_t vr = __reduce_or_sync(0xFFFFFFFFu, viol[q]);
            const int cr = __reduce_add_sync(0xFFFFFFFFu, cnt[q]);
            const uint32_t g = (uint32_t)(cfg.clause_lo + c);
            const int k0 = cfg.coalesced ? 0 : (int)(g / (uint32_t)cfg.clauses_per_class);
            // an empty clause matches (kernel.cu:273-276); a dropped one never fires
            const bool f = !(drop && drop[c] == 1u) && vr == 0u;
            if (lane == 0) {
                ninc_ws[c] = cr;
                sel_next[c] = f ? 0 : -1;
                if (f) patch_w[c] += 1;  // kernel.cu:305
            }
            if (f)
                for (int kk = lane; kk < nk; kk += 32)
                    atomicAdd(&cs_blk[k0 + kk], weights[(int64_t)c * K + k0 + kk]);
        }
    }
    // 2d. several patches: match every patch of sample i+1 testing only the
    //     clause's non-zero include words (fast_eval, kernel.cu:255-282), then
    //     pick one matching patch uniformly (select_active, kernel.cu:285-316)
    if (do_eval && P > 1) {
        uint32_t *lw = lw_s + wib * W, *li = li_s + wib * W, *mb = mb_s + wib * PW;
        const uint64_t t_next = t0 + (uint64_t)e_next;
#pragma unroll 1
        for (int q = 0; q < CPW; ++q) {
            const int c = (wib + q * FB_WARPS) * G + blockIdx.x;
            if (c >= C) break;
            const uint32_t g = (uint32_t)(cfg.clause_lo + c);
            const int k0 = cfg.coalesced ? 0 : (int)(g / (uint32_t)cfg.clauses_per_class);
            int n = 0, cr = 0;
            for (int w0 = 0; w0 < W; w0 += 32) {
                const int w = w0 + lane;
                const uint32_t top = w < W ? state[((int64_t)(NB - 1) * C + c) * W + w] : 0u;
                cr += __popc(top);
                const uint32_t m = __ballot_sync(0xFFFFFFFFu, top != 0u);
                if (top) {
                    const int pos = n + __popc(m & ((1u << lane) - 1u));
                    lw[pos] = (uint32_t)w;
                    li[pos] = top;
                }
                n += __popc(m);
            }
            cr = __reduce_add_sync(0xFFFFFFFFu, cr);
            __syncwarp();
            const bool dropped = drop && drop[c] == 1u;
            int count = 0;
            if (!dropped) {
                for (int p0 = 0; p0 < P; p0 += 32) {
                    const int p = p0 + lane;
                    bool ok = p < P;
                    if (ok) {
                        const uint32_t *xp = stage ? xs_s + p * SW : words_of(e_next) + (int64_t)p * W;
                        for (int j = 0; j < n; ++j)
                            if (li[j] & ~xp[lw[j]]) { ok = false; break; }
                    }
                    const uint32_t m = __ballot_sync(0xFFFFFFFFu, ok);
                    if (lane == 0) mb[p0 >> 5] = m;
                    count += __popc(m);
                }
            }
            __syncwarp();
            int32_t sp = -1;
            if (count > 0) {
                const uint32_t r = draw(cfg.seed, g, t_next, 0, TAG_PATCH, 0).x;  // t_next may change the high word
                uint32_t idx = (uint32_t)(((uint64_t)r * (uint64_t)count) >> 32);
                for (int jw = 0; jw < PW; ++jw) {
                    uint32_t word = mb[jw];
                    const uint32_t pc = (uint32_t)__popc(word);
                    if (idx < pc) {
                        for (uint32_t z = 0; z < idx; ++z) word &= word - 1u;
                        sp = jw * 32 + __ffs(word) - 1;
                        break;
                    }
                    idx -= pc;
                }
            }
            if (lane == 0) {
                ninc_ws[c] = cr;
                sel_next[c] = sp;
                if (sp >= 0) patch_w[(int64_t)c * P + sp] += 1;  // kernel.cu:305
            }
            if (sp >= 0)
                for (int kk = lane; kk < nk; kk += 32)
                    atomicAdd(&cs_blk[k0 + kk], weights[(int64_t)c * K + k0 + kk]);
            __syncwarp();
        }
    }
    __syncthreads();
    if (do_eval)
        for (int k = threadIdx.x; k < K; k += blockDim.x)
            if (cs_blk[k]) atomicAdd(&cs_next[k], cs_blk[k]);
}

}  // namespace ytm

using namespace ytm;

template <int NB, int CPB, bool IMG>
static ytm_status launch_b1(const ytm_config *cfg, uint32_t *state, int32_t *weights, const int32_t *bias,
                            const uint32_t *drop, const uint32_t *lits, const int32_t *Y, int64_t N, uint64_t t0,
                            int32_t *cs_ring, int32_t *sel, int32_t *ninc, int32_t *patch_w, uint32_t *ring,
                            cudaStream_t st) {
    ytm_status rc;
    if (ring) {  // sample 0's patch words; each launch forms the next one's
        k_patch_words<<<(unsigned)std::min<int64_t>(cdiv((int64_t)cfg->patches * cfg->words, 256), 1024), 256, 0,
                        st>>>(lit_src(cfg, lits), 0, ring);
        if ((rc = launch_check("patch words"))) return rc;
    }
    const int C = cfg->clause_count;
    const int blocks = (int)cdiv(C, CPB);
    const int nk = cfg->coalesced ? cfg->n_classes : 1;
    size_t smem = (size_t)cfg->n_classes * 12 + (size_t)CPB * ((nk + 31) / 32) * 12 + 16;
    // convolutional models stage each sample's patch words in shared memory
    // when they take at most 64 KB
    const size_t stage_bytes = (size_t)cfg->patches * (cfg->words | 1) * 4;
    const int stage = cfg->patches > 1 && stage_bytes <= 64 * 1024;
    if (cfg->patches > 1)
        smem += (size_t)FB_WARPS * (2 * cfg->words + (cfg->patches + 31) / 32) * 4 + (stage ? stage_bytes : 0);
    if (smem > 200 * 1024) return fail(YTM_ERR_UNSUPPORTED, "ytm_train_fit_b1: literal vector too long");
    if (smem > 48 * 1024 &&
        (rc = cuda_check(cudaFuncSetAttribute(k_fused_b1<NB, CPB, IMG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)smem), "fused b1 smem")))
        return rc;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)blocks);
    lc.blockDim = dim3(FB_WARPS * 32);
    lc.dynamicSmemBytes = smem;
    lc.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    const ytm_config c = *cfg;
    for (int64_t i = -1; i < N; ++i) {  // i = -1: the prologue evaluating sample 0
        const int64_t ii = i < 0 ? 0 : i;
        const int upd = i < 0 ? 0 : 1;
        const RoundKeys rk = round_keys(c.seed, (uint32_t)((t0 + (uint64_t)ii) >> 32));  // keys of sample ii
        if ((rc = cuda_check(cudaLaunchKernelEx(&lc, k_fused_b1<NB, CPB, IMG>, c, state, weights, bias, drop, lits, Y, ii,
                                                N, t0, upd, cs_ring, sel, ninc, patch_w, rk, ring, stage),
                             "fused b1 launch")))
            return rc;
    }
    return YTM_OK;
}

extern "C" ytm_status ytm_train_fit_b1(const ytm_config *cfg, uint32_t *state, int32_t *weights, const int32_t *bias,
                                       const uint32_t *drop, const uint32_t *lits, const int32_t *Y, int64_t N,
                                       uint64_t t0, int32_t *patch_w, void *workspace, void *stream) {
    ytm_status rc = check_cfg(cfg);
    if (rc) return rc;
    if (cfg->patches > 32 * 64) return fail(YTM_ERR_UNSUPPORTED, "ytm_train_fit_b1 handles at most 2048 patches");
    if (N < 0) return fail(YTM_ERR_ARG, "N < 0");
    if (N == 0) return YTM_OK;
    if (!state || !weights || !lits || !Y || !patch_w || !workspace) return fail(YTM_ERR_ARG, "null pointer");
    if (cfg->coalesced && cfg->n_classes > 256)
        return fail(YTM_ERR_UNSUPPORTED, "ytm_train_fit_b1 handles at most 256 classes");
    cudaStream_t st = as_stream(stream);
    B1Ws l = b1_ws_layout(cfg);
    char *ws = (char *)workspace;
    int32_t *cs_ring = (int32_t *)(ws + l.cs);
    int32_t *sel = (int32_t *)(ws + l.fired);
    int32_t *ninc = (int32_t *)(ws + l.ninc);
    uint32_t *ring = cfg->input_images ? (uint32_t *)(ws + l.ring) : nullptr;
    if ((rc = cuda_check(cudaMemsetAsync(cs_ring, 0, 3 * (size_t)cfg->n_classes * 4, st), "memset"))) return rc;
    const int cpb = cfg->patches > 1 ? YTM_B1_CPB_CONV : YTM_B1_CPB;
    YTM_DISPATCH_PLANES(cfg->planes, {
        // bit images only come with several patches
        rc = ring ? launch_b1<NB, YTM_B1_CPB_CONV, true>(cfg, state, weights, bias, drop, lits, Y, N, t0, cs_ring, sel, ninc,
                                            patch_w, ring, st)
             : cpb == YTM_B1_CPB_CONV ? launch_b1<NB, YTM_B1_CPB_CONV, false>(cfg, state, weights, bias, drop, lits, Y, N, t0, cs_ring, sel,
                                                    ninc, patch_w, ring, st)
                         : launch_b1<NB, YTM_B1_CPB, false>(cfg, state, weights, bias, drop, lits, Y, N, t0, cs_ring, sel,
                                                    ninc, patch_w, ring, st);
        if (rc) return rc;
    });
    return launch_check("fused b1");
}
