// update.cu — Type I / Type II feedback of a training batch.
//
// Reference: clause_update with type1a_fb / type1b_fb / type2_fb
// (kernel.cu:397-613): one thread per clause walks classes and then all L
// literals as u32 states, drawing one curand uniform per eligible literal.
//
// Here a CTA owns one clause.  A one-block kernel first turns the batch's
// class sums into update thresholds and the list of (sample, class) pairs
// whose threshold is non-zero (only those can update any clause; once a model
// has converged most pairs drop out).  Then per chunk of up to 128 samples:
//  1. the Q-selection and update draws of the active pairs run in parallel;
//     threads over classes walk their active samples in order to fix each
//     feedback type (it depends on the weight sign), updating weights in
//     shared memory;
//  2. the decided events are compacted into a list in feedback order;
//  3. threads over literal words load the word's bit planes once, apply every
//     event of the chunk in order with bit-parallel ripple adders (32 literals
//     per instruction), and store the planes once.
// The state therefore makes one read-modify-write trip through memory per
// chunk, however many events the chunk holds.
//
// Small batches (at most 32 samples) run the same steps with one WARP per
// clause (WPC): the decision phases then cost warp syncs instead of CTA
// barriers, and a block holds 8 clauses.
#include "common.cuh"

namespace ytm {

// samples per chunk at most: list entries hold 8-bit rows, and a chunk is at
// most one Type Ib run window (run_window: 128 or 64 samples)
constexpr int UPD_BC_MAX = 128;
static_assert(UPD_BC_MAX <= 256, "event list rows are 8 bits");

// One block prepares the batch's decisions, which every clause shares.
//  * thr[b][k] = floor(p * 2^32) of the update probability, bit 63 set when
//    the target is -1 (kernel.cu:544-551, 569-571).
//  * The pair (b, k) is active when thr is non-zero (the update draw is
//    r < thr, so an inactive pair never updates a clause) and, under pytm's
//    rules, k is one of the sample's two classes.  Once a model has converged
//    most class sums sit at +-T and few pairs stay active.
//  * amask[b][k / 32] and colm[k][b / 32] hold the active pairs as bits per
//    sample and per class; alist lists them in feedback order (sample by
//    sample; classes in order, or pytm's true class first), each entry
//    (threshold - 1) << 32 | negative << 31 | sample << 16 | class, so that the
//    feedback reads a pair's decision inputs in one contiguous load; row_off[b]
//    is the position of sample b's first pair in it (row_off[B] = the count).
//    With the negative-class selection drawn as a set (q_select), each
//    sample's target +1 pairs come first and npos[b] counts them.
// An active pair's list entry (its threshold is at least 1, at most 2^32).
__device__ __forceinline__ uint64_t pair_entry(const uint64_t *__restrict__ thr, int b, int k, int K) {
    const uint64_t th = thr[(int64_t)b * K + k];
    return (((th & ~(1ull << 63)) - 1ull) << 32) | ((th >> 63) << 31) | ((uint64_t)b << 16) | (uint64_t)k;
}

__global__ void __launch_bounds__(1024) k_thresholds(const int32_t *__restrict__ cs, const int32_t *__restrict__ Y,
                                                     int B, int K, int T, int one_neg,
                                                     const int32_t *__restrict__ pair, uint64_t *__restrict__ thr,
                                                     uint32_t *__restrict__ amask, uint32_t *__restrict__ colm,
                                                     int32_t *__restrict__ row_off, uint64_t *__restrict__ alist,
                                                     int qsel, int32_t *__restrict__ npos) {
    constexpr int AM_SMEM = 8192;  // words of amask kept in shared memory
    __shared__ uint32_t am_s[AM_SMEM];
    __shared__ int wsum[32];
    __shared__ int base_s;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int KWm = (K + 31) >> 5, BW = (B + 31) >> 5;
    const int64_t nam = (int64_t)B * KWm;
    const bool in_smem = nam <= AM_SMEM;
    if (in_smem) {  // a thread per pair; the bits gather in shared memory
        for (int i = threadIdx.x; i < nam; i += blockDim.x) am_s[i] = 0u;
        __syncthreads();
        for (int i = threadIdx.x; i < B * K; i += blockDim.x) {
            const int b = i / K, k = i - b * K;
            int32_t v = cs[i];
            v = v > T ? T : (v < -T ? -T : v);  // clip_cs, kernel.cu:397
            const int32_t y = Y[i];
            uint64_t t = update_threshold(y, v);
            if (t != 0ull && (!one_neg || k == pair[2 * b] || k == pair[2 * b + 1]))
                atomicOr(&am_s[b * KWm + (k >> 5)], 1u << (k & 31));
            if (v > y) t |= 1ull << 63;
            thr[i] = t;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < nam; i += blockDim.x) amask[i] = am_s[i];
    } else {  // a warp per (sample, 32 classes)
        for (int64_t u = wid; u < nam; u += nw) {
            const int64_t b = u / KWm;
            const int k = (int)(u - b * KWm) * 32 + lane;
            bool act = false;
            if (k < K) {
                int32_t v = cs[b * K + k];
                v = v > T ? T : (v < -T ? -T : v);
                const int32_t y = Y[b * K + k];
                uint64_t t = update_threshold(y, v);
                act = t != 0ull && (!one_neg || k == pair[2 * b] || k == pair[2 * b + 1]);
                if (v > y) t |= 1ull << 63;
                thr[b * K + k] = t;
            }
            const uint32_t m = __ballot_sync(0xFFFFFFFFu, act);
            if (lane == 0) amask[u] = m;
        }
    }
    const uint32_t *am_all = in_smem ? am_s : amask;
    if (threadIdx.x == 0) base_s = 0;
    __syncthreads();
    for (int64_t u = wid; u < (int64_t)K * BW; u += nw) {
        const int k = (int)(u / BW), row = (int)(u - (int64_t)k * BW) * 32 + lane;
        const bool a = row < B && ((am_all[(int64_t)row * KWm + (k >> 5)] >> (k & 31)) & 1u);
        const uint32_t m = __ballot_sync(0xFFFFFFFFu, a);
        if (lane == 0) colm[u] = m;
    }
    for (int r0 = 0; r0 < B; r0 += blockDim.x) {
        const int row = r0 + threadIdx.x;
        int n = 0;
        if (row < B)
            for (int m = 0; m < KWm; ++m) n += __popc(am_all[(int64_t)row * KWm + m]);
        int incl = n;
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
            if (lane >= o) incl += v;
        }
        if (lane == 31) wsum[wid] = incl;
        __syncthreads();
        if (wid == 0) {
            int v = lane < nw ? wsum[lane] : 0;
            for (int o = 1; o < 32; o <<= 1) {
                const int x = __shfl_up_sync(0xFFFFFFFFu, v, o);
                if (lane >= o) v += x;
            }
            wsum[lane] = v;
        }
        __syncthreads();
        int pos = base_s + (wid ? wsum[wid - 1] : 0) + incl - n;
        if (row < B) {
            row_off[row] = pos;
            const uint32_t *am = am_all + (int64_t)row * KWm;
            if (one_neg) {
                for (int q = 0; q < 2; ++q) {
                    const int k = pair[2 * row + q];
                    if (k >= 0 && ((am[k >> 5] >> (k & 31)) & 1u)) alist[pos++] = pair_entry(thr, row, k, K);
                }
            }
        }
        __syncthreads();
        if (threadIdx.x == 0) base_s += wsum[nw - 1];
        __syncthreads();
    }
    if (threadIdx.x == 0) row_off[B] = base_s;
    if (one_neg) return;
    // the pair lists: a warp per sample, 32 classes per ballot, classes in
    // ascending order (with qsel: the target +1 pairs, then the target -1
    // ones); row_off was written by this block before the barrier above
    for (int row = wid; row < B; row += nw) {
        int pos = row_off[row], np = 0;
        const uint32_t *am = am_all + (int64_t)row * KWm;
        for (int pass = 0; pass < (qsel ? 2 : 1); ++pass) {
            for (int m = 0; m < KWm; ++m) {
                const int k = m * 32 + lane;
                bool a = (am[m] >> lane) & 1u;
                if (a && qsel) a = (int)(thr[(int64_t)row * K + k] >> 63) == pass;
                const uint32_t bal = __ballot_sync(0xFFFFFFFFu, a);
                if (a) alist[pos + __popc(bal & ((1u << lane) - 1u))] = pair_entry(thr, row, k, K);
                pos += __popc(bal);
                if (pass == 0) np += __popc(bal);
            }
        }
        if (qsel && lane == 0) npos[row] = np;
    }
}

// Patch literal words u32 [B][P][W] of samples 0..B-1 of the bit images.
__global__ void k_batch_words(const LitSrc src, int64_t B, uint32_t *__restrict__ out) {
    const int64_t PW = (int64_t)src.P * src.g.W, total = B * PW;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = idx / PW;
        const int64_t r = idx - n * PW;
        const int p = (int)(r / src.g.W);
        out[idx] = src.word<true>(n, p, (int)(r - (int64_t)p * src.g.W));
    }
}

// Optional per-phase cycle counts of the feedback kernel (measurement
// builds with -DYTM_PHASE_TIMING only: counters[6..11] receive the cycles
// thread 0 of each clause spent in each phase).
#ifdef YTM_PHASE_TIMING
#define YTM_PHASE_START() long long ph_last_ = clock64()
#define YTM_PHASE(i)                                       \
    do {                                                   \
        const long long ph_now_ = clock64();               \
        ph_cyc[i] += (unsigned long long)(ph_now_ - ph_last_); \
        ph_last_ = ph_now_;                                \
    } while (0)
#else
#define YTM_PHASE_START() ((void)0)
#define YTM_PHASE(i) ((void)0)
#endif

template <bool WPC>
__device__ __forceinline__ void block_sync() {
    if (WPC)
        __syncwarp();
    else
        __syncthreads();
}

// Shared memory of one clause: weights [nk], picks [bc], count, event list
// [bc*nk], fired samples [bc/32], event types [bc*nk], simple classes [nk],
// pairs with an event as bits [bc][ceil(nk/32)].
// An event list entry is row << 24 | type << 22 | run piece << 18 | class
// (piece: 0 for a single event, mi + 1 for the first event of a Type Ib run
// piece of 8 (mi + 1) events).
// update_smem() (without the last two small arrays' padding) sizes the chunk.
static __host__ __device__ inline size_t update_smem(int nk, int bc) {
    return (size_t)nk * 4 + (size_t)bc * 4 + 4 + (size_t)bc * nk * 4 + (size_t)bc * nk + 16;
}
static __host__ __device__ inline size_t update_smem_total(int nk, int bc) {
    return update_smem(nk, bc) + (size_t)(bc / 32) * 4 + (size_t)nk + 4 + (size_t)bc * ((nk + 31) / 32) * 4;
}
static __host__ __device__ inline size_t update_smem_aligned(int nk, int bc) {
    return (update_smem_total(nk, bc) + 15) & ~(size_t)15;
}

enum : uint32_t { EV_NONE = 0, EV_T1A = 1, EV_T1B = 2, EV_T2 = 3 };

__global__ void k_pairs(uint64_t seed, const int32_t *__restrict__ Y, int B, int K, uint64_t t0,
                        int32_t *__restrict__ pair) {
    for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < B; b += gridDim.x * blockDim.x) {
        int kt, ko;
        true_other_pair(seed, Y + (int64_t)b * K, K, t0 + (uint64_t)b, &kt, &ko);
        pair[2 * b] = kt;
        pair[2 * b + 1] = ko;
    }
}

// The decision of clause g for the active pair (b, k) from its two decision
// uniforms (class_words): 1 = update with target +1, 2 = with target -1, 0 =
// none.  Pairs reach here only when active (under pytm's rules: one of the
// sample's two classes).
__device__ __forceinline__ uint8_t decide_words(const ytm_config &cfg, const uint64_t *__restrict__ thr, int b, int k,
                                                int K, uint2 u) {
    uint64_t th = thr[(int64_t)b * K + k];
    const bool neg = (th >> 63) != 0;
    th &= ~(1ull << 63);
    const bool pass = cfg.one_negative || !(neg && !((uint64_t)u.x < cfg.q_threshold));  // kernel.cu:573
    return (pass && (uint64_t)u.y < th) ? (neg ? 2 : 1) : 0;                             // kernel.cu:582
}

__device__ __forceinline__ u32x4 pair_draw(const ytm_config &cfg, const RoundKeys &rk, int rk_ok, uint32_t g,
                                           uint64_t tb, int k) {
    return rk_ok ? class_pair_draw_rk(rk, g, tb, (uint32_t)k) : class_pair_draw(cfg.seed, g, tb, (uint32_t)k);
}

template <int NB, bool WPC>
#ifndef YTM_UPD_MINB
#define YTM_UPD_MINB 4  // 64 registers: measured fastest (no spills)
#endif
#ifndef YTM_UPD_MINB_WIDE
// 12 planes and more: 80 registers (no spills); such models' event lists
// (at least 4096 states go with wide, many-class workloads) mostly leave
// shared memory for 3 CTAs of 256 threads anyway
#define YTM_UPD_MINB_WIDE 3
#endif
__global__ void __launch_bounds__(256, (NB >= 12 ? YTM_UPD_MINB_WIDE : YTM_UPD_MINB)) k_update(ytm_config cfg, uint32_t *__restrict__ state,
                                                int32_t *__restrict__ weights, const uint64_t *__restrict__ thr,
                                                const uint32_t *__restrict__ drop,
                                                const LitSrc src, int B, uint64_t t0,
                                                const int32_t *__restrict__ sel, int32_t *__restrict__ patch_w,
                                                int BC, const RoundKeys rk, int rk_ok,
                                                int count_patch, const int32_t *__restrict__ pair,
                                                const uint32_t *__restrict__ amask, const uint32_t *__restrict__ colm,
                                                const int32_t *__restrict__ row_off,
                                                const uint64_t *__restrict__ alist,
                                                const uint32_t *__restrict__ fcm,
                                                const int32_t *__restrict__ npos,
                                                unsigned long long *__restrict__ counters) {
    extern __shared__ __align__(16) unsigned char small[];
    const int C = cfg.clause_count, W = cfg.words, K = cfg.n_classes;
    // the Type Ib run thresholds' plane masks, after the clauses' arrays
    uint4 *kmt = (uint4 *)(small + (WPC ? (blockDim.x >> 5) : 1u) * update_smem_aligned(cfg.coalesced ? K : 1, BC));
    run_table_fill(cfg, kmt, (int)threadIdx.x, (int)blockDim.x);
    __syncthreads();
    const int c = WPC ? (int)(blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) : (int)blockIdx.x;
    if (c >= C) return;
    const uint32_t g = (uint32_t)(cfg.clause_lo + c);
    if (drop && drop[c] == 1u) return;  // kernel.cu:555
    const int k0 = cfg.coalesced ? 0 : (int)(g / (uint32_t)cfg.clauses_per_class);
    const int nk = cfg.coalesced ? K : 1;
    const int BW = (B + 31) >> 5, KWm = (K + 31) >> 5;
    unsigned char *smraw = WPC ? small + (threadIdx.x >> 5) * update_smem_aligned(nk, BC) : small;
    int32_t *wk = (int32_t *)smraw;                       // [nk]
    int32_t *sel_s = wk + nk;                             // [BC]
    int32_t *cnt = sel_s + BC;                            // [1]
    uint32_t *list = (uint32_t *)(cnt + 1);               // [BC * nk]
    uint32_t *fm = list + BC * nk;                        // [BC / 32] samples whose clause output is 1
    uint8_t *evt = (uint8_t *)(fm + BC / 32);             // [BC * nk], valid at active pairs only
    uint8_t *simple = evt + BC * nk;                      // [nk] no active sample of the class fired
    uint32_t *enz = (uint32_t *)(((uintptr_t)(simple + nk) + 3) & ~(uintptr_t)3);  // [BC][KWm] pairs with an event
    const int tid = WPC ? (int)(threadIdx.x & 31) : (int)threadIdx.x, nt = WPC ? 32 : (int)blockDim.x;
    const int lane = tid & 31;
    // include count of the batch-start state (pack_clauses, kernel.cu:155-204):
    // this CTA alone writes the clause, so its top plane is still unchanged.
    // Not needed when the cap cannot bind.
    bool ok_inc = true;
    if (cfg.max_included_literals < cfg.literals) {
        int n = 0;
        for (int w = tid; w < W; w += nt) n += __popc(state[((int64_t)(NB - 1) * C + c) * W + w]);
        for (int o = 16; o; o >>= 1) n += __shfl_xor_sync(0xFFFFFFFFu, n, o);
        if (WPC) {
            ok_inc = n <= cfg.max_included_literals;
        } else {
            __shared__ int ninc_s;
            if (tid == 0) ninc_s = 0;
            __syncthreads();
            if ((tid & 31) == 0 && n) atomicAdd(&ninc_s, n);
            __syncthreads();
            ok_inc = ninc_s <= cfg.max_included_literals;
        }
    }
    int fired_count = 0;  // single-patch models: patch 0 picks of this clause (select_active, kernel.cu:305)
    const uint32_t win_shift = run_window(cfg) == 128 ? 7u : 6u;  // Type Ib run windows
    // measurement counters: (event, word) pairs applied, Philox4x32-7 calls
    // of the literal masks, state words streamed, events
    uint32_t n_units = 0, n_calls = 0, n_words = 0, n_events = 0, n_dcalls = 0, n_tests = 0;
#ifdef YTM_PHASE_TIMING
    unsigned long long ph_cyc[6] = {0, 0, 0, 0, 0, 0};
#endif
    const uint32_t max_s = (uint32_t)(cfg.max_state + cfg.state_offset);
    const uint32_t zero_s = (uint32_t)cfg.state_offset;
    const bool top2 = NB >= 2 && (uint32_t)cfg.state_offset + 1u == (1u << (NB >= 2 ? NB - 2 : 0));
    // the stored maximum is 2^(NB-1) + 2^(NB-2) - 1 (power-of-two state counts)
    const bool max_pow2 = NB >= 3 && max_s == (1u << (NB - 1)) + (1u << (NB >= 2 ? NB - 2 : 0)) - 1u;
    const uint32_t *mycol = colm + (int64_t)k0 * BW;  // non-coalesced: the active samples of the bank's class
    // the pairs holding an event, as bits kept by the decision phases (the
    // compaction over all threads reads them)
    const bool use_enz = !WPC && cfg.coalesced && !cfg.one_negative;
    // negative-class selection drawn as a set per (clause, sample)
    const bool use_qsel = cfg.coalesced && cfg.q_select && !cfg.one_negative;

    for (int kk = tid; kk < nk; kk += nt) wk[kk] = weights[(int64_t)c * K + k0 + kk];

    for (int b0 = 0; b0 < B; b0 += BC) {  // BC is a multiple of 32
        YTM_PHASE_START();
        const int bc = min(BC, B - b0);
        for (int q0 = tid & ~31; q0 < bc; q0 += nt) {  // warp-uniform
            const int q = q0 + lane;
            int32_t sv = -1;
            if (fcm) {  // single patch: the clause's fired bits (pick = patch 0)
                const uint32_t f = fcm[(int64_t)c * BW + ((b0 + q0) >> 5)];
                if (q < bc) sv = ((f >> lane) & 1u) ? 0 : -1;
            } else if (q < bc) {
                sv = sel[(int64_t)(b0 + q) * C + c];
            }
            if (q < bc) {
                sel_s[q] = sv;
                fired_count += sv >= 0;
            }
            const uint32_t f = __ballot_sync(0xFFFFFFFFu, sv >= 0);
            if (lane == 0) fm[q0 >> 5] = f;
        }
        block_sync<WPC>();
        YTM_PHASE(0);
        // A class none of whose active samples fired the clause is simple:
        // its events are Type Ib or none, fixed by the weight's sign, and its
        // weight stays as it is for the chunk (kernel.cu:584-606).
        for (int kk = tid; kk < nk; kk += nt) {
            const uint32_t *cm = colm + (int64_t)(k0 + kk) * BW + (b0 >> 5);
            uint32_t hit = 0u;
            for (int gi = 0; gi < (bc + 31) >> 5; ++gi) hit |= cm[gi] & fm[gi];
            simple[kk] = hit == 0u;
        }
        if (use_enz)
            for (int i = tid; i < bc * KWm; i += nt) enz[i] = 0u;
        block_sync<WPC>();
        YTM_PHASE(1);
        const int lo = cfg.coalesced ? row_off[b0] : 0, hi = cfg.coalesced ? row_off[b0 + bc] : 0;
        // 1a. the Q-selection and update draws of the active pairs, in
        //     parallel: 1 = update with target +1, 2 = with target -1; simple
        //     classes get their event type here (Ib when target and weight
        //     sign agree)
        if (use_qsel) {
            // the negative-class selection drawn as a set per sample
            // (kernel.cu:573); only events are written, so the chunk's event
            // types start cleared
            const int nb = bc * nk;
            for (int i = tid; i < (nb >> 2); i += nt) ((uint32_t *)evt)[i] = 0u;
            for (int i = (nb & ~3) + tid; i < nb; i += nt) evt[i] = 0;
            if (tid == 0) cnt[0] = 0;  // the candidate count (the event count later)
            block_sync<WPC>();
            // (a) a thread per (sample, task): the sample's selected classes
            //     with target -1 and an active pair, or its target +1 pairs,
            //     into a candidate list (the event list's space, unused until
            //     the compaction; candidates are distinct pairs of the chunk)
            for (int x = tid; x < 2 * bc; x += nt) {
                const int bl = x >> 1, b = b0 + bl;
                const int lo_b = row_off[b], hi_b = row_off[b + 1], np = npos[b];
                if (x & 1) {  // target +1: no selection (kernel.cu:573)
                    for (int i = lo_b; i < lo_b + np; ++i)
                        list[atomicAdd(cnt, 1)] = ((uint32_t)bl << 16) | (uint32_t)(alist[i] & 0xFFFFu);
                } else if (hi_b - lo_b > np) {  // some target -1 pair is active
                    const uint64_t tb = t0 + (uint64_t)b;
                    uint16_t qs[32];
                    int nq = 0;
                    qselect(cfg, [&](uint32_t sub) {
                        ++n_dcalls;
                        return rk_ok ? draw_rk<7>(rk, g, tb, sub, TAG_CLASS, 0)
                                     : draw<7>(cfg.seed, g, tb, sub, TAG_CLASS, 0);
                    }, [&](int v) {
                        for (int j = 0; j < nq; ++j)
                            if (qs[j] == (uint16_t)v) return false;
                        qs[nq++] = (uint16_t)v;
                        const uint64_t th = thr[(int64_t)b * K + v];
                        if ((th >> 63) && (th & ~(1ull << 63)))  // target -1, active
                            list[atomicAdd(cnt, 1)] = ((uint32_t)bl << 16) | (uint32_t)v;
                        return true;
                    });
                }
            }
            block_sync<WPC>();
            // (b) a thread per candidate pair: its update draw (kernel.cu:582)
            const int ncand = cnt[0];
            for (int j = tid; j < ncand; j += nt) {
                const uint32_t ce = list[j];
                const int bl = (int)(ce >> 16), k = (int)(ce & 0xFFFFu);
                const uint64_t th = thr[(int64_t)(b0 + bl) * K + k];
                const uint2 u = class_words(pair_draw(cfg, rk, rk_ok, g, t0 + (uint64_t)(b0 + bl), k), (uint32_t)k);
                ++n_dcalls;
                if ((uint64_t)u.y < (th & ~(1ull << 63))) {
                    uint8_t a = (th >> 63) ? 2 : 1;
                    if (simple[k]) a = ((a == 1) == (wk[k] >= 0)) ? EV_T1B : EV_NONE;
                    if (a) {
                        evt[bl * nk + k] = a;
                        if (use_enz) atomicOr(&enz[bl * KWm + (k >> 5)], 1u << (k & 31));
                    }
                }
            }
        }
        // otherwise four consecutive list entries per thread, loaded together;
        // when two neighbours are the two classes of one class pair of one
        // sample, one Philox call serves both
        for (int i0 = lo + 4 * tid; !use_qsel && i0 < hi; i0 += 4 * nt) {  // coalesced: the chunk's pairs
            uint64_t ent[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) ent[j] = i0 + j < hi ? alist[i0 + j] : 0ull;
            u32x4 r{};
            uint32_t rkey = 0xFFFFFFFFu;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (i0 + j >= hi) break;
                const uint64_t e = ent[j];
                const int b = (int)((e >> 16) & 0x7FFFu), k = (int)(e & 0xFFFFu);
                const uint32_t key = ((uint32_t)e & 0x7FFFFFFFu) >> 1;  // (sample, class pair)
                if (key != rkey) {
                    r = pair_draw(cfg, rk, rk_ok, g, t0 + (uint64_t)b, k);
                    rkey = key;
                    ++n_dcalls;
                }
                const uint2 u = class_words(r, (uint32_t)k);
                const bool neg = (e >> 31) & 1u;
                const bool pass = cfg.one_negative || !neg || (uint64_t)u.x < cfg.q_threshold;  // kernel.cu:573
                uint8_t a = (pass && u.y <= (uint32_t)(e >> 32)) ? (neg ? 2 : 1) : 0;          // kernel.cu:582
                if (simple[k]) a = (a && ((a == 1) == (wk[k] >= 0))) ? EV_T1B : EV_NONE;
                evt[(b - b0) * nk + k] = a;
                if (use_enz && a) atomicOr(&enz[(b - b0) * KWm + (k >> 5)], 1u << (k & 31));
            }
        }
        if (!cfg.coalesced)
            for (int bl = tid; bl < bc; bl += nt)
                if ((mycol[(b0 + bl) >> 5] >> ((b0 + bl) & 31)) & 1u) {
                    uint8_t a = decide_words(cfg, thr, b0 + bl, k0, K,
                                             class_words(pair_draw(cfg, rk, rk_ok, g, t0 + (uint64_t)(b0 + bl), k0),
                                                         (uint32_t)k0));
                    if (simple[0]) a = (a && ((a == 1) == (wk[0] >= 0))) ? EV_T1B : EV_NONE;
                    evt[bl] = a;
                    ++n_dcalls;
                }
        block_sync<WPC>();
        YTM_PHASE(2);
        // 1b. feedback types, class-parallel and sample-sequential over the
        //     class's active samples (weights evolve)
        for (int kk = tid; kk < nk; kk += nt) {
            if (simple[kk]) continue;
            int32_t wv = wk[kk];
            const uint32_t *cm = colm + (int64_t)(k0 + kk) * BW + (b0 >> 5);
            for (int gi = 0; gi < (bc + 31) >> 5; ++gi) {
                for (uint32_t mm = cm[gi]; mm; mm &= mm - 1u) {
                    const int bl = gi * 32 + __ffs(mm) - 1;
                    const uint8_t a = evt[bl * nk + kk];
                    uint8_t ev = EV_NONE;
                    if (a) {
                        const int target = a == 1 ? 1 : -1;
                        const int sign = (wv >= 0) - (wv < 0);
                        const bool fired = sel_s[bl] > -1;
                        const int ts = target * sign;
                        if (ts > 0 && fired && ok_inc) {
                            ev = EV_T1A;
                            wv += sign;
                        } else if (ts > 0) {
                            ev = EV_T1B;
                        } else if (ts < 0 && fired) {
                            ev = EV_T2;
                            wv -= sign;
                            if (!cfg.negative_polarity && wv < 1) wv = 1;  // kernel.cu:603-606
                        }
                    }
                    evt[bl * nk + kk] = ev;
                    if (use_enz && a && ev == EV_NONE) atomicAnd(&enz[bl * KWm + (kk >> 5)], ~(1u << (kk & 31)));
                }
            }
            wk[kk] = wv;
        }
        block_sync<WPC>();
        YTM_PHASE(3);
        // 2. the events in feedback order: a lane per sample counts and then
        //    writes its events (classes in order; pytm's rules: the true
        //    class first); only active pairs hold event types
        if (!WPC && cfg.coalesced && !cfg.one_negative) {
            // all threads: a thread per (sample, 32 classes) unit in feedback
            // order, an exclusive scan of their event counts over the block,
            // then each writes its events in class order
            __shared__ int psum_s[8];
            const int nwarp = nt >> 5, wid = tid >> 5;
            const int units = bc * KWm;
            int base = 0;
            for (int u0 = 0; u0 < units; u0 += nt) {
                const int u = u0 + tid;
                uint32_t em = 0u;
                int row = 0, m = 0;
                if (u < units) {
                    row = u / KWm;
                    m = u - row * KWm;
                    em = enz[row * KWm + m];
                }
                const int n = __popc(em);
                int incl = n;
                for (int o = 1; o < 32; o <<= 1) {
                    const int v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
                    if (lane >= o) incl += v;
                }
                if (lane == 31) psum_s[wid] = incl;
                __syncthreads();
                if (tid < 32) {
                    int v = lane < nwarp ? psum_s[lane] : 0;
                    for (int o = 1; o < 32; o <<= 1) {
                        const int x = __shfl_up_sync(0xFFFFFFFFu, v, o);
                        if (lane >= o) v += x;
                    }
                    if (lane < nwarp) psum_s[lane] = v;
                }
                __syncthreads();
                int pos = base + (wid ? psum_s[wid - 1] : 0) + incl - n;
                for (uint32_t v = em; v; v &= v - 1u) {
                    const int k = m * 32 + __ffs(v) - 1;
                    list[pos++] = ((uint32_t)row << 24) | ((uint32_t)evt[row * nk + k] << 22) | (uint32_t)k;
                }
                base += psum_s[nwarp - 1];
                __syncthreads();
            }
            if (tid == 0) cnt[0] = base;
        } else if (tid < 32) {  // WPC: the whole warp
            int base = 0;
            for (int r0 = 0; r0 < bc; r0 += 32) {
                const int row = r0 + lane;
                const int64_t b = b0 + row;
                int n = 0;
                if (row < bc) {
                    if (cfg.coalesced) {
                        for (int m = 0; m < KWm; ++m)
                            for (uint32_t v = amask[b * KWm + m]; v; v &= v - 1u)
                                n += evt[row * nk + m * 32 + __ffs(v) - 1] != EV_NONE;
                    } else {
                        n = ((mycol[b >> 5] >> (b & 31)) & 1u) && evt[row] != EV_NONE;
                    }
                }
                int incl = n;
                for (int o = 1; o < 32; o <<= 1) {
                    const int v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
                    if (lane >= o) incl += v;
                }
                int pos = base + incl - n;
                if (n && !cfg.coalesced) {
                    list[pos] = ((uint32_t)row << 24) | ((uint32_t)evt[row] << 22);
                } else if (n && cfg.one_negative) {
                    for (int q = 0; q < 2; ++q) {
                        const int k = pair[2 * b + q];
                        if (k < 0 || !((amask[b * KWm + (k >> 5)] >> (k & 31)) & 1u)) continue;
                        const uint32_t ev = evt[row * nk + k];
                        if (ev != EV_NONE) list[pos++] = ((uint32_t)row << 24) | (ev << 22) | (uint32_t)k;
                    }
                } else if (n) {
                    for (int m = 0; m < KWm; ++m)
                        for (uint32_t v = amask[b * KWm + m]; v; v &= v - 1u) {
                            const int k = m * 32 + __ffs(v) - 1;
                            const uint32_t ev = evt[row * nk + k];
                            if (ev != EV_NONE) list[pos++] = ((uint32_t)row << 24) | (ev << 22) | (uint32_t)k;
                        }
                }
                base += __shfl_sync(0xFFFFFFFFu, incl, 31);
            }
            if (lane == 0) cnt[0] = base;
        }
        block_sync<WPC>();
        const int nev = cnt[0];
        // 2b. Type Ib run pieces, once per chunk: the first event of each run
        //     of consecutive Type Ib events inside a run window marks its
        //     pieces (from the run start, each the longest multiple of 8
        //     events up to 64 that the rest holds; fewer than 8 remain
        //     single events) with code mi + 1 in bits 18..21 of their first
        //     entry
        for (int e = tid; e < nev; e += nt) {
            const uint32_t ent = list[e];
            if (((ent >> 22) & 3u) != EV_T1B) continue;
            const uint32_t win = (ent >> 24) >> win_shift;
            if (e > 0) {
                const uint32_t ep = list[e - 1];
                if (((ep >> 22) & 3u) == EV_T1B && ((ep >> 24) >> win_shift) == win) continue;  // not a run start
            }
            int run = 1;
            while (e + run < nev) {
                const uint32_t en = list[e + run];
                if (((en >> 22) & 3u) != EV_T1B || ((en >> 24) >> win_shift) != win) break;
                ++run;
            }
            for (int q = e; run >= 8;) {
                const int m = min(run, 64) & ~7;
                list[q] |= (uint32_t)(m >> 3) << 18;
                q += m;
                run -= m;
            }
        }
        block_sync<WPC>();
        YTM_PHASE(4);
        // 3. stream the literal words
        if (nev > 0) {
            if (counters && tid == 0) n_events += (uint32_t)nev;
            for (int w = tid; w < W; w += nt) {
                ++n_words;
                Counter<NB> ctr;
#pragma unroll
                for (int i = 0; i < NB; ++i) ctr.p[i] = state[((int64_t)i * C + c) * W + w];
                const uint32_t vm = valid_mask(w, W, cfg.literals);
                for (int e = 0; e < nev; ++e) {
                    const uint32_t ent = list[e];
                    const int bl = (int)(ent >> 24);
                    const uint32_t ev = (ent >> 22) & 3u;
                    const int k = k0 + (int)(ent & 0xFFFFu);
                    const int b = b0 + bl;
                    const uint64_t t = t0 + (uint64_t)b;
                    ++n_units;
                    {
                        const uint32_t piece = (ent >> 18) & 15u;
                        if (piece) {  // a Type Ib run piece of 8 (mi + 1) events
                            const int mi = (int)piece - 1;
                            uint32_t D[7];
                            run_counts(cfg, mi, [&](uint32_t i) {
                                const uint32_t sub = 0x40000000u | ((uint32_t)w << 2) | i;
                                return rk_ok ? draw_rk<7>(rk, g, t, sub, TAG_SMASK, (uint32_t)k)
                                             : draw<7>(cfg.seed, g, t, sub, TAG_SMASK, (uint32_t)k);
                            }, D, n_calls, n_tests, kmt + 4 * run_table_base(cfg, mi));
#pragma unroll
                            for (int i = 0; i < 7; ++i) D[i] &= vm;
                            ctr.sub_floor(D, zero_s, top2);
                            e += 8 * (mi + 1) - 1;
                            continue;
                        }
                    }
                    if (ev == EV_T2) {  // type2_fb, kernel.cu:481-506
                        const uint32_t x = src.word<false>(b, sel_s[bl], w);
                        ctr.inc(~x & vm & ctr.below_top());
                    } else {
                        uint32_t cand;
                        if (ev == EV_T1A) {  // type1a_fb, kernel.cu:410-443
                            const uint32_t x = src.word<false>(b, sel_s[bl], w);
                            ctr.inc(x & vm & ctr.lt_max(max_s, max_pow2));
                            cand = ~x & vm & ctr.nonzero(zero_s, top2);
                        } else {  // type1b_fb, kernel.cu:453-470
                            cand = vm & ctr.nonzero(zero_s, top2);
                        }
                        if (cand)
                            ctr.dec(cand & (rk_ok ? smask_word_rk(cfg, rk, g, t, (uint32_t)k, (uint32_t)w, n_calls)
                                                  : smask_word(cfg, g, t, (uint32_t)k, (uint32_t)w, n_calls)));
                    }
                }
#pragma unroll
                for (int i = 0; i < NB; ++i) state[((int64_t)i * C + c) * W + w] = ctr.p[i];
            }
        }
        block_sync<WPC>();
        YTM_PHASE(5);
    }
    for (int kk = tid; kk < nk; kk += nt) weights[(int64_t)c * K + k0 + kk] = wk[kk];
#ifdef YTM_PHASE_TIMING
    if (counters && tid == 0)
        for (int i = 0; i < 6; ++i) atomicAdd(&counters[6 + i], ph_cyc[i]);
#endif
    if (counters) {
        unsigned long long v[6] = {n_units, n_calls, n_words, n_events, n_dcalls, n_tests};
#pragma unroll
        for (int i = 0; i < 6; ++i) {
            for (int o = 16; o; o >>= 1) v[i] += __shfl_xor_sync(0xFFFFFFFFu, v[i], o);
            if ((tid & 31) == 0 && v[i]) atomicAdd(&counters[i], v[i]);
        }
    }
    if (count_patch) {
        for (int o = 16; o; o >>= 1) fired_count += __shfl_xor_sync(0xFFFFFFFFu, fired_count, o);
        if ((tid & 31) == 0 && fired_count) atomicAdd(&patch_w[c], fired_count);
    }
}

}  // namespace ytm

using namespace ytm;

extern "C" ytm_status ytm_train_update_counted(const ytm_config *cfg, uint32_t *state, int32_t *weights,
                                               const int32_t *cs, const int32_t *Y, const uint32_t *drop,
                                               const uint32_t *lits, int32_t B, uint64_t t0,
                                               const int32_t *sel_override, int32_t *patch_w, void *workspace,
                                               uint64_t *counters, void *stream) {
    unsigned long long *ctrs = reinterpret_cast<unsigned long long *>(counters);
    ytm_status rc = check_cfg(cfg);
    if (rc) return rc;
    if (B <= 0) return fail(YTM_ERR_ARG, "batch must be positive");
    if (!state || !weights || !cs || !Y || !lits || !workspace) return fail(YTM_ERR_ARG, "null pointer");
    const int count_patch = single_patch_eval(cfg) ? 1 : 0;
    if (count_patch && !patch_w) return fail(YTM_ERR_ARG, "patch_w is NULL");
    // active-pair list entries hold sample << 16 | class (and a sign bit above)
    if (cfg->n_classes > 65535 || B > 32767)
        return fail(YTM_ERR_UNSUPPORTED, "feedback handles at most 65,535 classes and 32,767 samples per batch");
    if ((int64_t)B * cfg->n_classes >= (1ll << 32)) return fail(YTM_ERR_UNSUPPORTED, "batch x classes above 2^32");
    cudaStream_t st = as_stream(stream);
    TrainWs l = train_ws_layout(cfg, B);
    char *ws = (char *)workspace;
    const int32_t *sel = sel_override ? sel_override : (const int32_t *)(ws + l.sel);
    // single-patch batches evaluated by ytm_train_eval leave clause-major
    // fired bits, which the feedback reads instead of the [B][C] picks
    const uint32_t *fcm = (!sel_override && count_patch) ? (const uint32_t *)(ws + l.fcm) : nullptr;
    uint64_t *thr = (uint64_t *)(ws + l.thr);
    int32_t *pair = (int32_t *)(ws + l.pair);
    uint32_t *amask = (uint32_t *)(ws + l.amask);
    uint32_t *colm = (uint32_t *)(ws + l.colm);
    int32_t *row_off = (int32_t *)(ws + l.row_off);
    uint64_t *alist = (uint64_t *)(ws + l.alist);
    if (cfg->one_negative) {
        k_pairs<<<(unsigned)cdiv(B, 256), 256, 0, st>>>(cfg->seed, Y, B, cfg->n_classes, t0, pair);
        if ((rc = launch_check("class pairs"))) return rc;
    }
    const int qsel = cfg->coalesced && cfg->q_select && !cfg->one_negative;
    int32_t *npos = (int32_t *)(ws + l.npos);
    k_thresholds<<<1, 1024, 0, st>>>(cs, Y, B, cfg->n_classes, cfg->T, cfg->one_negative, pair, thr, amask, colm,
                                     row_off, alist, qsel, npos);
    if ((rc = launch_check("update thresholds"))) return rc;
    const int nk = cfg->coalesced ? cfg->n_classes : 1;
    // chunks hold whole Type Ib run windows: the whole batch when it is at
    // most one window, else one window (128 samples, or 64 above 256 classes)
    const int win = run_window(*cfg);
    int BC = B <= win ? ((B + 31) / 32) * 32 : win;
    const size_t smem = update_smem_aligned(nk, BC) + run_table_bytes(*cfg);
    if (smem > 227 * 1024) return fail(YTM_ERR_UNSUPPORTED, "too many classes for the feedback kernel");
    // round keys for the batch's samples when they share the counter's high word
    // the literal source of the feedback: the batch's patch literal words;
    // from bit images they are formed once into the workspace when they fit
    LitSrc src = lit_src(cfg, lits);
    if (cfg->input_images) {
        uint32_t *pw = (uint32_t *)(ws + l.pwords);
        const int64_t total = (int64_t)B * cfg->patches * cfg->words;
        k_batch_words<<<(unsigned)std::min<int64_t>(cdiv(total, 256), (int64_t)sm_count() * 16), 256, 0, st>>>(
            src, B, pw);
        if ((rc = launch_check("batch patch words"))) return rc;
        src.p = pw;
        src.img = 0;
    }
    const RoundKeys rk = round_keys(cfg->seed, (uint32_t)(t0 >> 32));
    const int rk_ok = (t0 >> 32) == ((t0 + (uint64_t)B - 1) >> 32);
    const int W = cfg->words;
    // small batches: one warp per clause, 8 clauses per block
    const size_t smem_wpc = 8 * update_smem_aligned(nk, 32) + run_table_bytes(*cfg);
    if (B <= 32 && smem_wpc <= 48 * 1024) {
        YTM_DISPATCH_PLANES(cfg->planes, {
            k_update<NB, true><<<(unsigned)cdiv(cfg->clause_count, 8), 256, smem_wpc, st>>>(
                *cfg, state, weights, thr, drop, src, B, t0, sel, patch_w, 32, rk, rk_ok, count_patch, pair, amask,
                colm, row_off,
                alist, fcm, npos, ctrs);
        });
        return launch_check("feedback");
    }
    const int tpb = W <= 32 ? 32 : (W <= 64 ? 64 : (W <= 128 ? 128 : 256));
    YTM_DISPATCH_PLANES(cfg->planes, {
        if (smem > 48 * 1024) {
            if ((rc = cuda_check(cudaFuncSetAttribute(k_update<NB, false>,
                                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                                 "update smem")))
                return rc;
        }
        k_update<NB, false><<<cfg->clause_count, tpb, smem, st>>>(*cfg, state, weights, thr, drop, src, B,
                                                                  t0, sel,
                                                                  patch_w, BC, rk, rk_ok, count_patch, pair,
                                                                  amask, colm, row_off, alist, fcm, npos, ctrs);
    });
    return launch_check("feedback");
}

extern "C" ytm_status ytm_train_update(const ytm_config *cfg, uint32_t *state, int32_t *weights, const int32_t *cs,
                                       const int32_t *Y, const uint32_t *drop, const uint32_t *lits, int32_t B,
                                       uint64_t t0, const int32_t *sel_override, int32_t *patch_w, void *workspace,
                                       void *stream) {
    return ytm_train_update_counted(cfg, state, weights, cs, Y, drop, lits, B, t0, sel_override, patch_w, workspace,
                                    nullptr, stream);
}
