// common.cuh — shared device code of libytm: error plumbing, Philox4x32-10,
// the decision rules of training, and bit-sliced counter arithmetic.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/ytm.h"

namespace ytm {

// ------------------------------------------------------------------ errors

void set_error(const std::string &msg);
ytm_status fail(ytm_status code, const std::string &msg);
ytm_status cuda_check(cudaError_t e, const char *what);
// Checks the launch that was just issued.
ytm_status launch_check(const char *what);

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

inline uint64_t cdiv(uint64_t a, uint64_t b) { return (a + b - 1) / b; }
inline uint64_t align_up(uint64_t a, uint64_t b) { return cdiv(a, b) * b; }

int sm_count();

// ------------------------------------------------------------ Philox4x32-10
// Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3",
// SC'11.  Round: (c0,c1,c2,c3) -> (hi(M1*c2)^c1^k0, lo(M1*c2), hi(M0*c0)^c3^k1,
// lo(M0*c0)) with M0 = 0xD2511F53, M1 = 0xCD9E8D57; Weyl key schedule.

struct u32x4 {
    uint32_t x, y, z, w;
};

template <int R>
__device__ __forceinline__ u32x4 philox(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0,
                                        uint32_t k1) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
        if (r) {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
        uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
        uint32_t n0 = hi1 ^ c1 ^ k0;
        uint32_t n2 = hi0 ^ c3 ^ k1;
        c0 = n0;
        c1 = lo1;
        c2 = n2;
        c3 = lo0;
    }
    return {c0, c1, c2, c3};
}

// Decision streams.  counter = (global clause, sample counter low word,
// sub-index, tag | class << 2); key = (seed low, seed high ^ sample high).
enum : uint32_t { TAG_PATCH = 0, TAG_CLASS = 1, TAG_SMASK = 2, TAG_INIT = 3 };

// Decision draws use Philox4x32-10; the bulk literal-mask draws use the
// 7-round variant, which Salmon et al. report as passing BigCrush.
template <int R = 10>
__device__ __forceinline__ u32x4 draw(uint64_t seed, uint32_t clause, uint64_t t, uint32_t sub, uint32_t tag,
                                      uint32_t k) {
    return philox<R>(clause, (uint32_t)t, sub, tag | (k << 2), (uint32_t)seed,
                     (uint32_t)(seed >> 32) ^ (uint32_t)(t >> 32));
}

// Round keys of one (seed, sample-counter high word): the Weyl schedule
// k_r = k_0 + r * constant, computed once on the host and passed as a kernel
// parameter, so the rounds read their keys from the constant bank.
struct RoundKeys {
    uint32_t a[10], b[10];
};

inline RoundKeys round_keys(uint64_t seed, uint32_t t_hi) {
    RoundKeys k;
    uint32_t a = (uint32_t)seed, b = (uint32_t)(seed >> 32) ^ t_hi;
    for (int r = 0; r < 10; ++r) {
        k.a[r] = a;
        k.b[r] = b;
        a += 0x9E3779B9u;
        b += 0xBB67AE85u;
    }
    return k;
}

template <int R>
__device__ __forceinline__ u32x4 philox_rk(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3,
                                           const RoundKeys &rk) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
        uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
        uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
        uint32_t n0 = hi1 ^ c1 ^ rk.a[r];
        uint32_t n2 = hi0 ^ c3 ^ rk.b[r];
        c0 = n0;
        c1 = lo1;
        c2 = n2;
        c3 = lo0;
    }
    return {c0, c1, c2, c3};
}

// draw() with precomputed round keys (valid for samples t whose high word is
// the one the keys were made for).
template <int R = 10>
__device__ __forceinline__ u32x4 draw_rk(const RoundKeys &rk, uint32_t clause, uint64_t t, uint32_t sub,
                                         uint32_t tag, uint32_t k) {
    return philox_rk<R>(clause, (uint32_t)t, sub, tag | (k << 2), rk);
}

// Bernoulli(thr/4096) bits for the 32 literals of word w of clause g in the
// feedback for class k of sample t: literal j is set iff the 12-bit number
// whose bit 11-i is bit j of random word i is below thr; three Philox4x32-7
// draws give the 12 words.  (Stands in for the reference's per-literal
// `curand_uniform(rng) <= S_INV`.)  Only the literals in `cand` are wanted:
// the comparison runs most significant bit first, so once every candidate
// literal is decided the remaining draws cannot change the result and are
// skipped.  Returns the bits within cand.
// One Philox draw j of the comparison: planes 11-4j .. 8-4j of the 12-bit
// values against the same bits of thr (branch-free: thr is uniform).
__device__ __forceinline__ void smask_planes(uint32_t thr, int j, const u32x4 &r, uint32_t &lt, uint32_t &eq) {
    const uint32_t R[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t tb = 0u - ((thr >> (11 - (4 * j + i))) & 1u);
        lt |= eq & ~R[i] & tb;
        eq &= ~(R[i] ^ tb);
    }
}

template <typename DrawFn>
__device__ __forceinline__ uint32_t smask_compare(uint32_t thr, uint32_t cand, DrawFn drawj) {
    if (thr >= 4096u) return cand;
    if (thr == 0u) return 0u;
    uint32_t lt = 0u, eq = cand;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        if (eq == 0u) break;
        smask_planes(thr, j, drawj((uint32_t)j), lt, eq);
    }
    return lt;
}

__device__ __forceinline__ uint32_t smask_word(uint64_t seed, uint32_t thr, uint32_t cand, uint32_t g, uint64_t t,
                                               uint32_t k, uint32_t w) {
    return smask_compare(thr, cand, [&](uint32_t j) { return draw<7>(seed, g, t, w * 4u + j, TAG_SMASK, k); });
}

// smask_word with precomputed round keys.
__device__ __forceinline__ uint32_t smask_word_rk(const RoundKeys &rk, uint32_t thr, uint32_t cand, uint32_t g,
                                                  uint64_t t, uint32_t k, uint32_t w) {
    return smask_compare(thr, cand, [&](uint32_t j) { return draw_rk<7>(rk, g, t, w * 4u + j, TAG_SMASK, k); });
}

// pytm's per-sample pick (pytm/base.py:139-141): the true class (the first
// with a positive target, -1 if none) and one other class drawn uniformly
// among the rest from the counter (clause 0xFFFFFFFF, t, 1, CLASS).
__device__ __forceinline__ void true_other_pair(uint64_t seed, const int32_t *Yrow, int K, uint64_t t, int *kt,
                                                int *ko) {
    int y = -1;
    for (int k = 0; k < K; ++k)
        if (Yrow[k] > 0) { y = k; break; }
    const uint32_t r = draw(seed, 0xFFFFFFFFu, t, 1, TAG_CLASS, 0).x;
    if (y < 0) {
        *ko = (int)(((uint64_t)r * (uint64_t)K) >> 32);
    } else {
        const int idx = K > 1 ? (int)(((uint64_t)r * (uint64_t)(K - 1)) >> 32) : 0;
        *ko = K > 1 ? (idx < y ? idx : idx + 1) : -1;
    }
    *kt = y;
}

// floor(p * 2^32) for the update probability p = (y - v) / (2y)
// (reference update_probability, kernel.cu:508-529).  IEEE double division is
// correctly rounded on host and device alike.
__host__ __device__ __forceinline__ uint64_t update_threshold(int32_t y, int32_t v) {
    double p = ((double)y - (double)v) / (2.0 * (double)y);
    if (!(p > 0.0)) return 0ull;
    if (p >= 1.0) return 4294967296ull;
    return (uint64_t)floor(p * 4294967296.0);
}

// ------------------------------------------------- bit-sliced TA counters
// NB planes hold (state + offset) for 32 literals; plane NB-1 is the include
// mask.  All operations act on the literals selected by a 32-bit mask.

template <int NB>
struct Counter {
    uint32_t p[NB];

    __device__ __forceinline__ void inc(uint32_t m) {  // ripple-carry +1
#pragma unroll
        for (int i = 0; i < NB; ++i) {
            uint32_t c = p[i] & m;
            p[i] ^= m;
            m = c;
        }
    }
    __device__ __forceinline__ void dec(uint32_t m) {  // ripple-borrow -1
#pragma unroll
        for (int i = 0; i < NB; ++i) {
            uint32_t b = ~p[i] & m;
            p[i] ^= m;
            m = b;
        }
    }
    // literals whose stored value != v
    __device__ __forceinline__ uint32_t ne(uint32_t v) const {
        uint32_t d = 0u;
#pragma unroll
        for (int i = 0; i < NB; ++i) d |= p[i] ^ (((v >> i) & 1u) ? 0xFFFFFFFFu : 0u);
        return d;
    }
    // literals whose stored value < v (MSB-first comparator)
    __device__ __forceinline__ uint32_t lt(uint32_t v) const {
        uint32_t l = 0u, e = 0xFFFFFFFFu;
#pragma unroll
        for (int i = NB - 1; i >= 0; --i) {
            if ((v >> i) & 1u) {
                l |= e & ~p[i];
                e &= p[i];
            } else {
                e &= ~p[i];
            }
        }
        return l;
    }
    // literals whose stored value is not all ones (below the top)
    // literals whose stored value is not v (= the stored zero state, offset):
    // when offset + 1 == 2^(NB-2) (state counts that are powers of two, e.g.
    // 256 on 9 planes) a stored value is above the offset exactly when one of
    // the two top planes is set
    __device__ __forceinline__ uint32_t nonzero(uint32_t v, bool top2) const {
        if (NB >= 2 && top2) return p[NB - 1] | p[NB - 2];
        return ne(v);
    }
    __device__ __forceinline__ uint32_t below_top() const {
        uint32_t a = 0xFFFFFFFFu;
#pragma unroll
        for (int i = 0; i < NB; ++i) a &= p[i];
        return ~a;
    }
};

// Mask of the literal bits of word w that are real literals (< L).
__host__ __device__ __forceinline__ uint32_t valid_mask(int w, int W, int L) {
    if (w < W - 1) return 0xFFFFFFFFu;
    int r = L & 31;
    return r ? ((1u << r) - 1u) : 0xFFFFFFFFu;
}

// Dispatch a templated launcher on the plane count.
#define YTM_DISPATCH_PLANES(NBVAR, ...)                      \
    switch (NBVAR) {                                         \
        case 2: { constexpr int NB = 2; __VA_ARGS__; } break;   \
        case 3: { constexpr int NB = 3; __VA_ARGS__; } break;   \
        case 4: { constexpr int NB = 4; __VA_ARGS__; } break;   \
        case 5: { constexpr int NB = 5; __VA_ARGS__; } break;   \
        case 6: { constexpr int NB = 6; __VA_ARGS__; } break;   \
        case 7: { constexpr int NB = 7; __VA_ARGS__; } break;   \
        case 8: { constexpr int NB = 8; __VA_ARGS__; } break;   \
        case 9: { constexpr int NB = 9; __VA_ARGS__; } break;   \
        case 10: { constexpr int NB = 10; __VA_ARGS__; } break; \
        case 11: { constexpr int NB = 11; __VA_ARGS__; } break; \
        case 12: { constexpr int NB = 12; __VA_ARGS__; } break; \
        case 13: { constexpr int NB = 13; __VA_ARGS__; } break; \
        case 14: { constexpr int NB = 14; __VA_ARGS__; } break; \
        case 15: { constexpr int NB = 15; __VA_ARGS__; } break; \
        case 16: { constexpr int NB = 16; __VA_ARGS__; } break; \
        default: return fail(YTM_ERR_UNSUPPORTED, "number_of_ta_states needs more than 16 bit planes"); \
    }

// Single-patch models with up to 256 classes evaluate training batches in one
// fused kernel that leaves patch counting to the feedback kernel.
inline bool single_patch_eval(const ytm_config *cfg) { return cfg->patches == 1 && cfg->n_classes <= 256; }

// Validates the pieces of a config every entry point relies on.
ytm_status check_cfg(const ytm_config *cfg);

// Workspace carve-up (offsets in bytes, 256-aligned).
struct TrainWs {
    uint64_t ninc, mbits, sel, fired, fcm, thr, amask, colm, row_off, alist, pair, sparse, total;
};
TrainWs train_ws_layout(const ytm_config *cfg, int64_t B);
struct InferWs {
    uint64_t ninc, fired, total;
};
InferWs infer_ws_layout(const ytm_config *cfg, int64_t N);
struct B1Ws {
    uint64_t cs, fired, ninc, total;
};
B1Ws b1_ws_layout(const ytm_config *cfg);
uint64_t cs_planes_bytes(const ytm_config *cfg);  // class-sum weight planes scratch (eval.cu)
uint64_t sparse_ws_bytes(const ytm_config *cfg);  // sparse patch-match scratch (eval.cu)

// Peer all-reduce (peer.cu), used by the training loop.
extern "C" ytm_status ytm_peer_allreduce_i32(void *ctx, int32_t *data, int64_t n, int64_t limit, void *stream);

// Shared launchers (eval.cu) used by several entry points.
ytm_status launch_ninc(const ytm_config *cfg, const uint32_t *state, int32_t *ninc, cudaStream_t st);

}  // namespace ytm
