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

// The patch pick and pytm's other-class draw use Philox4x32-10; the
// per-class decision draws and the bulk literal-mask draws use the 7-round
// variant, which Salmon et al. report as passing BigCrush.
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

// Bernoulli(1/s) bits for the 32 literals of word w of clause g in the
// feedback for class k of sample t (stands in for the reference's per-literal
// `curand_uniform(rng) <= S_INV`, kernel.cu:425-428, 457-460), by count and
// placement, so that a word costs one Philox4x32-7 call in all but rare
// cases: the first random word r0 of counter sub-index 4w gives the number n
// of set literals, the smallest n with r0 < cdf[n] (32 if none), which is
// Binomial(32, 1/s); then n distinct positions (when n > 16: the 32 - n unset
// ones) are drawn uniformly by rejection from 5-bit fields (bits 0-4, ...,
// 25-29) of r1, r2, r3 and, if those run out, of all four words of further
// calls at sub-indices 4w+1, 4w+2, ...  Given n every n-subset is equally
// likely, so the 32 bits are independent Bernoulli(1/s) (to the table's 2^-32
// resolution).  `calls` is increased by the number of Philox calls made.
// The count scan's index is the same in every lane still scanning, so the
// table reads are uniform (kernel-parameter space).
// The count and the first six placements run branch-free (the same
// sequential rejection, unrolled), so that the lanes of a warp stay together;
// only counts of 8 or more and words whose first six fields did not finish
// the placement continue in the loops.
template <typename DrawFn>
__device__ __forceinline__ uint32_t smask_place(const ytm_config &cfg, DrawFn drawj, uint32_t &calls) {
    u32x4 r = drawj(0u);
    uint32_t n = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) n += r.x >= cfg.s_count_cdf[j] ? 1u : 0u;
    if (n == 8u)
        while (n < 32u && r.x >= cfg.s_count_cdf[n]) ++n;
    const bool holes = n > 16u;
    uint32_t need = holes ? 32u - n : n, m = 0u;
    ++calls;
#pragma unroll
    for (int f = 0; f < 6; ++f) {  // fields 0-5: bits 0-29 of r.y
        const uint32_t b = 1u << ((r.y >> (5 * f)) & 31u);
        const bool take = need != 0u && !(m & b);
        m |= take ? b : 0u;
        need -= take ? 1u : 0u;
    }
    uint32_t cur = r.z, sub = 0;
    int wi = 2, left = 6;
    // large 1/s (counts above 6 common: P(count <= 6) < 0.9, a uniform test):
    // fields 6-11 (r.z) branch-free as well
    if (cfg.s_count_cdf[6] < 0xE6666666u) {
#pragma unroll
        for (int f = 0; f < 6; ++f) {
            const uint32_t b = 1u << ((r.z >> (5 * f)) & 31u);
            const bool take = need != 0u && !(m & b);
            m |= take ? b : 0u;
            need -= take ? 1u : 0u;
        }
        cur = r.w;
        wi = 3;
    }
    while (need) {
        if (left == 0) {
            if (++wi == 4) {
                r = drawj(++sub);
                ++calls;
                wi = 0;
            }
            cur = wi == 0 ? r.x : (wi == 1 ? r.y : (wi == 2 ? r.z : r.w));
            left = 6;
        }
        const uint32_t b = 1u << (cur & 31u);
        cur >>= 5;
        --left;
        if (!(m & b)) {
            m |= b;
            --need;
        }
    }
    return holes ? ~m : m;
}

__device__ __forceinline__ uint32_t smask_word(const ytm_config &cfg, uint32_t g, uint64_t t, uint32_t k, uint32_t w,
                                               uint32_t &calls) {
    return smask_place(cfg, [&](uint32_t j) { return draw<7>(cfg.seed, g, t, w * 4u + j, TAG_SMASK, k); }, calls);
}

// smask_word with precomputed round keys.
__device__ __forceinline__ uint32_t smask_word_rk(const ytm_config &cfg, const RoundKeys &rk, uint32_t g, uint64_t t,
                                                  uint32_t k, uint32_t w, uint32_t &calls) {
    return smask_place(cfg, [&](uint32_t j) { return draw_rk<7>(rk, g, t, w * 4u + j, TAG_SMASK, k); }, calls);
}

// A run of m = 8 (mi + 1) (8 to 64) consecutive Type Ib events of one clause (type1b_fb,
// kernel.cu:453-470, applied by the reference one event at a time: each
// decrements every literal with a positive state with probability 1/s).
// Decrements with a floor at 0 commute, so the run leaves state - d clamped
// at 0, with d the literal's number of successes, Binomial(m, 1/s), drawn by
// inverse CDF from a 16-bit uniform: d = #{e : u >= run_cdf16[mi][e]}.  The
// uniforms of the 32 literals of word w come as bit planes: plane b (bit b of
// every literal's uniform, literal j at bit j) is word b & 3 of the
// Philox4x32-7 call b >> 2 at sub-index 0x40000000 | 4w | (b >> 2), keyed on
// the run's first event.  So all 32 comparisons with one threshold c are one
// bit-sliced carry chain: u >= c exactly when u + (65536 - c) carries out of
// bit 15, and the carry through plane b is the majority of the plane, bit b
// of the constant and the incoming carry (one LOP3 per plane).  The masks
// "d >= j" are nested, so bit b of d is the parity of the masks of the j
// divisible by 2^b; D receives the counts as bit planes (d <= 64 needs 7).
// Thresholds outside run_range (0: certain, 65536: never) are not tested,
// and the chain stops once no literal of the thread reaches the next one.
__device__ __forceinline__ uint32_t maj3(uint32_t a, uint32_t b, uint32_t c) {
    return (a & b) | (c & (a | b));
}

// The thresholds' plane masks (16 per threshold: all ones where the constant
// 65536 - c has a one) for every run size, in shared memory: the table of run
// size mi starts at threshold run_table_base(cfg, mi); a kernel that keeps it
// saves the 32 instructions per threshold that forming the masks takes.
__host__ __device__ inline int run_table_base(const ytm_config &cfg, int mi) {
    int n = 0;
    for (int i = 0; i < mi; ++i) n += (int)(cfg.run_range[i] >> 16) - (int)(cfg.run_range[i] & 0xFFFFu);
    return n;
}
__host__ __device__ inline size_t run_table_bytes(const ytm_config &cfg) { return (size_t)run_table_base(cfg, 8) * 64; }
__device__ inline void run_table_fill(const ytm_config &cfg, uint4 *tab, int tid, int nt) {
    const int n = run_table_base(cfg, 8);
    for (int i = tid; i < n * 4; i += nt) {
        int e = i >> 2, mi = 0;
        for (; mi < 7; ++mi) {
            const int len = (int)(cfg.run_range[mi] >> 16) - (int)(cfg.run_range[mi] & 0xFFFFu);
            if (e < len) break;
            e -= len;
        }
        const int j = (int)(cfg.run_range[mi] & 0xFFFFu) + 1 + e;
        const uint32_t k = 65536u - cfg.run_cdf16[mi][j - 1], q = (uint32_t)(i & 3) * 4u;
        tab[i] = make_uint4(0u - ((k >> q) & 1u), 0u - ((k >> (q + 1)) & 1u), 0u - ((k >> (q + 2)) & 1u),
                            0u - ((k >> (q + 3)) & 1u));
    }
}

// km: the plane masks of run size mi (run_table_fill's table at
// run_table_base(cfg, mi)), or nullptr to form them in registers.
template <typename DrawFn>
__device__ __forceinline__ void run_counts(const ytm_config &cfg, int mi, DrawFn drawi, uint32_t (&D)[7],
                                           uint32_t &calls, uint32_t &tests, const uint4 *km) {
    uint32_t R[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const u32x4 r = drawi((uint32_t)i);
        R[4 * i] = r.x;
        R[4 * i + 1] = r.y;
        R[4 * i + 2] = r.z;
        R[4 * i + 3] = r.w;
    }
    calls += 4u;
    const uint32_t rr = cfg.run_range[mi];
    const int lo = (int)(rr & 0xFFFFu), hi = (int)(rr >> 16);
#pragma unroll
    for (int b = 0; b < 7; ++b) D[b] = ((lo >> b) & 1) ? 0xFFFFFFFFu : 0u;  // d >= lo for every literal
#pragma unroll 1
    for (int j = lo + 1; j <= hi; ++j) {
        uint32_t cy = 0u;
        if (km) {
            const uint4 *m = km + (j - lo - 1) * 4;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint4 mm = m[q];
                cy = maj3(R[4 * q], mm.x, cy);
                cy = maj3(R[4 * q + 1], mm.y, cy);
                cy = maj3(R[4 * q + 2], mm.z, cy);
                cy = maj3(R[4 * q + 3], mm.w, cy);
            }
        } else {
            const uint32_t k = 65536u - cfg.run_cdf16[mi][j - 1];
#pragma unroll
            for (int b = 0; b < 16; ++b) cy = maj3(R[b], 0u - ((k >> b) & 1u), cy);
        }
        ++tests;
        if (!cy) break;  // d < j for all 32 literals, and the masks are nested
        const int tz = __ffs(j) - 1;
#pragma unroll
        for (int b = 0; b < 7; ++b)
            if (b <= tz) D[b] ^= cy;
    }
}

// The decision draws of class k for clause g at sample t: the Philox4x32-7
// call of the class pair k >> 1 (counter sub-index 0, tag CLASS) gives words
// (x, y) to the even class and (z, w) to the odd one; the first is the
// negative-class selection uniform (kernel.cu:573), the second the update
// uniform (kernel.cu:582).  Two classes share one call.
__device__ __forceinline__ uint2 class_words(const u32x4 &r, uint32_t k) {
    return (k & 1u) ? make_uint2(r.z, r.w) : make_uint2(r.x, r.y);
}
__device__ __forceinline__ u32x4 class_pair_draw_rk(const RoundKeys &rk, uint32_t g, uint64_t t, uint32_t k) {
    return draw_rk<7>(rk, g, t, 0, TAG_CLASS, k >> 1);
}
__device__ __forceinline__ u32x4 class_pair_draw(uint64_t seed, uint32_t g, uint64_t t, uint32_t k) {
    return draw<7>(seed, g, t, 0, TAG_CLASS, k >> 1);
}

// The negative-class selection (kernel.cu:573: each class with target -1
// takes part with probability Q) drawn as a set for clause g at sample t when
// cfg.q_select: the Philox4x32-7 call at sub-index 2 (class field 0) gives in
// word 0 the count n of selected classes among all K, the smallest n with
// r0 < q_count_cdf[n] (min(K, 32) if none), i.e. Binomial(K, Q); then n distinct
// classes by rejection from b-bit fields (b = bits of K - 1, floor(32 / b)
// fields per word from bit 0) of words 1-3 and of all words of further calls
// at sub-indices 3, 4, ...: a value >= K or already drawn is skipped.  take(v)
// records class v and returns false when it was drawn before.
template <typename DrawFn, typename TakeFn>
__device__ __forceinline__ void qselect(const ytm_config &cfg, DrawFn drawsub, TakeFn take) {
    const int K = cfg.n_classes;
    uint32_t sub = 2;
    u32x4 r = drawsub(sub);
    // at most min(K, 32) classes: the saturated table entries would otherwise
    // let a word of all ones ask for more distinct classes than exist
    const uint32_t nmax = K < 32 ? (uint32_t)K : 32u;
    uint32_t n = 0;
    while (n < nmax && r.x >= cfg.q_count_cdf[n]) ++n;
    if (!n) return;
    const int b = 32 - __clz(K - 1);  // K >= 32
    const int per = 32 / b;
    const uint32_t fm = (1u << b) - 1u;
    int wi = 1, f = 0;
    uint32_t cur = r.y;
    while (n) {
        if (f == per) {
            f = 0;
            if (++wi == 4) {
                r = drawsub(++sub);
                wi = 0;
            }
            cur = wi == 0 ? r.x : (wi == 1 ? r.y : (wi == 2 ? r.z : r.w));
        }
        const uint32_t v = (cur >> (b * f)) & fm;
        ++f;
        if ((int)v < K && take((int)v)) --n;
    }
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
    // lt(v) for v = 2^(NB-1) + 2^(NB-2) - 1, the stored maximum state when
    // the state count is a power of two (offset + 1 = 2^(NB-2)): a value is
    // >= v iff its top plane is set and either the next plane or all lower
    // planes are
    __device__ __forceinline__ uint32_t lt_max_pow2() const {
        uint32_t low = 0xFFFFFFFFu;
#pragma unroll
        for (int i = 0; i + 2 < NB; ++i) low &= p[i];
        return ~(p[NB - 1] & (p[NB - 2] | low));
    }
    // lt(max_s) with the shortcut above when it applies (pow2 is uniform)
    __device__ __forceinline__ uint32_t lt_max(uint32_t max_s, bool pow2) const {
        if (NB >= 3 && pow2) return lt_max_pow2();
        return lt(max_s);
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
    // stored value := max(z, value - D) for the literals of D (bit planes,
    // seven of them): a run of Type Ib decrements with the floor at state 0
    // (stored value z = offset).  top2: z + 1 = 2^(NB-2), so a value is at
    // most z exactly when its two top planes are clear.
    __device__ __forceinline__ void sub_floor(const uint32_t (&D)[7], uint32_t z, bool top2) {
        uint32_t q[NB], br = 0u;
#pragma unroll
        for (int i = 0; i < NB; ++i) {
            const uint32_t d = i < 7 ? D[i] : 0u;
            q[i] = p[i] ^ d ^ br;
            br = (~p[i] & (d | br)) | (d & br);
        }
        uint32_t low;  // literals whose difference is below z + 1 (or negative)
        if (NB >= 3 && top2) {
            low = ~(q[NB - 1] | q[NB - 2]);
        } else {
            uint32_t l = 0u, e = 0xFFFFFFFFu;
            const uint32_t v = z + 1u;
#pragma unroll
            for (int i = NB - 1; i >= 0; --i) {
                if ((v >> i) & 1u) {
                    l |= e & ~q[i];
                    e &= q[i];
                } else {
                    e &= ~q[i];
                }
            }
            low = l;
        }
        low |= br;
#pragma unroll
        for (int i = 0; i < NB; ++i) p[i] = (q[i] & ~low) | (((z >> i) & 1u) ? low : 0u);
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

// ------------------------------------------- patch literals from bit images
// With cfg->input_images set, the `lits` arguments of the data path hold one
// packed bit image per sample, u32 [N][image_words] (bit j = input j of the
// D0*D1*D2 inputs, any nonzero value a 1; one zero word of padding at the
// end), and the literal words of a patch are formed where they are used,
// exactly as encode_batch (kernel.cu:76-152) lays them out: for patch (py, px)
// bits [0, py) and [D1-P1, D1-P1+px) are the location thermometers (set even
// without encode_loc, as the reference does), bit loc + ry*P0*D2 + rx*D2 + z
// is pixel (py+ry, px+rx, z), and bit L/2 + j is NOT literal j.
struct PatchGeom {
    int D2, dx, seg, loc, npix, Lh, thx, W, L, neg;
    int64_t rowbits;
    __host__ __device__ explicit PatchGeom(const ytm_config &c)
        : D2(c.dim2), dx(c.dim0 - c.patch_dim0 + 1), seg(c.patch_dim0 * c.dim2),
          loc(c.encode_loc ? c.loc_literals : 0), npix(c.patch_dim0 * c.patch_dim1 * c.dim2), Lh(c.half_literals),
          thx(c.dim1 - c.patch_dim1), W(c.words), L(c.literals), neg(c.append_negated),
          rowbits((int64_t)c.dim0 * c.dim2) {}
};

// nbits (1..32) bits of a packed image starting at bit q (the image's padding
// word keeps the second read inside it).
__device__ __forceinline__ uint32_t img_bits(const uint32_t *__restrict__ img, int64_t q, int nbits) {
    const uint32_t lo = img[q >> 5], hi = img[(q >> 5) + 1];
    const uint32_t v = __funnelshift_r(lo, hi, (uint32_t)(q & 31));
    return nbits >= 32 ? v : (v & ((1u << nbits) - 1u));
}

// Bits [a, a+32) of patch (py, px)'s positive literal vector (zero outside
// [0, L/2)); a may be negative.
__device__ __forceinline__ uint32_t pos_window(const uint32_t *__restrict__ img, const PatchGeom &g, int py, int px,
                                               int a) {
    if (a <= -32 || a >= g.Lh) return 0u;
    uint32_t v = 0u;
    // location thermometers
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int s0 = r ? g.thx : 0, s1 = r ? g.thx + px : py;
        const int l0 = max(s0, a), l1 = min(s1, a + 32);
        if (l0 < l1) {
            const int n = l1 - l0;
            v |= (n >= 32 ? 0xFFFFFFFFu : ((1u << n) - 1u)) << (l0 - a);
        }
    }
    // pixels: segments of one patch row (P0 * D2 bits) each
    int lo = max(a, g.loc);
    const int hi = min(a + 32, g.loc + g.npix);
    if (lo < hi) {
        const int rel = lo - g.loc;
        int ry = rel / g.seg, o = rel - ry * g.seg;
        int64_t q = (int64_t)(py + ry) * g.rowbits + (int64_t)px * g.D2 + o;
        while (lo < hi) {
            const int n = min(hi - lo, g.seg - o);
            v |= img_bits(img, q, n) << (lo - a);
            lo += n;
            q += g.rowbits - o;  // next patch row, from its first bit
            o = 0;
        }
    }
    const int keep = g.Lh - a;
    return keep >= 32 ? v : (v & ((1u << keep) - 1u));
}

// Literal word w of patch `patch` of the sample whose bit image is img.
__device__ __forceinline__ uint32_t patch_word(const uint32_t *__restrict__ img, const PatchGeom &g, int patch,
                                               int w) {
    const int py = patch / g.dx, px = patch - py * g.dx;
    const int a = w * 32;
    uint32_t v = pos_window(img, g, py, px, a);
    const int rem = g.L - a;
    const uint32_t vm = rem >= 32 ? 0xFFFFFFFFu : ((1u << rem) - 1u);
    if (g.neg && a + 32 > g.Lh) {
        const int k = g.Lh - a;  // bits of this word in the positive half
        const uint32_t mpos = k >= 32 ? 0xFFFFFFFFu : (k <= 0 ? 0u : ((1u << k) - 1u));
        v = (v & mpos) | (~pos_window(img, g, py, px, a - g.Lh) & ~mpos & vm);
    } else {
        v &= vm;
    }
    return v;
}

// The literal input of a data-path call: per-patch literal words
// u32 [N][P][W], or packed bit images u32 [N][iws] (cfg->input_images).
struct LitSrc {
    const uint32_t *p;
    PatchGeom g;
    int P, img;
    int64_t iws;
    // literal word w of patch `patch` of sample n; kernels instantiate IMG =
    // img so that the per-patch-word instantiation carries no image code
    // (its register count would otherwise grow)
    template <bool IMG>
    __device__ __forceinline__ uint32_t word(int64_t n, int patch, int w) const {
        if (IMG) return patch_word(p + n * iws, g, patch, w);
        return __ldg(&p[(n * P + patch) * (int64_t)g.W + w]);
    }
    // the same source starting at sample n0
    __host__ __device__ LitSrc from(int64_t n0) const {
        LitSrc s = *this;
        s.p += n0 * (img ? iws : (int64_t)P * g.W);
        return s;
    }
};

__host__ __device__ inline LitSrc lit_src_dev(const ytm_config &cfg, const uint32_t *lits) {
    LitSrc s{lits, PatchGeom(cfg), cfg.patches, cfg.input_images ? 1 : 0, cfg.image_words};
    return s;
}
inline LitSrc lit_src(const ytm_config *cfg, const uint32_t *lits) { return lit_src_dev(*cfg, lits); }

// Type Ib runs are taken inside windows of this many samples of the batch
// (batch-relative): 128, or 64 when a clause sees more than 256 classes (the
// feedback kernel's event list of 128 samples would then not fit shared memory)
__host__ __device__ inline int run_window(const ytm_config &c) {
    return (c.coalesced ? c.n_classes : 1) <= 256 ? 128 : 64;
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
    uint64_t ninc, mbits, sel, fired, fcm, thr, amask, colm, row_off, npos, alist, pair, sparse, pwords, total;
};
TrainWs train_ws_layout(const ytm_config *cfg, int64_t B);
// Bit-image input: the feedback reads the batch's patch literal words from a
// transient [B][P][W] buffer in the training workspace, formed from the
// images by one kernel per batch (the per-sample arrays of the batch, such
// as the patch match bits [B][C][P/32], are larger still).
inline uint64_t batch_words_bytes(const ytm_config *cfg, int64_t B) {
    return cfg->input_images ? (uint64_t)B * cfg->patches * cfg->words * 4 : 0;
}
struct InferWs {
    uint64_t ninc, fired, total;
};
InferWs infer_ws_layout(const ytm_config *cfg, int64_t N);
struct B1Ws {
    uint64_t cs, fired, ninc, ring, total;
};
B1Ws b1_ws_layout(const ytm_config *cfg);
uint64_t cs_planes_bytes(const ytm_config *cfg);  // class-sum weight planes scratch (eval.cu)
uint64_t sparse_ws_bytes(const ytm_config *cfg);  // sparse patch-match scratch (eval.cu)

// Peer all-reduce (peer.cu), used by the training loop.
extern "C" ytm_status ytm_peer_allreduce_i32(void *ctx, int32_t *data, int64_t n, int64_t limit, void *stream);

// Shared launchers (eval.cu) used by several entry points.
ytm_status launch_ninc(const ytm_config *cfg, const uint32_t *state, int32_t *ninc, cudaStream_t st);

}  // namespace ytm
