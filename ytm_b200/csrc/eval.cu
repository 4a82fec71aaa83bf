// eval.cu — clause evaluation: inference class sums, transforms, and the
// evaluation half of a training batch.
//
// A clause matches a patch iff no included literal is 0 in it:
//     OR_w (inc[c][w] & ~x[row][w]) == 0          (one LOP3 per word test)
// which is the reference's clause_match (kernel.cu:207-216): its FILTER mask of
// the last word is implied because include bits beyond L are never set.
//
// The match kernel treats (sample, patch) rows x clauses like a GEMM tile:
// 64 rows x 64 clauses per CTA, 32-word K-chunks staged in shared memory, 4x4
// (row, clause) pairs per thread held in registers.  Its epilogue writes one of
// three outputs: any-patch fired bits, per-patch match bits, or u32 per
// (sample, clause, patch).  Class sums are then a sparse sum of weight rows
// over the fired bits (int32 atomics: exact and order independent).
#include "common.cuh"

namespace ytm {

__global__ void k_ninc(int C, int W, const uint32_t *__restrict__ inc, int32_t *__restrict__ ninc,
                       uint32_t *__restrict__ inc_out);

enum { MODE_ANY = 0, MODE_PBITS = 1, MODE_PATCHWISE = 2 };

constexpr int RT = 64, CT = 64, KW = 32, XS = RT + 4;

// Violations v[i][j] = OR_w (inc & ~x) of the 4 rows x 4 clauses a thread
// owns in the 64 x 64 tile at (row0, c0); 32-word chunks staged in shared
// memory, no work on words past W.
template <bool IMG>
__device__ __forceinline__ int tile_violations(const uint32_t *__restrict__ inc, const LitSrc &src,
                                                int64_t R, int C, int W, int64_t row0, int c0,
                                                uint32_t (*xs)[XS], uint32_t (*is)[XS], uint32_t (&v)[4][4]) {
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    // out-of-range pairs start violated (callers bounds-check before reading
    // v), so that the exit test below is the minimum of the 16 words
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) v[i][j] = (row0 + ty * 4 + i < R && c0 + tx * 4 + j < C) ? 0u : 0xFFFFFFFFu;
    int nch = 0;
    for (int w0 = 0; w0 < W; w0 += KW) {
        const int kwn = min(KW, W - w0);  // no work on words past W
#pragma unroll
        for (int q = 0; q < (RT * KW) / 256; ++q) {
            int idx = tid + q * 256;
            int r = idx / KW, kw = idx % KW;
            int w = w0 + kw;
            int64_t row = row0 + r;
            int c = c0 + r;
            uint32_t x = 0xFFFFFFFFu;
            if (row < R && w < W) {
                if (IMG) {  // row = sample * P + patch
                    const int64_t n = row / src.P;
                    x = src.word<true>(n, (int)(row - n * src.P), w);
                } else {
                    x = __ldg(&src.p[row * W + w]);
                }
            }
            xs[kw][r] = x;
            is[kw][r] = (c < C && w < W) ? __ldg(&inc[(int64_t)c * W + w]) : 0u;
        }
        __syncthreads();
#pragma unroll 8
        for (int kw = 0; kw < kwn; ++kw) {
            uint4 xv = *reinterpret_cast<const uint4 *>(&xs[kw][ty * 4]);
            uint4 iv = *reinterpret_cast<const uint4 *>(&is[kw][tx * 4]);
            uint32_t xa[4] = {xv.x, xv.y, xv.z, xv.w};
            uint32_t ia[4] = {iv.x, iv.y, iv.z, iv.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) v[i][j] |= ia[j] & ~xa[i];
        }
        // early exit: once every in-range (row, clause) pair of the tile has a
        // violation, the remaining words cannot make any of them match (only
        // v == 0 is read by the callers)
        uint32_t m = v[0][0];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) m = min(m, v[i][j]);
        ++nch;
        if (!__syncthreads_or((int)(m == 0u))) break;
    }
    return nch;
}

// Executed work of the inference / transform match: [0] tiles, [1] 32-word
// chunks those tiles processed (read and cleared by ytm_match_counters).
static __device__ unsigned long long g_match_counts[2];

template <int MODE, bool IMG>
__global__ void __launch_bounds__(256) k_match(const uint32_t *__restrict__ inc, const LitSrc src,
                                               int64_t R, int C, int W, int P, uint32_t *__restrict__ out) {
    __shared__ __align__(16) uint32_t xs[KW][XS];
    __shared__ __align__(16) uint32_t is[KW][XS];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int64_t row0 = (int64_t)blockIdx.x * RT;
    const int c0 = blockIdx.y * CT;
    uint32_t v[4][4];
    const int nch = tile_violations<IMG>(inc, src, R, C, W, row0, c0, xs, is, v);
    if (tid == 0) {
        atomicAdd(&g_match_counts[0], 1ull);
        atomicAdd(&g_match_counts[1], (unsigned long long)nch);
    }

    const int cb = c0 + tx * 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int64_t row = row0 + ty * 4 + i;
        if (row >= R) continue;
        int64_t n = row / P;
        int p = (int)(row % P);
        if (MODE == MODE_ANY) {
            uint32_t nib = 0u;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (v[i][j] == 0u && cb + j < C) nib |= 1u << j;
            if (nib) {
                const int CWn = (C + 31) / 32;
                atomicOr(&out[n * CWn + (cb >> 5)], nib << (cb & 31));
            }
        } else if (MODE == MODE_PBITS) {
            const int PW = (P + 31) / 32;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (v[i][j] == 0u && cb + j < C)
                    atomicOr(&out[(n * C + cb + j) * PW + (p >> 5)], 1u << (p & 31));
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (cb + j < C) out[(n * C + cb + j) * P + p] = v[i][j] == 0u ? 1u : 0u;
        }
    }
}

template <int MODE>
static ytm_status launch_match(const uint32_t *inc, const LitSrc &src, int64_t R, int C, int W, int P,
                               uint32_t *out, cudaStream_t st) {
    if (R <= 0) return YTM_OK;
    int64_t gx = (int64_t)cdiv(R, RT), gy = (int64_t)cdiv(C, CT);
    if (gx > 0x7FFFFFFFll || gy > 65535) return fail(YTM_ERR_UNSUPPORTED, "match grid too large; split the batch");
    if (src.img)
        k_match<MODE, true><<<dim3((unsigned)gx, (unsigned)gy), 256, 0, st>>>(inc, src, R, C, W, P, out);
    else
        k_match<MODE, false><<<dim3((unsigned)gx, (unsigned)gy), 256, 0, st>>>(inc, src, R, C, W, P, out);
    return launch_check("clause match");
}

// ---- sparse patch match ---------------------------------------------------
// Trained clauses include few literals: most include words are zero.  The
// compacted list of a clause's non-zero include words (index, word) lets a
// warp test 128 patches against only those words.  The patch tile of one
// sample is staged word-major in shared memory, [W][SP_STRIDE] with
// SP_STRIDE = 129, so that the 32 lanes (32 consecutive patches) read 32
// banks and the staging writes (consecutive words) do too.

static unsigned grid1(int64_t threads);

constexpr int SP_PT = 128, SP_STRIDE = SP_PT + 1, SP_WARPS = 32;

// the patch tile, plus the sample's bit image when the input is bit images
inline size_t sparse_smem_bytes(int W, int64_t img_words = 0) { return ((size_t)W * SP_STRIDE + img_words) * 4; }
inline bool sparse_match_fits(int W, int64_t img_words = 0) { return sparse_smem_bytes(W, img_words) <= 220 * 1024; }

// One warp per clause: cnt[c] = non-zero include words, ent[c][0..cnt) =
// (word index, include word) in word order.
__global__ void k_compact(const uint32_t *__restrict__ inc, int C, int W, int32_t *__restrict__ cnt,
                          uint2 *__restrict__ ent) {
    const int lane = threadIdx.x & 31;
    for (int64_t c = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; c < C;
         c += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        const uint32_t *row = inc + c * W;
        uint2 *out = ent + c * W;
        int base = 0;
        for (int w0 = 0; w0 < W; w0 += 32) {
            const int w = w0 + lane;
            const uint32_t v = w < W ? row[w] : 0u;
            const uint32_t m = __ballot_sync(0xFFFFFFFFu, v != 0u);
            if (v) out[base + __popc(m & ((1u << lane) - 1u))] = make_uint2((uint32_t)w, v);
            base += __popc(m);
        }
        if (lane == 0) cnt[c] = base;
    }
}

// MODE_PBITS: out[n][c][PW] = patches of sample n that clause c matches (an
// empty clause matches all); every word is written once (no clear needed).
// MODE_ANY: bit c of out[n][CW] is set when clause c matches some patch
// (out cleared beforehand).  Grid: x = 128-patch tiles, y = clause blocks of
// cpb clauses, z = samples.
template <int MODE, bool IMG>
__global__ void __launch_bounds__(SP_WARPS * 32, 2) k_match_sparse(const LitSrc src,
                                                                const int32_t *__restrict__ cnt,
                                                                const uint2 *__restrict__ ent, int C, int W, int P,
                                                                int cpb, uint32_t *__restrict__ out) {
    extern __shared__ uint32_t sl[];  // [W][SP_STRIDE], then (bit images) the sample's image
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t n = blockIdx.z;
    const int p0 = blockIdx.x * SP_PT;
    const int np = min(SP_PT, P - p0);
    if (IMG) {
        // the tile's patch words formed from the sample's bit image, staged
        // in shared memory first (sliding-window patches of one image)
        uint32_t *im = sl + W * SP_STRIDE;
        const uint32_t *gi = src.p + n * src.iws;
        for (int i = tid; i < src.iws; i += SP_WARPS * 32) im[i] = __ldg(&gi[i]);
        __syncthreads();
        for (int idx = tid; idx < SP_PT * W; idx += SP_WARPS * 32) {
            const int p = idx / W, w = idx - p * W;
            sl[w * SP_STRIDE + p] = p < np ? patch_word(im, src.g, p0 + p, w) : 0u;
        }
    } else {
        const uint32_t *gp = src.p + ((int64_t)n * P + p0) * W;
        for (int idx = tid; idx < SP_PT * W; idx += SP_WARPS * 32) {
            const int p = idx / W, w = idx - p * W;
            sl[w * SP_STRIDE + p] = p < np ? __ldg(&gp[idx]) : 0u;
        }
    }
    __syncthreads();
    const int PW = (P + 31) / 32;
    const int c_lo = blockIdx.y * cpb, c_hi = min(C, c_lo + cpb);
    const int ng = (np + 31) / 32;
    // the count and the first 32 entries of the next clause are loaded while
    // the current one is tested (entries past the count are never used; a
    // row holds W entries, so lanes below W stay inside it)
    int c = c_lo + warp;
    int k_nx = 0;
    uint2 e_nx = make_uint2(0u, 0u);
    if (c < c_hi) {
        k_nx = __ldg(&cnt[c]);
        if (lane < W) e_nx = ent[(int64_t)c * W + lane];
    }
    for (; c < c_hi; c += SP_WARPS) {
        const int k = k_nx;
        uint2 my = e_nx;
        const int cn = c + SP_WARPS;
        if (cn < c_hi) {
            k_nx = __ldg(&cnt[cn]);
            if (lane < W) e_nx = ent[(int64_t)cn * W + lane];
        }
        const uint2 *e = ent + (int64_t)c * W;
        uint32_t v0 = 0u, v1 = 0u, v2 = 0u, v3 = 0u;
        for (int e0 = 0; e0 < k; e0 += 32) {
            if (e0 > 0) my = e0 + lane < k ? e[e0 + lane] : make_uint2(0u, 0u);
            const int m = min(32, k - e0);
            for (int j = 0; j < m; ++j) {
                const uint32_t off = __shfl_sync(0xFFFFFFFFu, my.x, j) * SP_STRIDE + lane;
                const uint32_t iv = __shfl_sync(0xFFFFFFFFu, my.y, j);
                v0 |= iv & ~sl[off];
                v1 |= iv & ~sl[off + 32];
                v2 |= iv & ~sl[off + 64];
                v3 |= iv & ~sl[off + 96];
                // every patch of the tile already violated: nothing can match
                if ((j & 3) == 3 && __all_sync(0xFFFFFFFFu, (v0 != 0u) & (v1 != 0u) & (v2 != 0u) & (v3 != 0u)))
                    goto done;
            }
        }
    done:
        const uint32_t v[4] = {v0, v1, v2, v3};
        if (MODE == MODE_PBITS) {
            uint32_t *o = out + ((int64_t)n * C + c) * PW + (p0 >> 5);
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                if (g < ng) {
                    const uint32_t b = __ballot_sync(0xFFFFFFFFu, v[g] == 0u && g * 32 + lane < np);
                    if (lane == 0) o[g] = b;
                }
            }
        } else {
            bool any = false;
#pragma unroll
            for (int g = 0; g < 4; ++g) any |= v[g] == 0u && g * 32 + lane < np;
            if (__any_sync(0xFFFFFFFFu, any) && lane == 0)
                atomicOr(&out[(int64_t)n * ((C + 31) / 32) + (c >> 5)], 1u << (c & 31));
        }
    }
}

// Scratch of the sparse match: include-word counts [C] and lists [C][W].
uint64_t sparse_ws_bytes(const ytm_config *cfg) {
    if (cfg->patches <= 1) return 0;
    const uint64_t C = cfg->clause_count;
    return align_up(C * 4, 256) + align_up(C * (uint64_t)cfg->words * 8, 256);
}

inline bool use_sparse_match(const ytm_config *cfg) {
    return cfg->patches > 1 && sparse_match_fits(cfg->words, cfg->input_images ? cfg->image_words : 0);
}

// Samples [0, N) of src; out as k_match_sparse<MODE> describes.
template <int MODE>
static ytm_status launch_match_sparse(const uint32_t *inc, const LitSrc &src, int64_t N, int C, int W, int P,
                                      void *scratch, uint32_t *out, cudaStream_t st) {
    int32_t *cnt = (int32_t *)scratch;
    uint2 *ent = (uint2 *)((char *)scratch + align_up((uint64_t)C * 4, 256));
    k_compact<<<grid1((int64_t)C * 32), 256, 0, st>>>(inc, C, W, cnt, ent);
    ytm_status rc = launch_check("include compaction");
    if (rc) return rc;
    const size_t smem = sparse_smem_bytes(W, src.img ? src.iws : 0);
    if (smem > 48 * 1024 &&
        (rc = cuda_check(cudaFuncSetAttribute(src.img ? k_match_sparse<MODE, true> : k_match_sparse<MODE, false>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                         "sparse match smem")))
        return rc;
    const int tiles = (int)cdiv(P, SP_PT);
    const int64_t PW = (int64_t)cdiv(P, 32), CW = (int64_t)cdiv(C, 32);
    for (int64_t n0 = 0; n0 < N; n0 += 65535) {
        const int64_t nb = std::min<int64_t>(65535, N - n0);
        // about two CTAs per SM over the whole grid; at least 32 clauses a block
        int64_t cb = std::max<int64_t>(1, (int64_t)sm_count() * 2 / ((int64_t)tiles * nb));
        cb = std::min<int64_t>(cb, std::max<int64_t>(1, C / 32));
        const int cpb = (int)cdiv(C, cb);
        cb = cdiv(C, cpb);
        uint32_t *o = out + n0 * (MODE == MODE_PBITS ? (int64_t)C * PW : CW);
        const dim3 grid((unsigned)tiles, (unsigned)cb, (unsigned)nb);
        if (src.img)
            k_match_sparse<MODE, true><<<grid, SP_WARPS * 32, smem, st>>>(src.from(n0), cnt, ent, C, W, P, cpb, o);
        else
            k_match_sparse<MODE, false><<<grid, SP_WARPS * 32, smem, st>>>(src.from(n0), cnt, ent, C, W, P, cpb, o);
        if ((rc = launch_check("sparse match"))) return rc;
    }
    return YTM_OK;
}

// The fired bitmap of inference and transforms (out cleared beforehand).
static ytm_status launch_match_any(const ytm_config *cfg, const uint32_t *inc, const uint32_t *lits, int64_t N,
                                   void *sparse_scratch, uint32_t *fired, cudaStream_t st) {
    const int C = cfg->clause_count, W = cfg->words, P = cfg->patches;
    const LitSrc src = lit_src(cfg, lits);
    if (sparse_scratch && use_sparse_match(cfg))
        return launch_match_sparse<MODE_ANY>(inc, src, N, C, W, P, sparse_scratch, fired, st);
    return launch_match<MODE_ANY>(inc, src, N * P, C, W, P, fired, st);
}

// Training evaluation of single-patch models in one kernel: the tile's
// matches give each (sample, clause) its pick (patch 0, or -1 when it does not
// fire or is dropped: fast_eval + select_active, kernel.cu:255-316), the fired
// bits, and the class sums: per row the weights of the fired clauses
// (staged in shared memory; non-coalesced clauses count for their own class
// only, kernel.cu:306-312) are summed over the 16 threads that share the row
// and added with one int32 atomic per (row, class) and tile.
__global__ void __launch_bounds__(256) k_train_eval1(ytm_config cfg, const uint32_t *__restrict__ inc,
                                                     const uint32_t *__restrict__ lits, int B,
                                                     const int32_t *__restrict__ weights,
                                                     const uint32_t *__restrict__ drop, int32_t *__restrict__ sel,
                                                     uint32_t *__restrict__ fcm, int32_t *__restrict__ cs) {
    __shared__ __align__(16) uint32_t xs[KW][XS];
    __shared__ __align__(16) uint32_t is[KW][XS];
    extern __shared__ int32_t w_s[];  // [CT][K]
    const int C = cfg.clause_count, W = cfg.words, K = cfg.n_classes;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int64_t row0 = (int64_t)blockIdx.x * RT;
    const int c0 = blockIdx.y * CT;
    for (int q = tid; q < CT * K; q += 256) {
        const int cl = q / K, k = q % K, c = c0 + cl;
        int32_t v = 0;
        if (c < C && !(drop && drop[c] == 1u)) {
            const int own = (cfg.clause_lo + c) / cfg.clauses_per_class;
            if (cfg.coalesced || k == own) v = weights[(int64_t)c * K + k];
        }
        w_s[q] = v;
    }
    uint32_t v[4][4];
    tile_violations<false>(inc, lit_src_dev(cfg, lits), B, C, W, row0, c0, xs, is, v);  // its syncs also publish w_s
    const int cb = c0 + tx * 4;
    uint32_t keep = 0u;  // clauses of this thread that exist and are not dropped
#pragma unroll
    for (int j = 0; j < 4; ++j)
        if (cb + j < C && !(drop && drop[cb + j] == 1u)) keep |= 1u << j;
    uint32_t cbits[4] = {0u, 0u, 0u, 0u};  // per clause of this thread: its 4 rows' outputs
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t row = row0 + ty * 4 + i;
        const bool rv = row < B;
        uint32_t nib = 0u;
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (v[i][j] == 0u) nib |= 1u << j;
        nib &= keep;
        if (!rv) nib = 0u;
#pragma unroll
        for (int j = 0; j < 4; ++j) cbits[j] |= ((nib >> j) & 1u) << i;
        if (rv) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (cb + j < C) sel[row * C + cb + j] = ((nib >> j) & 1u) ? 0 : -1;

        }
        for (int k = 0; k < K; ++k) {
            int32_t part = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if ((nib >> j) & 1u) part += w_s[(tx * 4 + j) * K + k];
            part += __shfl_xor_sync(0xFFFFFFFFu, part, 8);
            part += __shfl_xor_sync(0xFFFFFFFFu, part, 4);
            part += __shfl_xor_sync(0xFFFFFFFFu, part, 2);
            part += __shfl_xor_sync(0xFFFFFFFFu, part, 1);
            if (tx == 0 && rv && part != 0) atomicAdd(&cs[row * K + k], part);
        }
    }
    if (fcm) {  // clause-major fired bits [C][ceil(B/32)] for the feedback kernel
        const int BWn = (B + 31) / 32;
        const int64_t r4 = row0 + ty * 4;  // 4-aligned: the 4 rows share one word
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (cbits[j]) atomicOr(&fcm[(int64_t)(cb + j) * BWn + (r4 >> 5)], cbits[j] << (r4 & 31));
    }
}

__global__ void k_cs_init(int32_t *__restrict__ cs, const int32_t *__restrict__ bias, int64_t N, int K,
                          uint32_t *__restrict__ zero = nullptr, int64_t nzero = 0) {
    int64_t total = N * K;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x)
        cs[i] = bias ? bias[i % K] : 0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nzero; i += (int64_t)gridDim.x * blockDim.x)
        zero[i] = 0u;
}

// cs[n][k] += sum over fired clauses c of w[c][k].  A warp takes 32 bitmap
// words (1024 clauses) of one sample; lanes own classes k = lane + 32 m.
// ninc (inference): clauses with no include are skipped (kernel.cu:328).
// own_class (training, non-coalesced): clause c adds only to its bank's class
// (kernel.cu:306-312).
constexpr int CS_WARPS = 4, CS_KREG = 8;

__global__ void __launch_bounds__(CS_WARPS * 32) k_class_sums(const uint32_t *__restrict__ fired,
                                                              const int32_t *__restrict__ ninc,
                                                              const int32_t *__restrict__ w, int C, int K,
                                                              int64_t N, int own_class, int clause_lo, int cpc,
                                                              int32_t *__restrict__ cs) {
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int CWn = (C + 31) / 32;
    const int64_t chunks = (CWn + 31) / 32;
    const int64_t units = N * chunks;
    for (int64_t u = (int64_t)blockIdx.x * CS_WARPS + wib; u < units; u += (int64_t)gridDim.x * CS_WARPS) {
        const int64_t n = u / chunks;
        const int wbase = (int)(u % chunks) * 32;
        uint32_t mine = (wbase + lane < CWn) ? fired[n * CWn + wbase + lane] : 0u;
        if (__ballot_sync(0xFFFFFFFFu, mine != 0u) == 0u) continue;
        for (int k0 = 0; k0 < K; k0 += 32 * CS_KREG) {
            int32_t acc[CS_KREG];
#pragma unroll
            for (int m = 0; m < CS_KREG; ++m) acc[m] = 0;
            for (int j = 0; j < 32; ++j) {
                uint32_t bits = __shfl_sync(0xFFFFFFFFu, mine, j);
                while (bits) {
                    int b = __ffs(bits) - 1;
                    bits &= bits - 1;
                    int c = (wbase + j) * 32 + b;
                    if (ninc && ninc[c] == 0) continue;
                    const int32_t *wr = w + (int64_t)c * K;
                    if (own_class) {
                        int k = (clause_lo + c) / cpc;
                        int m = (k - k0) >> 5;
                        if (k >= k0 && m < CS_KREG && ((k - k0) & 31) == lane) acc[m] += wr[k];
                    } else {
#pragma unroll
                        for (int m = 0; m < CS_KREG; ++m) {
                            int k = k0 + m * 32 + lane;
                            if (k < K) acc[m] += wr[k];
                        }
                    }
                }
            }
#pragma unroll
            for (int m = 0; m < CS_KREG; ++m) {
                int k = k0 + m * 32 + lane;
                if (k < K && acc[m] != 0) atomicAdd(&cs[n * K + k], acc[m]);
            }
        }
    }
}

static ytm_status launch_class_sums(const uint32_t *fired, const int32_t *ninc, const int32_t *w,
                                    const ytm_config *cfg, int64_t N, int own_class, int32_t *cs, cudaStream_t st) {
    const int C = cfg->clause_count;
    int64_t chunks = (int64_t)cdiv(cdiv(C, 32), 32);
    int64_t blocks = std::min<int64_t>((int64_t)cdiv(N * chunks, CS_WARPS), (int64_t)sm_count() * 16);
    if (blocks < 1) blocks = 1;
    k_class_sums<<<(unsigned)blocks, CS_WARPS * 32, 0, st>>>(fired, ninc, w, C, cfg->n_classes, N, own_class,
                                                              cfg->clause_lo, cfg->clauses_per_class, cs);
    return launch_check("class sums");
}

static unsigned grid1(int64_t threads) {
    int64_t b = (int64_t)cdiv(threads, 256);
    int64_t cap = (int64_t)sm_count() * 32;
    if (b > cap) b = cap;
    return (unsigned)(b < 1 ? 1 : b);
}

// ---- class sums from weight bit planes ------------------------------------
// For every 32-clause word w and class k, the weights u = w[c][k] + OFF
// (offset binary, OFF = 2^(npl-1), npl bits) are stored as npl bit planes;
// then sum_c fired_c * w[c][k] = sum_b 2^b popc(f & plane_b) - OFF * popc(f)
// for f = the word's fired bits, evaluated modulo 2^32 (exact: the true sum
// fits int32).  Words where nothing fired are skipped; every class sum has
// one writer.

constexpr int CSP_KCH = 16;

__global__ void k_wmax(const int32_t *__restrict__ w, int C, int K, int own_class, int clause_lo, int cpc,
                       int32_t *__restrict__ wmax) {
    int m = 0;
    const int64_t total = (int64_t)C * K;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i / K), k = (int)(i % K);
        if (own_class && k != (clause_lo + c) / cpc) continue;
        const int v = w[i];
        m = max(m, v < 0 ? -v : v);
    }
    for (int o = 16; o; o >>= 1) m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if ((threadIdx.x & 31) == 0 && m) atomicMax(wmax, m);
}

__device__ __forceinline__ int planes_for(int wmax) { return 33 - __clz(wmax | 1) > 32 ? 32 : 33 - __clz(wmax | 1); }

// One warp per (clause word, class): lane = clause.  planes [K][32][CW]
// (class-major, clause words innermost, so that lanes walking consecutive
// clause words read consecutive plane words); keep [CW] = clauses that count
// (non-empty when ninc is given).
__global__ void k_wplanes(const int32_t *__restrict__ w, const int32_t *__restrict__ ninc, int C, int K,
                          int own_class, int clause_lo, int cpc, const int32_t *__restrict__ wmax,
                          uint32_t *__restrict__ planes, uint32_t *__restrict__ keep) {
    const int lane = threadIdx.x & 31;
    const int CWn = (C + 31) / 32;
    const int npl = planes_for(*wmax);
    const uint32_t off = 1u << (npl - 1);
    const int64_t units = (int64_t)CWn * K;
    for (int64_t u = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; u < units;
         u += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        const int wd = (int)(u / K), k = (int)(u % K);
        const int c = wd * 32 + lane;
        int32_t v = 0;
        if (c < C && !(own_class && k != (clause_lo + c) / cpc)) v = w[(int64_t)c * K + k];
        const uint32_t x = (uint32_t)v + off;
        uint32_t *pl = planes + (int64_t)k * 32 * CWn + wd;
        for (int b = 0; b < npl; ++b) {
            const uint32_t m = __ballot_sync(0xFFFFFFFFu, (x >> b) & 1u);
            if (lane == 0) pl[(int64_t)b * CWn] = m;
        }
        if (k == 0) {
            const uint32_t m = __ballot_sync(0xFFFFFFFFu, c < C && (!ninc || ninc[c] > 0));
            if (lane == 0) keep[wd] = m;
        }
    }
}

// WARP: one warp per (sample, 16 classes, segment of seg_words clause words),
// lanes striding over the segment's words (coalesced fired-bit and plane
// reads); with more than one segment (gridDim.y) the partial sums are added
// atomically onto cs, which then holds the bias already.  Else one thread per
// (sample, 16 classes) walking all words (models with few clause words).
template <bool WARP>
__global__ void __launch_bounds__(256) k_cs_planes(const uint32_t *__restrict__ fired,
                                                   const uint32_t *__restrict__ keep,
                                                   const uint32_t *__restrict__ planes,
                                                   const int32_t *__restrict__ wmax, const int32_t *__restrict__ bias,
                                                   int C, int K, int64_t N, int seg_words,
                                                   int32_t *__restrict__ cs) {
    const int lane = WARP ? (threadIdx.x & 31) : 0;
    const int step = WARP ? 32 : 1;
    const int CWn = (C + 31) / 32;
    const int KC = (K + CSP_KCH - 1) / CSP_KCH;
    const int npl = planes_for(*wmax);
    const uint32_t off = 1u << (npl - 1);
    const int64_t units = N * KC;
    const int64_t u0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / step;
    const int64_t us = ((int64_t)gridDim.x * blockDim.x) / step;
    for (int64_t u = u0; u < units; u += us) {
        // consecutive units: consecutive samples of the same classes
        const int64_t n = u % N;
        const int k0 = (int)(u / N) * CSP_KCH;
        const int kn = min(CSP_KCH, K - k0);
        uint32_t acc[CSP_KCH];
#pragma unroll
        for (int j = 0; j < CSP_KCH; ++j) acc[j] = 0u;
        uint32_t nf = 0u;
        const uint32_t *fr = fired + n * CWn;
        const int wlo = WARP ? (int)blockIdx.y * seg_words : 0;
        const int whi = WARP ? min(CWn, wlo + seg_words) : CWn;
        for (int wd = wlo + lane; wd < whi; wd += step) {
            const uint32_t f = fr[wd] & keep[wd];
            if (!f) continue;
            nf += (uint32_t)__popc(f);
            const uint32_t *pl = planes + (int64_t)k0 * 32 * CWn + wd;
#pragma unroll
            for (int j = 0; j < CSP_KCH; ++j) {
                if (j < kn) {
                    uint32_t a = 0u;
                    for (int b = 0; b < npl; ++b) a += (uint32_t)__popc(f & pl[((int64_t)j * 32 + b) * CWn]) << b;
                    acc[j] += a;
                }
            }
        }
        if (WARP) nf = __reduce_add_sync(0xFFFFFFFFu, nf);
#pragma unroll
        for (int j = 0; j < CSP_KCH; ++j) {
            if (j < kn) {
                const uint32_t t = WARP ? __reduce_add_sync(0xFFFFFFFFu, acc[j]) : acc[j];
                if (lane == 0) {
                    if (WARP && gridDim.y > 1)
                        atomicAdd(&cs[n * K + k0 + j], (int32_t)(t - off * nf));
                    else
                        cs[n * K + k0 + j] = (int32_t)(t - off * nf) + (bias ? bias[k0 + j] : 0);
                }
            }
        }
    }
}

uint64_t cs_planes_bytes(const ytm_config *cfg) {
    const uint64_t CW = cdiv(cfg->clause_count, 32);
    return 256 + align_up(CW * cfg->n_classes * 32 * 4, 256) + align_up(CW * 4, 256);
}

// cs [N][K] = bias + class sums of the fired bits (all classes, or only each
// clause's own class when own_class); scratch: cs_planes_bytes(cfg).
static ytm_status launch_cs_planes(const uint32_t *fired, const int32_t *ninc, const int32_t *w, const int32_t *bias,
                                   const ytm_config *cfg, int64_t N, int own_class, int32_t *cs, void *scratch,
                                   cudaStream_t st, bool wmax_cleared = false) {
    const int C = cfg->clause_count, K = cfg->n_classes;
    const int64_t CW = (int64_t)cdiv(C, 32);
    char *p = (char *)scratch;
    int32_t *wmax = (int32_t *)p;
    uint32_t *planes = (uint32_t *)(p + 256);
    uint32_t *keep = (uint32_t *)(p + 256 + align_up(CW * K * 32 * 4, 256));
    ytm_status rc;
    if (!wmax_cleared && (rc = cuda_check(cudaMemsetAsync(wmax, 0, 4, st), "memset"))) return rc;
    k_wmax<<<grid1((int64_t)C * K), 256, 0, st>>>(w, C, K, own_class, cfg->clause_lo, cfg->clauses_per_class, wmax);
    if ((rc = launch_check("weight range"))) return rc;
    k_wplanes<<<grid1(CW * K * 32), 256, 0, st>>>(w, ninc, C, K, own_class, cfg->clause_lo, cfg->clauses_per_class,
                                                   wmax, planes, keep);
    if ((rc = launch_check("weight planes"))) return rc;
    const int64_t units = N * (int64_t)cdiv(K, CSP_KCH);
    const int sms = sm_count();
    if (units < (int64_t)sms * 32 || CW >= 64) {
        // split the clause words so that about 16 warps per SM run; a segment
        // keeps at least 4 words (batch 1 with 4000 clauses ran on 3 warps
        // when segments kept one word per lane: 23 us instead of a few)
        int64_t segs = std::max<int64_t>(1, (int64_t)sms * 16 / units);
        segs = std::min<int64_t>(segs, std::max<int64_t>(1, CW / 4));
        const int seg_words = (int)cdiv(CW, segs);
        segs = cdiv(CW, seg_words);
        if (segs > 1) {
            k_cs_init<<<grid1(N * K), 256, 0, st>>>(cs, bias, N, K);
            if ((rc = launch_check("class sums init"))) return rc;
        }
        k_cs_planes<true><<<dim3((unsigned)cdiv(units * 32, 256), (unsigned)segs), 256, 0, st>>>(
            fired, keep, planes, wmax, bias, C, K, N, seg_words, cs);
    } else {
        k_cs_planes<false><<<(unsigned)std::min<int64_t>(cdiv(units, 256), (int64_t)sms * 64), 256, 0, st>>>(
            fired, keep, planes, wmax, bias, C, K, N, 0, cs);
    }
    return launch_check("class sums");
}

__global__ void k_expand(const uint32_t *__restrict__ fired, int64_t N, int C, uint32_t *__restrict__ out) {
    const int CWn = (C + 31) / 32;
    int64_t total = N * C;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t n = i / C;
        int c = (int)(i % C);
        out[i] = (fired[n * CWn + (c >> 5)] >> (c & 31)) & 1u;
    }
}

// One thread per (sample, clause): pick a matching patch uniformly
// (reference select_active, kernel.cu:285-316, reservoir sampling; here the
// TAG_PATCH draw r gives index floor(r * count / 2^32) among the matches in
// patch order), count it in patch_w and set the fired bit.
// Also: thread 0 clears the weight-range slot of the class-sum planes that
// follow.
__global__ void k_pick(ytm_config cfg, const uint32_t *__restrict__ mbits, const uint32_t *__restrict__ drop,
                       int B, uint64_t t0, int32_t *__restrict__ sel, uint32_t *__restrict__ fired,
                       int32_t *__restrict__ patch_w, int32_t *__restrict__ wmax) {
    const int C = cfg.clause_count, P = cfg.patches, PW = (P + 31) / 32, CWn = (C + 31) / 32;
    if (blockIdx.x == 0 && threadIdx.x == 0) *wmax = 0;
    int64_t total = (int64_t)B * C;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int b = (int)(i / C), c = (int)(i % C);

        int32_t s = -1;
        if (!(drop && drop[c] == 1u)) {
            const uint32_t *m = mbits + i * PW;
            int cnt = 0;
            for (int j = 0; j < PW; ++j) cnt += __popc(m[j]);
            if (cnt > 0) {
                uint32_t r = draw(cfg.seed, (uint32_t)(cfg.clause_lo + c), t0 + (uint64_t)b, 0, TAG_PATCH, 0).x;
                uint32_t idx = (uint32_t)(((uint64_t)r * (uint64_t)cnt) >> 32);
                for (int j = 0; j < PW; ++j) {
                    uint32_t word = m[j];
                    uint32_t pc = (uint32_t)__popc(word);
                    if (idx < pc) {
                        for (uint32_t q = 0; q < idx; ++q) word &= word - 1u;
                        s = j * 32 + __ffs(word) - 1;
                        break;
                    }
                    idx -= pc;
                }
                atomicAdd(&patch_w[(int64_t)c * P + s], 1);
                atomicOr(&fired[(int64_t)b * CWn + (c >> 5)], 1u << (c & 31));
            }
        }
        sel[i] = s;
    }
}


}  // namespace ytm

using namespace ytm;

extern "C" {

ytm_status ytm_infer(const ytm_config *cfg, const uint32_t *state, const int32_t *weights, const int32_t *bias,
                     const uint32_t *lits, int64_t N, int32_t *cs, void *workspace, void *stream) {
    ytm_status rc = check_cfg(cfg);
    if (rc) return rc;
    if (N < 0) return fail(YTM_ERR_ARG, "N < 0");
    if (N == 0) return YTM_OK;
    if (!state || !weights || !lits || !cs || !workspace) return fail(YTM_ERR_ARG, "null pointer");
    cudaStream_t st = as_stream(stream);
    const int C = cfg->clause_count, W = cfg->words;
    InferWs l = infer_ws_layout(cfg, N);
    char *ws = (char *)workspace;
    int32_t *ninc = (int32_t *)(ws + l.ninc);
    uint32_t *fired = (uint32_t *)(ws + l.fired);
    const uint32_t *inc = state + (int64_t)(cfg->planes - 1) * C * W;
    if ((rc = launch_ninc(cfg, state, ninc, st))) return rc;
    if ((rc = cuda_check(cudaMemsetAsync(fired, 0, (size_t)N * cdiv(C, 32) * 4, st), "memset"))) return rc;
    if ((rc = launch_match_any(cfg, inc, lits, N, ws + l.total + cs_planes_bytes(cfg), fired, st))) return rc;
    return launch_cs_planes(fired, cfg->count_empty ? nullptr : ninc, weights, bias, cfg, N, 0, cs, ws + l.total,
                            st);
}

ytm_status ytm_infer_include(const ytm_config *cfg, const uint32_t *inc, const int32_t *weights,
                             const int32_t *bias, const uint32_t *lits, int64_t N, int32_t *cs, void *workspace,
                             void *stream) {
    ytm_status rc = check_cfg(cfg);
    if (rc) return rc;
    if (N < 0) return fail(YTM_ERR_ARG, "N < 0");
    if (N == 0) return YTM_OK;
    if (!inc || !weights || !lits || !cs || !workspace) return fail(YTM_ERR_ARG, "null pointer");
    cudaStream_t st = as_stream(stream);
    const int C = cfg->clause_count, W = cfg->words;
    InferWs l = infer_ws_layout(cfg, N);
    char *ws = (char *)workspace;
    int32_t *ninc = (int32_t *)(ws + l.ninc);
    uint32_t *fired = (uint32_t *)(ws + l.fired);
    k_ninc<<<grid1((int64_t)C * 32), 256, 0, st>>>(C, W, inc, ninc, nullptr);
    if ((rc = launch_check("include counts"))) return rc;
    if ((rc = cuda_check(cudaMemsetAsync(fired, 0, (size_t)N * cdiv(C, 32) * 4, st), "memset"))) return rc;
    if ((rc = launch_match_any(cfg, inc, lits, N, ws + l.total + cs_planes_bytes(cfg), fired, st))) return rc;
    return launch_cs_planes(fired, cfg->count_empty ? nullptr : ninc, weights, bias, cfg, N, 0, cs, ws + l.total,
                            st);
}

ytm_status ytm_transform(const ytm_config *cfg, const uint32_t *state, const uint32_t *lits, int64_t N,
                         uint32_t *out, void *workspace, void *stream) {
    ytm_status rc = check_cfg(cfg);
    if (rc) return rc;
    if (N < 0) return fail(YTM_ERR_ARG, "N < 0");
    if (N == 0) return YTM_OK;
    if (!state || !lits || !out || !workspace) return fail(YTM_ERR_ARG, "null pointer");
    cudaStream_t st = as_stream(stream);
    const int C = cfg->clause_count, W = cfg->words;
    InferWs l = infer_ws_layout(cfg, N);
    uint32_t *fired = (uint32_t *)((char *)workspace + l.fired);
    const uint32_t *inc = state + (int64_t)(cfg->planes - 1) * C * W;
    if ((rc = cuda_check(cudaMemsetAsync(fired, 0, (size_t)N * cdiv(C, 32) * 4, st), "memset"))) return rc;
    // empty clauses match every patch, so they come out as 1 (kernel.cu:354-357)
    if ((rc = launch_match_any(cfg, inc, lits, N, (char *)workspace + l.total + cs_planes_bytes(cfg), fired, st)))
        return rc;
    k_expand<<<grid1(N * C), 256, 0, st>>>(fired, N, C, out);
    return launch_check("transform expand");
}

ytm_status ytm_transform_patchwise(const ytm_config *cfg, const uint32_t *state, const uint32_t *lits, int64_t N,
                                   uint32_t *out, void *stream) {
    ytm_status rc = check_cfg(cfg);
    if (rc) return rc;
    if (N < 0) return fail(YTM_ERR_ARG, "N < 0");
    if (N == 0) return YTM_OK;
    if (!state || !lits || !out) return fail(YTM_ERR_ARG, "null pointer");
    const int C = cfg->clause_count, W = cfg->words, P = cfg->patches;
    const uint32_t *inc = state + (int64_t)(cfg->planes - 1) * C * W;
    return launch_match<MODE_PATCHWISE>(inc, lit_src(cfg, lits), N * P, C, W, P, out, as_stream(stream));
}

ytm_status ytm_train_eval(const ytm_config *cfg, const uint32_t *state, const int32_t *weights, const int32_t *bias,
                          const uint32_t *drop, const uint32_t *lits, int32_t B, uint64_t t0, int32_t add_bias,
                          int32_t *cs, int32_t *patch_w, void *workspace, void *stream) {
    ytm_status rc = check_cfg(cfg);
    if (rc) return rc;
    if (B <= 0) return fail(YTM_ERR_ARG, "batch must be positive");
    if (!state || !weights || !lits || !cs || !patch_w || !workspace) return fail(YTM_ERR_ARG, "null pointer");
    cudaStream_t st = as_stream(stream);
    const int C = cfg->clause_count, W = cfg->words, P = cfg->patches;
    TrainWs l = train_ws_layout(cfg, B);
    char *ws = (char *)workspace;
    uint32_t *mbits = (uint32_t *)(ws + l.mbits);
    int32_t *sel = (int32_t *)(ws + l.sel);
    uint32_t *fired = (uint32_t *)(ws + l.fired);
    const uint32_t *inc = state + (int64_t)(cfg->planes - 1) * C * W;
    if (single_patch_eval(cfg)) {
        // single patch: one fused kernel (picks and class sums; the feedback
        // kernel counts the picks in patch_w)
        uint32_t *fcm = (uint32_t *)(ws + l.fcm);
        const int64_t nfcm = (int64_t)C * cdiv(B, 32);
        k_cs_init<<<grid1(std::max<int64_t>((int64_t)B * cfg->n_classes, nfcm)), 256, 0, st>>>(
            cs, add_bias ? bias : nullptr, B, cfg->n_classes, fcm, nfcm);
        if ((rc = launch_check("cs init"))) return rc;
        const size_t smem = (size_t)CT * cfg->n_classes * 4;
        if (smem > 48 * 1024 &&
            (rc = cuda_check(cudaFuncSetAttribute(k_train_eval1, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  (int)smem), "train eval smem")))
            return rc;
        const int64_t gx = (int64_t)cdiv(B, RT), gy = (int64_t)cdiv(C, CT);
        if (gy > 65535) return fail(YTM_ERR_UNSUPPORTED, "too many clauses for one launch");
        k_train_eval1<<<dim3((unsigned)gx, (unsigned)gy), 256, smem, st>>>(*cfg, inc, lits, B, weights, drop, sel,
                                                                           fcm, cs);
        return launch_check("train eval");
    }
    // training semantics: an empty clause matches every patch (kernel.cu:273-276)
    if (use_sparse_match(cfg)) {
        if ((rc = cuda_check(cudaMemsetAsync(fired, 0, l.sel - l.fired, st), "memset"))) return rc;
        if ((rc = launch_match_sparse<MODE_PBITS>(inc, lit_src(cfg, lits), B, C, W, P, ws + l.sparse, mbits, st)))
            return rc;
    } else {
        // match bits and fired bits are adjacent in the workspace: one clear
        if ((rc = cuda_check(cudaMemsetAsync(mbits, 0, l.sel - l.mbits, st), "memset"))) return rc;
        if ((rc = launch_match<MODE_PBITS>(inc, lit_src(cfg, lits), (int64_t)B * P, C, W, P, mbits, st))) return rc;
    }
    int32_t *wmax = (int32_t *)(ws + l.total);  // the class-sum planes scratch starts with the weight range
    k_pick<<<grid1((int64_t)B * C), 256, 0, st>>>(*cfg, mbits, drop, B, t0, sel, fired, patch_w, wmax);
    if ((rc = launch_check("patch pick"))) return rc;
    return launch_cs_planes(fired, nullptr, weights, add_bias ? bias : nullptr, cfg, B, cfg->coalesced ? 0 : 1, cs,
                            ws + l.total, st, true);
}

ytm_status ytm_train_selection(const ytm_config *cfg, int32_t B, const void *workspace, int32_t *sel,
                               void *stream) {
    ytm_status rc = check_cfg(cfg);
    if (rc) return rc;
    if (B <= 0 || !workspace || !sel) return fail(YTM_ERR_ARG, "bad argument");
    TrainWs l = train_ws_layout(cfg, B);
    return cuda_check(cudaMemcpyAsync(sel, (const char *)workspace + l.sel, (size_t)B * cfg->clause_count * 4,
                                      cudaMemcpyDeviceToDevice, as_stream(stream)),
                      "selection copy");
}

ytm_status ytm_match_counters(uint64_t *out, void *stream) {
    if (!out) return fail(YTM_ERR_ARG, "bad argument");
    cudaStream_t st = as_stream(stream);
    unsigned long long h[2] = {0ull, 0ull};
    ytm_status rc = cuda_check(cudaMemcpyFromSymbolAsync(h, g_match_counts, sizeof h, 0, cudaMemcpyDeviceToHost, st),
                               "match counters");
    if (!rc) rc = cuda_check(cudaStreamSynchronize(st), "match counters");
    if (rc) return rc;
    const unsigned long long z[2] = {0ull, 0ull};
    if ((rc = cuda_check(cudaMemcpyToSymbolAsync(g_match_counts, z, sizeof z, 0, cudaMemcpyHostToDevice, st),
                         "match counters")))
        return rc;
    if ((rc = cuda_check(cudaStreamSynchronize(st), "match counters"))) return rc;
    out[0] = h[0];
    out[1] = h[1];
    return YTM_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free inference.
//
// Some callers cannot allocate device memory: embedders whose device memory
// is carved up in advance by another runtime or pool allocator (a cudaMalloc
// of their own would fail or break that runtime's accounting), and services
// that forbid allocation after start-up so that a request can never fail or
// stall on it.  ytm_infer_noalloc gives them inference without a workspace
// argument.  Its scratch (include
// counts and the fired-clause bitmap) lives in the fixed array below, which
// every GPU that loads this library holds until the process exits.
//
// Host code must not pass `g_noalloc_scratch` itself to a kernel: in host code
// that name is only a host-side stand-in for the symbol.  The device address is
// looked up once per device with cudaGetSymbolAddress, with that device
// current, the first time the entry point runs on it; that first call should
// therefore come before any stream capture.  The address is cached for the
// life of the process: after cudaDeviceReset (which unloads this module from
// the device) the cache is stale, so a process that resets a device must not
// call ytm_infer_noalloc on it afterwards.
//
// All calls share the array and it keeps the previous call's contents; the
// bitmap is cleared on every call.  Calls that overlap on the GPU (different
// streams, or other threads) race on the array and must be serialised by the
// caller.
// ---------------------------------------------------------------------------
#include <mutex>

namespace ytm {

static __device__ __align__(256) unsigned char g_noalloc_scratch[YTM_NOALLOC_SCRATCH_BYTES];

static std::mutex g_noalloc_mu;
static void *g_noalloc_ptr[64];

static ytm_status noalloc_scratch(void **out) {
    int dev = 0;
    ytm_status rc = cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
    if (rc) return rc;
    if (dev < 0 || dev >= 64) return fail(YTM_ERR_UNSUPPORTED, "device index above 63");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        if ((rc = cuda_check(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress"))) return rc;
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return YTM_OK;
}

}  // namespace ytm

extern "C" ytm_status ytm_infer_noalloc(const ytm_config *cfg, const uint32_t *state, const int32_t *weights,
                                        const int32_t *bias, const uint32_t *lits, int64_t N, int32_t *cs,
                                        void *stream) {
    ytm_status rc = check_cfg(cfg);
    if (rc) return rc;
    if (N < 0) return fail(YTM_ERR_ARG, "N < 0");
    if (N == 0) return YTM_OK;
    if (!state || !weights || !lits || !cs) return fail(YTM_ERR_ARG, "null pointer");
    InferWs l = infer_ws_layout(cfg, N);
    if (l.total > (uint64_t)YTM_NOALLOC_SCRATCH_BYTES)
        return fail(YTM_ERR_ARG, "ytm_infer_noalloc: " + std::to_string(l.total) +
                                     " bytes of scratch needed, the fixed scratch holds " +
                                     std::to_string((uint64_t)YTM_NOALLOC_SCRATCH_BYTES) +
                                     "; pass fewer samples per call");
    void *scratch = nullptr;
    if ((rc = noalloc_scratch(&scratch))) return rc;
    cudaStream_t st = as_stream(stream);
    const int C = cfg->clause_count, W = cfg->words, P = cfg->patches;
    char *ws = (char *)scratch;
    int32_t *ninc = (int32_t *)(ws + l.ninc);
    uint32_t *fired = (uint32_t *)(ws + l.fired);
    const uint32_t *inc = state + (int64_t)(cfg->planes - 1) * C * W;
    if ((rc = launch_ninc(cfg, state, ninc, st))) return rc;
    if ((rc = cuda_check(cudaMemsetAsync(fired, 0, (size_t)N * cdiv(C, 32) * 4, st), "memset"))) return rc;
    if ((rc = launch_match<MODE_ANY>(inc, lit_src(cfg, lits), N * P, C, W, P, fired, st))) return rc;
    k_cs_init<<<grid1(N * cfg->n_classes), 256, 0, st>>>(cs, bias, N, cfg->n_classes);
    if ((rc = launch_check("cs init"))) return rc;
    return launch_class_sums(fired, cfg->count_empty ? nullptr : ninc, weights, cfg, N, 0, cs, st);
}
