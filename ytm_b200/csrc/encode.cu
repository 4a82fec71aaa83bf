// encode.cu — raw inputs to per-patch literal words.
//
// Same output as the reference's encode_batch (kernel.cu:76-152): for patch
// (py, px), literal bits are
//   [0, py)                         y-location thermometer
//   [D1-P1, D1-P1+px)               x-location thermometer
//   loc + ry*P0*D2 + rx*D2 + z      pixel (py+ry, px+rx, z), loc = D1-P1+D0-P0
//                                   when encode_loc, else 0
//   L/2 + j                         NOT literal j (append_negated)
// (the location bits are set even without encode_loc, as the reference does).
//
// Two passes instead of one thread per (sample, patch) doing scattered
// read-modify-writes: (1) the u32-per-pixel input is packed to one bit per
// pixel with warp ballots (coalesced 128-byte reads); (2) one warp per
// (sample, patch) builds the positive literal words in shared memory with
// funnel shifts out of the packed image rows, then writes all W words
// (positive and negated halves) with coalesced stores.
#include "common.cuh"

namespace ytm {

// X u32 [N][D] -> img u32 [N][IWS] (IWS = IW + 1, last word zero padding).
__global__ void k_bitpack(const uint32_t *__restrict__ X, int64_t N, int64_t D, int64_t IWS,
                          uint32_t *__restrict__ img) {
    int64_t total = N * IWS * 32;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t n = i / (IWS * 32), j = i % (IWS * 32);
        uint32_t v = (j < D) ? X[n * D + j] : 0u;
        uint32_t b = __ballot_sync(0xFFFFFFFFu, v > 0u);
        if ((threadIdx.x & 31) == 0) img[n * IWS + j / 32] = b;
    }
}

// nbits (<= 32) bits of a packed row starting at bit q.
__device__ __forceinline__ uint32_t bits_at(const uint32_t *__restrict__ row, int64_t q, int nbits) {
    uint32_t lo = row[q >> 5], hi = row[(q >> 5) + 1];
    uint32_t v = __funnelshift_r(lo, hi, (uint32_t)(q & 31));
    return nbits >= 32 ? v : (v & ((1u << nbits) - 1u));
}

// 32 bits of the positive literal vector (in shared memory, PWn words, zero
// beyond) starting at bit a, which may be negative (zeros there).
__device__ __forceinline__ uint32_t pos_at(const uint32_t *pos, int PWn, int64_t a) {
    if (a <= -32 || a >= (int64_t)PWn * 32) return 0u;
    if (a < 0) return pos[0] << (uint32_t)(-a);
    int64_t w = a >> 5;
    uint32_t lo = pos[w], hi = (w + 1 < PWn) ? pos[w + 1] : 0u;
    return __funnelshift_r(lo, hi, (uint32_t)(a & 31));
}

__global__ void k_literals(ytm_config cfg, const uint32_t *__restrict__ img, int64_t IWS, int64_t N,
                           uint32_t *__restrict__ lits) {
    extern __shared__ uint32_t sm[];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5, wpb = blockDim.x >> 5;
    const int P = cfg.patches, W = cfg.words, L = cfg.literals, Lh = cfg.half_literals;
    const int PWn = (Lh + 31) / 32;
    const int D0 = cfg.dim0, D1 = cfg.dim1, D2 = cfg.dim2, P0 = cfg.patch_dim0, P1 = cfg.patch_dim1;
    const int seg = P0 * D2;               // bits per patch row
    const int64_t rowbits = (int64_t)D0 * D2;
    const int loc = cfg.encode_loc ? cfg.loc_literals : 0;
    const int npix = P0 * P1 * D2;
    uint32_t *pos = sm + wib * PWn;
    const int64_t total = N * P;
    for (int64_t ep = (int64_t)blockIdx.x * wpb + wib; ep < total; ep += (int64_t)gridDim.x * wpb) {
        const int64_t e = ep / P;
        const int patch = (int)(ep % P);
        const int py = patch / (D0 - P0 + 1), px = patch % (D0 - P0 + 1);
        const uint32_t *row = img + e * IWS;
        for (int w = lane; w < PWn; w += 32) {
            const int a = w * 32;
            uint32_t v = 0u;
            // pixel literals [loc, loc + npix)
            int lo = max(a, loc), hi = min(a + 32, loc + npix);
            while (lo < hi) {
                int rel = lo - loc;
                int ry = rel / seg, o = rel % seg;
                int n = min(hi - lo, seg - o);
                int64_t q = (int64_t)(py + ry) * rowbits + (int64_t)px * D2 + o;
                v |= bits_at(row, q, n) << (lo - a);
                lo += n;
            }
            // y thermometer [0, py), x thermometer [D1-P1, D1-P1+px)
            for (int r = 0; r < 2; ++r) {
                int s0 = r ? (D1 - P1) : 0, s1 = r ? (D1 - P1 + px) : py;
                int l0 = max(s0, a), l1 = min(s1, a + 32);
                if (l0 < l1) {
                    int n = l1 - l0;
                    uint32_t m = n >= 32 ? 0xFFFFFFFFu : ((1u << n) - 1u);
                    v |= m << (l0 - a);
                }
            }
            if (a + 32 > Lh) v &= (Lh - a >= 32) ? 0xFFFFFFFFu : ((1u << (Lh - a)) - 1u);
            pos[w] = v;
        }
        __syncwarp();
        uint32_t *out = lits + ep * W;
        for (int w = lane; w < W; w += 32) {
            const int64_t a = (int64_t)w * 32;
            uint32_t v = pos_at(pos, PWn, a);
            if (cfg.append_negated) {
                uint32_t mpos = (Lh - a >= 32) ? 0xFFFFFFFFu : (Lh - a <= 0 ? 0u : ((1u << (Lh - a)) - 1u));
                uint32_t mneg = ~mpos & valid_mask(w, W, L);
                v = (v & mpos) | (~pos_at(pos, PWn, a - Lh) & mneg);
            } else {
                v &= valid_mask(w, W, L);
            }
            out[w] = v;
        }
        __syncwarp();
    }
}

// Thermometer binarisation fused into the bit packing: img u8 [N][pixels][ch]
// -> bit image [N][IWS] with bit (pixel * ch + c) * levels + j set iff
// img >= thr[j] (thr[j] = ceil((j+1) * 255 / (levels+1)), the integer form of
// ThermometerBinarizer's float thresholds, tm_utils/binarizer.py:11-21; thr =
// NULL computes them as ((j+1) * 255 + levels) / (levels+1), the same exact
// ceiling).
__global__ void k_thermo_bitpack(const uint8_t *__restrict__ img, int64_t N, int64_t pixels, int ch, int levels,
                                 const uint32_t *__restrict__ thr, int64_t IWS, uint32_t *__restrict__ out) {
    const int64_t D = pixels * ch * levels;
    const int64_t total = N * IWS * 32;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = i / (IWS * 32), q = i % (IWS * 32);
        bool v = false;
        if (q < D) {
            const int64_t pc = q / levels;  // pixel * ch + c
            const int j = (int)(q % levels);
            // thr == NULL: the same thresholds in exact integer form
            const uint32_t t = thr ? thr[j] : (uint32_t)(((j + 1) * 255 + levels) / (levels + 1));
            v = img[n * pixels * ch + pc] >= t;
        }
        const uint32_t b = __ballot_sync(0xFFFFFFFFu, v);
        if ((threadIdx.x & 31) == 0) out[n * IWS + q / 32] = b;
    }
}

}  // namespace ytm

using namespace ytm;

extern "C" ytm_status ytm_encode_thermometer(const ytm_config *cfg, const uint8_t *img, int64_t N, int32_t levels,
                                             uint32_t *lits, void *workspace, void *stream) {
    ytm_status rc = check_cfg(cfg);
    if (rc) return rc;
    if (N < 0 || levels <= 0 || levels > 255) return fail(YTM_ERR_ARG, "bad N or levels");
    if (cfg->dim2 % levels) return fail(YTM_ERR_ARG, "dim2 must be channels * levels");
    if (N == 0) return YTM_OK;
    if (!img || !lits || !workspace) return fail(YTM_ERR_ARG, "null pointer");
    cudaStream_t st = as_stream(stream);
    const int ch = cfg->dim2 / levels;
    const int64_t pixels = (int64_t)cfg->dim0 * cfg->dim1;
    const int64_t D = pixels * cfg->dim2;
    const int64_t IWS = (int64_t)cdiv(D, 32) + 1;
    uint32_t *bits = (uint32_t *)workspace;
    uint32_t *thr = bits + N * IWS;  // levels thresholds after the bit images
    uint32_t h[256];
    for (int j = 0; j < levels; ++j) h[j] = (uint32_t)ceil((double)(j + 1) * 255.0 / (double)(levels + 1));
    if ((rc = cuda_check(cudaMemcpyAsync(thr, h, levels * 4, cudaMemcpyHostToDevice, st), "thresholds"))) return rc;
    const int sms = sm_count();
    {
        int64_t blocks = std::min<int64_t>(cdiv(N * IWS * 32, 256), (int64_t)sms * 16);
        k_thermo_bitpack<<<(unsigned)blocks, 256, 0, st>>>(img, N, pixels, ch, levels, thr, IWS, bits);
        if ((rc = launch_check("thermometer bitpack"))) return rc;
    }
    const int PWn = (cfg->half_literals + 31) / 32;
    int wpb = 8;
    size_t smem = (size_t)wpb * PWn * 4;
    while (smem > 48 * 1024 && wpb > 1) { wpb >>= 1; smem = (size_t)wpb * PWn * 4; }
    if (smem > 48 * 1024 &&
        (rc = cuda_check(cudaFuncSetAttribute(k_literals, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                         "encode smem")))
        return rc;
    int64_t blocks = std::min<int64_t>(cdiv(N * cfg->patches, wpb), (int64_t)sms * 32);
    k_literals<<<(unsigned)blocks, wpb * 32, smem, st>>>(*cfg, bits, IWS, N, lits);
    return launch_check("encode literals");
}

extern "C" ytm_status ytm_pack_images(const ytm_config *cfg, const uint32_t *X, int64_t N, uint32_t *img,
                                      void *stream) {
    ytm_status rc = check_cfg(cfg);
    if (rc) return rc;
    if (N < 0) return fail(YTM_ERR_ARG, "N < 0");
    if (N == 0) return YTM_OK;
    if (!X || !img) return fail(YTM_ERR_ARG, "null pointer");
    const int64_t D = (int64_t)cfg->dim0 * cfg->dim1 * cfg->dim2;
    const int64_t IWS = cfg->image_words;
    if (IWS != (int64_t)cdiv(D, 32) + 1) return fail(YTM_ERR_ARG, "config image_words does not match its dims");
    int64_t blocks = std::min<int64_t>(cdiv(N * IWS * 32, 256), (int64_t)sm_count() * 16);
    k_bitpack<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(X, N, D, IWS, img);
    return launch_check("image bitpack");
}

extern "C" ytm_status ytm_pack_images_thermometer(const ytm_config *cfg, const uint8_t *img, int64_t N,
                                                  int32_t levels, uint32_t *bits, void *stream) {
    ytm_status rc = check_cfg(cfg);
    if (rc) return rc;
    if (N < 0 || levels <= 0 || levels > 255) return fail(YTM_ERR_ARG, "bad N or levels");
    if (cfg->dim2 % levels) return fail(YTM_ERR_ARG, "dim2 must be channels * levels");
    if (N == 0) return YTM_OK;
    if (!img || !bits) return fail(YTM_ERR_ARG, "null pointer");
    const int ch = cfg->dim2 / levels;
    const int64_t pixels = (int64_t)cfg->dim0 * cfg->dim1;
    const int64_t IWS = cfg->image_words;
    if (IWS != (int64_t)cdiv(pixels * cfg->dim2, 32) + 1)
        return fail(YTM_ERR_ARG, "config image_words does not match its dims");
    cudaStream_t st = as_stream(stream);
    int64_t blocks = std::min<int64_t>(cdiv(N * IWS * 32, 256), (int64_t)sm_count() * 16);
    // thresholds computed in the kernel (thr = NULL): no scratch memory
    k_thermo_bitpack<<<(unsigned)blocks, 256, 0, st>>>(img, N, pixels, ch, levels, nullptr, IWS, bits);
    return launch_check("thermometer image bitpack");
}

extern "C" ytm_status ytm_encode(const ytm_config *cfg, const uint32_t *X, int64_t N, uint32_t *lits,
                                 void *workspace, void *stream) {
    ytm_status rc = check_cfg(cfg);
    if (rc) return rc;
    if (N < 0) return fail(YTM_ERR_ARG, "N < 0");
    if (N == 0) return YTM_OK;
    if (!X || !lits || !workspace) return fail(YTM_ERR_ARG, "null pointer");
    cudaStream_t st = as_stream(stream);
    const int64_t D = (int64_t)cfg->dim0 * cfg->dim1 * cfg->dim2;
    const int64_t IWS = (int64_t)cdiv(D, 32) + 1;
    uint32_t *img = (uint32_t *)workspace;
    const int sms = sm_count();
    {
        int64_t threads = N * IWS * 32;
        int64_t blocks = std::min<int64_t>(cdiv(threads, 256), (int64_t)sms * 16);
        k_bitpack<<<(unsigned)blocks, 256, 0, st>>>(X, N, D, IWS, img);
        if ((rc = launch_check("encode bitpack"))) return rc;
    }
    {
        const int PWn = (cfg->half_literals + 31) / 32;
        int wpb = 8;
        size_t smem = (size_t)wpb * PWn * 4;
        while (smem > 48 * 1024 && wpb > 1) { wpb >>= 1; smem = (size_t)wpb * PWn * 4; }
        if (smem > 48 * 1024) {
            if ((rc = cuda_check(cudaFuncSetAttribute(k_literals, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                      (int)smem), "encode smem")))
                return rc;
        }
        int64_t units = N * cfg->patches;
        int64_t blocks = std::min<int64_t>(cdiv(units, wpb), (int64_t)sms * 32);
        k_literals<<<(unsigned)blocks, wpb * 32, smem, st>>>(*cfg, img, IWS, N, lits);
        if ((rc = launch_check("encode literals"))) return rc;
    }
    return YTM_OK;
}
