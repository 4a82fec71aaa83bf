// ref_launcher.cu — host launcher for the reference's own kernels.
//
// TEST INFRASTRUCTURE ONLY.  Compiled by oracle/ref_build.py into
// oracle/_ref/ref_<shape>.so with the reference's macro preamble (the string
// Mayur1009/YTM src/cutm/base.py:129-152 builds) force-included and the
// reference's src/cutm/cuda/kernel.cu #included from where it lies (REF_KERNEL).
// It replaces pycuda's prepared_call with plain CUDA runtime launches, using the
// reference's launch geometry (cuda_utils.py:27-41), and moves host arrays in
// and out.  Nothing of the reference's source is copied here.
#include <cuda_runtime.h>
#include <stdint.h>

#include REF_KERNEL

namespace {

int g_sms = 0;

void geometry(long long n, int bs, dim3 *grid, dim3 *block) {
    // kernel_config, cuda_utils.py:27-41
    if (!g_sms) cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, 0);
    long long g = (n + bs - 1) / bs;
    long long cap = 4LL * g_sms < 65535 ? 4LL * g_sms : 65535;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    *grid = dim3((unsigned)g);
    *block = dim3((unsigned)bs);
}

__global__ void seed_rng(curandState *s, unsigned long long seed, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) curand_init(seed + (unsigned long long)i, 0, 0, &s[i]);
}

template <class T>
T *dev(const T *host, size_t n) {
    T *d = nullptr;
    if (cudaMalloc(&d, n * sizeof(T) + 16) != cudaSuccess) return nullptr;
    if (host) cudaMemcpy(d, host, n * sizeof(T), cudaMemcpyHostToDevice);
    else cudaMemset(d, 0, n * sizeof(T));
    return d;
}

template <class T>
void back(T *host, const T *d, size_t n) { cudaMemcpy(host, d, n * sizeof(T), cudaMemcpyDeviceToHost); }

int status() {
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? 0 : (int)e;
}

}  // namespace

extern "C" {

void ref_sizes(int *out) {
    out[0] = CLAUSES; out[1] = CLASSES; out[2] = LITERALS; out[3] = NUM_LITERAL_CHUNKS; out[4] = PATCHES;
}

// encode (base.py:224-263): X u32 [N][D0*D1*D2] -> out u32 [N][P][W]
int ref_encode(const uint32_t *X, int N, uint32_t *out) {
    size_t nx = (size_t)N * DIM0 * DIM1 * DIM2, no = (size_t)N * PATCHES * NUM_LITERAL_CHUNKS;
    uint32_t *dX = dev(X, nx), *dO = dev<uint32_t>(nullptr, no);
    dim3 g, b;
    geometry((long long)N * PATCHES, 128, &g, &b);
    encode_batch<<<g, b>>>(dX, dO, N);
    int rc = status();
    back(out, dO, no);
    cudaFree(dX); cudaFree(dO);
    return rc;
}

// pack_clauses: ta u32 [C][L] -> packed [C][W], ninc [C]
int ref_pack(const uint32_t *ta, uint32_t *packed, int32_t *ninc) {
    uint32_t *dT = dev(ta, (size_t)CLAUSES * LITERALS);
    uint32_t *dP = dev<uint32_t>(nullptr, (size_t)CLAUSES * NUM_LITERAL_CHUNKS);
    int *dN = dev<int>(nullptr, CLAUSES);
    dim3 g, b;
    geometry(CLAUSES, 128, &g, &b);
    pack_clauses<<<g, b>>>(dT, dP, dN);
    int rc = status();
    back(packed, dP, (size_t)CLAUSES * NUM_LITERAL_CHUNKS);
    back(ninc, dN, CLAUSES);
    cudaFree(dT); cudaFree(dP); cudaFree(dN);
    return rc;
}

// _score_batch (base.py:375-420): cs f32 [N][K] enters holding the bias rows.
int ref_infer(const uint32_t *ta, const float *w, const uint32_t *lits, int N, float *cs) {
    uint32_t *dT = dev(ta, (size_t)CLAUSES * LITERALS);
    uint32_t *dP = dev<uint32_t>(nullptr, (size_t)CLAUSES * NUM_LITERAL_CHUNKS);
    int *dN = dev<int>(nullptr, CLAUSES);
    float *dW = dev(w, (size_t)CLAUSES * CLASSES);
    uint32_t *dX = dev(lits, (size_t)N * PATCHES * NUM_LITERAL_CHUNKS);
    float *dC = dev(cs, (size_t)N * CLASSES);
    dim3 g, b;
    geometry(CLAUSES, 128, &g, &b);
    pack_clauses<<<g, b>>>(dT, dP, dN);
    geometry((long long)N * CLAUSES, 512, &g, &b);
    calc_class_sums_infer_batch<<<g, b>>>(dP, dW, dN, dX, N, dC);
    int rc = status();
    back(cs, dC, (size_t)N * CLASSES);
    cudaFree(dT); cudaFree(dP); cudaFree(dN); cudaFree(dW); cudaFree(dX); cudaFree(dC);
    return rc;
}

// transform (base.py:465-502) / transform_patchwise (base.py:504-542)
int ref_transform(const uint32_t *ta, const uint32_t *lits, int N, int patchwise, uint32_t *out) {
    size_t no = (size_t)N * CLAUSES * (patchwise ? PATCHES : 1);
    uint32_t *dT = dev(ta, (size_t)CLAUSES * LITERALS);
    uint32_t *dP = dev<uint32_t>(nullptr, (size_t)CLAUSES * NUM_LITERAL_CHUNKS);
    int *dN = dev<int>(nullptr, CLAUSES);
    uint32_t *dX = dev(lits, (size_t)N * PATCHES * NUM_LITERAL_CHUNKS);
    uint32_t *dO = dev<uint32_t>(nullptr, no);
    dim3 g, b;
    geometry(CLAUSES, 128, &g, &b);
    pack_clauses<<<g, b>>>(dT, dP, dN);
    geometry((long long)no, 128, &g, &b);
    if (patchwise) transform_patchwise<<<g, b>>>(dP, dN, dX, N, dO);
    else transform<<<g, b>>>(dP, dN, dX, N, dO);
    int rc = status();
    back(out, dO, no);
    cudaFree(dT); cudaFree(dP); cudaFree(dN); cudaFree(dX); cudaFree(dO);
    return rc;
}

// init_weights (kernel.cu:46-73): w f32 [C][K]
int ref_init_weights(unsigned long long seed, float *w) {
    dim3 g, b;
    geometry(CLAUSES, 128, &g, &b);
    int n = g.x * b.x;
    curandState *rng = nullptr;
    cudaMalloc(&rng, sizeof(curandState) * n);
    seed_rng<<<(n + 127) / 128, 128>>>(rng, seed, n);
    float *dW = dev<float>(nullptr, (size_t)CLAUSES * CLASSES);
    init_weights<<<g, b>>>(rng, dW);
    int rc = status();
    back(w, dW, (size_t)CLAUSES * CLASSES);
    cudaFree(rng); cudaFree(dW);
    return rc;
}

// One iteration of the training loop of _fit (base.py:305-357) for sample e:
// pack_clauses, fast_eval, class_sum <- bias, select_active, clause_update.
// ta, w, patch_w are updated in place; sel [C] and cs [K] report what the
// feedback used.  drop [C] may be NULL (no clause dropped).
int ref_train_step(uint32_t *ta, float *w, int32_t *patch_w, const uint32_t *lits, const int32_t *Y, int N,
                   int e, const uint32_t *drop, unsigned long long seed, int32_t *sel, float *cs) {
    const int bs = 16;  // the block_size the reference's scripts train with (mnist_conv.py:19)
    dim3 gc, bc, gp, bp;
    geometry(CLAUSES, bs, &gc, &bc);
    geometry((long long)CLAUSES * PATCHES, bs, &gp, &bp);
    int n = gc.x * bc.x;
    curandState *rng = nullptr;
    cudaMalloc(&rng, sizeof(curandState) * n);
    seed_rng<<<(n + 127) / 128, 128>>>(rng, seed, n);
    uint32_t *dT = dev(ta, (size_t)CLAUSES * LITERALS);
    float *dW = dev(w, (size_t)CLAUSES * CLASSES);
    int *dPW = dev(patch_w, (size_t)CLAUSES * PATCHES);
    float *dBias = dev<float>(nullptr, CLASSES);
    uint32_t *dX = dev(lits, (size_t)N * PATCHES * NUM_LITERAL_CHUNKS);
    int *dY = dev(Y, (size_t)N * CLASSES);
    double *dTrue = nullptr, *dFalse = nullptr;
    {
        double ones[CLASSES];
        for (int k = 0; k < CLASSES; ++k) ones[k] = 1.0;
        dTrue = dev(ones, CLASSES);
        dFalse = dev(ones, CLASSES);
    }
    uint32_t *dDrop = dev(drop, CLAUSES);
    uint32_t *dPk = dev<uint32_t>(nullptr, (size_t)CLAUSES * NUM_LITERAL_CHUNKS);
    float *dCS = dev<float>(nullptr, CLASSES);
    uint32_t *dCO = dev<uint32_t>(nullptr, (size_t)CLAUSES * PATCHES);
    int *dSel = dev<int>(nullptr, CLAUSES);
    int *dN = dev<int>(nullptr, CLAUSES);

    pack_clauses<<<gc, bc>>>(dT, dPk, dN);
    fast_eval<<<gp, bp>>>(dPk, dN, dDrop, dX, dCO, e);
    cudaMemcpy(dCS, dBias, CLASSES * sizeof(float), cudaMemcpyDeviceToDevice);
    select_active<<<gc, bc>>>(rng, dW, dCO, dPW, dSel, dCS);
    cudaDeviceSynchronize();
    back(sel, dSel, CLAUSES);
    back(cs, dCS, CLASSES);
    clause_update<<<gc, bc>>>(rng, dT, dW, dBias, dCS, dSel, dN, dTrue, dFalse, dDrop, dX, dY, e, 0, 0);
    int rc = status();
    back(ta, dT, (size_t)CLAUSES * LITERALS);
    back(w, dW, (size_t)CLAUSES * CLASSES);
    back(patch_w, dPW, (size_t)CLAUSES * PATCHES);
    cudaFree(rng); cudaFree(dT); cudaFree(dW); cudaFree(dPW); cudaFree(dBias); cudaFree(dX); cudaFree(dY);
    cudaFree(dTrue); cudaFree(dFalse); cudaFree(dDrop); cudaFree(dPk); cudaFree(dCS); cudaFree(dCO);
    cudaFree(dSel); cudaFree(dN);
    return rc;
}

// One epoch of _fit (base.py:266-359) over samples 0..N-1 in order, all on the
// device: per sample pack_clauses, fast_eval, class_sum <- bias,
// select_active, clause_update, with one curand state per thread seeded once.
int ref_fit(uint32_t *ta, float *w, int32_t *patch_w, const uint32_t *lits, const int32_t *Y, int N,
            unsigned long long seed) {
    const int bs = 16;
    dim3 gc, bc, gp, bp;
    geometry(CLAUSES, bs, &gc, &bc);
    geometry((long long)CLAUSES * PATCHES, bs, &gp, &bp);
    int n = gc.x * bc.x;
    curandState *rng = nullptr;
    cudaMalloc(&rng, sizeof(curandState) * n);
    seed_rng<<<(n + 127) / 128, 128>>>(rng, seed, n);
    uint32_t *dT = dev(ta, (size_t)CLAUSES * LITERALS);
    float *dW = dev(w, (size_t)CLAUSES * CLASSES);
    int *dPW = dev(patch_w, (size_t)CLAUSES * PATCHES);
    float *dBias = dev<float>(nullptr, CLASSES);
    uint32_t *dX = dev(lits, (size_t)N * PATCHES * NUM_LITERAL_CHUNKS);
    int *dY = dev(Y, (size_t)N * CLASSES);
    double ones[CLASSES];
    for (int k = 0; k < CLASSES; ++k) ones[k] = 1.0;
    double *dTrue = dev(ones, CLASSES), *dFalse = dev(ones, CLASSES);
    uint32_t *dDrop = dev<uint32_t>(nullptr, CLAUSES);
    uint32_t *dPk = dev<uint32_t>(nullptr, (size_t)CLAUSES * NUM_LITERAL_CHUNKS);
    float *dCS = dev<float>(nullptr, CLASSES);
    uint32_t *dCO = dev<uint32_t>(nullptr, (size_t)CLAUSES * PATCHES);
    int *dSel = dev<int>(nullptr, CLAUSES);
    int *dN = dev<int>(nullptr, CLAUSES);
    for (int e = 0; e < N; ++e) {
        pack_clauses<<<gc, bc>>>(dT, dPk, dN);
        fast_eval<<<gp, bp>>>(dPk, dN, dDrop, dX, dCO, e);
        cudaMemcpyAsync(dCS, dBias, CLASSES * sizeof(float), cudaMemcpyDeviceToDevice);
        select_active<<<gc, bc>>>(rng, dW, dCO, dPW, dSel, dCS);
        clause_update<<<gc, bc>>>(rng, dT, dW, dBias, dCS, dSel, dN, dTrue, dFalse, dDrop, dX, dY, e, 0, 0);
    }
    int rc = status();
    back(ta, dT, (size_t)CLAUSES * LITERALS);
    back(w, dW, (size_t)CLAUSES * CLASSES);
    back(patch_w, dPW, (size_t)CLAUSES * PATCHES);
    cudaFree(rng); cudaFree(dT); cudaFree(dW); cudaFree(dPW); cudaFree(dBias); cudaFree(dX); cudaFree(dY);
    cudaFree(dTrue); cudaFree(dFalse); cudaFree(dDrop); cudaFree(dPk); cudaFree(dCS); cudaFree(dCO);
    cudaFree(dSel); cudaFree(dN);
    return rc;
}

}  // extern "C"
