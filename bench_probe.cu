// bench_probe.cu — measurement helper of bench.py (not part of libytm's
// ABI): a LOP3 throughput probe giving the INT/logic-pipe ceiling that the
// clause-evaluation kernels (one LOP3 per word test) are measured against.
// Built into bench_probe.so by ytm_b200.build.build_probe().
#include <cuda_runtime.h>
#include <stdint.h>

namespace {

constexpr int PROBE_CHAINS = 8;

__global__ void __launch_bounds__(256) k_probe_lop3(int iters, uint32_t seed, uint32_t *__restrict__ out) {
    uint32_t a[PROBE_CHAINS];
    const uint32_t b = seed ^ threadIdx.x, c = seed * 0x9E3779B9u + blockIdx.x;
#pragma unroll
    for (int j = 0; j < PROBE_CHAINS; ++j) a[j] = seed + j * 0x1234567u + threadIdx.x;
    for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int j = 0; j < PROBE_CHAINS; ++j)  // a = a | (b & ~c): the word-test operation
            asm volatile("lop3.b32 %0, %0, %1, %2, 0xF2;" : "+r"(a[j]) : "r"(b), "r"(c));
    }
    uint32_t r = 0;
#pragma unroll
    for (int j = 0; j < PROBE_CHAINS; ++j) r ^= a[j];
    if (r == 0x12345678u) out[0] = r;  // keeps the chains alive
}

// Philox4x32-7 calls back to back, 4 independent counters per thread: the
// throughput ceiling of the literal-mask draws of the feedback kernels.
__global__ void __launch_bounds__(256) k_probe_philox7(int iters, uint32_t seed, uint32_t *__restrict__ out) {
    uint32_t c[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        c[j][0] = blockIdx.x * blockDim.x + threadIdx.x;
        c[j][1] = j;
        c[j][2] = seed;
        c[j][3] = 2u;
    }
    for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t k0 = seed, k1 = seed ^ 0x5bd1e995u;
            uint32_t c0 = c[j][0], c1 = c[j][1], c2 = c[j][2], c3 = c[j][3];
#pragma unroll
            for (int r = 0; r < 7; ++r) {
                if (r) {
                    k0 += 0x9E3779B9u;
                    k1 += 0xBB67AE85u;
                }
                const uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
                const uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
                const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
                c0 = n0;
                c1 = lo1;
                c2 = n2;
                c3 = lo0;
            }
            c[j][0] = c0 + (uint32_t)it;  // next counter depends on this output
            c[j][1] = c1;
            c[j][2] = c2;
            c[j][3] = c3;
        }
    }
    uint32_t r = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) r ^= c[j][0] ^ c[j][1] ^ c[j][2] ^ c[j][3];
    if (r == 0x12345678u) out[0] = r;
}

}  // namespace

extern "C" int bench_probe_philox7(int32_t blocks, int32_t iters, uint32_t *out, uint64_t *calls, void *stream) {
    if (blocks <= 0 || iters <= 0 || !out || !calls) return (int)cudaErrorInvalidValue;
    k_probe_philox7<<<blocks, 256, 0, (cudaStream_t)stream>>>(iters, 0x2545F491u, out);
    *calls = (uint64_t)blocks * 256 * (uint64_t)iters * 4;
    return (int)cudaGetLastError();
}

// Launch `blocks` x 256 threads that each run `iters` x 8 dependent-free LOP3
// operations (the word-test operation a |= b & ~c); *ops receives the
// operation count.  Time it with events on `stream`.  Returns a cudaError_t.
extern "C" int bench_probe_lop3(int32_t blocks, int32_t iters, uint32_t *out, uint64_t *ops, void *stream) {
    if (blocks <= 0 || iters <= 0 || !out || !ops) return (int)cudaErrorInvalidValue;
    k_probe_lop3<<<blocks, 256, 0, (cudaStream_t)stream>>>(iters, 0x2545F491u, out);
    *ops = (uint64_t)blocks * 256 * (uint64_t)iters * PROBE_CHAINS;
    return (int)cudaGetLastError();
}
