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

}  // namespace

// Launch `blocks` x 256 threads that each run `iters` x 8 dependent-free LOP3
// operations (the word-test operation a |= b & ~c); *ops receives the
// operation count.  Time it with events on `stream`.  Returns a cudaError_t.
extern "C" int bench_probe_lop3(int32_t blocks, int32_t iters, uint32_t *out, uint64_t *ops, void *stream) {
    if (blocks <= 0 || iters <= 0 || !out || !ops) return (int)cudaErrorInvalidValue;
    k_probe_lop3<<<blocks, 256, 0, (cudaStream_t)stream>>>(iters, 0x2545F491u, out);
    *ops = (uint64_t)blocks * 256 * (uint64_t)iters * PROBE_CHAINS;
    return (int)cudaGetLastError();
}
