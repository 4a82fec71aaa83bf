// probe.cu — LOP3 throughput probe: the INT/logic-pipe ceiling that the
// clause-evaluation kernels (one LOP3 per word test) are measured against.
#include "common.cuh"

namespace ytm {

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

}  // namespace ytm

using namespace ytm;

extern "C" ytm_status ytm_probe_lop3(int32_t blocks, int32_t iters, uint32_t *out, uint64_t *ops, void *stream) {
    if (blocks <= 0 || iters <= 0 || !out || !ops) return fail(YTM_ERR_ARG, "bad argument");
    k_probe_lop3<<<blocks, 256, 0, as_stream(stream)>>>(iters, 0x2545F491u, out);
    *ops = (uint64_t)blocks * 256 * (uint64_t)iters * PROBE_CHAINS;
    return launch_check("lop3 probe");
}
