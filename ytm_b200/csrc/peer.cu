// peer.cu — one-shot int32 all-reduce of the class sums over NVLink peer
// memory (CUDA IPC), for clause-sharded training on the GPUs of one node.
//
// Every rank owns one buffer: data slots [2][world][max_n] (one set per call
// parity, one row per source rank) and flags [AR_BLOCKS][world].  Call e
// (epoch, counted by the host, from 1), CTA j owning slice j of the values:
//   1. store the slice into row `rank` of slot set e&1 of EVERY rank's buffer
//      (fire-and-forget stores over NVLink; the own buffer locally);
//   2. store e, with release semantics at system scope, into flag[j][rank]
//      of every rank's buffer;
//   3. wait until flag[j][p] of the own buffer reaches e for every rank p (a
//      bounded spin: on timeout an error code is recorded and the CTA leaves
//      its slice unchanged);
//   4. sum row p of slot set e&1 of the own buffer over p (local loads).
// A rank writes slot set e&1 into a peer again only in call e+2, which it
// starts after that peer signalled call e+1 — which the peer does only after
// its call e finished reading — so one flag exchange per call suffices.  No
// multicast and no TMA: plain stores to peer memory, loads of local memory.
#include "common.cuh"

namespace ytm {

constexpr int AR_MAX_RANKS = 8;

struct PeerAr {
    int rank = 0, world = 1;
    int64_t max_n = 0;
    uint64_t epoch = 0;
    char *own = nullptr;                  // own buffer (cudaMalloc)
    char *peers[AR_MAX_RANKS] = {};       // every rank's buffer, mapped here (own included)
    int32_t *status = nullptr;            // device status word: 0 ok, else 1 + a missing peer's index
    int device = 0;
};

constexpr int AR_BLOCKS = 16;

struct PeerPtrs {
    int32_t *data[AR_MAX_RANKS];              // slot region of every rank's buffer
    unsigned long long *flags[AR_MAX_RANKS];  // flag region of every rank's buffer
};

static inline uint64_t ar_data_bytes(int64_t n, int world) { return align_up((uint64_t)2 * world * n * 4, 256); }
static inline uint64_t ar_buffer_bytes(int64_t n, int world) {
    return ar_data_bytes(n, world) + align_up((uint64_t)AR_BLOCKS * AR_MAX_RANKS * 8, 256);
}

__device__ __forceinline__ void st_release_sys(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// AR_BLOCKS CTAs, each owning one slice.  limit: spin iterations before a
// missing peer is reported.
__global__ void __launch_bounds__(256) k_peer_allreduce(PeerPtrs pp, int rank, int world, uint64_t epoch,
                                                        int64_t max_n, int32_t *__restrict__ data, int64_t n,
                                                        int64_t limit, int32_t *__restrict__ status) {
    __shared__ int ok;
    const int j = blockIdx.x;
    const int64_t chunk = (n + AR_BLOCKS - 1) / AR_BLOCKS;
    const int64_t lo = j * chunk, hi = min(n, lo + chunk);
    const int64_t set = (int64_t)(epoch & 1) * world * max_n;
    // 1. push the slice to every rank (row `rank`)
    for (int p = 0; p < world; ++p) {
        int32_t *dst = pp.data[p] + set + (int64_t)rank * max_n;
        for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) dst[i] = data[i];
    }
    if (threadIdx.x == 0) ok = 1;
    __syncthreads();
    // 2. signal: release at system scope orders the CTA's stores above
    if (threadIdx.x < world) st_release_sys(&pp.flags[threadIdx.x][j * AR_MAX_RANKS + rank], epoch);
    // 3. wait for every rank's slice
    if (threadIdx.x < world) {
        const unsigned long long *f = &pp.flags[rank][j * AR_MAX_RANKS + threadIdx.x];
        int64_t it = 0;
        while (ld_acquire_sys(f) < epoch) {
            if (++it > limit) {
                atomicExch(&ok, 0);
                atomicMax(status, (int)threadIdx.x + 1);  // the missing peer's index + 1
                break;
            }
        }
    }
    __syncthreads();
    if (!ok) return;
    // 4. sum the rows locally
    const int32_t *own = pp.data[rank] + set;
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        int32_t acc = 0;
        for (int p = 0; p < world; ++p) acc += own[(int64_t)p * max_n + i];
        data[i] = acc;
    }
}

}  // namespace ytm

using namespace ytm;

extern "C" {

ytm_status ytm_peer_ar_create(int32_t rank, int32_t world, int64_t max_n, void **ctx_out, uint8_t *handle_out) {
    if (!ctx_out || !handle_out || world < 1 || world > AR_MAX_RANKS || rank < 0 || rank >= world || max_n <= 0)
        return fail(YTM_ERR_ARG, "bad argument");
    PeerAr *a = new PeerAr();
    a->rank = rank;
    a->world = world;
    a->max_n = max_n;
    ytm_status rc;
    if ((rc = cuda_check(cudaGetDevice(&a->device), "cudaGetDevice"))) { delete a; return rc; }
    if ((rc = cuda_check(cudaMalloc(&a->own, ar_buffer_bytes(max_n, world)), "cudaMalloc"))) { delete a; return rc; }
    if ((rc = cuda_check(cudaMemset(a->own, 0, ar_buffer_bytes(max_n, world)), "cudaMemset")) ||
        (rc = cuda_check(cudaMalloc(&a->status, 4), "cudaMalloc")) ||
        (rc = cuda_check(cudaMemset(a->status, 0, 4), "cudaMemset"))) {
        cudaFree(a->own);
        delete a;
        return rc;
    }
    cudaIpcMemHandle_t h;
    if ((rc = cuda_check(cudaIpcGetMemHandle(&h, a->own), "cudaIpcGetMemHandle"))) {
        cudaFree(a->own);
        cudaFree(a->status);
        delete a;
        return rc;
    }
    memcpy(handle_out, &h, sizeof(h));
    a->peers[rank] = a->own;
    *ctx_out = a;
    return YTM_OK;
}

// handles: world x 64 bytes (cudaIpcMemHandle_t) in rank order; the own entry is ignored.
ytm_status ytm_peer_ar_open(void *ctx, const uint8_t *handles) {
    PeerAr *a = (PeerAr *)ctx;
    if (!a || !handles) return fail(YTM_ERR_ARG, "null pointer");
    for (int p = 0; p < a->world; ++p) {
        if (p == a->rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, handles + (size_t)p * sizeof(h), sizeof(h));
        void *ptr = nullptr;
        ytm_status rc = cuda_check(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
        if (rc) return rc;
        a->peers[p] = (char *)ptr;
    }
    return YTM_OK;
}

// Sums data[0..n) (int32, device) over the ranks, in place, on `stream`.
// limit: spin iterations before a missing peer is reported (<= 0: default).
ytm_status ytm_peer_allreduce_i32(void *ctx, int32_t *data, int64_t n, int64_t limit, void *stream) {
    PeerAr *a = (PeerAr *)ctx;
    if (!a || !data || n < 0) return fail(YTM_ERR_ARG, "bad argument");
    if (n > a->max_n) return fail(YTM_ERR_ARG, "all-reduce larger than the buffer");
    if (n == 0 || a->world == 1) return YTM_OK;
    for (int p = 0; p < a->world; ++p)
        if (!a->peers[p]) return fail(YTM_ERR_ARG, "peer buffers not opened");
    PeerPtrs pp = {};
    const uint64_t db = ar_data_bytes(a->max_n, a->world);
    for (int p = 0; p < a->world; ++p) {
        pp.data[p] = (int32_t *)a->peers[p];
        pp.flags[p] = (unsigned long long *)(a->peers[p] + db);
    }
    a->epoch += 1;
    k_peer_allreduce<<<AR_BLOCKS, 256, 0, as_stream(stream)>>>(pp, a->rank, a->world, a->epoch, a->max_n, data, n,
                                                              limit > 0 ? limit : (int64_t)1 << 26, a->status);
    return launch_check("peer all-reduce");
}

// 0 if every call since the last read completed; else (peer index + 1) of
// a peer that never signalled.  Synchronises the device and clears the
// status word (the kernel only raises it, with atomicMax).
ytm_status ytm_peer_ar_status(void *ctx, int32_t *status_out) {
    PeerAr *a = (PeerAr *)ctx;
    if (!a || !status_out) return fail(YTM_ERR_ARG, "bad argument");
    ytm_status rc = cuda_check(cudaMemcpy(status_out, a->status, 4, cudaMemcpyDeviceToHost), "status copy");
    if (rc == YTM_OK && *status_out != 0) rc = cuda_check(cudaMemset(a->status, 0, 4), "status clear");
    return rc;
}

ytm_status ytm_peer_ar_destroy(void *ctx) {
    PeerAr *a = (PeerAr *)ctx;
    if (!a) return YTM_OK;
    cudaDeviceSynchronize();
    for (int p = 0; p < a->world; ++p)
        if (p != a->rank && a->peers[p]) cudaIpcCloseMemHandle(a->peers[p]);
    cudaFree(a->own);
    cudaFree(a->status);
    delete a;
    return YTM_OK;
}

}  // extern "C"
