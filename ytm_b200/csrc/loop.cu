// loop.cu — whole training runs queued from C: per mini-batch, clause
// evaluation, the int32 all-reduce of the class sums over the clause shards
// (NCCL over NVLink, on the caller's stream), and the feedback.  The
// reference's _fit loop (base.py:305-357) runs in Python with a host sync
// after each kernel; here no host code runs between batches.
#include <nccl.h>

#include "common.cuh"

using namespace ytm;

static ytm_status nccl_check(ncclResult_t r, const char *what) {
    if (r == ncclSuccess) return YTM_OK;
    return fail(YTM_ERR_CUDA, std::string(what) + ": " + ncclGetErrorString(r));
}

extern "C" {

ytm_status ytm_nccl_unique_id(uint8_t *id_out) {
    if (!id_out) return fail(YTM_ERR_ARG, "null pointer");
    ncclUniqueId id;
    ytm_status rc = nccl_check(ncclGetUniqueId(&id), "ncclGetUniqueId");
    if (rc) return rc;
    memcpy(id_out, id.internal, NCCL_UNIQUE_ID_BYTES);
    return YTM_OK;
}

ytm_status ytm_nccl_comm_init(const uint8_t *id_in, int32_t rank, int32_t world, void **comm_out) {
    if (!id_in || !comm_out || world <= 0 || rank < 0 || rank >= world) return fail(YTM_ERR_ARG, "bad argument");
    ncclUniqueId id;
    memcpy(id.internal, id_in, NCCL_UNIQUE_ID_BYTES);
    ncclComm_t comm = nullptr;
    ytm_status rc = nccl_check(ncclCommInitRank(&comm, world, id, rank), "ncclCommInitRank");
    if (rc) return rc;
    *comm_out = comm;
    return YTM_OK;
}

ytm_status ytm_nccl_comm_destroy(void *comm) {
    if (!comm) return YTM_OK;
    return nccl_check(ncclCommDestroy((ncclComm_t)comm), "ncclCommDestroy");
}

ytm_status ytm_train_fit_batches(const ytm_config *cfg, uint32_t *state, int32_t *weights, const int32_t *bias,
                                 const uint32_t *drop, const uint32_t *lits, const int32_t *Y, int64_t N, int32_t B,
                                 uint64_t t0, int32_t add_bias, int32_t *patch_w, void *comm, void *peer_ar,
                                 void *workspace, void *stream) {
    ytm_status rc = check_cfg(cfg);
    if (rc) return rc;
    if (N < 0 || B <= 0) return fail(YTM_ERR_ARG, "bad N or batch size");
    if (N == 0) return YTM_OK;
    if (!lits || !Y || !workspace) return fail(YTM_ERR_ARG, "null pointer");
    // words per sample of the input: per-patch literal words, or a bit image
    const int64_t PW = cfg->input_images ? (int64_t)cfg->image_words : (int64_t)cfg->patches * cfg->words;
    const int K = cfg->n_classes;
    char *ws = (char *)workspace;
    int32_t *cs = (int32_t *)ws;  // [B][K] class sums
    void *train_ws = ws + align_up((uint64_t)B * K * 4, 256);
    for (int64_t i = 0; i < N; i += B) {
        const int32_t b = (int32_t)std::min<int64_t>(B, N - i);
        const uint32_t *lb = lits + i * PW;
        const uint64_t t = t0 + (uint64_t)i;
        if ((rc = ytm_train_eval(cfg, state, weights, bias, drop, lb, b, t, add_bias, cs, patch_w, train_ws, stream)))
            return rc;
        if (peer_ar) {
            if ((rc = ytm_peer_allreduce_i32(peer_ar, cs, (int64_t)b * K, 0, stream))) return rc;
        } else if (comm &&
                   (rc = nccl_check(ncclAllReduce(cs, cs, (size_t)b * K, ncclInt32, ncclSum, (ncclComm_t)comm,
                                                  as_stream(stream)),
                                    "ncclAllReduce"))) {
            return rc;
        }
        if ((rc = ytm_train_update(cfg, state, weights, cs, Y + i * K, drop, lb, b, t, nullptr, patch_w, train_ws,
                                   stream)))
            return rc;
    }
    return YTM_OK;
}

}  // extern "C"
