/*
 * ytm.h — C ABI of libytm.so, the B200 (sm_100a) Tsetlin Machine engine.
 *
 * This ABI replaces the pycuda launch boundary of the reference engine
 * (Mayur1009/YTM, src/cutm/base.py:128-206 builds a macro preamble, JIT-compiles
 * src/cutm/cuda/kernel.cu and launches its extern "C" kernels through
 * `prepared_call`).  Every entry point here is a host function taking plain
 * device pointers, sizes and a CUDA stream (`void *stream`, a cudaStream_t);
 * no torch or pycuda type crosses the boundary.
 *
 * Conventions
 *  - The caller owns every buffer.  Functions that need scratch memory take a
 *    `workspace` pointer whose size is given by ytm_workspace_bytes().
 *  - Launches are asynchronous on `stream`; nothing synchronises the device.
 *  - Every function returns a ytm_status; on failure ytm_last_error() returns a
 *    message (thread-local).  Nothing calls exit() or abort().
 *  - Hyper-parameters are runtime values in ytm_config (the reference bakes them
 *    into #defines and compiles one kernel module per model, base.py:129-152).
 *
 * Data layouts in device memory (C = cfg->clause_count clauses held by this
 * process, K = classes, L = literals, W = literal words, P = patches):
 *  - literals   u32 [N][P][W]   bit j of word w = literal 32*w+j of a patch;
 *                               identical to the reference's encoded X
 *                               (kernel.cu:76-152, base.py:238).
 *  - state      u32 [B][C][W]   bit-sliced TA states, B = cfg->planes.  Bit j of
 *                               plane b, word w of clause c is bit b of
 *                               (state + cfg->state_offset) of literal 32*w+j.
 *                               Plane B-1 is the include mask.
 *  - weights    i32 [C][K]      clause weights (reference: f32, base.py:190).
 *  - class sums i32 [N][K].
 *  - patch_w    i32 [C][P]      patch selection counts (base.py:191).
 */
#ifndef YTM_H_
#define YTM_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int ytm_status;
#define YTM_OK 0
#define YTM_ERR_ARG 1         /* bad argument: shape, null pointer, range      */
#define YTM_ERR_CUDA 2        /* a CUDA runtime call failed                    */
#define YTM_ERR_UNSUPPORTED 3 /* configuration outside what the engine builds  */

/* Model configuration.  Filled by ytm_config_init() from the reference's
 * constructor arguments (base.py:42-125); the derived fields follow
 * base.py:94-121. */
typedef struct ytm_config {
    /* reference constructor arguments */
    int32_t clauses_per_class; /* number_of_clauses_per_class                  */
    int32_t T;                 /* threshold (THRESH, base.py:131)               */
    double s;                  /* specificity (S)                               */
    double q;                  /* min(q, n_classes) (base.py:81)                */
    int32_t dim0, dim1, dim2;
    int32_t n_classes;
    int32_t patch_dim0, patch_dim1;
    int32_t number_of_ta_states; /* MAX_TA_STATE (base.py:146)                */
    int32_t max_included_literals; /* MAX_INCLUDED_LITERALS (base.py:141)     */
    int32_t append_negated, init_neg_weights, negative_polarity;
    int32_t encode_loc, coalesced;
    uint64_t seed;
    /* derived sizes (base.py:94-121) */
    int32_t clause_banks;      /* 1 if coalesced else n_classes                 */
    int32_t clauses;           /* clause_banks * clauses_per_class (global)     */
    int32_t literals;          /* L                                             */
    int32_t words;             /* W = (L-1)/32 + 1                              */
    int32_t patches;           /* P                                             */
    int32_t half_literals;     /* L/2 (first negated literal when appended)     */
    int32_t loc_literals;      /* (D1-P1) + (D0-P0) location literals           */
    /* bit-sliced TA state encoding */
    int32_t max_state;         /* = number_of_ta_states                         */
    int32_t half_state;        /* = max_state / 2; include iff state > half     */
    int32_t planes;            /* bits per counter                              */
    int32_t state_offset;      /* stored value = state + state_offset           */
    int32_t state_top;         /* largest representable state                  */
    /* decision thresholds (fractions of 2^32) */
    uint32_t s_count_cdf[32];  /* literal mask: number of set literals among 32,
                                  Binomial(32, 1/s); entry n = floor(2^32 *
                                  P(count <= n)), saturated at 2^32 - 1     */
    uint64_t q_threshold;      /* negative-class selection, thr / 2^32          */
    uint32_t q_count_cdf[32];  /* negative-class selection drawn per (clause,
                                  sample) as a set (q_select): count of
                                  selected classes among K, Binomial(K, Q);
                                  entry n = floor(2^32 * P(count <= n)),
                                  saturated at 2^32 - 1                     */
    int32_t q_select;          /* 1: coalesced, K >= 32, K * Q <= 2 (the set is
                                  drawn at once), 0: one draw per class       */
    uint32_t run_cdf16[8][65]; /* Type Ib runs of m = 8, 16, ..., 64 events: per
                                  literal decrement count Binomial(m, 1/s);
                                  entry d = 65536 * P(count <= d) rounded to
                                  nearest, 65536 from d = m on               */
    /* clause shard held by this process */
    int32_t clause_lo;         /* first global clause index                     */
    int32_t clause_count;      /* clauses held (C above)                        */
    /* rule variants of the reference's CPU TM, pytm/base.py (0 = cutm rules;
     * set after ytm_config_init) */
    int32_t one_negative;      /* per sample: feedback for the true class, then
                                  for ONE uniformly drawn other class, no
                                  Q-selection (pytm/base.py:139-143)           */
    int32_t count_empty;       /* inference counts clauses without includes
                                  (pytm/base.py:59-67)                         */
    /* input form of the data path (set after ytm_config_init) */
    int32_t input_images;      /* 0: `lits` arguments are per-patch literal
                                  words u32 [N][P][W] (ytm_encode); 1: they
                                  are packed bit images u32 [N][image_words]
                                  (ytm_pack_images) and the patch literal words
                                  are formed on the fly where they are read
                                  (models with several patches only)          */
    int32_t image_words;       /* ceil(dim0*dim1*dim2 / 32) + 1 (one padding
                                  word)                                        */
    uint32_t run_range[8];     /* per run size: lo | hi << 16, run_cdf16
                                  entries below lo are 0 and entries from hi
                                  on are 65536 (the thresholds a draw tests
                                  lie in [lo, hi))                             */
} ytm_config;

/* Fill *cfg.  Arguments mirror BaseTM.__init__ (base.py:42-92) and its defaults
 * (base.py:60-74); max_included_literals < 0 means "None" (= literals).
 * The whole clause range is held (clause_lo = 0, clause_count = clauses). */
ytm_status ytm_config_init(ytm_config *cfg, int32_t clauses_per_class, int32_t T, double s,
                           int32_t dim0, int32_t dim1, int32_t dim2, int32_t n_classes,
                           double q, int32_t patch_dim0, int32_t patch_dim1,
                           int32_t number_of_ta_states, int32_t max_included_literals,
                           int32_t append_negated, int32_t init_neg_weights,
                           int32_t negative_polarity, int32_t encode_loc, int32_t coalesced,
                           uint64_t seed);

/* Restrict *cfg to the contiguous clause shard of `rank` out of `world`
 * processes (no reference counterpart: the reference is single-GPU). */
ytm_status ytm_config_shard(ytm_config *cfg, int32_t rank, int32_t world);

/* Scratch sizes.  op is one of the YTM_OP_* values, n the sample count of the
 * call (batch size for training). */
#define YTM_OP_ENCODE 1
#define YTM_OP_INFER 2
#define YTM_OP_TRANSFORM 3
#define YTM_OP_TRAIN 4
#define YTM_OP_TRAIN_B1 5   /* ytm_train_fit_b1 (n ignored) */
#define YTM_OP_ENCODE_THERMO 6
#define YTM_OP_TRAIN_LOOP 7  /* ytm_train_fit_batches, n = batch size */
uint64_t ytm_workspace_bytes(const ytm_config *cfg, int32_t op, int64_t n);

/* Encode raw inputs into per-patch literal words.
 * Replaces encode_batch (kernel.cu:76-152) as driven by BaseTM.encode
 * (base.py:224-263).  X: u32 [N][dim0*dim1*dim2] (any nonzero value is a 1);
 * lits: u32 [N][P][W].  workspace: ytm_workspace_bytes(cfg, YTM_OP_ENCODE, N). */
ytm_status ytm_encode(const ytm_config *cfg, const uint32_t *X, int64_t N, uint32_t *lits,
                      void *workspace, void *stream);

/* Encode raw 8-bit images without the host u32-per-bit expansion: img u8
 * [N][dim0*dim1][ch] with ch = dim2 / levels is thermometer-binarised as
 * ThermometerBinarizer(levels).binarize_rgb / binarize_gray would
 * (tm_utils/binarizer.py:5-21: bit c*levels+j of a pixel is
 * img[c] >= (j+1)*255/(levels+1)) and encoded as ytm_encode would encode the
 * binarised array.  workspace: ytm_workspace_bytes(cfg, YTM_OP_ENCODE_THERMO, N). */
ytm_status ytm_encode_thermometer(const ytm_config *cfg, const uint8_t *img, int64_t N, int32_t levels,
                                  uint32_t *lits, void *workspace, void *stream);

/* Pack raw inputs into one bit image per sample, the input form of
 * cfg->input_images = 1: X u32 [N][dim0*dim1*dim2] (any nonzero value is a 1)
 * -> img u32 [N][cfg->image_words] (bit j = input j; last word zero padding).
 * With it, convolutional models never hold the reference's per-patch literal
 * tensor (encode_batch, kernel.cu:76-152: P*W words per sample, 324 KB at
 * 32x32x24 with 10x10 patches): the data-path kernels form each patch's
 * literal words from the image where they read them.  No workspace. */
ytm_status ytm_pack_images(const ytm_config *cfg, const uint32_t *X, int64_t N, uint32_t *img, void *stream);

/* Same from raw 8-bit images, thermometer-binarised as in
 * ytm_encode_thermometer (tm_utils/binarizer.py:5-21): img u8
 * [N][dim0*dim1][ch], ch = dim2 / levels -> bits u32 [N][cfg->image_words].
 * No workspace. */
ytm_status ytm_pack_images_thermometer(const ytm_config *cfg, const uint8_t *img, int64_t N, int32_t levels,
                                       uint32_t *bits, void *stream);

/* Set every TA state of the shard to number_of_ta_states/2.
 * Replaces _reset_clauses (base.py:208-209). */
ytm_status ytm_state_init(const ytm_config *cfg, uint32_t *state, void *stream);

/* Convert flat u32 TA states [C][L] (the reference's ta_state layout,
 * base.py:189, get_state_dict base.py:561-582) into bit-sliced planes and back.
 * from_u32 saturates values above cfg->state_top; callers validate first. */
ytm_status ytm_state_from_u32(const ytm_config *cfg, const uint32_t *ta, uint32_t *state,
                              void *stream);
ytm_status ytm_state_to_u32(const ytm_config *cfg, const uint32_t *state, uint32_t *ta,
                            void *stream);

/* Include masks u32 [C][W] and include counts i32 [C] of the shard.
 * Replaces pack_clauses (kernel.cu:155-204). */
ytm_status ytm_include_mask(const ytm_config *cfg, const uint32_t *state, uint32_t *inc,
                            int32_t *num_includes, void *stream);

/* Initial clause weights i32 [C][K] of the shard.
 * Replaces init_weights (kernel.cu:46-73) via _reset_weights (base.py:211-222). */
ytm_status ytm_weights_init(const ytm_config *cfg, int32_t *weights, void *stream);

/* Inference class sums: cs[n][k] = bias[k] + sum of weights[c][k] over the
 * non-empty clauses c of the shard that match at least one patch of sample n.
 * Replaces calc_class_sums_infer_batch (kernel.cu:319-343) as driven by
 * _score_batch (base.py:375-420).  bias may be NULL (zero).  cs: i32 [N][K],
 * fully overwritten.  workspace: ytm_workspace_bytes(cfg, YTM_OP_INFER, N). */
ytm_status ytm_infer(const ytm_config *cfg, const uint32_t *state, const int32_t *weights,
                     const int32_t *bias, const uint32_t *lits, int64_t N, int32_t *cs,
                     void *workspace, void *stream);

/* Same as ytm_infer, but from include masks u32 [C][W] (the layout of
 * ytm_include_mask / the reference's packed clauses, kernel.cu:155-204)
 * instead of the bit-sliced state: used by sample-sharded inference, where
 * every rank holds a replica of all clauses' include masks.
 * workspace: ytm_workspace_bytes(cfg, YTM_OP_INFER, N). */
ytm_status ytm_infer_include(const ytm_config *cfg, const uint32_t *inc, const int32_t *weights,
                             const int32_t *bias, const uint32_t *lits, int64_t N, int32_t *cs,
                             void *workspace, void *stream);

/* Clause outputs u32 [N][C] (1 if any patch matches; empty clauses give 1).
 * Replaces transform (kernel.cu:346-368, base.py:465-502).
 * workspace: ytm_workspace_bytes(cfg, YTM_OP_TRANSFORM, N). */
ytm_status ytm_transform(const ytm_config *cfg, const uint32_t *state, const uint32_t *lits,
                         int64_t N, uint32_t *out, void *workspace, void *stream);

/* Per-patch clause outputs u32 [N][C][P] (empty clauses give 1).
 * Replaces transform_patchwise (kernel.cu:370-394, base.py:504-542). */
ytm_status ytm_transform_patchwise(const ytm_config *cfg, const uint32_t *state,
                                   const uint32_t *lits, int64_t N, uint32_t *out,
                                   void *stream);

/* Training, part 1, for a batch of B samples whose first global sample
 * counter is t0: freeze include counts, evaluate every clause of the shard on
 * every patch (training semantics: empty clause matches, dropped clause never
 * fires), pick one matching patch per (sample, clause), count it in patch_w
 * (single-patch models: ytm_train_update counts the picks),
 * and write the shard's partial class sums cs i32 [B][K] (bias added when
 * add_bias != 0).  Replaces pack_clauses + fast_eval + select_active
 * (kernel.cu:155-204, 255-316) of the per-sample loop (base.py:305-337).
 * drop: u32 [C] clause-drop mask or NULL.  workspace holds the batch's
 * selections for ytm_train_update: ytm_workspace_bytes(cfg, YTM_OP_TRAIN, B). */
ytm_status ytm_train_eval(const ytm_config *cfg, const uint32_t *state, const int32_t *weights,
                          const int32_t *bias, const uint32_t *drop, const uint32_t *lits,
                          int32_t B, uint64_t t0, int32_t add_bias, int32_t *cs,
                          int32_t *patch_w, void *workspace, void *stream);

/* Training, part 2: Type I / Type II feedback of the batch, applied clause by
 * clause in sample order with the class sums cs i32 [B][K] (summed over all
 * shards) and targets Y i32 [B][K] (+T / -T).  Replaces clause_update and
 * type1a_fb / type1b_fb / type2_fb (kernel.cu:397-613, base.py:339-357).
 * sel_override: i32 [B][C] patch picks to use instead of the ones
 * ytm_train_eval chose (-1 = clause did not fire), or NULL.  patch_w: for
 * single-patch models with up to 256 classes, ytm_train_eval leaves the
 * counting of picks (kernel.cu:305) to this call, which adds them here.
 * workspace: the one ytm_train_eval filled for this batch; without
 * sel_override this call reads the picks from it (single-patch models: the
 * clause outputs, kept there clause by clause).  Limits: at most 65,535
 * classes and 32,767 samples per batch; for batches above 64 samples, at
 * most about 700 classes (a chunk's event list lives in shared memory);
 * beyond them YTM_ERR_UNSUPPORTED. */
ytm_status ytm_train_update(const ytm_config *cfg, uint32_t *state, int32_t *weights,
                            const int32_t *cs, const int32_t *Y, const uint32_t *drop,
                            const uint32_t *lits, int32_t B, uint64_t t0,
                            const int32_t *sel_override, int32_t *patch_w, void *workspace,
                            void *stream);

/* ytm_train_update that also adds measurement counts of its feedback into
 * counters u64[6] (device memory, accumulated, never cleared here):
 * [0] literal-word operations applied (one per word for each single event
 * and for each piece of a Type Ib run), [1] Philox4x32-7 calls made for
 * literal masks and run counts, [2] state words streamed (each a read and a
 * write of every bit plane), [3] feedback events, [4] Philox4x32-7 calls
 * made for the decisions of the active (sample, class) pairs, [5] run-count
 * thresholds tested (each a 16-plane carry chain over 32 literals).  Measurement variant with no reference
 * counterpart; counters == NULL gives ytm_train_update. */
ytm_status ytm_train_update_counted(const ytm_config *cfg, uint32_t *state, int32_t *weights,
                                    const int32_t *cs, const int32_t *Y, const uint32_t *drop,
                                    const uint32_t *lits, int32_t B, uint64_t t0,
                                    const int32_t *sel_override, int32_t *patch_w, void *workspace,
                                    uint64_t *counters, void *stream);

/* Train on samples 0..N-1 one at a time, in order: the reference's
 * per-sample loop (_fit, base.py:305-357: pack_clauses, fast_eval,
 * select_active, clause_update per sample).  Same result as ytm_train_eval +
 * ytm_train_update with B = 1 for each sample, t = t0 + i, but one fused
 * launch per sample (feedback of sample i and evaluation of sample i+1) queued
 * from C++.  Up to 2048 patches; one process (the class sums are not
 * all-reduced).  lits u32 [N][P][W], Y i32
 * [N][K].  workspace: ytm_workspace_bytes(cfg, YTM_OP_TRAIN_B1, 0). */
ytm_status ytm_train_fit_b1(const ytm_config *cfg, uint32_t *state, int32_t *weights, const int32_t *bias,
                            const uint32_t *drop, const uint32_t *lits, const int32_t *Y, int64_t N,
                            uint64_t t0, int32_t *patch_w, void *workspace, void *stream);

/* NCCL communicator for clause-sharded training (no reference counterpart:
 * the reference is single-GPU).  Rank 0 makes the 128-byte id, every rank
 * passes it to ytm_nccl_comm_init (the caller distributes it). */
ytm_status ytm_nccl_unique_id(uint8_t *id_out);
ytm_status ytm_nccl_comm_init(const uint8_t *id_in, int32_t rank, int32_t world, void **comm_out);
ytm_status ytm_nccl_comm_destroy(void *comm);

/* Train on samples 0..N-1 in mini-batches of B (the last one ragged), all
 * queued on `stream` from C: per batch ytm_train_eval, the int32 sum of the
 * class sums over the clause shards (ncclAllReduce on `comm`; NULL for one
 * process), ytm_train_update.  The reference's _fit loop (base.py:305-357)
 * with batch B.  add_bias: add the bias on this shard (one shard only).
 * workspace: ytm_workspace_bytes(cfg, YTM_OP_TRAIN_LOOP, B). */
ytm_status ytm_train_fit_batches(const ytm_config *cfg, uint32_t *state, int32_t *weights, const int32_t *bias,
                                 const uint32_t *drop, const uint32_t *lits, const int32_t *Y, int64_t N,
                                 int32_t B, uint64_t t0, int32_t add_bias, int32_t *patch_w, void *comm,
                                 void *peer_ar, void *workspace, void *stream);

/* One-shot int32 all-reduce over NVLink peer memory for the ranks of one
 * node (no reference counterpart).  create: allocate this rank's buffer (room
 * for max_n values) and return its 64-byte CUDA IPC handle; open: map every
 * rank's buffer from the handles (world x 64 bytes, rank order); allreduce:
 * sum data[0..n) over the ranks in place on `stream` (every rank must call it
 * the same number of times); a rank that never arrives is reported after
 * `limit` spin iterations (<= 0: default, tens of seconds) through status
 * (0 = all calls since the last status read completed, else 1 + the index
 * of the missing peer; reading it synchronises the device and clears it) and
 * the call leaves data unchanged: the caller must treat a non-zero status as
 * fatal for the training run.  ytm_train_fit_batches uses it when peer_ar is
 * given (instead of comm). */
ytm_status ytm_peer_ar_create(int32_t rank, int32_t world, int64_t max_n, void **ctx_out, uint8_t *handle_out);
ytm_status ytm_peer_ar_open(void *ctx, const uint8_t *handles);
ytm_status ytm_peer_allreduce_i32(void *ctx, int32_t *data, int64_t n, int64_t limit, void *stream);
ytm_status ytm_peer_ar_status(void *ctx, int32_t *status_out);
ytm_status ytm_peer_ar_destroy(void *ctx);

/* Read back the patch picks of the last ytm_train_eval on this workspace:
 * sel i32 [B][C] (-1 = not fired).  Device-to-device copy on `stream`. */
ytm_status ytm_train_selection(const ytm_config *cfg, int32_t B, const void *workspace,
                               int32_t *sel, void *stream);

/* Inference without a workspace, for callers that cannot allocate device
 * memory (embedders whose device memory is handed out by another runtime,
 * services that forbid allocation after start-up).  No counterpart in the
 * reference.
 * Same inputs and output as ytm_infer; scratch comes from a fixed array of
 * YTM_NOALLOC_SCRATCH_BYTES that every GPU loading the library keeps until
 * exit.  Calls needing more scratch (include counts + N * ceil(C/32) words of
 * fired bits) fail with YTM_ERR_ARG: split N.  The first call on a device
 * looks up the array's device address and should precede any stream capture;
 * the address stays cached, so do not call this after cudaDeviceReset of that
 * device.  Calls share the array: calls that overlap on the GPU race. */
#define YTM_NOALLOC_SCRATCH_BYTES (16u << 20)
ytm_status ytm_infer_noalloc(const ytm_config *cfg, const uint32_t *state, const int32_t *weights,
                             const int32_t *bias, const uint32_t *lits, int64_t N, int32_t *cs,
                             void *stream);

/* Executed work of the dense clause match (inference and transforms of the
 * current device) since the previous call: out[0] = 64 x 64 (row, clause)
 * tiles, out[1] = 32-word chunks they processed (a tile stops after the chunk
 * at which every one of its pairs has a violation).  Reads and clears the
 * counts; synchronizes the stream.  Measurement entry point with no
 * reference counterpart. */
ytm_status ytm_match_counters(uint64_t *out, void *stream);

/* Message of the last failing call on this thread ("" if none). */
const char *ytm_last_error(void);

/* Library version string. */
const char *ytm_version(void);

/* sizeof(ytm_config) as compiled into the library (bindings check their
 * mirror of the struct against it). */
int32_t ytm_config_size(void);

#ifdef __cplusplus
}
#endif

#endif /* YTM_H_ */
