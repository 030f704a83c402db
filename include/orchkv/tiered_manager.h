/*
 * tiered_manager.h — scheduler C ABI (tm_*) of the B200 implementation.
 *
 * Every tm_* entry point of the reference is kept with the same name,
 * arguments, return values and error behaviour
 * (src/scheduler/tiered_manager.h:44-222).  Per-slot tracker and classifier
 * state (src/scheduler/attention_tracker.h:23-30,
 * src/scheduler/hotcold_classifier.h:55-60) lives in GPU memory; the
 * O(capacity) sweeps (step_done, classification), threshold selection and
 * prefetch selection run as CUDA kernels on the manager's stream.
 *
 * The entry points marked "B200" below are new: tensor-level reporting and
 * batched selection that the reference does one block at a time through
 * Python (python/orchkv/fast_kvcache_manager.py:221-341).
 */
#ifndef ORCHKV_TIERED_MANAGER_H
#define ORCHKV_TIERED_MANAGER_H

#include <pthread.h>
#include "kv_types.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- caller-owned block record: layout of src/core/kv_block.h:22-52 ------ */
typedef struct kv_block {
    uint64_t         block_id;
    uint64_t         request_id;
    uint16_t         layer_id;
    uint16_t         head_id;
    uint32_t         token_start;
    uint16_t         token_count;
    uint16_t         _pad0;
    StorageTier      tier;
    void            *data_ptr;
    uint64_t         persistent_offset;
    float            hotness;
    uint64_t         last_access_step;
    uint32_t         access_count;
    KVBlockState     state;
    uint8_t          flags;
    pthread_rwlock_t lock;
    struct kv_block *prev;
    struct kv_block *next;
} kv_block_t;

/* ---- classifier (src/scheduler/hotcold_classifier.h:38-107) ------------- */
typedef enum { HEAT_HOT = 0, HEAT_WARM = 1, HEAT_COLD = 2 } HeatLevel;

#define HCC_DECAY_TABLE_MAX 512

typedef struct hcc_params {
    float alpha, beta, gamma;
    float recency_tau;
    float threshold_hot;
    float threshold_warm;
} hcc_params_t;

static inline void hcc_params_default(hcc_params_t *p)
{
    p->alpha = 0.5f; p->beta = 0.3f; p->gamma = 0.2f;
    p->recency_tau = 50.0f;
    p->threshold_hot = 0.5f; p->threshold_warm = 0.2f;
}

typedef struct hcc_stats {
    uint32_t n_hot, n_warm, n_cold, n_attn_sink;
    float    avg_hotness, max_hotness, min_hotness;
} hcc_stats_t;

/* ---- adaptive threshold (src/scheduler/adaptive_threshold.h:62-83) ------ */
typedef struct athresh_params {
    float  threshold_hot, threshold_warm;
    float  min_hot, max_hot;
    float  min_warm, max_warm;
    float  gpu_hwm, gpu_lwm;
    float  dram_hwm, dram_lwm;
    float  adjust_step;
    double cooldown_sec;
} athresh_params_t;

static inline void athresh_params_default(athresh_params_t *p)
{
    p->threshold_hot = 0.5f;  p->threshold_warm = 0.2f;
    p->min_hot = 0.2f;        p->max_hot = 0.9f;
    p->min_warm = 0.05f;      p->max_warm = 0.5f;
    p->gpu_hwm = 0.9f;        p->gpu_lwm = 0.7f;
    p->dram_hwm = 0.9f;       p->dram_lwm = 0.7f;
    p->adjust_step = 0.02f;   p->cooldown_sec = 0.5;
}

/* ---- prefetch + migration stats (prefetch_scheduler.h:45-52,
 *      migration_engine.h:36-72) ------------------------------------------- */
typedef struct prefetch_stats {
    uint64_t total_scanned, total_enqueued, total_dispatched;
    uint64_t prefetch_hits, prefetch_wasted;
    float    hit_rate;
} prefetch_stats_t;

typedef enum {
    MIGRATE_DEMOTE_GPU2DRAM   = 0,
    MIGRATE_DEMOTE_DRAM2STOR  = 1,
    MIGRATE_DEMOTE_GPU2STOR   = 2,
    MIGRATE_PROMOTE_STOR2DRAM = 3,
    MIGRATE_PROMOTE_DRAM2GPU  = 4,
    MIGRATE_PROMOTE_STOR2GPU  = 5,
    MIGRATE_OP_COUNT          = 6,
} MigrateOp;

typedef int (*mig_transfer_fn)(kv_block_t *blk, void *dst_buf, size_t size,
                               MigrateOp op, void *ctx);

typedef struct mig_stats {
    uint64_t op_count[MIGRATE_OP_COUNT];
    uint64_t op_bytes[MIGRATE_OP_COUNT];
    uint64_t op_errors;
    uint64_t blocks_migrated;
} mig_stats_t;

/* ---- manager configuration (src/scheduler/tiered_manager.h:39-80) ------- */
typedef void *(*tm_alloc_fn)(size_t size, StorageTier tier, void *ctx);
typedef void  (*tm_free_fn)(void *ptr, StorageTier tier, void *ctx);

typedef struct tm_config {
    uint32_t         tracker_capacity;
    float            ema_lambda;
    hcc_params_t     hcc_params;
    athresh_params_t athresh_params;
    float            w_heat, w_lru;
    uint32_t         tokens_per_block;
    uint32_t         prefetch_budget;
    float            threshold_to_gpu;
    float            threshold_to_dram;
    mig_transfer_fn  transfer_fn;
    void            *transfer_ctx;
    tm_alloc_fn      alloc_fn;
    tm_free_fn       free_fn;
    void            *alloc_ctx;
    size_t           block_data_size;
    uint32_t         schedule_interval_us;
    uint32_t         demote_batch_size;
    uint32_t         prefetch_batch_size;
    uint32_t         max_blocks;
    bool             auto_schedule;
} tm_config_t;

void tm_config_default(tm_config_t *cfg);

typedef struct tm_stats {
    uint64_t         schedule_cycles;
    uint64_t         gpu_demotes;
    uint64_t         dram_demotes;
    uint64_t         prefetches_dispatched;
    float            gpu_used_ratio;
    float            dram_used_ratio;
    hcc_stats_t      hcc_stats;
    prefetch_stats_t prefetch_stats;
    mig_stats_t      migration_stats;
} tm_stats_t;

/* The manager handle.  Callers allocate it (on the stack or heap) exactly as
 * with the reference; the state lives behind `impl` (host object + GPU
 * arrays), so only the size differs from the reference struct. */
typedef struct tiered_manager {
    void    *impl;
    uint64_t reserved[7];
} tiered_manager_t;

/* ---- reference entry points --------------------------------------------- */
int       tm_init(tiered_manager_t *m, const tm_config_t *cfg);
void      tm_destroy(tiered_manager_t *m);
int       tm_register_block(tiered_manager_t *m, kv_block_t *blk);
void      tm_unregister_block(tiered_manager_t *m, kv_block_t *blk);
void      tm_notify_attn(tiered_manager_t *m, uint64_t block_id, float attn_weight);
void      tm_notify_access(tiered_manager_t *m, kv_block_t *blk);
void      tm_step_done(tiered_manager_t *m);
void      tm_schedule_once(tiered_manager_t *m);
int       tm_start(tiered_manager_t *m);
void      tm_stop(tiered_manager_t *m);
void      tm_set_usage(tiered_manager_t *m, float gpu_used_ratio, float dram_used_ratio);
void      tm_set_policy(tiered_manager_t *m, float alpha, float beta, float gamma);
float     tm_get_block_score(const tiered_manager_t *m, uint64_t block_id);
HeatLevel tm_get_block_heat(const tiered_manager_t *m, uint64_t block_id);
void      tm_get_stats(const tiered_manager_t *m, tm_stats_t *out);

/* ---- B200: stream binding and state access ------------------------------ */

/* Run the manager's GPU work on `stream` (a cudaStream_t; NULL = the
 * manager's own stream, which is ordered with the legacy default stream).
 * Replaces tm_notify_attn's implicit ordering. */
int       tm_set_stream(tiered_manager_t *m, void *stream);
/* Block until all GPU work queued by the manager has finished. */
int       tm_sync(tiered_manager_t *m);
uint32_t  tm_capacity(const tiered_manager_t *m);
uint64_t  tm_current_step(const tiered_manager_t *m);
/* Per-block tier as seen by the selector; binding-owned records only
 * (bindings/orchkv_pybind.cpp:308-320 `tm_set_block_tier`). */
int       tm_set_block_tier_id(tiered_manager_t *m, uint64_t block_id, int tier);
/* Copy per-slot state to host arrays of tm_capacity() entries (any pointer may
 * be NULL).  last_hit uses UINT64_MAX for "never hit". */
int       tm_read_state(tiered_manager_t *m, float *sum, float *ema,
                        uint32_t *hits, uint64_t *last_hit, uint8_t *t_active,
                        float *hotness, uint8_t *heat, uint8_t *c_active);

/* ---- B200: tensor-level scoring ----------------------------------------- *
 *
 * Reduce per-token attention probabilities to per-block attention mass and
 * record it as tm_notify_attn would, for every block in one launch.
 *
 *   probs      fp32 [n_rows][n_q_heads][row_len]  (row = request*L+layer,
 *              decode q_len = 1)
 *   lens       uint32 [n_rows] valid tokens per row, or NULL (= row_len)
 *   block_ids  uint32 [n_rows][n_kv_heads][ceil(row_len/tpb)]: the block
 *              id receiving the mass of (row, kv head, token block);
 *              0xFFFFFFFF = none.  Ids may repeat or share a tracker slot
 *              (slot = id & (capacity - 1)), e.g. one block id per token
 *              position shared by every layer's row: such reports apply in
 *              (row, kv head, block) order, as that many tm_notify_attn calls
 *              in that order would (attn_tracker_update_batch,
 *              src/scheduler/attention_tracker.c:95-118).  A device pass over
 *              the ids detects shared slots; only a call that has them takes
 *              the slower ordered apply.
 *
 * mass(row,h,b) = sum over the n_q_heads/n_kv_heads query heads of KV group h
 * and the tokens of block b of probs.  A block's per-step sum, max and last
 * hit then update exactly as attn_tracker_update
 * (src/scheduler/attention_tracker.c:27-33,75-92).  Each array may be in
 * device memory (read in place) or in host memory, pinned or pageable
 * (copied once to the device on the manager's stream).  Asynchronous: a
 * pageable host array may be reused when the call returns (the copy has
 * taken it by then); a pinned one is read by the copy engine later and must
 * stay unchanged until the manager's stream has run the call (tm_sync). */
int tm_report_attn_probs(tiered_manager_t *m, const float *probs,
                         uint32_t n_rows, uint32_t n_q_heads, uint32_t n_kv_heads,
                         uint32_t row_len, uint32_t tokens_per_block,
                         const uint32_t *lens, const uint32_t *block_ids);

/* B200: device timing of tm_report_attn_probs, opt-in (on != 0 starts it):
 * tm_last_report_times gives the last call's duplicate-slot pass, score
 * kernel and ordered pass in ms (waiting for them); ORCHKV_ERR_STATE while
 * profiling is off.  No counterpart in the reference. */
int tm_profile_reports(tiered_manager_t *m, int on);
int tm_last_report_times(tiered_manager_t *m, float *mark_ms, float *score_ms,
                         float *ordered_ms);

/* B200: upload a host input of a later report call now, on the manager's
 * own copy stream, so the copy overlaps whatever runs meanwhile (the current
 * step's migrations, say).  The next tm_report_attn_probs /
 * tm_report_attn_ranges call given exactly this host pointer and byte count
 * for one of its arrays reads the uploaded copy (waiting for the upload on
 * the device) instead of copying the array then.  The caller keeps the host
 * bytes unchanged until that call; pinned memory makes the upload fully
 * asynchronous.  Two uploads may wait for their reports at once, taken
 * oldest first; a third returns ORCHKV_ERR_STATE.  host = NULL drops every
 * waiting upload.  No counterpart in the reference (its reports arrive as
 * per-block host floats). */
int tm_stage_input_async(tiered_manager_t *m, const void *host, size_t bytes);

/* The original KVCacheManager's per-block report in one call
 * (python/orchkv/kvcache_manager.py:317-347: one float(avg[:, s:e].sum()) and
 * one tm_report_attn per block).
 *
 *   avg        fp32 [heads][kv_len]: the attention weights averaged over batch
 *              and query positions (the manager's own mean)
 *   starts, ends, block_ids   uint32 [n]: block i covers tokens
 *              [starts[i], ends[i]) and reports to block_ids[i]
 *
 * Block i records sum over h and t in [starts[i], min(ends[i], kv_len)) of
 * avg[h][t] as tm_notify_attn would; a block whose range is empty is not
 * reported.  Ids that share a tracker slot apply in list order.  Each array
 * may be in device or host memory (host arrays are copied once on the
 * manager's stream).  Asynchronous; host arrays may be reused as for
 * tm_report_attn_probs (pageable ones on return, pinned ones after tm_sync). */
int tm_report_attn_ranges(tiered_manager_t *m, const float *avg, uint32_t heads,
                          uint32_t kv_len, const uint32_t *starts, const uint32_t *ends,
                          const uint32_t *block_ids, uint32_t n);

/* Report a batch of (id, weight) pairs already on the device, applied in
 * array order per block (attn_tracker_update_batch semantics,
 * src/scheduler/attention_tracker.c:95-118), repeated ids and ids sharing a
 * tracker slot included. */
int tm_report_attn_batch_dev(tiered_manager_t *m, const uint32_t *block_ids,
                             const float *weights, uint32_t n);

/* The vLLM attention hook's reduction and reports in one call
 * (python/orchkv/vllm_integration/attention_hook.py:105-115,118-140,155-189:
 * _blockwise_reduce, then tm_report_attn per (head, block)), without the
 * device-to-host copy and the per-block calls.
 *
 *   weights    device [batch][heads][q_len][kv_len], contiguous, of dtype
 *              0 = fp16, 1 = bf16, 2 = fp32 (the softmax output)
 *   scores     device fp32 [heads][n_blocks], n_blocks = ceil(kv_len /
 *              block_size), receives score(h, b) = the mean of weights over
 *              batch, q_len and the block_size positions of block b, positions
 *              at or past kv_len counting as zeros (the hook pads the last
 *              block), computed in fp32 and rounded to the weights' type (the
 *              type a mean over such a tensor returns)
 *   block_ids  device uint32 [heads][n_blocks]: the id each (h, b) is
 *              reported to, 0xFFFFFFFF = none; or NULL to compute the scores
 *              only.  Reports are recorded as tm_notify_attn would, the heads
 *              of one block b in order h = 0, 1, ...: ids of one block may
 *              share a tracker slot (the hook's block-table mode gives every
 *              head the same id); ids of different blocks must map to
 *              different slots (slot = id & (capacity - 1)).
 *
 * block_size <= 4096.  Asynchronous. */
int tm_report_attn_blockmean(tiered_manager_t *m, const void *weights, int dtype,
                             uint32_t batch, uint32_t heads, uint32_t q_len, uint32_t kv_len,
                             uint32_t block_size, const uint32_t *block_ids, float *scores);

/* step_done + classification fused into one sweep: equivalent to
 * tm_step_done followed by the classification pass of tm_schedule_once
 * (src/scheduler/tiered_manager.c:205-213,318), without the threshold update,
 * demotion or prefetch phases.  Asynchronous. */
int tm_step_and_classify(tiered_manager_t *m);

/* Coldest-k selection.  Candidates: registered blocks whose tier is GPU,
 * not flagged PIN or ATTN_SINK and not MIGRATING.  Order: ascending hotness,
 * ties by ascending block id (the FastKVCacheManager order,
 * python/orchkv/fast_kvcache_manager.py:307-321).  Writes min(k, #candidates)
 * block ids in ascending id order to out_ids (device, capacity >= k) and the
 * count to *out_count (device uint32).  Asynchronous. */
int tm_select_victims(tiered_manager_t *m, uint32_t k, uint32_t *out_ids,
                      uint32_t *out_count);

/* Same, restricted further to slots whose eligible[slot] (device uint8,
 * tm_capacity() entries, slot = block_id & (capacity - 1)) is non-zero: for
 * callers that keep their own evicted set, as FastKVCacheManager does
 * (python/orchkv/fast_kvcache_manager.py:300-318). */
int tm_select_victims_masked(tiered_manager_t *m, uint32_t k, const uint8_t *eligible,
                             uint32_t *out_ids, uint32_t *out_count);

/* Same, with k = floor(frac * #candidates) computed on the device. */
int tm_select_victims_frac(tiered_manager_t *m, float frac, uint32_t *out_ids,
                           uint32_t *out_count, uint32_t max_out);

/* Prefetch selection (src/scheduler/prefetch_scheduler.c:131-228 rules):
 * blocks not on GPU (and not NONE) with ema >= th_gpu (priority ema) or
 * ema >= th_dram and tier != DRAM (priority ema/2); the top k by priority,
 * ties by ascending id, written in ascending id order.  Asynchronous. */
int tm_select_prefetch(tiered_manager_t *m, uint32_t k, float th_gpu,
                       float th_dram, uint32_t *out_ids, uint32_t *out_count);

/* Coldest-k selection that allocates no memory.  No counterpart in the
 * reference: it is for callers that cannot call cudaMalloc while they run
 * (engines that reserve device memory for their own allocator up front,
 * paths that must not take the CUDA allocator's locks).  Same ordering and
 * output as tm_select_victims, over a caller's arrays: values[i] (device f32)
 * is eligible where eligible[i] (device u8) is non-zero; the min(k, #eligible)
 * winners go to out_ids in ascending index order, their number to *out_count
 * (device u32).  n is at most 1,048,576 (ORCHKV_ERR_INVALID beyond, with a
 * message).  Scratch is one static device array of ~4.1 MB in each GPU that
 * loads the library, kept until exit: the first call on a device looks its
 * address up (make that first call before any stream capture) and later
 * calls reuse it, looking it up again only when the device's context was
 * replaced (after cudaDeviceReset); every call shares the array, so calls
 * that overlap on the GPU race.  Asynchronous on
 * `stream` (a cudaStream_t, NULL = default stream). */
int orchkv_select_coldest_noalloc(const float *values, const uint8_t *eligible,
                                  uint32_t n, uint32_t k, uint32_t *out_ids,
                                  uint32_t *out_count, void *stream);

/* Threshold controller state (the fields the reference binding reads from
 * m->threshold, bindings/orchkv_pybind.cpp:408-411). */
int tm_get_threshold_state(const tiered_manager_t *m, float *threshold_hot,
                           float *threshold_warm, uint64_t *adjustments_up,
                           uint64_t *adjustments_down);

/* ---- B200: multi-GPU selection ------------------------------------------
 *
 * One rank per GPU, KV pool sharded by KV head.  With a communicator set,
 * every selection's k (or fraction) refers to the union of all ranks' blocks:
 * the per-pass key histograms are summed with ncclAllReduce and boundary ties
 * are split in (rank, block id) order via ncclAllGather, so each rank selects
 * exactly its share of the global order.  Communicator: orchkv_comm_create
 * (one rank takes the same path: its exchanges are local copies and its
 * picks those of a manager without one); at most 48 ranks (else
 * ORCHKV_ERR_INVALID).  NULL detaches. */
int   orchkv_comm_unique_id(unsigned char *out128);
void *orchkv_comm_create(int rank, int world, const unsigned char *id128, double timeout_s);
int   orchkv_comm_destroy(void *comm);
int   orchkv_comm_allreduce_u32(void *comm, const uint32_t *send, uint32_t *recv,
                                uint32_t n, void *stream);
/* Device time of the communicator's exchanges since the previous call (the
 * first 64 timed, waits for slower ranks included) and their number; resets. */
int   orchkv_comm_exchange_time(void *comm, float *ms, uint32_t *calls);
int   tm_set_comm(tiered_manager_t *m, void *comm);

#ifdef __cplusplus
}
#endif
#endif /* ORCHKV_TIERED_MANAGER_H */
