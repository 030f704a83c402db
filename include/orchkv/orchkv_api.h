/*
 * orchkv_api.h — data-plane C ABI (orchkv_*) of the B200 implementation.
 *
 * The reference entry points (src/api/orchkv_api.h:28-121) keep their names,
 * arguments and return codes.  Slab layout is the reference's
 * (src/api/orchkv_api.cu:8-18): one slab per (request, layer, KV head, token
 * block), K rows in the first half, V rows in the second, token t at
 * t*d_head*dtype_size within each half.
 *
 * What differs inside: the GPU slab pool, the pinned host-DRAM slab pool, the
 * free stacks and every block's location live in GPU-visible memory and are
 * changed only by CUDA kernels, so per-block calls and batched calls share one
 * state.  Per-block calls are one small kernel plus a stream synchronisation
 * (the reference issues one cudaMemcpyAsync + cudaStreamSynchronize per slab
 * half).  Host pointers passed to prefill/append may be pageable, pinned, or
 * device pointers (detected with cudaPointerGetAttributes).
 *
 * Entry points marked "B200" are new batched forms of the per-block calls.
 */
#ifndef ORCHKV_API_H
#define ORCHKV_API_H

#include <pthread.h>
#include "kv_types.h"
#include "tiered_manager.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct kv_request_ctx kv_request_ctx_t;   /* opaque request handle */

/* Pool snapshots returned by the accessors (fields as in
 * src/tiered_store/gpu_tier.h:10-20 and dram_tier.h:10-20; free_stack points
 * to a host copy refreshed at each accessor call). */
typedef struct gpu_tier {
    int             device_id;
    void           *pool_base;
    size_t          pool_size;
    size_t          slab_size;
    uint32_t        total_slabs;
    uint32_t        used_slabs;
    uint32_t       *free_stack;
    uint32_t        free_top;
    pthread_mutex_t lock;
} gpu_tier_t;

typedef struct dram_tier {
    void           *pool_base;
    size_t          pool_size;
    size_t          slab_size;
    uint32_t        total_slabs;
    uint32_t        used_slabs;
    uint32_t       *free_stack;
    uint32_t        free_top;
    bool            is_pinned;
    pthread_mutex_t lock;
} dram_tier_t;

/* The file tier's snapshot (fields as in src/tiered_store/orchfs_tier.h:40-51;
 * counters since orchkv_init: one write per slab written to a request's file,
 * one read per slab read back, as src/api/orchkv_api.cu:453,496 record them,
 * batched calls counting each slab). */
typedef struct orchfs_tier {
    bool            initialized;
    char            base_dir[256];
    size_t          slab_size;
    uint64_t        total_writes;
    uint64_t        total_reads;
    uint64_t        bytes_written;
    uint64_t        bytes_read;
    pthread_mutex_t lock;
} orchfs_tier_t;

static inline uint64_t orchfs_tier_writes(const orchfs_tier_t *t) { return t->total_writes; }
static inline uint64_t orchfs_tier_reads(const orchfs_tier_t *t) { return t->total_reads; }

/* ---- reference entry points --------------------------------------------- */
int  orchkv_init(const orchkv_config_t *config);
int  orchkv_shutdown(void);
bool orchkv_is_initialized(void);

kv_request_ctx_t *orchkv_request_create(uint64_t request_id, uint32_t n_layers,
                                        uint32_t n_kv_heads);
int  orchkv_request_destroy(kv_request_ctx_t *ctx);

/* k_data / v_data: [n_kv_heads][seq_len][d_head] of dtype. */
int  orchkv_prefill(kv_request_ctx_t *ctx, uint32_t layer_id, const void *k_data,
                    const void *v_data, uint32_t seq_len);
/* k_token / v_token: [n_kv_heads][d_head] of dtype. */
int  orchkv_append_token(kv_request_ctx_t *ctx, uint32_t layer_id,
                         const void *k_token, const void *v_token);
/* Promotes DRAM/storage blocks to GPU first; returns device pointers to the K
 * and V halves of the slab. */
int  orchkv_get_kv_block(kv_request_ctx_t *ctx, uint32_t layer_id, uint32_t head_id,
                         uint32_t block_idx, void **k_out, void **v_out);
int  orchkv_evict_to_dram(kv_request_ctx_t *ctx, uint32_t layer_id,
                          uint32_t head_id, uint32_t block_idx);
int  orchkv_promote_to_gpu(kv_request_ctx_t *ctx, uint32_t layer_id,
                           uint32_t head_id, uint32_t block_idx);
int  orchkv_evict_to_storage(kv_request_ctx_t *ctx, uint32_t layer_id,
                             uint32_t head_id, uint32_t block_idx);
int  orchkv_promote_from_storage(kv_request_ctx_t *ctx, uint32_t layer_id,
                                 uint32_t head_id, uint32_t block_idx);
int  orchkv_evict_cold(kv_request_ctx_t *ctx, uint32_t layer_id,
                       uint32_t head_id, uint32_t block_idx);
void orchkv_storage_flush(void);
int  orchkv_get_stats(orchkv_stats_t *stats);
gpu_tier_t  *orchkv_gpu_tier(void);
dram_tier_t *orchkv_dram_tier(void);
orchfs_tier_t *orchkv_orchfs_tier(void);   /* snapshot refreshed at each call */

/* ---- B200 ------------------------------------------------------------------ */

/* Extra sizing not present in orchkv_config_t (kept out of that struct so its
 * layout stays the reference's).  Zero fields take defaults. */
typedef struct orchkv_config_ext {
    uint32_t max_blocks;      /* block-id space; default gpu_slabs + dram_slabs
                                 rounded up to a power of two                  */
    uint32_t max_requests;    /* concurrent requests; default 4096             */
    uint64_t table_entries;   /* block-table entries for all requests; default
                                 max_blocks * 2                                 */
    uint32_t staging_mb;      /* device staging for batched evicts, in MiB;
                                 default 768 (three 256 MiB slots).  A swap
                                 overlaps its evict and promote only when the
                                 whole evict fits.                             */
    uint32_t reserved[11];
} orchkv_config_ext_t;

int  orchkv_init_ext(const orchkv_config_t *config, const orchkv_config_ext_t *ext);

/* All data-plane GPU work runs on this stream (cudaStream_t; NULL restores
 * the library's own stream, which is ordered with the legacy default
 * stream). */
int  orchkv_set_stream(void *stream);
int  orchkv_sync(void);

/* Block ids of the data plane become slots of `tm` (tm capacity must cover
 * max_blocks): new blocks register themselves, migrations keep the
 * scheduler's tier view current, destroyed requests unregister. */
int  orchkv_attach_scheduler(tiered_manager_t *tm);

/* orchkv_append_token for every (request, layer) pair, in request-major then
 * layer order, as one launch sequence.  All requests must share n_layers and
 * n_kv_heads.  k/v: [n][n_layers][n_kv_heads][d_head] of dtype, device or
 * host memory.  All-or-nothing: ERR_TIER_FULL if the pools cannot hold the
 * new blocks, ERR_STATE if some last block is not on the GPU. */
int  orchkv_append_token_batch(kv_request_ctx_t *const *ctxs, uint32_t n,
                               const void *k, const void *v);

/* Batched orchkv_evict_to_dram / orchkv_promote_to_gpu over a device list of
 * block ids, with exactly the per-block semantics applied in list order:
 * blocks in the wrong tier (or pinned, for evict) are skipped, as are
 * repeats of an id already listed and ids outside the block-id space; once
 * the destination pool is empty the rest fail with TIER_FULL.  `count` (device
 * uint32*) may be NULL to use max_n.  `result` (device uint32[2], may be NULL)
 * receives {migrated, skipped}.  Asynchronous. */
int  orchkv_evict_batch_to_dram(const uint32_t *block_ids, const uint32_t *count,
                                uint32_t max_n, uint32_t *result);
int  orchkv_promote_batch_to_gpu(const uint32_t *block_ids, const uint32_t *count,
                                 uint32_t max_n, uint32_t *result);

/* B200: orchkv_evict_to_storage / orchkv_promote_from_storage /
 * orchkv_evict_cold over a host list of n (layer, head, block) triples of one
 * request (lhb[3*i .. 3*i+2]), with the per-block semantics applied in list
 * order: entries not on the source tier (DRAM; storage; GPU for
 * evict_cold), pinned (evicts), repeated or naming no block are skipped, and
 * a promote that finds the DRAM pool empty skips the rest.  File I/O goes in
 * offset order; entries at consecutive offsets of the reference's file layout
 * move in one pwritev / preadv of up to 1 MiB straight from / into their
 * DRAM slabs.  result (host uint32[2], may be NULL) = {moved, skipped}.
 * Synchronous.  ORCHKV_ERR_IO when a write or read fails: no entry of the
 * call is committed (the file may hold part of the data). */
int  orchkv_evict_batch_to_storage(kv_request_ctx_t *ctx, const uint32_t *lhb, uint32_t n,
                                   uint32_t *result);
int  orchkv_promote_batch_from_storage(kv_request_ctx_t *ctx, const uint32_t *lhb,
                                       uint32_t n, uint32_t *result);
int  orchkv_evict_cold_batch(kv_request_ctx_t *ctx, const uint32_t *lhb, uint32_t n,
                             uint32_t *result);

/* Device-side timing of the last batched evict / promote (synchronises):
 * pack_ms sums the pack kernels of a staged (copy-engine) evict, pack_bytes
 * are the bytes they read and wrote, chunks the staging slots used (0 when the
 * fused zero-copy kernel ran instead); promote_ms is the last promote
 * kernel's duration. */
int  orchkv_last_migration_profile(float *pack_ms, unsigned long long *pack_bytes,
                                   uint32_t *chunks, float *promote_ms);

/* Per-chunk device time of the last staged evict's pack kernels, in chunk
 * order: ms[c] for c < min(*chunks, max_chunks) (synchronises).  *chunks = the
 * staging slots the evict used (0 when the zero-copy kernel ran alone). */
int  orchkv_last_pack_chunks(float *ms, uint32_t max_chunks, uint32_t *chunks);

/* Device time of each unpack launch of the last staged promote (or swap), in
 * launch order, and the bytes each moved (the ring read plus the GPU slab
 * write): ms[u], bytes[u] for u < min(*launches, max_launches) (synchronises).
 * *launches = 0 when the promote ran zero-copy only. */
int  orchkv_last_unpack_chunks(float *ms, unsigned long long *bytes, uint32_t max_launches,
                               uint32_t *launches);

/* How the last staged evict reached the DRAM tier: `runs` = runs of
 * consecutive DRAM slabs it filled, `ce_copies` = copy-engine copies issued
 * (one per run of at least 1 MiB, split at staging-slot boundaries),
 * `zero_copy_slabs` = blocks in shorter runs, written by a kernel straight
 * into mapped host memory.  All 0 when the zero-copy kernel ran alone. */
int  orchkv_last_evict_layout(uint32_t *runs, uint32_t *ce_copies,
                              uint32_t *zero_copy_slabs);

/* The same for the promote half of the last batched promote or swap (runs of
 * consecutive source slabs, copy-engine H2D copies, blocks read zero-copy),
 * and whether the last swap overlapped its evict and promote. */
int  orchkv_last_promote_layout(uint32_t *runs, uint32_t *ce_copies,
                                uint32_t *zero_copy_slabs, int *overlapped);

/* B200: evict one list and promote another in one call, with exactly the
 * effect of orchkv_evict_batch_to_dram(evict list) followed by
 * orchkv_promote_batch_to_gpu(promote list).  When the evict fits the
 * staging buffer (orchkv_config_ext_t.staging_mb) and no promoted block sits
 * in a DRAM slab this evict fills, the evict's device-to-host and the
 * promote's host-to-device transfers run at the same time on the two copy
 * engines.  `result` (device uint32[4], may be NULL) receives {evicted,
 * evict skipped, promoted, promote skipped}.  Asynchronous. */
int  orchkv_swap_batch(const uint32_t *evict_ids, const uint32_t *evict_count,
                       uint32_t max_evict, const uint32_t *promote_ids,
                       const uint32_t *promote_count, uint32_t max_promote,
                       uint32_t *result);

/* B200: copy token blocks between a caller's own contiguous KV buffers and
 * a packed store in one launch.  bufs: host array of n_bufs (<= 1024)
 * buffer pointers (device memory), each laid out [n_heads][tokens][row_bytes]
 * with heads head_stride_bytes apart -- e.g. K and V of every layer of the
 * managers' persistent buffers (python/orchkv/fast_kvcache_manager.py:79-88).
 * blocks: device array of n_blocks block indices; block b covers tokens
 * [b*block_tokens, min((b+1)*block_tokens, n_tokens)).  The store (device or
 * pinned host memory) is laid out [slot][n_bufs][n_heads][block_tokens]
 * [row_bytes]; the j-th listed block uses slot store_slots[j] (device array,
 * may be NULL for slot j).  Rows past n_tokens are left untouched.  dir 0:
 * buffers -> store, 1: store -> buffers.  row_bytes, head_stride_bytes and
 * every pointer must be 16-byte aligned.  Asynchronous on `stream`
 * (cudaStream_t).  With n_heads = 1, block_tokens = 1 and row_bytes = one
 * block's bytes it moves whole blocks of a [num_blocks, ...] cache tensor. */
int  orchkv_copy_token_blocks(void *const *bufs, uint32_t n_bufs, uint32_t n_heads,
                              uint64_t head_stride_bytes, uint32_t row_bytes,
                              uint32_t block_tokens, uint32_t n_tokens,
                              const uint32_t *blocks, uint32_t n_blocks, void *store,
                              const uint32_t *store_slots, int dir, void *stream);

/* Device table [n*n_layers][n_kv_heads][ceil(row_len/tpb)] of block ids of
 * the given requests (0xFFFFFFFF where a block does not exist), the layout
 * tm_report_attn_probs takes.  Asynchronous. */
int  orchkv_block_id_table(kv_request_ctx_t *const *ctxs, uint32_t n,
                           uint32_t row_len, uint32_t *out);

/* B200: a 64-bit checksum of each listed block's slab where it currently
 * lives (HBM or the DRAM tier): out[i] = sum_j x_j * (mix64(j) | 1) mod 2^64
 * over the slab's little-endian 64-bit words x_j, mix64 being splitmix64's
 * output function.  Blocks in no GPU or DRAM slab get 0 (tier_out[i] = 7).
 * ids, out and tier_out (may be NULL) are device memory, n entries.  Lets a
 * caller compare a block's bytes before and after a migration without
 * copying slabs out; no counterpart in the reference, whose tests compare
 * seed-pattern words (test/test_gpu_dram.cu:40-55).  Asynchronous. */
int  orchkv_block_checksums(const uint32_t *block_ids, uint32_t n,
                            unsigned long long *out, uint8_t *tier_out);

/* B200: the checked build (liborchkv_b200.so compiled with -DOKV_CHECKED,
 * built into orchkv_b200/_checked/).  Every slab, free-stack and block index
 * a data-plane kernel reads from memory is compared with its bound first; one
 * out of range is recorded and its access skipped, nothing traps, and
 * orchkv_sync / tm_sync return ORCHKV_ERR_CUDA from then on.  The regular
 * build compiles the comparisons away.  No counterpart in the reference.
 *   orchkv_checked_build: 1 in the checked build, else 0.
 *   orchkv_check_status: words[4] = {indices out of range, source line of
 *     the first, its value, its bound} since load or the last reset, shutdowns
 *     included (all 0 in the regular build); reset != 0 clears them.
 *   orchkv_check_inject: checked build only (else ORCHKV_ERR_INVALID):
 *     record one violation at `line` without touching any other memory, to
 *     test what a caller does with the error. */
int  orchkv_checked_build(void);
int  orchkv_check_status(uint32_t *words, int reset);
int  orchkv_check_inject(uint32_t line);

/* Introspection for tests and tools (synchronous). */
int  orchkv_block_info(kv_request_ctx_t *ctx, uint32_t layer_id, uint32_t head_id,
                       uint32_t block_idx, uint64_t *block_id, int *tier,
                       uint32_t *slab, int *state, uint32_t *token_count);
int  orchkv_set_block_flags(kv_request_ctx_t *ctx, uint32_t layer_id,
                            uint32_t head_id, uint32_t block_idx, uint8_t flags);
/* which: 0 = GPU pool, 1 = DRAM pool, 2 = block-id stack.  Copies the free
 * stack (all entries: pool slabs, or max_blocks ids) and its top. */
int  orchkv_read_pool(int which, uint32_t *stack_out, uint32_t *top_out);
/* Location words ((tier << 29) | slab) and states of all max_blocks ids. */
int  orchkv_read_block_locs(uint32_t *loc_out, uint8_t *state_out);
uint32_t orchkv_max_blocks(void);
/* CUDA kernel launches issued by the library since it was loaded. */
unsigned long long orchkv_kernel_launches(void);
void *orchkv_gpu_pool_base(void);
void *orchkv_dram_pool_base(void);

#ifdef __cplusplus
}
#endif
#endif /* ORCHKV_API_H */
