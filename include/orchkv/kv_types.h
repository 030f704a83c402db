/*
 * kv_types.h — shared types of the orchkv C ABI (B200 implementation).
 *
 * Binary layout and numeric values follow the OrchKvCache reference so that
 * callers compiled against the reference header keep working:
 *   error codes            src/core/kv_types.h:18-28
 *   StorageTier/DataType/KVBlockState enums   src/core/kv_types.h:34-58
 *   block flags            src/core/kv_types.h:90-94
 *   orchkv_config_t + defaults               src/core/kv_types.h:200-255
 *   orchkv_stats_t         src/core/kv_types.h:261-288
 */
#ifndef ORCHKV_KV_TYPES_H
#define ORCHKV_KV_TYPES_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- return codes: 0 on success, negative on failure ------------------- */
#define ORCHKV_OK             0
#define ORCHKV_ERR_OOM       -1   /* host or device allocation failed      */
#define ORCHKV_ERR_INVALID   -2   /* bad argument                          */
#define ORCHKV_ERR_NOT_FOUND -3   /* no such block / request               */
#define ORCHKV_ERR_TIER_FULL -4   /* destination tier has no free slab     */
#define ORCHKV_ERR_CUDA      -5   /* CUDA runtime or kernel-reported error */
#define ORCHKV_ERR_IO        -6   /* storage I/O failed                    */
#define ORCHKV_ERR_LOCKED    -7   /* block pinned or in flight             */
#define ORCHKV_ERR_STATE     -8   /* operation illegal in the block state  */
#define ORCHKV_ERR_INIT      -9   /* system not initialised                */
#define ORCHKV_ERR_ALREADY  -10   /* already initialised / duplicate       */

/* ---- where a block's bytes live ------------------------------------------ */
typedef enum {
    TIER_GPU_HBM   = 0,
    TIER_HOST_DRAM = 1,
    TIER_NVM       = 2,
    TIER_SSD       = 3,
    TIER_NONE      = 4,
} StorageTier;

typedef enum {
    DTYPE_FP16 = 0,
    DTYPE_BF16 = 1,
    DTYPE_FP32 = 2,
    DTYPE_INT8 = 3,
    DTYPE_INT4 = 4,   /* two values per byte; stored as 1 byte per element */
} DataType;

typedef enum {
    KV_STATE_FREE      = 0,
    KV_STATE_ALLOCATED = 1,
    KV_STATE_HOT       = 2,   /* on GPU                 */
    KV_STATE_WARM      = 3,   /* on host DRAM           */
    KV_STATE_COLD      = 4,   /* on the storage tier    */
    KV_STATE_MIGRATING = 5,
    KV_STATE_EVICTED   = 6,
} KVBlockState;

/* ---- sizes ------------------------------------------------------------- */
#define KV_TOKEN_GROUP_SIZE     64
#define KV_PAGE_SIZE            4096
#define KV_BLOCK_SIZE           (32 * 1024)
#define KV_DEFAULT_GPU_POOL_GB  40
#define KV_DEFAULT_DRAM_POOL_GB 64
#define KV_DEFAULT_NUM_STREAMS  4
#define KV_TRANSFER_QUEUE_CAP   1024
#define KV_ADDRMAP_INIT_CAP     (1 << 16)
#define KV_ADDRMAP_LOAD_FACTOR  0.75

/* ---- per-block flag bits ---------------------------------------------- */
#define KV_FLAG_NONE        0x00
#define KV_FLAG_PIN         0x01   /* never evicted                 */
#define KV_FLAG_DIRTY       0x02
#define KV_FLAG_PREFETCHING 0x04
#define KV_FLAG_ATTN_SINK   0x08   /* always classified HOT         */

#define ORCHKV_ALIGN_UP(x, a)   (((x) + (a) - 1) & ~((a) - 1))
#define ORCHKV_ALIGN_DOWN(x, a) ((x) & ~((a) - 1))
#define ORCHKV_MIN(a, b)        (((a) < (b)) ? (a) : (b))
#define ORCHKV_MAX(a, b)        (((a) > (b)) ? (a) : (b))
#define ORCHKV_DIV_CEIL(a, b)   (((a) + (b) - 1) / (b))

static inline size_t dtype_size(DataType dt)
{
    switch (dt) {
    case DTYPE_FP16: case DTYPE_BF16: return 2;
    case DTYPE_FP32: return 4;
    case DTYPE_INT8: case DTYPE_INT4: return 1;
    default: return 0;
    }
}

/* Printable names of the enums (src/core/kv_types.h:142-178). */
static inline const char *dtype_name(DataType dt)
{
    static const char *const n[] = {"fp16", "bf16", "fp32", "int8", "int4"};
    return (unsigned)dt < sizeof(n) / sizeof(n[0]) ? n[dt] : "unknown";
}

static inline const char *tier_name(StorageTier t)
{
    static const char *const n[] = {"GPU_HBM", "HOST_DRAM", "NVM", "SSD", "NONE"};
    return (unsigned)t < sizeof(n) / sizeof(n[0]) ? n[t] : "UNKNOWN";
}

static inline const char *block_state_name(KVBlockState s)
{
    static const char *const n[] = {"FREE", "ALLOCATED", "HOT", "WARM", "COLD", "MIGRATING",
                                    "EVICTED"};
    return (unsigned)s < sizeof(n) / sizeof(n[0]) ? n[s] : "UNKNOWN";
}

/* Bytes of one slab: K and V halves of tokens_per_block rows of d_head. */
static inline size_t kv_block_data_bytes(uint32_t token_count, uint32_t d_head,
                                         DataType dtype)
{
    return (size_t)token_count * d_head * 2 * dtype_size(dtype);
}

/* ---- system configuration (same field order as the reference) ---------- */
typedef struct orchkv_config {
    int          gpu_device_id;
    size_t       gpu_pool_bytes;
    size_t       dram_pool_bytes;
    bool         dram_use_pinned;     /* the B200 build always pins (zero-copy) */
    int          num_cuda_streams;
    uint32_t     tokens_per_block;
    uint32_t     d_head;
    DataType     dtype;
    float        gpu_hwm;
    float        gpu_lwm;
    float        dram_hwm;
    float        dram_lwm;
    const char  *orchfs_base_dir;
    const char  *orchfs_nvm_path;
    const char  *orchfs_ssd_path;
    int          nvm_io_threads;
    int          ssd_io_threads;
    int          orchfs_io_workers;
    uint32_t     max_blocks_per_head; /* also the block-table width per head */
} orchkv_config_t;

static inline void orchkv_config_default(orchkv_config_t *c)
{
    c->gpu_device_id       = 0;
    c->gpu_pool_bytes      = (size_t)KV_DEFAULT_GPU_POOL_GB << 30;
    c->dram_pool_bytes     = (size_t)KV_DEFAULT_DRAM_POOL_GB << 30;
    c->dram_use_pinned     = true;
    c->num_cuda_streams    = KV_DEFAULT_NUM_STREAMS;
    c->tokens_per_block    = KV_TOKEN_GROUP_SIZE;
    c->d_head              = 128;
    c->dtype               = DTYPE_FP16;
    c->gpu_hwm             = 0.9f;
    c->gpu_lwm             = 0.7f;
    c->dram_hwm            = 0.9f;
    c->dram_lwm            = 0.7f;
    c->orchfs_base_dir     = "/dev/shm/orchkv";
    c->orchfs_nvm_path     = NULL;
    c->orchfs_ssd_path     = NULL;
    c->nvm_io_threads      = 4;
    c->ssd_io_threads      = 16;
    c->orchfs_io_workers   = 4;
    c->max_blocks_per_head = 256;
}

typedef struct orchkv_stats {
    size_t   gpu_pool_total;
    size_t   gpu_pool_used;
    uint32_t gpu_slabs_total;
    uint32_t gpu_slabs_used;
    size_t   dram_pool_total;
    size_t   dram_pool_used;
    uint32_t dram_slabs_total;
    uint32_t dram_slabs_used;
    uint64_t total_blocks;
    uint64_t blocks_on_gpu;
    uint64_t blocks_on_dram;
    uint64_t blocks_on_nvm;
    uint64_t blocks_on_ssd;
    uint64_t transfers_d2h;
    uint64_t transfers_h2d;
    uint64_t bytes_d2h;
    uint64_t bytes_h2d;
    uint32_t active_requests;
} orchkv_stats_t;

#ifdef __cplusplus
}
#endif
#endif /* ORCHKV_KV_TYPES_H */
