// pool.h — device view of the data plane (slab pools, block records,
// request block tables) shared by pool_kernels.cu and api.cu.
#pragma once

#include "common.cuh"

namespace okv {

struct PoolCounters {
    uint32_t g_top, d_top, id_top, err;
    unsigned long long transfers_d2h, transfers_h2d, bytes_d2h, bytes_h2d;
    uint32_t last_done, last_skipped, live_blocks, pad;
    unsigned long long scratch[4];
};

struct PoolDev {
    char *gpu_base;
    char *dram_base;                 // pinned + mapped host memory (UVA pointer)
    unsigned long long slab, half;   // bytes
    uint32_t row;                    // d_head * dtype bytes
    uint32_t tpb;
    uint32_t g_total, d_total, max_blocks;
    uint32_t *g_stack, *d_stack, *id_stack;
    uint32_t *loc;                   // (tier << 29) | slab, per block id
    uint32_t *first;                 // per block id: first list position in a batch (else ~0)
    uint8_t *state, *flags;          // per block id
    PoolCounters *ctr;
    SchedDev sd;                     // attached scheduler (valid if attached)
    int attached;
    uint32_t *chk;                   // checked build: {count, line, index, bound} of the
                                     // first out-of-range index (device, 4 words)
};

// ---- checked build ------------------------------------------------------------
// Compiled with -DOKV_CHECKED, every slab, stack and block index a data-plane
// kernel takes from memory is compared with its bound before it is used.  An
// index out of range is counted in the check words (the first one's source
// line, value and bound recorded) and its access is skipped -- nothing traps;
// orchkv_sync / tm_sync then return ORCHKV_ERR_CUDA.  The regular build
// compiles every comparison to `true`.
#ifdef OKV_CHECKED
constexpr bool kCheckedBuild = true;
#else
constexpr bool kCheckedBuild = false;
#endif

__device__ __forceinline__ bool in_bounds(uint32_t *chk, unsigned long long i,
                                          unsigned long long n, uint32_t line)
{
    if (!kCheckedBuild || i < n) return true;
    if (chk && atomicAdd(chk, 1u) == 0) {
        chk[1] = line;
        chk[2] = (uint32_t)i;
        chk[3] = (uint32_t)n;
    }
    return false;
}
#define OKV_IN(chk, i, n) okv::in_bounds((chk), (i), (n), __LINE__)

// The pool sizes a kernel that only sees raw pointers checks against.
struct Bounds {
    uint32_t *chk;
    uint32_t g_total, d_total, max_blocks;
};
inline Bounds bounds_of(const PoolDev &p) { return Bounds{p.chk, p.g_total, p.d_total, p.max_blocks}; }

// A request's region in the block-table array:
//   [0]              seq_len
//   [1 .. L]         tokens held per layer (identical for all heads)
//   [1+L ..]         block ids, [layer][head][max_blocks_per_head]
struct ReqDev {
    uint32_t *region;
    uint32_t L, H, mbph;
};

__host__ __device__ inline uint32_t *req_tok(const ReqDev &r) { return r.region + 1; }
__host__ __device__ inline uint32_t *req_table(const ReqDev &r) { return r.region + 1 + r.L; }
__host__ __device__ inline size_t req_region_words(uint32_t L, uint32_t H, uint32_t mbph)
{
    return 1 + (size_t)L + (size_t)L * H * mbph;
}

// Result of a per-block (compat) operation, written by the kernel into
// pinned host memory and read after the stream synchronises.
struct CompatResult {
    int rc;
    uint32_t id;
    unsigned long long k_ptr, v_ptr;
    uint32_t loc, state, tok, flags;
    uint32_t aux, pad;
};

enum CompatOp : int {
    OP_EVICT = 0,
    OP_PROMOTE = 1,
    OP_GET = 2,          // promote if on DRAM, return pointers
    OP_INFO = 3,
    OP_SET_FLAGS = 4,
    OP_DRAM_POP = 5,     // pop a DRAM slab into res->aux (storage promotion)
    OP_SET_LOC = 6,      // loc := arg; state := arg2 & 0xFF; arg2 >> 8 = DRAM slab + 1 to push
};

// ---- launchers (pool_kernels.cu) -------------------------------------------
int launch_compat_op(const PoolDev &p, const ReqDev &r, int op, uint32_t l, uint32_t h,
                     uint32_t bi, uint32_t arg, uint32_t arg2, CompatResult *res,
                     cudaStream_t s);
int launch_append_one(const PoolDev &p, const ReqDev &r, uint32_t l, const char *k,
                      const char *v, CompatResult *res, cudaStream_t s);
int launch_prefill(const PoolDev &p, const ReqDev &r, uint32_t l, const char *k,
                   const char *v, uint32_t seq_len, uint32_t *scratch,
                   CompatResult *res, cudaStream_t s);
// Batched append over n requests x L layers.  regions: device array of n
// region pointers.  scratch: >= 2*n*L + 16 words.
int launch_append_batch(const PoolDev &p, uint32_t *const *regions, uint32_t n, uint32_t L,
                        uint32_t H, uint32_t mbph, const char *k, const char *v,
                        uint32_t *scratch, cudaStream_t s);
// Batched migration.  dir 0 = evict (GPU -> DRAM), 1 = promote (DRAM -> GPU).
// scratch: >= 3*max_n + tiles + 16 words where tiles = ceil(max_n/1024).
int launch_migrate_batch(const PoolDev &p, int dir, const uint32_t *ids,
                         const uint32_t *count, uint32_t max_n, uint32_t *result,
                         uint32_t *scratch, cudaStream_t s);

// Pieces of a batched migration for the staged (copy-engine) evict path.
// meta words: [0] done, [1] old dst top, [2] old src top, [3] lowest dst slab,
// [4] 1 if the popped dst slabs form one contiguous range, [5] its first slab.
// scratch: >= 3*max_n + tiles + 16 words.
struct MigPlan {
    uint32_t *meta, *plan_src, *plan_dst, *plan_id;
    uint32_t tiles, max_n;
    int rc;
};
MigPlan launch_migrate_plan(const PoolDev &p, int dir, const uint32_t *ids,
                            const uint32_t *count, uint32_t max_n, uint32_t *result,
                            uint32_t *scratch, cudaStream_t s);
int launch_migrate_zero_copy(const PoolDev &p, int dir, const MigPlan &mp, cudaStream_t s);
// Staged evict: the popped DRAM slabs are sorted (byte map over the pool),
// victim o gets the o-th smallest, and the runs of consecutive slabs are
// listed for the copy engine.  meta[6] receives the number of runs.
struct SortScratch {
    uint8_t *flags;      // [d_total]
    uint32_t *tile_cnt;  // [ceil(d_total / 1024)]
    uint32_t *sorted;    // [d_total]
    uint8_t *run_flag;   // [d_total]
    uint32_t *run_o;     // [max_runs] list position of each run start
    uint32_t *run_d;     // [max_runs] first slab of each run
    uint32_t max_runs;
    uint32_t *pos_of;    // [d_total] DRAM slab -> list position (staged promote only)
};
int launch_sorted_assign(const PoolDev &p, const MigPlan &mp, const SortScratch &ss,
                         cudaStream_t s);
// Pack entries [pos0, pos0 + n) into staging (entry w at staging + w*slab).
// min_len > 0: only entries in DRAM runs of >= min_len slabs (requires the
// run list of launch_sorted_assign, and meta[6] <= ss.max_runs).
int launch_pack(const PoolDev &p, const MigPlan &mp, char *staging, uint32_t pos0, uint32_t n,
                const SortScratch &ss, uint32_t min_len, cudaStream_t s);
// Entries of [pos0, pos0 + n) in DRAM runs shorter than min_len: written from
// their GPU slab straight into the DRAM tier (zero-copy).
// `staged` (may be null): the packed copies of entries [pos0, pos0 + n), read
// instead of the GPU slabs.
int launch_drain_short(const PoolDev &p, const MigPlan &mp, uint32_t pos0, uint32_t n,
                       const SortScratch &ss, uint32_t min_len, const char *staged,
                       cudaStream_t s);

// Staged promote (dir 1 plan): sort the source DRAM slabs (ss.sorted, with
// ss.pos_of mapping slab -> list position) and list their runs (meta[6]).
int launch_sorted_sources(const PoolDev &p, const MigPlan &mp, const SortScratch &ss,
                          cudaStream_t s);
// Sorted positions [j0, j0 + n) in runs of >= min_len slabs (all if 0):
// staging entry j - j0 -> the block's GPU slab.
int launch_unpack(const PoolDev &p, const MigPlan &mp, const SortScratch &ss,
                  const char *staging, uint32_t j0, uint32_t n, uint32_t min_len, cudaStream_t s);
// Sorted positions in runs shorter than min_len: DRAM slab -> GPU slab over
// the host link (no-op when min_len is 0).
int launch_promote_short(const PoolDev &p, const MigPlan &mp, const SortScratch &ss,
                         uint32_t min_len, cudaStream_t s);
// *conflicts = promote sources among the slabs an evict's sorted assignment
// popped (evict_ss.flags).
int launch_conflicts(const PoolDev &p, const MigPlan &promote, const SortScratch &evict_ss,
                     uint32_t *conflicts,
                     cudaStream_t s);
int launch_id_table(const PoolDev &p, uint32_t *const *regions, uint32_t n, uint32_t L,
                    uint32_t H, uint32_t mbph, uint32_t row_len, uint32_t *out,
                    cudaStream_t s);
// Batched storage moves: triples lhb[3n] -> out[3n] = {id, loc word, flags}.
int launch_lhb_lookup(const PoolDev &p, const ReqDev &r, const uint32_t *lhb, uint32_t n,
                      uint32_t *out, cudaStream_t s);
// Commit n storage moves in list order (dir 0: DRAM -> storage, pushing
// DRAM slabs[j]; dir 1: storage -> DRAM, popping the DRAM stack's top n
// slabs; dir 2: GPU -> storage, pushing GPU slabs[j]).
int launch_storage_commit(const PoolDev &p, const uint32_t *ids, const uint32_t *slabs,
                          uint32_t n, int dir, cudaStream_t s);
// Checked build: record a violation at `line` without any other access (a
// test of the check words' plumbing).
int launch_check_inject(const PoolDev &p, uint32_t line, cudaStream_t s);
// Per-block checksums of listed blocks' slabs (integrity_kernels.cu).
int launch_block_checksums(const PoolDev &p, const uint32_t *ids, uint32_t n,
                           unsigned long long *out, uint8_t *tier_out, cudaStream_t s);
// scratch: >= 3 * ceil(L*H*mbph / 1024) words.
int launch_request_free(const PoolDev &p, const ReqDev &r, uint32_t *scratch, cudaStream_t s);

}  // namespace okv
