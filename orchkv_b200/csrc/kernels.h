// kernels.h — host-side launchers of the orchkv B200 CUDA kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace okv {

// ---- scoring (sched_kernels.cu) ---------------------------------------------

// Ordering of one report call whose ids may share tracker slots.  A mark pass
// stamps every listed active slot with `epoch` (a value unique to the call)
// and sets *flag = epoch when a slot is stamped twice.  Report kernels read
// the flag: when it is not set they record straight into the tracker (no two
// writers per slot); when it is, they leave the tracker alone and write each
// entry's id and mass to ids_eff / mass, and the ordered pass applies them per
// slot in entry order -- the sums consecutive single reports would give.
struct ReportOrder {
    uint32_t *mark;      // [cap] last epoch that stamped each slot
    uint32_t *flag;      // one word: == epoch when this call has aliasing ids
    uint32_t epoch;
    uint32_t *ids_eff;   // [n] per entry: id, or kNoBlock when not reported
    float *mass;         // [n] per entry mass
};
int launch_alias_mark(const uint32_t *ids, uint32_t n, const SchedDev &d, const ReportOrder &o,
                      cudaStream_t s);
// Applies (ids[i], w[i]) for i in [0, n) in entry order per slot, only when
// the call's flag is set (otherwise returns at once on the device).
int launch_report_ordered(const uint32_t *ids, const float *w, uint32_t n, const SchedDev &d,
                          unsigned long long step, const ReportOrder &o, cudaStream_t s);
int launch_score(const float *probs, uint32_t R, uint32_t Hq, uint32_t Hkv,
                 uint32_t T, uint32_t tpb, const uint32_t *lens,
                 const uint32_t *ids, const SchedDev &d, unsigned long long step,
                 const ReportOrder &o, cudaStream_t s);
int launch_report_apply(const uint32_t *slots, const float *psum, const float *pmax,
                        uint32_t n, const SchedDev &d, unsigned long long step,
                        cudaStream_t s);
int launch_report_batch(const uint32_t *ids, const float *w, uint32_t n,
                        const SchedDev &d, unsigned long long step, const ReportOrder &o,
                        cudaStream_t s);
// Per-block mass over token ranges: sum over heads and tokens [start, min(end,
// kv_len)) of avg [heads][kv_len], recorded for ids[i]; empty ranges skipped.
int launch_range_mass(const float *avg, uint32_t heads, uint32_t kv_len, const uint32_t *start,
                      const uint32_t *end, const uint32_t *ids, uint32_t n, const SchedDev &d,
                      unsigned long long step, const ReportOrder &o, cudaStream_t s);
// Block means of attention weights [batch][heads][q_len][kv_len] (dtype 0
// fp16, 1 bf16, 2 fp32) into scores [heads][ceil(kv_len/bs)]; with ids and d,
// each (h, b) is then recorded in the tracker, heads of one block in order.
int launch_blockmean(const void *w, int dtype, uint32_t batch, uint32_t heads, uint32_t q_len,
                     uint32_t kv_len, uint32_t bs, const uint32_t *ids, float *scores,
                     const SchedDev *d, unsigned long long step, cudaStream_t s);
int launch_sweep(const SchedDev &d, const SchedParams &p, bool step_done,
                 bool classify, ClassCounts *counts, cudaStream_t s);
int launch_registry_count(const uint32_t *reg_slot, const uint8_t *reg_tier,
                          uint32_t n, const SchedDev &d, float th_gpu,
                          float th_dram, uint32_t *count, cudaStream_t s);
// Slot writes applied in list order: op 0 = register (tracker + classifier
// reset, flags, tier, state), 1 = unregister, 2 = update tier/flags/state.
// `b` packs per entry {op, flags, tier, state}.
int launch_slot_ops(const uint32_t *slots, const uint8_t *b, uint32_t n,
                    const SchedDev &d, cudaStream_t s);

// ---- selection (select_kernels.cu) -------------------------------------------
// kSelectExternal: keys from a caller's value array (SchedDev.hot) where the
// caller's byte array (SchedDev.tact) is non-zero; ascending value order.
enum SelectMode { kSelectColdest = 0, kSelectPrefetch = 1, kSelectExternal = 2 };

struct SelectScratch {
    uint32_t *hist_local;    // [4096 + 16]
    uint32_t *hist_global;   // [4096 + 16]
    uint32_t *state;         // SelState words
    uint32_t *tile_counts;   // [2 * max_tiles]
    uint32_t *tile_offsets;  // [2 * max_tiles]
    uint32_t max_tiles;
};

// Host hook run between passes (multi-GPU): reduce `hist_local` into
// `hist_global` over `nwords` words.  NULL = single device (device copy).
typedef int (*hist_reduce_fn)(const uint32_t *local, uint32_t *global, uint32_t nwords,
                              cudaStream_t s, void *ctx);
typedef int (*tie_gather_fn)(const uint32_t *local_one, uint32_t *all_out,
                             cudaStream_t s, void *ctx);

struct SelectArgs {
    SelectMode mode;
    uint32_t k;          // explicit k (used when frac < 0)
    float frac;          // >= 0: k = floor(frac * eligible)
    float th_gpu, th_dram;
    uint32_t max_out;
    uint32_t *out_ids;
    uint32_t *out_count;
    hist_reduce_fn reduce;
    tie_gather_fn gather;
    void *comm_ctx;
    int rank, world;
    uint32_t *gather_buf;  // device [world]
    const uint8_t *mask;   // coldest mode: optional device [cap]; 0 excludes slot
};

int launch_select(const SchedDev &d, const SelectScratch &sc, const SelectArgs &a,
                  cudaStream_t s);
size_t select_scratch_words(uint32_t cap, uint32_t *max_tiles);

}  // namespace okv
