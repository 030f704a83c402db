/*
 * orchkv_oracle.h — CPU restatement of OrchKvCache's scheduling path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the checker the CUDA path is compared
 * against; it is never linked into, loaded by, or called from the product
 * library (liborchkv_b200.so) or the orchkv_core module.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg use it.
 *
 * Every function restates one piece of the reference algorithm in fresh
 * code and names the reference file:line it follows (paths are relative to
 * the OrchKvCache source tree).  Floating point is evaluated in IEEE single
 * precision one operation at a time, in the reference's operation order; the
 * Makefile builds this file with -ffp-contract=off so no FMA is formed.
 */
#ifndef ORCHKV_ORACLE_H
#define ORCHKV_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OC_DECAY_TABLE 512           /* src/scheduler/hotcold_classifier.h:63 */
#define OC_STEP_NEVER  UINT64_MAX    /* src/scheduler/attention_tracker.c:189 */

/* Scheduler state for one manager, structure-of-arrays indexed by slot =
 * block_id & mask (src/scheduler/attention_tracker.c:21-24). */
typedef struct oc_sched {
    uint32_t  cap, mask;
    uint64_t  step;
    float     lambda;
    /* tracker (C1) — src/scheduler/attention_tracker.h:23-30 */
    float    *sum, *max, *ema;
    uint32_t *hits;
    uint64_t *last;
    uint8_t  *t_active;
    /* classifier (C2) — src/scheduler/hotcold_classifier.h:55-60 */
    float    *hot;
    uint8_t  *heat;
    uint8_t  *c_flags;
    uint8_t  *c_active;
    float     alpha, beta, gamma, tau, th_hot, th_warm;
    float     table[OC_DECAY_TABLE];
} oc_sched_t;

int   oc_sched_init(oc_sched_t *s, uint32_t capacity, float lambda,
                    float alpha, float beta, float gamma, float tau,
                    float th_hot, float th_warm);
void  oc_sched_free(oc_sched_t *s);
void  oc_register(oc_sched_t *s, uint64_t id, uint8_t flags);
void  oc_unregister(oc_sched_t *s, uint64_t id);
void  oc_update(oc_sched_t *s, uint64_t id, float w);
void  oc_update_batch(oc_sched_t *s, const uint64_t *ids, const float *w, uint32_t n);
void  oc_step_done(oc_sched_t *s);
void  oc_update_all(oc_sched_t *s);
void  oc_set_thresholds(oc_sched_t *s, float th_hot, float th_warm);
void  oc_set_weights(oc_sched_t *s, float a, float b, float g);
void  oc_build_decay_table(float *table, float tau);
float oc_hotness_one(const oc_sched_t *s, uint32_t slot, uint64_t step);

/* Adaptive threshold (C3) — src/scheduler/adaptive_threshold.c:82-169.
 * Cooldown is evaluated by the caller (elapsed flag), the rest is here. */
typedef struct oc_athresh {
    float th_hot, th_warm, min_hot, max_hot, min_warm, max_warm;
    float gpu_hwm, gpu_lwm, dram_hwm, dram_lwm, step;
    uint64_t up, down, checks;
} oc_athresh_t;
int   oc_athresh_update(oc_athresh_t *a, float gpu_ratio, float dram_ratio);

/* Orderable 32-bit key of a float: ascending key == ascending value, with
 * -0.0 folded onto +0.0 (the two compare equal in the callers' sort) and
 * NaN placed after every number. */
uint32_t oc_orderable(float f);

/* Coldest-k among eligible slots, ordered by (hotness asc, slot asc) — the
 * FastKVCacheManager ordering (python/orchkv/fast_kvcache_manager.py:307-321,
 * Python's stable sort over ascending block ids).  Writes the chosen slots in
 * ascending slot order; returns how many were written (min(k, #eligible)). */
uint32_t oc_select_coldest(const float *hot, const uint8_t *eligible,
                           uint32_t n, uint32_t k, uint32_t *out);

/* Prefetch candidates (src/scheduler/prefetch_scheduler.c:131-172): for
 * tier not GPU(0) and not NONE(4): ema >= th_gpu -> prio = ema; else if
 * ema >= th_dram and tier != DRAM(1) -> prio = 0.5*ema; else skipped.
 * Picks the top-k by (prio desc, slot asc); output ascending slot order. */
uint32_t oc_select_prefetch(const float *ema, const uint8_t *active,
                            const uint8_t *tier, uint32_t n,
                            float th_gpu, float th_dram, uint32_t k,
                            uint32_t *out);

/* Per-block attention mass (python/orchkv/fast_kvcache_manager.py:221-235,
 * python/orchkv/kvcache_manager.py:317-347, restated per KV group): for row r
 * (= request*L + layer), KV head h and token block b:
 *   out[(r*Hkv + h)*nb + b] = sum_{g < Hq/Hkv} sum_{t in block b, t < len}
 *                               probs[(r*Hq + h*G + g)*T + t]
 * accumulated in exactly that loop order in fp32.  len = lens ? lens[r] : T. */
void oc_score_blocks(const float *probs, uint32_t R, uint32_t Hq, uint32_t Hkv,
                     uint32_t T, uint32_t tpb, const uint32_t *lens, float *out);

/* LIFO slab pool (src/tiered_store/gpu_tier.cu:36-93): stack filled so the
 * first pops return 0,1,2,...; pop takes stack[--top], push does
 * stack[top++] = idx. */
typedef struct oc_pool { uint32_t total, top; uint32_t *stack; } oc_pool_t;
int      oc_pool_init(oc_pool_t *p, uint32_t total);
void     oc_pool_free(oc_pool_t *p);
int      oc_pool_pop(oc_pool_t *p, uint32_t *idx);
void     oc_pool_push(oc_pool_t *p, uint32_t idx);

/* Batched migration with the reference's per-block semantics applied in list
 * order (src/api/orchkv_api.cu:353-428): loc[] encodes (tier<<29)|slab.
 * Evict: block must be on GPU and not pinned (else it is skipped, as
 * mig_demote_batch skips, src/scheduler/migration_engine.c:222-245); pop a
 * DRAM slab, copy the slab bytes, mark WARM, push the GPU slab.  Once the
 * destination pool is empty every later block fails with TIER_FULL.
 * Returns the number of blocks migrated; *n_skipped gets the others. */
uint32_t oc_evict_batch(oc_pool_t *gpu, oc_pool_t *dram, uint32_t *loc,
                        uint8_t *state, const uint8_t *flags,
                        const uint32_t *handles, uint32_t n,
                        const uint8_t *gpu_base, uint8_t *dram_base,
                        size_t slab, uint32_t *n_skipped);
uint32_t oc_promote_batch(oc_pool_t *gpu, oc_pool_t *dram, uint32_t *loc,
                          uint8_t *state, const uint32_t *handles, uint32_t n,
                          uint8_t *gpu_base, const uint8_t *dram_base,
                          size_t slab, uint32_t *n_skipped);

/* Location word helpers: tier in bits 29-31, slab index in bits 0-28. */
#define OC_LOC(tier, slab) (((uint32_t)(tier) << 29) | (uint32_t)(slab))
#define OC_LOC_TIER(w)     ((uint32_t)(w) >> 29)
#define OC_LOC_SLAB(w)     ((uint32_t)(w) & 0x1FFFFFFFu)

#ifdef __cplusplus
}
#endif
#endif /* ORCHKV_ORACLE_H */
