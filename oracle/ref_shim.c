/*
 * ref_shim.c — ctypes-friendly wrappers around the reference's own scheduler
 * and data-plane code, compiled together with the reference sources into
 * oracle/_ref/liborchkv_ref.so by oracle/Makefile.
 *
 * TEST INFRASTRUCTURE ONLY: used to pin the oracle restatement, to generate
 * tests/golden fixtures, and as bench.py's reference (CPU) arm.  Nothing in
 * the product links or loads it.
 *
 * The manager wrapper mirrors what the reference's Python binding does
 * (bindings/orchkv_pybind.cpp:215-306): tm_config_default, the pybind
 * keyword set, and binding-owned kv_block_t records registered by id.
 */
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include "scheduler/tiered_manager.h"
#include "api/orchkv_api.h"

typedef struct ref_tm {
    tiered_manager_t m;
    kv_block_t     **blks;
    uint32_t         n, cap;
} ref_tm_t;

void *ref_tm_create(uint32_t tracker_cap, float ema_lambda, float alpha,
                    float beta, float gamma, uint32_t prefetch_budget,
                    float gpu_hwm, float gpu_lwm, float dram_hwm,
                    float dram_lwm, uint32_t max_blocks, float th_gpu,
                    float th_dram, float tau, double cooldown_sec,
                    float adjust_step, uint32_t demote_batch,
                    uint32_t prefetch_batch)
{
    ref_tm_t *w = calloc(1, sizeof(*w));
    if (!w) return NULL;
    tm_config_t cfg;
    tm_config_default(&cfg);
    cfg.tracker_capacity = tracker_cap;
    cfg.ema_lambda = ema_lambda;
    cfg.hcc_params.alpha = alpha;
    cfg.hcc_params.beta = beta;
    cfg.hcc_params.gamma = gamma;
    cfg.hcc_params.recency_tau = tau;
    cfg.prefetch_budget = prefetch_budget;
    cfg.auto_schedule = false;
    cfg.athresh_params.gpu_hwm = gpu_hwm;
    cfg.athresh_params.gpu_lwm = gpu_lwm;
    cfg.athresh_params.dram_hwm = dram_hwm;
    cfg.athresh_params.dram_lwm = dram_lwm;
    cfg.athresh_params.cooldown_sec = cooldown_sec;
    cfg.athresh_params.adjust_step = adjust_step;
    cfg.max_blocks = max_blocks;
    cfg.threshold_to_gpu = th_gpu;
    cfg.threshold_to_dram = th_dram;
    if (demote_batch) cfg.demote_batch_size = demote_batch;
    if (prefetch_batch) cfg.prefetch_batch_size = prefetch_batch;
    if (tm_init(&w->m, &cfg) != ORCHKV_OK) { free(w); return NULL; }
    return w;
}

void ref_tm_destroy(void *h)
{
    ref_tm_t *w = h;
    if (!w) return;
    tm_destroy(&w->m);
    for (uint32_t i = 0; i < w->n; i++) free(w->blks[i]);
    free(w->blks);
    free(w);
}

int ref_tm_register_id(void *h, uint64_t id, int tier, uint8_t flags)
{
    ref_tm_t *w = h;
    kv_block_t *b = calloc(1, sizeof(*b));
    b->block_id = id;
    b->tier = (StorageTier)tier;
    b->flags = flags;
    int rc = tm_register_block(&w->m, b);
    if (rc != ORCHKV_OK) { free(b); return rc; }
    if (w->n == w->cap) {
        w->cap = w->cap ? 2 * w->cap : 256;
        w->blks = realloc(w->blks, w->cap * sizeof(*w->blks));
    }
    w->blks[w->n++] = b;
    return rc;
}

void ref_tm_set_block_tier(void *h, uint64_t id, int tier)
{
    ref_tm_t *w = h;
    for (uint32_t i = 0; i < w->n; i++)
        if (w->blks[i]->block_id == id) { w->blks[i]->tier = (StorageTier)tier; return; }
}

/* Bulk forms for large samples: register ids 0..n-1 in order, and set the
 * tier of a list of ids (direct index when ids were registered in order,
 * a scan otherwise). */
int ref_tm_register_range(void *h, uint32_t n)
{
    for (uint32_t i = 0; i < n; i++) {
        int rc = ref_tm_register_id(h, i, 0, 0);
        if (rc != ORCHKV_OK) return rc;
    }
    return ORCHKV_OK;
}

void ref_tm_set_tiers(void *h, const uint64_t *ids, uint32_t n, int tier)
{
    ref_tm_t *w = h;
    for (uint32_t i = 0; i < n; i++) {
        uint64_t id = ids[i];
        if (id < w->n && w->blks[id]->block_id == id)
            w->blks[id]->tier = (StorageTier)tier;
        else
            ref_tm_set_block_tier(h, id, tier);
    }
}

void ref_tm_notify_access(void *h, uint64_t id)
{
    ref_tm_t *w = h;
    for (uint32_t i = 0; i < w->n; i++)
        if (w->blks[i]->block_id == id) { tm_notify_access(&w->m, w->blks[i]); return; }
}

void ref_tm_report(void *h, uint64_t id, float wgt) { tm_notify_attn(&((ref_tm_t *)h)->m, id, wgt); }
void ref_tm_report_batch(void *h, const uint64_t *ids, const float *wgt, uint32_t n)
{
    attn_tracker_update_batch(&((ref_tm_t *)h)->m.tracker, ids, wgt, n);
}
void ref_tm_step_done(void *h) { tm_step_done(&((ref_tm_t *)h)->m); }
void ref_tm_set_usage(void *h, float g, float d) { tm_set_usage(&((ref_tm_t *)h)->m, g, d); }
void ref_tm_schedule_once(void *h) { tm_schedule_once(&((ref_tm_t *)h)->m); }
void ref_tm_update_all(void *h) { hcc_update_all(&((ref_tm_t *)h)->m.classifier); }
void ref_tm_set_policy(void *h, float a, float b, float g) { tm_set_policy(&((ref_tm_t *)h)->m, a, b, g); }
float ref_tm_score(void *h, uint64_t id) { return tm_get_block_score(&((ref_tm_t *)h)->m, id); }
int ref_tm_heat(void *h, uint64_t id) { return (int)tm_get_block_heat(&((ref_tm_t *)h)->m, id); }
uint32_t ref_tm_capacity(void *h) { return ((ref_tm_t *)h)->m.tracker.capacity; }
uint64_t ref_tm_step(void *h) { return ((ref_tm_t *)h)->m.tracker.current_step; }

/* Flattened tm_get_stats plus the threshold fields the binding exposes
 * (bindings/orchkv_pybind.cpp:388-415). */
void ref_tm_stats(void *h, double *o)
{
    ref_tm_t *w = h;
    tm_stats_t s;
    tm_get_stats(&w->m, &s);
    o[0] = (double)s.schedule_cycles;
    o[1] = (double)s.gpu_demotes;
    o[2] = (double)s.dram_demotes;
    o[3] = (double)s.prefetches_dispatched;
    o[4] = s.gpu_used_ratio;
    o[5] = s.dram_used_ratio;
    o[6] = (double)s.migration_stats.blocks_migrated;
    o[7] = (double)s.migration_stats.op_errors;
    o[8] = (double)s.prefetch_stats.prefetch_hits;
    o[9] = (double)s.prefetch_stats.prefetch_wasted;
    o[10] = s.prefetch_stats.hit_rate;
    o[11] = (double)s.hcc_stats.n_hot;
    o[12] = (double)s.hcc_stats.n_warm;
    o[13] = (double)s.hcc_stats.n_cold;
    o[14] = (double)w->m.threshold.adjustments_up;
    o[15] = (double)w->m.threshold.adjustments_down;
    o[16] = w->m.threshold.threshold_hot;
    o[17] = w->m.threshold.threshold_warm;
    o[18] = (double)s.prefetch_stats.total_scanned;
    o[19] = (double)s.prefetch_stats.total_enqueued;
    o[20] = (double)s.prefetch_stats.total_dispatched;
    o[21] = (double)s.hcc_stats.n_attn_sink;
    o[22] = s.hcc_stats.avg_hotness;
    o[23] = s.hcc_stats.max_hotness;
    o[24] = s.hcc_stats.min_hotness;
    o[25] = (double)w->m.threshold.demote_checks;
}

/* Copy the per-slot tracker/classifier state out (arrays of capacity). */
void ref_tm_dump(void *h, float *sum, float *ema, uint32_t *hits,
                 uint64_t *last, uint8_t *tact, float *hot, uint8_t *heat,
                 uint8_t *cact)
{
    ref_tm_t *w = h;
    uint32_t cap = w->m.tracker.capacity;
    for (uint32_t i = 0; i < cap; i++) {
        const attn_stats_t *a = &w->m.tracker.stats[i];
        const hcc_slot_t *c = &w->m.classifier.slots[i];
        sum[i] = a->sum; ema[i] = a->ema; hits[i] = a->query_hits;
        last[i] = a->last_hit_step; tact[i] = a->active;
        hot[i] = c->hotness; heat[i] = (uint8_t)c->heat_level; cact[i] = c->active;
    }
}

/* C4 victim selection on the manager's own LRU list. */
uint32_t ref_tm_select_gpu_victims(void *h, uint32_t n, uint64_t *ids, float *scores)
{
    ref_tm_t *w = h;
    eviction_candidate_t *c = calloc(n ? n : 1, sizeof(*c));
    uint32_t f = evpol_select_gpu_victims(&w->m.evpol, n, c);
    for (uint32_t i = 0; i < f; i++) { ids[i] = c[i].block->block_id; scores[i] = c[i].score; }
    free(c);
    return f;
}

/* Decay table of the classifier (src/scheduler/hotcold_classifier.c:27-34). */
void ref_tm_decay_table(void *h, float *out)
{
    memcpy(out, ((ref_tm_t *)h)->m.classifier.decay_table, sizeof(float) * HCC_DECAY_TABLE_MAX);
}

/* DRAM slab pool on plain host memory (no CUDA needed): used to pin the
 * oracle's LIFO pool semantics against src/tiered_store/dram_tier.cu. */
void *ref_dram_pool_create(uint32_t slabs, uint32_t slab_size)
{
    dram_tier_t *t = calloc(1, sizeof(*t));
    if (dram_tier_init(t, (size_t)slabs * slab_size, slab_size, false) != ORCHKV_OK) { free(t); return NULL; }
    return t;
}
long long ref_dram_pool_alloc(void *h)
{
    dram_tier_t *t = h;
    void *p;
    int rc = dram_tier_alloc(t, &p);
    if (rc != ORCHKV_OK) return rc;
    return (long long)(((char *)p - (char *)t->pool_base) / (long long)t->slab_size);
}
int ref_dram_pool_free(void *h, uint32_t idx)
{
    dram_tier_t *t = h;
    return dram_tier_free(t, (char *)t->pool_base + (size_t)idx * t->slab_size);
}
void ref_dram_pool_destroy(void *h) { dram_tier_destroy(h); free(h); }

/* Read one slab of a request's storage file with the reference's own
 * orchfs_tier_read (POSIX path, src/tiered_store/orchfs_tier.c:246-317), to
 * check that files written by another implementation use its layout.  The
 * file is opened, not removed. */
int ref_storage_read(const char *base_dir, uint64_t request_id, uint32_t L, uint32_t H,
                     uint32_t mbph, size_t slab, uint32_t l, uint32_t h, uint32_t bi,
                     void *buf)
{
    orchfs_tier_t t;
    if (orchfs_tier_init(&t, base_dir, slab) != ORCHKV_OK) return ORCHKV_ERR_INIT;
    orchfs_file_ctx_t *f = orchfs_file_open(&t, request_id, L, H, mbph);
    if (!f) { orchfs_tier_destroy(&t); return ORCHKV_ERR_IO; }
    int rc = orchfs_tier_read(f, l, h, bi, buf, slab);
    close(f->fd);
    free(f);
    orchfs_tier_destroy(&t);
    return rc;
}

/* ------------------------------------------------------------------------
 * Callback scenario for the C4/C7 demotion path (tm_schedule_once with a
 * transfer callback and an allocator, as test/test_tiered_manager.c:24-60
 * sets up): memcpy transfer, calloc allocator, free.  Blocks get 64-byte
 * payloads.  touch[] is a sequence of block indices passed to
 * tm_notify_access; rep_off[s]..rep_off[s+1] are step s's reports.
 * Outputs: final tier, state and last payload byte (-1 when data_ptr is
 * NULL) per block, and stats o[0..15] =
 * gpu_demotes, dram_demotes, blocks_migrated, op_errors, op_count[6],
 * op_bytes[6] (bytes / 64).
 * ------------------------------------------------------------------------ */
/* ctx: {calls, fail_every}; every fail_every-th transfer fails with
 * ORCHKV_ERR_IO, as test/test_migration_engine.c:43-48's failing mock does */
static int sc_transfer(kv_block_t *blk, void *dst, size_t size, MigrateOp op, void *ctx)
{
    (void)op;
    uint32_t *c = ctx;
    if (c) {
        c[0]++;
        if (c[1] && c[0] % c[1] == 0) return ORCHKV_ERR_IO;
    }
    if (blk->data_ptr && dst) memcpy(dst, blk->data_ptr, size);
    return ORCHKV_OK;
}
static void *sc_alloc(size_t size, StorageTier tier, void *ctx) { (void)tier; (void)ctx; return calloc(1, size); }
static void sc_free(void *p, StorageTier tier, void *ctx) { (void)tier; (void)ctx; free(p); }

int ref_c4_scenario(uint32_t n, const uint64_t *ids, const int *tiers, const uint8_t *flags,
                    const uint32_t *touch, uint32_t n_touch, uint32_t steps,
                    const uint64_t *rep_ids, const float *rep_w, const uint32_t *rep_off,
                    const float *gpu_ratio, const float *dram_ratio, uint32_t demote_batch,
                    float alpha, float beta, float gamma, int *out_tier, int *out_state,
                    int *out_byte, double *o, uint32_t fail_every)
{
    uint32_t xfer_ctx[2] = {0, fail_every};
    tiered_manager_t m;
    tm_config_t cfg;
    tm_config_default(&cfg);
    cfg.tracker_capacity = 4096;
    cfg.max_blocks = 4096;
    cfg.hcc_params.alpha = alpha;
    cfg.hcc_params.beta = beta;
    cfg.hcc_params.gamma = gamma;
    cfg.transfer_fn = sc_transfer;
    cfg.transfer_ctx = xfer_ctx;
    cfg.alloc_fn = sc_alloc;
    cfg.free_fn = sc_free;
    cfg.block_data_size = 64;
    cfg.demote_batch_size = demote_batch;
    cfg.athresh_params.cooldown_sec = 0.0;
    if (tm_init(&m, &cfg) != ORCHKV_OK) return -1;
    kv_block_t *b = calloc(n, sizeof(kv_block_t));
    for (uint32_t i = 0; i < n; i++) {
        b[i].block_id = ids[i];
        b[i].tier = (StorageTier)tiers[i];
        b[i].flags = flags[i];
        b[i].state = tiers[i] == 0 ? KV_STATE_HOT : KV_STATE_WARM;
        b[i].data_ptr = calloc(1, 64);
        memset(b[i].data_ptr, (int)(i & 0xFF), 64);
        tm_register_block(&m, &b[i]);
    }
    for (uint32_t t = 0; t < n_touch; t++) tm_notify_access(&m, &b[touch[t]]);
    for (uint32_t s = 0; s < steps; s++) {
        for (uint32_t r = rep_off[s]; r < rep_off[s + 1]; r++) tm_notify_attn(&m, rep_ids[r], rep_w[r]);
        tm_step_done(&m);
        tm_set_usage(&m, gpu_ratio[s], dram_ratio[s]);
        tm_schedule_once(&m);
    }
    tm_stats_t st;
    tm_get_stats(&m, &st);
    o[0] = (double)st.gpu_demotes;
    o[1] = (double)st.dram_demotes;
    o[2] = (double)st.migration_stats.blocks_migrated;
    o[3] = (double)st.migration_stats.op_errors;
    for (int i = 0; i < 6; i++) {
        o[4 + i] = (double)st.migration_stats.op_count[i];
        o[10 + i] = (double)st.migration_stats.op_bytes[i] / 64.0;
    }
    for (uint32_t i = 0; i < n; i++) {
        out_tier[i] = (int)b[i].tier;
        out_state[i] = (int)b[i].state;
        out_byte[i] = b[i].data_ptr ? (int)((unsigned char *)b[i].data_ptr)[63] : -1;
        free(b[i].data_ptr);
    }
    tm_destroy(&m);
    free(b);
    return 0;
}

static double now_s(void)
{
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + (double)ts.tv_nsec * 1e-9;
}

/* ------------------------------------------------------------------------
 * Reference CPU arm for one decode step over a sample of blocks.
 *
 * ids[n] are the sample's block ids, w[n] their per-step attention mass
 * (computed by the caller with the oracle's fixed-order reduction, timed
 * separately).  One step = attn_tracker_update_batch + tm_step_done +
 * tm_set_usage + tm_schedule_once, then the FastKVCacheManager eviction order
 * (python/orchkv/fast_kvcache_manager.py:307-321: sort by
 * tm_get_block_score) restated as a C sort over the same getter, taking the
 * coldest k_evict.  Times in seconds go to t[0..2]: update+step_done,
 * schedule_once, selection.
 * ------------------------------------------------------------------------ */
typedef struct { float s; uint64_t id; } sc_t;
static int cmp_sc(const void *a, const void *b)
{
    const sc_t *x = a, *y = b;
    if (x->s < y->s) return -1;
    if (x->s > y->s) return 1;
    return x->id < y->id ? -1 : (x->id > y->id);
}

uint32_t ref_arm_sched_step(void *h, const uint64_t *ids, const float *w,
                            uint32_t n, float gpu_ratio, uint32_t k_evict,
                            uint64_t *victims, double *t)
{
    ref_tm_t *r = h;
    double t0 = now_s();
    attn_tracker_update_batch(&r->m.tracker, ids, w, n);
    tm_step_done(&r->m);
    double t1 = now_s();
    tm_set_usage(&r->m, gpu_ratio, 0.0f);
    tm_schedule_once(&r->m);
    double t2 = now_s();
    sc_t *v = malloc((size_t)(n ? n : 1) * sizeof(sc_t));
    uint32_t m = 0;
    for (uint32_t i = 0; i < r->n; i++) {
        kv_block_t *b = r->blks[i];
        if (b->tier != TIER_GPU_HBM) continue;
        v[m].s = tm_get_block_score(&r->m, b->block_id);
        v[m].id = b->block_id;
        m++;
    }
    qsort(v, m, sizeof(sc_t), cmp_sc);
    uint32_t c = k_evict < m ? k_evict : m;
    for (uint32_t i = 0; i < c; i++) victims[i] = v[i].id;
    free(v);
    double t3 = now_s();
    t[0] = t1 - t0; t[1] = t2 - t1; t[2] = t3 - t2;
    return c;
}

/* ------------------------------------------------------------------------
 * Reference data plane (real CUDA copies through the reference's own
 * orchkv_api): create requests, prefill from host, and migrate per block.
 * ------------------------------------------------------------------------ */
int ref_api_init(int dev, size_t gpu_pool, size_t dram_pool, uint32_t tpb,
                 uint32_t d_head, int dtype, int streams, uint32_t mbph,
                 const char *base_dir)
{
    orchkv_config_t cfg;
    orchkv_config_default(&cfg);
    cfg.gpu_device_id = dev;
    cfg.gpu_pool_bytes = gpu_pool;
    cfg.dram_pool_bytes = dram_pool;
    cfg.tokens_per_block = tpb;
    cfg.d_head = d_head;
    cfg.dtype = (DataType)dtype;
    cfg.num_cuda_streams = streams;
    cfg.max_blocks_per_head = mbph;
    if (base_dir) cfg.orchfs_base_dir = base_dir;
    return orchkv_init(&cfg);
}
int   ref_api_shutdown(void) { return orchkv_shutdown(); }
void *ref_api_request_create(uint64_t id, uint32_t L, uint32_t H) { return orchkv_request_create(id, L, H); }
int   ref_api_request_destroy(void *c) { return orchkv_request_destroy(c); }
int   ref_api_prefill(void *c, uint32_t l, const void *k, const void *v, uint32_t n) { return orchkv_prefill(c, l, k, v, n); }
int   ref_api_append(void *c, uint32_t l, const void *k, const void *v) { return orchkv_append_token(c, l, k, v); }
int   ref_api_evict(void *c, uint32_t l, uint32_t h, uint32_t b) { return orchkv_evict_to_dram(c, l, h, b); }
int   ref_api_promote(void *c, uint32_t l, uint32_t h, uint32_t b) { return orchkv_promote_to_gpu(c, l, h, b); }
int   ref_api_evict_cold(void *c, uint32_t l, uint32_t h, uint32_t b) { return orchkv_evict_cold(c, l, h, b); }
int   ref_api_promote_storage(void *c, uint32_t l, uint32_t h, uint32_t b) { return orchkv_promote_from_storage(c, l, h, b); }
int   ref_api_get(void *c, uint32_t l, uint32_t h, uint32_t b, void **k, void **v) { return orchkv_get_kv_block(c, l, h, b, k, v); }
void *ref_api_dram_base(void) { dram_tier_t *d = orchkv_dram_tier(); return d ? d->pool_base : NULL; }
void *ref_api_gpu_base(void) { gpu_tier_t *g = orchkv_gpu_tier(); return g ? g->pool_base : NULL; }
/* tier and data pointer of block (l, h, b) of a request, without migrating it */
int ref_api_block(void *c, uint32_t l, uint32_t h, uint32_t b, int *tier, void **data)
{
    kv_block_t *blk = kv_request_get_block((kv_request_ctx_t *)c, l, h, b);
    if (!blk) return ORCHKV_ERR_NOT_FOUND;
    *tier = (int)blk->tier;
    *data = blk->data_ptr;
    return ORCHKV_OK;
}

/* Evict then promote a list of (layer, head, block) triples of one request,
 * timing each phase (seconds in t[0], t[1]). */
int ref_api_migrate_list(void *c, const uint32_t *lhb, uint32_t n_evict,
                         uint32_t n_promote, double *t)
{
    double t0 = now_s();
    for (uint32_t i = 0; i < n_evict; i++) {
        int rc = orchkv_evict_to_dram(c, lhb[3 * i], lhb[3 * i + 1], lhb[3 * i + 2]);
        if (rc != ORCHKV_OK) return rc;
    }
    double t1 = now_s();
    for (uint32_t i = 0; i < n_promote; i++) {
        int rc = orchkv_promote_to_gpu(c, lhb[3 * i], lhb[3 * i + 1], lhb[3 * i + 2]);
        if (rc != ORCHKV_OK) return rc;
    }
    double t2 = now_s();
    t[0] = t1 - t0; t[1] = t2 - t1;
    return ORCHKV_OK;
}
