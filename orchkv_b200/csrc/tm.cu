// tm.cu — host side of the tiered manager (tm_* C ABI).
//
// Scheduler semantics follow src/scheduler/tiered_manager.c and its
// components; per-slot arrays and every O(capacity) pass live on the GPU
// (sched_kernels.cu, select_kernels.cu).  What stays on the host is what the
// reference keeps in caller-owned host structures: the registry of borrowed
// kv_block_t records, the intrusive LRU list threaded through them, the
// bounded 4n LRU-tail victim scan, the transfer/alloc callbacks, the scalar
// threshold controller and the counters.
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include <cmath>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "kernels.h"
#include "orchkv/tiered_manager.h"
#include "tm_internal.h"

using namespace okv;

namespace {

constexpr uint32_t kHeapCap = 1024;    // prefetch_init(..., heap_cap 0 -> 1024)
constexpr uint32_t kTrackCap = 512;    // PREFETCH_TRACK_CAP

double now_sec()
{
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + (double)ts.tv_nsec * 1e-9;
}

uint32_t pow2_cap(uint32_t v)
{
    uint32_t c = 64;
    if (v < 64) v = 64;
    while (c < v) c <<= 1;
    return c;
}

float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

}  // namespace

TmImpl *tm_impl(const tiered_manager_t *m)
{
    return m ? static_cast<TmImpl *>(m->impl) : nullptr;
}

// ---------------------------------------------------------------------------
// Device state lifetime
// ---------------------------------------------------------------------------

static int alloc_device(TmImpl *t)
{
    const size_t n = t->cap;
    SchedDev &d = t->d;
    memset(&d, 0, sizeof(d));
    d.cap = t->cap;
    d.mask = t->mask;
    uint32_t tiles = 0;
    const size_t sel_words = select_scratch_words(t->cap, &tiles);
    // every sub-array below is rounded up to 256 bytes: 32 slots of padding
    const size_t bytes = n * (4 * 4 + 4 + 8 + 4 + 7 + 4) + 512 * 4 + sel_words * 4 +
                         sizeof(ClassCounts) + 64 * 4 + 256 + 34 * 256;
    OKV_CUDA_TRY(cudaMalloc((void **)&t->dev_block, bytes));
    OKV_CUDA_TRY(cudaMemsetAsync(t->dev_block, 0, bytes, t->stream));
    char *p = t->dev_block;
    auto take = [&](size_t sz) { char *q = p; p += (sz + 255) & ~size_t(255); return q; };
    d.sum = (float *)take(n * 4);
    d.mx = (float *)take(n * 4);
    d.ema = (float *)take(n * 4);
    d.hot = (float *)take(n * 4);
    d.hits = (uint32_t *)take(n * 4);
    d.last = (unsigned long long *)take(n * 8);
    d.key = (uint32_t *)take(n * 4);
    d.tact = (uint8_t *)take(n);
    d.cact = (uint8_t *)take(n);
    d.cflags = (uint8_t *)take(n);
    d.heat = (uint8_t *)take(n);
    d.tier = (uint8_t *)take(n);
    d.bflags = (uint8_t *)take(n);
    d.bstate = (uint8_t *)take(n);
    float *table = (float *)take(512 * 4);
    d.table = table;
    t->sc.hist_local = (uint32_t *)take((4096 + 16) * 4);
    t->sc.hist_global = (uint32_t *)take((4096 + 16) * 4);
    t->sc.state = (uint32_t *)take(16 * 4);
    t->sc.max_tiles = tiles;
    t->sc.tile_counts = (uint32_t *)take((size_t)2 * tiles * 4);
    t->sc.tile_offsets = (uint32_t *)take((size_t)2 * tiles * 4);
    t->counts = (ClassCounts *)take(sizeof(ClassCounts));
    t->small = (uint32_t *)take(64 * 4);
    t->report_mark = (uint32_t *)take(n * 4);
    t->report_flag = (uint32_t *)take(4);
    t->report_epoch = 0;
    // TIER_NONE for never-registered slots keeps them out of every selection
    OKV_CUDA_TRY(cudaMemsetAsync(d.tier, TIER_NONE, n, t->stream));
    OKV_CUDA_TRY(cudaMemcpyAsync(table, t->table, 512 * 4, cudaMemcpyHostToDevice, t->stream));

    // pinned host mirrors for the getters and pinned staging for uploads
    OKV_CUDA_TRY(cudaMallocHost((void **)&t->m_hot, n * 4));
    OKV_CUDA_TRY(cudaMallocHost((void **)&t->m_heat, n));
    OKV_CUDA_TRY(cudaMallocHost((void **)&t->m_cact, n));
    OKV_CUDA_TRY(cudaMallocHost((void **)&t->m_cflags, n));
    OKV_CUDA_TRY(cudaMallocHost((void **)&t->h_small, 64 * 4));
    OKV_CUDA_TRY(cudaStreamSynchronize(t->stream));
    return ORCHKV_OK;
}

static void free_device(TmImpl *t)
{
    if (t->stream) cudaStreamSynchronize(t->stream);
    cudaFree(t->dev_block);
    cudaFree(t->up_dev);
    cudaFree(t->reg_dev);
    cudaFree(t->in_stage);
    cudaFree(t->report_scratch);
    if (t->early_copy) cudaStreamSynchronize(t->early_copy);
    for (StagedInput &e : t->early) {
        cudaFree(e.dev);
        if (e.ready) cudaEventDestroy(e.ready);
        if (e.consumed) cudaEventDestroy(e.consumed);
        e = StagedInput();
    }
    if (t->early_copy) cudaStreamDestroy(t->early_copy);
    t->early_copy = nullptr;
    for (auto &e : t->rep_ev) if (e) { cudaEventDestroy(e); e = nullptr; }
    cudaFreeHost(t->m_hot);
    cudaFreeHost(t->m_heat);
    cudaFreeHost(t->m_cact);
    cudaFreeHost(t->m_cflags);
    cudaFreeHost(t->h_small);
    cudaFreeHost(t->up_host);
    cudaFreeHost(t->reg_host);
    if (t->own_stream) cudaStreamDestroy(t->own_stream);
}

// Grow-on-demand pinned staging + device buffer for uploads of `bytes`.
static int ensure_upload(TmImpl *t, size_t bytes)
{
    if (bytes <= t->up_cap) return ORCHKV_OK;
    size_t cap = t->up_cap ? t->up_cap : 4096;
    while (cap < bytes) cap *= 2;
    if (t->stream) cudaStreamSynchronize(t->stream);
    cudaFreeHost(t->up_host);
    cudaFree(t->up_dev);
    t->up_host = nullptr;
    t->up_dev = nullptr;
    OKV_CUDA_TRY(cudaMallocHost((void **)&t->up_host, cap));
    OKV_CUDA_TRY(cudaMalloc((void **)&t->up_dev, cap));
    t->up_cap = cap;
    return ORCHKV_OK;
}

// ---------------------------------------------------------------------------
// Pending host-side work: slot ops (register/unregister/tier changes) and
// per-block reports, applied on the device in one upload.
// ---------------------------------------------------------------------------

int tm_flush_locked(TmImpl *t)
{
    const uint32_t n_ops = (uint32_t)t->ops_slot.size();
    const uint32_t n_rep = (uint32_t)t->pending.size();
    if (n_ops == 0 && n_rep == 0) return ORCHKV_OK;
    const size_t bytes = (size_t)n_ops * 8 + (size_t)n_rep * 12 + 64;
    // the previous upload must have been consumed before the staging is reused
    OKV_CUDA_TRY(cudaStreamSynchronize(t->stream));
    int rc = ensure_upload(t, bytes);
    if (rc) return rc;
    char *h = t->up_host;
    uint32_t *ops_slot = (uint32_t *)h;
    memcpy(ops_slot, t->ops_slot.data(), (size_t)n_ops * 4);
    uint8_t *ops_b = (uint8_t *)(h + (size_t)n_ops * 4);
    memcpy(ops_b, t->ops_b.data(), (size_t)n_ops * 4);
    size_t off = (size_t)n_ops * 8;
    uint32_t *rs = (uint32_t *)(h + off);
    float *rsum = (float *)(h + off + (size_t)n_rep * 4);
    float *rmax = (float *)(h + off + (size_t)n_rep * 8);
    uint32_t j = 0;
    for (auto &kv : t->pending) {
        rs[j] = kv.first;
        rsum[j] = kv.second.sum;
        rmax[j] = kv.second.max;
        j++;
    }
    OKV_CUDA_TRY(cudaMemcpyAsync(t->up_dev, h, bytes, cudaMemcpyHostToDevice, t->stream));
    char *dv = t->up_dev;
    rc = launch_slot_ops((const uint32_t *)dv, (const uint8_t *)(dv + (size_t)n_ops * 4),
                         n_ops, t->d, t->stream);
    if (rc) return rc;
    rc = launch_report_apply((const uint32_t *)(dv + off),
                             (const float *)(dv + off + (size_t)n_rep * 4),
                             (const float *)(dv + off + (size_t)n_rep * 8), n_rep, t->d,
                             t->step, t->stream);
    if (rc) return rc;
    t->ops_slot.clear();
    t->ops_b.clear();
    t->pending.clear();
    t->mirror_dirty = true;
    return ORCHKV_OK;
}

static void queue_op(TmImpl *t, uint32_t slot, uint8_t op, uint8_t flags, uint8_t tier,
                     uint8_t state)
{
    t->ops_slot.push_back(slot);
    t->ops_b.push_back(op);
    t->ops_b.push_back(flags);
    t->ops_b.push_back(tier);
    t->ops_b.push_back(state);
}

// Bring the device's per-slot tier/flags/state view up to date with the
// borrowed kv_block_t records (callers may change them in place).
static void sync_registry_view(TmImpl *t)
{
    for (size_t i = 0; i < t->blocks.size(); i++) {
        kv_block_t *b = t->blocks[i];
        RegShadow &s = t->shadow[i];
        if (s.tier != (uint8_t)b->tier || s.flags != b->flags || s.state != (uint8_t)b->state) {
            s.tier = (uint8_t)b->tier;
            s.flags = b->flags;
            s.state = (uint8_t)b->state;
            queue_op(t, (uint32_t)(b->block_id & t->mask), 2, s.flags, s.tier, s.state);
        }
    }
}

int tm_refresh_mirror_locked(TmImpl *t)
{
    int rc = tm_flush_locked(t);
    if (rc) return rc;
    if (!t->mirror_dirty) return ORCHKV_OK;
    const size_t n = t->cap;
    OKV_CUDA_TRY(cudaMemcpyAsync(t->m_hot, t->d.hot, n * 4, cudaMemcpyDeviceToHost, t->stream));
    OKV_CUDA_TRY(cudaMemcpyAsync(t->m_heat, t->d.heat, n, cudaMemcpyDeviceToHost, t->stream));
    OKV_CUDA_TRY(cudaMemcpyAsync(t->m_cact, t->d.cact, n, cudaMemcpyDeviceToHost, t->stream));
    OKV_CUDA_TRY(cudaMemcpyAsync(t->m_cflags, t->d.cflags, n, cudaMemcpyDeviceToHost, t->stream));
    OKV_CUDA_TRY(cudaStreamSynchronize(t->stream));
    t->mirror_dirty = false;
    return ORCHKV_OK;
}

// ---------------------------------------------------------------------------
// LRU list through kv_block_t.prev/next (src/scheduler/eviction_policy.c:9-48)
// ---------------------------------------------------------------------------

static bool lru_in(TmImpl *t, kv_block_t *b) { return b == t->lru_head || b->prev != nullptr; }

static void lru_detach(TmImpl *t, kv_block_t *b)
{
    if (b->prev) b->prev->next = b->next; else t->lru_head = b->next;
    if (b->next) b->next->prev = b->prev; else t->lru_tail = b->prev;
    b->prev = b->next = nullptr;
    t->lru_count--;
}

static void lru_push_front(TmImpl *t, kv_block_t *b)
{
    b->prev = nullptr;
    b->next = t->lru_head;
    if (t->lru_head) t->lru_head->prev = b; else t->lru_tail = b;
    t->lru_head = b;
    t->lru_count++;
}

static void lru_touch(TmImpl *t, kv_block_t *b)
{
    if (lru_in(t, b)) lru_detach(t, b);
    lru_push_front(t, b);
}

static void lru_remove(TmImpl *t, kv_block_t *b)
{
    if (lru_in(t, b)) lru_detach(t, b);
}

// ---------------------------------------------------------------------------
// Threshold controller (src/scheduler/adaptive_threshold.c:82-169)
// ---------------------------------------------------------------------------

static bool athresh_update(TmImpl *t)
{
    if (now_sec() - t->last_adjust < t->cooldown_sec) return false;
    bool changed = false;
    const float st = t->adjust_step;
    if (t->gpu_ratio > t->gpu_hwm) {
        float nh = clampf(t->th_hot + st, t->min_hot, t->max_hot);
        if (nh != t->th_hot) { t->th_hot = nh; t->adj_up++; changed = true; }
    } else if (t->gpu_ratio < t->gpu_lwm) {
        float nh = clampf(t->th_hot - st, t->min_hot, t->max_hot);
        if (nh != t->th_hot) { t->th_hot = nh; t->adj_down++; changed = true; }
    }
    if (t->dram_ratio > t->dram_hwm) {
        float nw = clampf(t->th_warm + st, t->min_warm, t->max_warm);
        if (nw != t->th_warm) { t->th_warm = nw; t->adj_up++; changed = true; }
    } else if (t->dram_ratio < t->dram_lwm) {
        float nw = clampf(t->th_warm - st, t->min_warm, t->max_warm);
        if (nw != t->th_warm) { t->th_warm = nw; t->adj_down++; changed = true; }
    }
    if (changed) t->last_adjust = now_sec();
    return changed;
}

// ---------------------------------------------------------------------------
// Migration engine restated for the callback path
// (src/scheduler/migration_engine.c:36-245)
// ---------------------------------------------------------------------------

static MigrateOp determine_op(StorageTier from, StorageTier to)
{
    if (from == to) return MIGRATE_OP_COUNT;
    const bool fs = from == TIER_NVM || from == TIER_SSD, ts = to == TIER_NVM || to == TIER_SSD;
    if (from == TIER_GPU_HBM && to == TIER_HOST_DRAM) return MIGRATE_DEMOTE_GPU2DRAM;
    if (from == TIER_HOST_DRAM && ts) return MIGRATE_DEMOTE_DRAM2STOR;
    if (from == TIER_GPU_HBM && ts) return MIGRATE_DEMOTE_GPU2STOR;
    if (fs && to == TIER_HOST_DRAM) return MIGRATE_PROMOTE_STOR2DRAM;
    if (from == TIER_HOST_DRAM && to == TIER_GPU_HBM) return MIGRATE_PROMOTE_DRAM2GPU;
    if (fs && to == TIER_GPU_HBM) return MIGRATE_PROMOTE_STOR2GPU;
    return MIGRATE_OP_COUNT;
}

static KVBlockState target_state(StorageTier t)
{
    switch (t) {
    case TIER_GPU_HBM: return KV_STATE_HOT;
    case TIER_HOST_DRAM: return KV_STATE_WARM;
    case TIER_NVM: case TIER_SSD: return KV_STATE_COLD;
    default: return KV_STATE_EVICTED;
    }
}

static int mig_execute_one(TmImpl *t, kv_block_t *b, StorageTier target, void *dst,
                           size_t size)
{
    if (!t->transfer_fn) return ORCHKV_ERR_INIT;
    if (b->flags & KV_FLAG_PIN) return ORCHKV_ERR_LOCKED;
    if (b->state == KV_STATE_MIGRATING) return ORCHKV_ERR_STATE;
    const MigrateOp op = determine_op(b->tier, target);
    if (op >= MIGRATE_OP_COUNT) return ORCHKV_ERR_INVALID;
    const bool two_hop = op == MIGRATE_DEMOTE_GPU2STOR || op == MIGRATE_PROMOTE_STOR2GPU;
    if (two_hop) return ORCHKV_ERR_INVALID;   // no intermediate buffer on this path
    const KVBlockState saved = b->state;
    b->state = KV_STATE_MIGRATING;
    const int rc = t->transfer_fn(b, dst, size, op, t->transfer_ctx);
    if (rc != ORCHKV_OK) {
        b->state = saved;
        t->mig_errors++;
        return rc;
    }
    // single-hop ops are counted here and again below, as the reference does
    t->op_count[op]++;
    t->op_bytes[op] += size;
    b->tier = target;
    b->data_ptr = (target == TIER_NVM || target == TIER_SSD) ? nullptr : dst;
    b->state = target_state(target);
    t->op_count[op]++;
    t->op_bytes[op] += size;
    t->blocks_migrated++;
    if (target == TIER_NVM || target == TIER_SSD) lru_remove(t, b);
    else lru_touch(t, b);
    return ORCHKV_OK;
}

struct Cand { kv_block_t *blk; float score; };

// eviction_policy.c:55-143: scan at most 4n blocks from the LRU tail.
static uint32_t select_victims(TmImpl *t, StorageTier tier, uint32_t n, Cand *out)
{
    if (n == 0) return 0;
    uint32_t found = 0, scanned = 0, pos = 0;
    const uint32_t max_scan = n * 4;
    for (kv_block_t *cur = t->lru_tail; cur && scanned < max_scan; cur = cur->prev, pos++) {
        scanned++;
        if (cur->tier != tier || (cur->flags & KV_FLAG_PIN) || cur->state == KV_STATE_MIGRATING)
            continue;
        const uint32_t s = (uint32_t)(cur->block_id & t->mask);
        const float h = t->m_cact[s] ? t->m_hot[s] : 0.0f;
        const float heat_part = (1.0f - h) * t->w_heat;
        const float lru_part = t->lru_count > 1
            ? ((float)(t->lru_count - 1 - pos) / (float)(t->lru_count - 1)) * t->w_lru
            : 0.0f;
        Cand c{cur, heat_part + lru_part};
        if (found < n) {
            uint32_t i = found;
            while (i > 0 && out[i - 1].score < c.score) { out[i] = out[i - 1]; i--; }
            out[i] = c;
            found++;
        } else if (c.score > out[found - 1].score) {
            uint32_t i = found - 1;
            while (i > 0 && out[i - 1].score < c.score) { out[i] = out[i - 1]; i--; }
            out[i] = c;
        }
    }
    return found;
}

static void do_demote(TmImpl *t, bool gpu)
{
    t->demote_checks++;
    const bool need = gpu ? t->gpu_ratio > t->gpu_hwm : t->dram_ratio > t->dram_hwm;
    if (!need) return;
    // without a transfer callback every migration returns ERR_INIT before any
    // state changes (migration_engine.c:111-119): nothing observable happens
    if (!t->transfer_fn) return;
    if (tm_refresh_mirror_locked(t) != ORCHKV_OK) return;
    std::vector<Cand> c(t->demote_batch_size);
    const StorageTier from = gpu ? TIER_GPU_HBM : TIER_HOST_DRAM;
    const StorageTier to = gpu ? TIER_HOST_DRAM : TIER_NVM;
    const uint32_t found = select_victims(t, from, t->demote_batch_size, c.data());
    for (uint32_t i = 0; i < found; i++) {
        kv_block_t *b = c[i].blk;
        void *dst = t->alloc_fn ? t->alloc_fn(t->block_data_size, to, t->alloc_ctx) : nullptr;
        if (!dst && t->alloc_fn) break;
        void *old = b->data_ptr;
        const int rc = mig_execute_one(t, b, to, dst, t->block_data_size);
        if (rc == ORCHKV_OK) {
            if (t->free_fn && old) t->free_fn(old, from, t->alloc_ctx);
            if (gpu) t->gpu_demotes++; else t->dram_demotes++;
        } else if (t->free_fn && dst) {
            t->free_fn(dst, to, t->alloc_ctx);
        }
    }
    sync_registry_view(t);
}

// tiered_manager.c:284-312 + prefetch_scheduler.c:131-228: only the counters
// are observable from this path, so the scan is a device count.
static int do_prefetch(TmImpl *t)
{
    const uint32_t n = (uint32_t)t->blocks.size();
    uint32_t scan_n = 0;
    t->reg_tmp.resize(n);
    uint32_t m = 0;
    for (uint32_t i = 0; i < n; i++) {
        kv_block_t *b = t->blocks[i];
        if (b->tier != TIER_GPU_HBM && b->tier != TIER_NONE) {
            t->reg_tmp[m].slot = (uint32_t)(b->block_id & t->mask);
            t->reg_tmp[m].tier = (uint8_t)b->tier;
            m++;
            scan_n++;
        }
    }
    t->total_scanned += scan_n;
    uint32_t qualifying = 0;
    if (m > 0) {
        const size_t need = (size_t)m * 5 + 64;
        if (need > t->reg_cap) {
            size_t cap = t->reg_cap ? t->reg_cap : 4096;
            while (cap < need) cap *= 2;
            cudaStreamSynchronize(t->stream);
            cudaFreeHost(t->reg_host);
            cudaFree(t->reg_dev);
            t->reg_host = nullptr;
            t->reg_dev = nullptr;
            OKV_CUDA_TRY(cudaMallocHost((void **)&t->reg_host, cap));
            OKV_CUDA_TRY(cudaMalloc((void **)&t->reg_dev, cap));
            t->reg_cap = cap;
        }
        uint32_t *hs = (uint32_t *)t->reg_host;
        uint8_t *ht = (uint8_t *)(t->reg_host + (size_t)m * 4);
        for (uint32_t i = 0; i < m; i++) { hs[i] = t->reg_tmp[i].slot; ht[i] = t->reg_tmp[i].tier; }
        OKV_CUDA_TRY(cudaMemcpyAsync(t->reg_dev, t->reg_host, (size_t)m * 5,
                                     cudaMemcpyHostToDevice, t->stream));
        int rc = launch_registry_count((const uint32_t *)t->reg_dev,
                                       (const uint8_t *)(t->reg_dev + (size_t)m * 4), m, t->d,
                                       t->th_gpu_pf, t->th_dram_pf, t->small, t->stream);
        if (rc) return rc;
        OKV_CUDA_TRY(cudaMemcpyAsync(t->h_small, t->small, 4, cudaMemcpyDeviceToHost, t->stream));
        OKV_CUDA_TRY(cudaStreamSynchronize(t->stream));
        qualifying = t->h_small[0];
    }
    const uint32_t room = kHeapCap - t->heap_size;
    const uint32_t enq = qualifying < room ? qualifying : room;
    t->heap_size += enq;
    t->total_enqueued += enq;
    uint32_t lim = t->prefetch_batch_size < t->prefetch_budget ? t->prefetch_batch_size
                                                               : t->prefetch_budget;
    const uint32_t d = lim < t->heap_size ? lim : t->heap_size;
    t->heap_size -= d;
    for (uint32_t i = 0; i < d; i++)
        if (t->tracked < kTrackCap) t->tracked++;
    t->total_dispatched += d;
    t->prefetches_dispatched += d;
    return ORCHKV_OK;
}

static SchedParams params_of(const TmImpl *t)
{
    SchedParams p;
    p.lambda = t->lambda;
    p.one_minus = 1.0f - t->lambda;
    p.alpha = t->alpha;
    p.beta = t->beta;
    p.gamma = t->gamma;
    p.th_hot = t->th_hot;
    p.th_warm = t->th_warm;
    p.step = t->step;
    return p;
}

static void *sched_loop(void *arg)
{
    tiered_manager_t *m = (tiered_manager_t *)arg;
    TmImpl *t = tm_impl(m);
    while (t->running) {
        usleep(t->schedule_interval_us);
        tm_schedule_once(m);
    }
    return nullptr;
}

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------

extern "C" {

void tm_config_default(tm_config_t *c)
{
    if (!c) return;
    memset(c, 0, sizeof(*c));
    c->tracker_capacity = 4096;
    c->ema_lambda = 0.9f;
    hcc_params_default(&c->hcc_params);
    athresh_params_default(&c->athresh_params);
    c->w_heat = 0.7f;
    c->w_lru = 0.3f;
    c->tokens_per_block = 64;
    c->prefetch_budget = 16;
    c->threshold_to_gpu = 0.5f;
    c->threshold_to_dram = 0.2f;
    c->block_data_size = 32 * 1024;
    c->schedule_interval_us = 1000;
    c->demote_batch_size = 8;
    c->prefetch_batch_size = 8;
    c->max_blocks = 4096;
    c->auto_schedule = false;
}

int tm_init(tiered_manager_t *m, const tm_config_t *cfg)
{
    if (!m || !cfg) return ORCHKV_ERR_INVALID;
    memset(m, 0, sizeof(*m));
    if (cfg->tracker_capacity == 0) return ORCHKV_ERR_INVALID;
    TmImpl *t = new (std::nothrow) TmImpl();
    if (!t) return ORCHKV_ERR_OOM;
    cudaGetDevice(&t->device);
    t->cap = pow2_cap(cfg->tracker_capacity);
    t->mask = t->cap - 1;
    t->lambda = (cfg->ema_lambda > 0.0f && cfg->ema_lambda < 1.0f) ? cfg->ema_lambda : 0.9f;
    t->alpha = cfg->hcc_params.alpha;
    t->beta = cfg->hcc_params.beta;
    t->gamma = cfg->hcc_params.gamma;
    t->tau = cfg->hcc_params.recency_tau;
    {   // hotcold_classifier.c:27-34: the table is built here with libm expf
        float tau = t->tau < 1.0f ? 1.0f : t->tau;
        const float inv = 1.0f / tau;
        for (int k = 0; k < 512; k++) t->table[k] = expf(-(float)k * inv);
    }
    const athresh_params_t &ap = cfg->athresh_params;
    t->th_hot = ap.threshold_hot;
    t->th_warm = ap.threshold_warm;
    t->min_hot = ap.min_hot; t->max_hot = ap.max_hot;
    t->min_warm = ap.min_warm; t->max_warm = ap.max_warm;
    t->gpu_hwm = ap.gpu_hwm; t->gpu_lwm = ap.gpu_lwm;
    t->dram_hwm = ap.dram_hwm; t->dram_lwm = ap.dram_lwm;
    t->adjust_step = ap.adjust_step > 0.0f ? ap.adjust_step : 0.02f;
    t->cooldown_sec = ap.cooldown_sec >= 0.0 ? ap.cooldown_sec : 0.5;
    t->last_adjust = now_sec();
    t->w_heat = cfg->w_heat;
    t->w_lru = cfg->w_lru;
    t->prefetch_budget = cfg->prefetch_budget > 0 ? cfg->prefetch_budget : 16;
    t->th_gpu_pf = cfg->threshold_to_gpu;
    t->th_dram_pf = cfg->threshold_to_dram;
    t->transfer_fn = cfg->transfer_fn;
    t->transfer_ctx = cfg->transfer_ctx;
    t->alloc_fn = cfg->alloc_fn;
    t->free_fn = cfg->free_fn;
    t->alloc_ctx = cfg->alloc_ctx;
    t->block_data_size = cfg->block_data_size;
    t->schedule_interval_us = cfg->schedule_interval_us;
    t->demote_batch_size = cfg->demote_batch_size;
    t->prefetch_batch_size = cfg->prefetch_batch_size;
    t->max_blocks = cfg->max_blocks > 0 ? cfg->max_blocks : 4096;
    // blocking: ordered with the legacy default stream until tm_set_stream
    if (cudaStreamCreate(&t->own_stream) != cudaSuccess) {
        delete t;
        return ORCHKV_ERR_CUDA;
    }
    t->stream = t->own_stream;
    int rc = alloc_device(t);
    if (rc != ORCHKV_OK) {
        free_device(t);
        delete t;
        return rc;
    }
    m->impl = t;
    if (cfg->auto_schedule) tm_start(m);
    return ORCHKV_OK;
}

void tm_destroy(tiered_manager_t *m)
{
    TmImpl *t = tm_impl(m);
    if (!t) return;
    tm_stop(m);
    okv_manager_destroyed(m);
    free_device(t);
    delete t;
    m->impl = nullptr;
}

int tm_register_block(tiered_manager_t *m, kv_block_t *blk)
{
    TmImpl *t = tm_impl(m);
    if (!t || !blk) return ORCHKV_ERR_INVALID;
    std::lock_guard<std::mutex> g(t->mu);
    if (t->blocks.size() >= t->max_blocks) return ORCHKV_ERR_TIER_FULL;
    t->blocks.push_back(blk);
    t->shadow.push_back(RegShadow{(uint8_t)blk->tier, blk->flags, (uint8_t)blk->state});
    const uint32_t s = (uint32_t)(blk->block_id & t->mask);
    t->pending.erase(s);   // registration zeroes the slot, dropping earlier reports
    queue_op(t, s, 0, blk->flags, (uint8_t)blk->tier, (uint8_t)blk->state);
    lru_touch(t, blk);
    t->mirror_dirty = true;
    return ORCHKV_OK;
}

void tm_unregister_block(tiered_manager_t *m, kv_block_t *blk)
{
    TmImpl *t = tm_impl(m);
    if (!t || !blk) return;
    std::lock_guard<std::mutex> g(t->mu);
    for (size_t i = 0; i < t->blocks.size(); i++) {
        if (t->blocks[i] == blk) {
            t->blocks[i] = t->blocks.back();
            t->shadow[i] = t->shadow.back();
            t->blocks.pop_back();
            t->shadow.pop_back();
            break;
        }
    }
    lru_remove(t, blk);
    const uint32_t s = (uint32_t)(blk->block_id & t->mask);
    t->pending.erase(s);
    queue_op(t, s, 1, 0, TIER_NONE, 0);
    t->mirror_dirty = true;
}

void tm_notify_attn(tiered_manager_t *m, uint64_t block_id, float w)
{
    TmImpl *t = tm_impl(m);
    if (!t) return;
    std::lock_guard<std::mutex> g(t->mu);
    // in-order accumulation per slot, exactly attn_tracker_update's arithmetic
    // (sum starts at 0 after step_done / registration)
    PendingReport &p = t->pending[(uint32_t)(block_id & t->mask)];
    p.sum = p.sum + w;
    if (w > p.max) p.max = w;
}

void tm_notify_access(tiered_manager_t *m, kv_block_t *blk)
{
    TmImpl *t = tm_impl(m);
    if (!t || !blk) return;
    std::lock_guard<std::mutex> g(t->mu);
    lru_touch(t, blk);
}

void tm_step_done(tiered_manager_t *m)
{
    TmImpl *t = tm_impl(m);
    if (!t) return;
    std::lock_guard<std::mutex> g(t->mu);
    if (tm_flush_locked(t) != ORCHKV_OK) return;
    launch_sweep(t->d, params_of(t), true, false, nullptr, t->stream);
    t->step++;
    // prefetch_step_reset (prefetch_scheduler.c:242-256)
    t->prefetch_wasted += t->tracked;
    t->tracked = 0;
    t->heap_size = 0;
    t->mirror_dirty = true;
}

void tm_schedule_once(tiered_manager_t *m)
{
    OKV_RANGE("tm_schedule_once");
    TmImpl *t = tm_impl(m);
    if (!t) return;
    std::lock_guard<std::mutex> g(t->mu);
    sync_registry_view(t);
    if (tm_flush_locked(t) != ORCHKV_OK) return;
    launch_sweep(t->d, params_of(t), false, true, t->counts, t->stream);
    t->mirror_dirty = true;
    athresh_update(t);
    do_demote(t, true);
    do_demote(t, false);
    do_prefetch(t);
    t->schedule_cycles++;
}

int tm_start(tiered_manager_t *m)
{
    TmImpl *t = tm_impl(m);
    if (!t || t->running) return ORCHKV_ERR_STATE;
    t->running = true;
    if (pthread_create(&t->thread, nullptr, sched_loop, m) != 0) {
        t->running = false;
        return ORCHKV_ERR_INIT;
    }
    return ORCHKV_OK;
}

void tm_stop(tiered_manager_t *m)
{
    TmImpl *t = tm_impl(m);
    if (!t || !t->running) return;
    t->running = false;
    pthread_join(t->thread, nullptr);
}

void tm_set_usage(tiered_manager_t *m, float g, float d)
{
    TmImpl *t = tm_impl(m);
    if (!t) return;
    std::lock_guard<std::mutex> lk(t->mu);
    t->gpu_ratio = g;
    t->dram_ratio = d;
}

void tm_set_policy(tiered_manager_t *m, float a, float b, float g)
{
    TmImpl *t = tm_impl(m);
    if (!t) return;
    std::lock_guard<std::mutex> lk(t->mu);
    t->alpha = a;
    t->beta = b;
    t->gamma = g;
}

float tm_get_block_score(const tiered_manager_t *m, uint64_t id)
{
    TmImpl *t = tm_impl(m);
    if (!t) return 0.0f;
    std::lock_guard<std::mutex> g(t->mu);
    if (tm_refresh_mirror_locked(t) != ORCHKV_OK) return 0.0f;
    const uint32_t s = (uint32_t)(id & t->mask);
    return t->m_cact[s] ? t->m_hot[s] : 0.0f;
}

HeatLevel tm_get_block_heat(const tiered_manager_t *m, uint64_t id)
{
    TmImpl *t = tm_impl(m);
    if (!t) return HEAT_COLD;
    std::lock_guard<std::mutex> g(t->mu);
    if (tm_refresh_mirror_locked(t) != ORCHKV_OK) return HEAT_COLD;
    const uint32_t s = (uint32_t)(id & t->mask);
    return t->m_cact[s] ? (HeatLevel)t->m_heat[s] : HEAT_COLD;
}

void tm_get_stats(const tiered_manager_t *m, tm_stats_t *out)
{
    TmImpl *t = tm_impl(m);
    if (!t || !out) return;
    memset(out, 0, sizeof(*out));
    std::lock_guard<std::mutex> g(t->mu);
    out->schedule_cycles = t->schedule_cycles;
    out->gpu_demotes = t->gpu_demotes;
    out->dram_demotes = t->dram_demotes;
    out->prefetches_dispatched = t->prefetches_dispatched;
    out->gpu_used_ratio = t->gpu_ratio;
    out->dram_used_ratio = t->dram_ratio;
    if (tm_refresh_mirror_locked(t) == ORCHKV_OK) {
        // hcc_get_stats (hotcold_classifier.c:286-319): slot order, float sum
        hcc_stats_t &h = out->hcc_stats;
        float sum = 0.0f, mx = -3.402823466e+38f, mn = 3.402823466e+38f;
        uint32_t n_active = 0;
        for (uint32_t i = 0; i < t->cap; i++) {
            if (!t->m_cact[i]) continue;
            n_active++;
            const float v = t->m_hot[i];
            sum += v;
            if (v > mx) mx = v;
            if (v < mn) mn = v;
            switch (t->m_heat[i]) {
            case HEAT_HOT: h.n_hot++; break;
            case HEAT_WARM: h.n_warm++; break;
            case HEAT_COLD: h.n_cold++; break;
            }
            if (t->m_cflags[i] & KV_FLAG_ATTN_SINK) h.n_attn_sink++;
        }
        if (n_active) {
            h.avg_hotness = sum / (float)n_active;
            h.max_hotness = mx;
            h.min_hotness = mn;
        }
    }
    prefetch_stats_t &p = out->prefetch_stats;
    p.total_scanned = t->total_scanned;
    p.total_enqueued = t->total_enqueued;
    p.total_dispatched = t->total_dispatched;
    p.prefetch_hits = t->prefetch_hits;
    p.prefetch_wasted = t->prefetch_wasted;
    p.hit_rate = t->total_dispatched ? (float)t->prefetch_hits / (float)t->total_dispatched : 0.0f;
    mig_stats_t &ms = out->migration_stats;
    for (int i = 0; i < MIGRATE_OP_COUNT; i++) {
        ms.op_count[i] = t->op_count[i];
        ms.op_bytes[i] = t->op_bytes[i];
    }
    ms.op_errors = t->mig_errors;
    ms.blocks_migrated = t->blocks_migrated;
}

// ---- B200 ------------------------------------------------------------------

int tm_set_stream(tiered_manager_t *m, void *stream)
{
    TmImpl *t = tm_impl(m);
    if (!t) return ORCHKV_ERR_INVALID;
    std::lock_guard<std::mutex> g(t->mu);
    OKV_CUDA_TRY(cudaStreamSynchronize(t->stream));
    t->stream = stream ? (cudaStream_t)stream : t->own_stream;
    return ORCHKV_OK;
}

int tm_sync(tiered_manager_t *m)
{
    TmImpl *t = tm_impl(m);
    if (!t) return ORCHKV_ERR_INVALID;
    std::lock_guard<std::mutex> g(t->mu);
    int rc = tm_flush_locked(t);
    if (rc) return rc;
    OKV_CUDA_TRY(cudaStreamSynchronize(t->stream));
    return okv_data_plane_check();
}

uint32_t tm_capacity(const tiered_manager_t *m)
{
    TmImpl *t = tm_impl(m);
    return t ? t->cap : 0;
}

uint64_t tm_current_step(const tiered_manager_t *m)
{
    TmImpl *t = tm_impl(m);
    return t ? t->step : 0;
}

int tm_set_block_tier_id(tiered_manager_t *m, uint64_t block_id, int tier)
{
    TmImpl *t = tm_impl(m);
    if (!t) return ORCHKV_ERR_INVALID;
    std::lock_guard<std::mutex> g(t->mu);
    for (size_t i = 0; i < t->blocks.size(); i++) {
        if (t->blocks[i]->block_id == block_id) {
            t->blocks[i]->tier = (StorageTier)tier;
            return ORCHKV_OK;
        }
    }
    return ORCHKV_ERR_NOT_FOUND;
}

int tm_read_state(tiered_manager_t *m, float *sum, float *ema, uint32_t *hits,
                  uint64_t *last_hit, uint8_t *t_active, float *hotness, uint8_t *heat,
                  uint8_t *c_active)
{
    TmImpl *t = tm_impl(m);
    if (!t) return ORCHKV_ERR_INVALID;
    std::lock_guard<std::mutex> g(t->mu);
    int rc = tm_flush_locked(t);
    if (rc) return rc;
    const size_t n = t->cap;
    cudaStream_t s = t->stream;
    if (sum) OKV_CUDA_TRY(cudaMemcpyAsync(sum, t->d.sum, n * 4, cudaMemcpyDeviceToHost, s));
    if (ema) OKV_CUDA_TRY(cudaMemcpyAsync(ema, t->d.ema, n * 4, cudaMemcpyDeviceToHost, s));
    if (hits) OKV_CUDA_TRY(cudaMemcpyAsync(hits, t->d.hits, n * 4, cudaMemcpyDeviceToHost, s));
    if (last_hit) OKV_CUDA_TRY(cudaMemcpyAsync(last_hit, t->d.last, n * 8, cudaMemcpyDeviceToHost, s));
    if (t_active) OKV_CUDA_TRY(cudaMemcpyAsync(t_active, t->d.tact, n, cudaMemcpyDeviceToHost, s));
    if (hotness) OKV_CUDA_TRY(cudaMemcpyAsync(hotness, t->d.hot, n * 4, cudaMemcpyDeviceToHost, s));
    if (heat) OKV_CUDA_TRY(cudaMemcpyAsync(heat, t->d.heat, n, cudaMemcpyDeviceToHost, s));
    if (c_active) OKV_CUDA_TRY(cudaMemcpyAsync(c_active, t->d.cact, n, cudaMemcpyDeviceToHost, s));
    OKV_CUDA_TRY(cudaStreamSynchronize(s));
    return ORCHKV_OK;
}

// Inputs of tm_report_attn_probs in host memory (pinned or pageable) are
// copied once into the manager's staging buffer on its stream; device and
// managed memory is read in place.  The buffer grows before any copy is
// queued, so no pointer handed out earlier in the same call is stranded.
static bool on_device(const void *p)
{
    cudaPointerAttributes a;
    const cudaError_t e = cudaPointerGetAttributes(&a, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// The oldest staged upload of exactly this host range, if any: the report
// then reads the uploaded copy, after its upload, instead of copying again.
static StagedInput *take_staged(TmImpl *t, const void *host, size_t bytes)
{
    StagedInput *best = nullptr;
    for (StagedInput &e : t->early)
        if (e.pending && e.host == host && e.bytes == bytes && (!best || e.seq < best->seq))
            best = &e;
    if (!best) return nullptr;
    if (cudaStreamWaitEvent(t->stream, best->ready, 0) != cudaSuccess) return nullptr;
    best->pending = false;
    best->in_use = true;
    return best;
}

// After a report's launches: staged inputs it read may be reused once they end.
static int release_staged(TmImpl *t)
{
    for (StagedInput &e : t->early) {
        if (!e.in_use) continue;
        e.in_use = false;
        OKV_CUDA_TRY(cudaEventRecord(e.consumed, t->stream));
    }
    return ORCHKV_OK;
}

static int stage_inputs(TmImpl *t, const void **ptrs, const size_t *bytes, int n)
{
    size_t off[4] = {0}, need = 0;
    bool host[4] = {false};
    for (int i = 0; i < n; i++) {
        host[i] = ptrs[i] && bytes[i] && !on_device(ptrs[i]);
        if (host[i]) {
            if (StagedInput *e = take_staged(t, ptrs[i], bytes[i])) {
                ptrs[i] = e->dev;
                host[i] = false;
                continue;
            }
            off[i] = need;
            need += (bytes[i] + 255) & ~size_t(255);
        }
    }
    if (need == 0) return ORCHKV_OK;
    if (need > t->in_stage_cap) {
        size_t cap = t->in_stage_cap ? t->in_stage_cap : (1 << 20);
        while (cap < need) cap *= 2;
        OKV_CUDA_TRY(cudaStreamSynchronize(t->stream));   // earlier launches may still read it
        cudaFree(t->in_stage);
        t->in_stage = nullptr;
        t->in_stage_cap = 0;
        OKV_CUDA_TRY(cudaMalloc((void **)&t->in_stage, cap));
        t->in_stage_cap = cap;
    }
    for (int i = 0; i < n; i++) {
        if (!host[i]) continue;
        OKV_CUDA_TRY(cudaMemcpyAsync(t->in_stage + off[i], ptrs[i], bytes[i],
                                     cudaMemcpyHostToDevice, t->stream));
        ptrs[i] = t->in_stage + off[i];
    }
    return ORCHKV_OK;
}

// A report call's ordering state (okv::ReportOrder): a new epoch, and when
// the call computes its masses itself (scratch), room for n entry ids and
// masses in case its ids turn out to share slots.
static int begin_report(TmImpl *t, size_t n, bool scratch, okv::ReportOrder *o)
{
    if (++t->report_epoch == 0) {
        // the stamps wrapped: clear them so no old stamp equals a new epoch
        OKV_CUDA_TRY(cudaMemsetAsync(t->report_mark, 0, (size_t)t->cap * 4, t->stream));
        OKV_CUDA_TRY(cudaMemsetAsync(t->report_flag, 0, 4, t->stream));
        t->report_epoch = 1;
    }
    const size_t half = (n * 4 + 255) & ~size_t(255);
    if (scratch && 2 * half > t->report_scratch_cap) {
        size_t cap = t->report_scratch_cap ? t->report_scratch_cap : (1 << 20);
        while (cap < 2 * half) cap *= 2;
        OKV_CUDA_TRY(cudaStreamSynchronize(t->stream));   // an earlier call may still use it
        cudaFree(t->report_scratch);
        t->report_scratch = nullptr;
        t->report_scratch_cap = 0;
        OKV_CUDA_TRY(cudaMalloc((void **)&t->report_scratch, cap));
        t->report_scratch_cap = cap;
    }
    o->mark = t->report_mark;
    o->flag = t->report_flag;
    o->epoch = t->report_epoch;
    o->ids_eff = scratch ? (uint32_t *)t->report_scratch : nullptr;
    o->mass = scratch ? (float *)(t->report_scratch + half) : nullptr;
    return ORCHKV_OK;
}

int tm_report_attn_probs(tiered_manager_t *m, const float *probs, uint32_t n_rows,
                         uint32_t n_q_heads, uint32_t n_kv_heads, uint32_t row_len,
                         uint32_t tpb, const uint32_t *lens, const uint32_t *block_ids)
{
    OKV_RANGE("tm_report_attn_probs");
    TmImpl *t = tm_impl(m);
    if (!t) return ORCHKV_ERR_INVALID;
    if (!probs || !block_ids || n_rows == 0 || n_q_heads == 0 || n_kv_heads == 0 ||
        row_len == 0 || tpb == 0 || n_q_heads % n_kv_heads != 0)
        return ORCHKV_ERR_INVALID;
    std::lock_guard<std::mutex> g(t->mu);
    int rc = tm_flush_locked(t);
    if (rc) return rc;
    const size_t nb = (row_len + tpb - 1) / tpb;
    const void *in[3] = {probs, lens, block_ids};
    const size_t bytes[3] = {(size_t)n_rows * n_q_heads * row_len * sizeof(float),
                             lens ? (size_t)n_rows * sizeof(uint32_t) : 0,
                             (size_t)n_rows * n_kv_heads * nb * sizeof(uint32_t)};
    const size_t n_ent = (size_t)n_rows * n_kv_heads * nb;
    if (n_ent > 0xFFFFFFFFull) return ORCHKV_ERR_INVALID;
    rc = stage_inputs(t, in, bytes, 3);
    if (rc) return rc;
    okv::ReportOrder o;
    rc = begin_report(t, n_ent, true, &o);
    if (rc) return rc;
    t->mirror_dirty = true;
    const uint32_t *ids = (const uint32_t *)in[2];
    auto mark = [&](int i) { if (t->rep_prof) cudaEventRecord(t->rep_ev[i], t->stream); };
    mark(0);
    rc = launch_alias_mark(ids, (uint32_t)n_ent, t->d, o, t->stream);
    mark(1);
    if (!rc) rc = launch_score((const float *)in[0], n_rows, n_q_heads, n_kv_heads, row_len, tpb,
                               (const uint32_t *)in[1], ids, t->d, t->step, o, t->stream);
    mark(2);
    if (!rc) rc = launch_report_ordered(o.ids_eff, o.mass, (uint32_t)n_ent, t->d, t->step, o,
                                        t->stream);
    mark(3);
    const int rr = release_staged(t);
    return rc ? rc : rr;
}

int tm_profile_reports(tiered_manager_t *m, int on)
{
    TmImpl *t = tm_impl(m);
    if (!t) return ORCHKV_ERR_INVALID;
    std::lock_guard<std::mutex> g(t->mu);
    for (auto &e : t->rep_ev)
        if (!e) OKV_CUDA_TRY(cudaEventCreate(&e));
    t->rep_prof = on != 0;
    return ORCHKV_OK;
}

int tm_last_report_times(tiered_manager_t *m, float *mark_ms, float *score_ms, float *ordered_ms)
{
    TmImpl *t = tm_impl(m);
    if (!t) return ORCHKV_ERR_INVALID;
    std::lock_guard<std::mutex> g(t->mu);
    if (!t->rep_prof) return ORCHKV_ERR_STATE;
    OKV_CUDA_TRY(cudaEventSynchronize(t->rep_ev[3]));
    float x = 0.f;
    if (mark_ms) { OKV_CUDA_TRY(cudaEventElapsedTime(&x, t->rep_ev[0], t->rep_ev[1])); *mark_ms = x; }
    if (score_ms) { OKV_CUDA_TRY(cudaEventElapsedTime(&x, t->rep_ev[1], t->rep_ev[2])); *score_ms = x; }
    if (ordered_ms) { OKV_CUDA_TRY(cudaEventElapsedTime(&x, t->rep_ev[2], t->rep_ev[3])); *ordered_ms = x; }
    return ORCHKV_OK;
}

int tm_stage_input_async(tiered_manager_t *m, const void *host, size_t bytes)
{
    OKV_RANGE("tm_stage_input_async");
    TmImpl *t = tm_impl(m);
    if (!t) return ORCHKV_ERR_INVALID;
    std::lock_guard<std::mutex> g(t->mu);
    if (!host) {                              // drop staged inputs nobody consumed
        if (t->early_copy) OKV_CUDA_TRY(cudaStreamSynchronize(t->early_copy));
        for (StagedInput &e : t->early) e.pending = false;
        return ORCHKV_OK;
    }
    if (bytes == 0 || on_device(host)) return ORCHKV_ERR_INVALID;
    StagedInput *e = nullptr;
    for (StagedInput &x : t->early)
        if (!x.pending && (!e || x.seq < e->seq)) e = &x;
    if (!e) return ORCHKV_ERR_STATE;          // two uploads already wait for their reports
    if (!t->early_copy)
        OKV_CUDA_TRY(cudaStreamCreateWithFlags(&t->early_copy, cudaStreamNonBlocking));
    if (!e->ready) OKV_CUDA_TRY(cudaEventCreateWithFlags(&e->ready, cudaEventDisableTiming));
    if (!e->consumed) OKV_CUDA_TRY(cudaEventCreateWithFlags(&e->consumed, cudaEventDisableTiming));
    if (bytes > e->cap) {
        OKV_CUDA_TRY(cudaEventSynchronize(e->consumed));   // its last reader is done
        cudaFree(e->dev);
        e->dev = nullptr;
        e->cap = 0;
        OKV_CUDA_TRY(cudaMalloc((void **)&e->dev, bytes));
        e->cap = bytes;
    }
    // the slot's previous report must have read it before it is overwritten
    OKV_CUDA_TRY(cudaStreamWaitEvent(t->early_copy, e->consumed, 0));
    OKV_CUDA_TRY(cudaMemcpyAsync(e->dev, host, bytes, cudaMemcpyHostToDevice, t->early_copy));
    OKV_CUDA_TRY(cudaEventRecord(e->ready, t->early_copy));
    e->host = host;
    e->bytes = bytes;
    e->pending = true;
    e->seq = ++t->early_seq;
    return ORCHKV_OK;
}

int tm_report_attn_ranges(tiered_manager_t *m, const float *avg, uint32_t heads,
                          uint32_t kv_len, const uint32_t *starts, const uint32_t *ends,
                          const uint32_t *block_ids, uint32_t n)
{
    OKV_RANGE("tm_report_attn_ranges");
    TmImpl *t = tm_impl(m);
    if (!t || !avg || heads == 0 || kv_len == 0 || (n && (!starts || !ends || !block_ids)))
        return ORCHKV_ERR_INVALID;
    std::lock_guard<std::mutex> g(t->mu);
    int rc = tm_flush_locked(t);
    if (rc) return rc;
    if (n == 0) return ORCHKV_OK;
    const void *in[4] = {avg, starts, ends, block_ids};
    const size_t bytes[4] = {(size_t)heads * kv_len * sizeof(float), (size_t)n * 4,
                             (size_t)n * 4, (size_t)n * 4};
    rc = stage_inputs(t, in, bytes, 4);
    if (rc) return rc;
    okv::ReportOrder o;
    rc = begin_report(t, n, true, &o);
    if (rc) return rc;
    t->mirror_dirty = true;
    const uint32_t *ids = (const uint32_t *)in[3];
    rc = launch_alias_mark(ids, n, t->d, o, t->stream);
    if (!rc) rc = launch_range_mass((const float *)in[0], heads, kv_len, (const uint32_t *)in[1],
                                    (const uint32_t *)in[2], ids, n, t->d, t->step, o, t->stream);
    if (!rc) rc = launch_report_ordered(o.ids_eff, o.mass, n, t->d, t->step, o, t->stream);
    const int rr = release_staged(t);
    return rc ? rc : rr;
}

int tm_report_attn_batch_dev(tiered_manager_t *m, const uint32_t *ids, const float *w,
                             uint32_t n)
{
    TmImpl *t = tm_impl(m);
    if (!t || (n && (!ids || !w))) return ORCHKV_ERR_INVALID;
    std::lock_guard<std::mutex> g(t->mu);
    int rc = tm_flush_locked(t);
    if (rc) return rc;
    if (n == 0) return ORCHKV_OK;
    okv::ReportOrder o;
    rc = begin_report(t, n, false, &o);
    if (rc) return rc;
    t->mirror_dirty = true;
    rc = launch_alias_mark(ids, n, t->d, o, t->stream);
    if (!rc) rc = launch_report_batch(ids, w, n, t->d, t->step, o, t->stream);
    if (!rc) rc = launch_report_ordered(ids, w, n, t->d, t->step, o, t->stream);
    return rc;
}

int tm_report_attn_blockmean(tiered_manager_t *m, const void *weights, int dtype,
                             uint32_t batch, uint32_t heads, uint32_t q_len, uint32_t kv_len,
                             uint32_t block_size, const uint32_t *block_ids, float *scores)
{
    OKV_RANGE("tm_report_attn_blockmean");
    TmImpl *t = tm_impl(m);
    if (!t) return ORCHKV_ERR_INVALID;
    std::lock_guard<std::mutex> g(t->mu);
    int rc = tm_flush_locked(t);
    if (rc) return rc;
    if (block_ids) t->mirror_dirty = true;
    return launch_blockmean(weights, dtype, batch, heads, q_len, kv_len, block_size, block_ids,
                            scores, block_ids ? &t->d : nullptr, t->step, t->stream);
}

int tm_step_and_classify(tiered_manager_t *m)
{
    OKV_RANGE("tm_step_and_classify");
    TmImpl *t = tm_impl(m);
    if (!t) return ORCHKV_ERR_INVALID;
    std::lock_guard<std::mutex> g(t->mu);
    int rc = tm_flush_locked(t);
    if (rc) return rc;
    rc = launch_sweep(t->d, params_of(t), true, true, nullptr, t->stream);
    if (rc) return rc;
    t->step++;
    t->prefetch_wasted += t->tracked;
    t->tracked = 0;
    t->heap_size = 0;
    t->mirror_dirty = true;
    return ORCHKV_OK;
}

static int select_common(TmImpl *t, SelectMode mode, uint32_t k, float frac, float thg,
                         float thd, uint32_t *out_ids, uint32_t *out_count, uint32_t max_out,
                         const uint8_t *mask = nullptr)
{
    if (!out_ids || !out_count) return ORCHKV_ERR_INVALID;
    std::lock_guard<std::mutex> g(t->mu);
    sync_registry_view(t);
    int rc = tm_flush_locked(t);
    if (rc) return rc;
    SelectArgs a;
    memset(&a, 0, sizeof(a));
    a.mode = mode;
    a.k = k;
    a.frac = frac;
    a.th_gpu = thg;
    a.th_dram = thd;
    a.max_out = max_out;
    a.out_ids = out_ids;
    a.out_count = out_count;
    a.mask = mask;
    a.world = 1;
    if (t->comm_reduce) {
        a.reduce = t->comm_reduce;
        a.gather = t->comm_gather;
        a.comm_ctx = t->comm_ctx;
        a.rank = t->comm_rank;
        a.world = t->comm_world;
        a.gather_buf = t->small + 16;
    }
    return launch_select(t->d, t->sc, a, t->stream);
}

int tm_select_victims(tiered_manager_t *m, uint32_t k, uint32_t *out_ids, uint32_t *out_count)
{
    OKV_RANGE("tm_select_victims");
    TmImpl *t = tm_impl(m);
    if (!t) return ORCHKV_ERR_INVALID;
    return select_common(t, kSelectColdest, k, -1.0f, 0.f, 0.f, out_ids, out_count, k);
}

int tm_select_victims_masked(tiered_manager_t *m, uint32_t k, const uint8_t *eligible,
                             uint32_t *out_ids, uint32_t *out_count)
{
    OKV_RANGE("tm_select_victims_masked");
    TmImpl *t = tm_impl(m);
    if (!t || !eligible) return ORCHKV_ERR_INVALID;
    return select_common(t, kSelectColdest, k, -1.0f, 0.f, 0.f, out_ids, out_count, k,
                         eligible);
}

int tm_select_victims_frac(tiered_manager_t *m, float frac, uint32_t *out_ids,
                           uint32_t *out_count, uint32_t max_out)
{
    OKV_RANGE("tm_select_victims_frac");
    TmImpl *t = tm_impl(m);
    if (!t || !(frac >= 0.0f) || frac > 1.0f) return ORCHKV_ERR_INVALID;
    return select_common(t, kSelectColdest, 0, frac, 0.f, 0.f, out_ids, out_count, max_out);
}

int tm_select_prefetch(tiered_manager_t *m, uint32_t k, float th_gpu, float th_dram,
                       uint32_t *out_ids, uint32_t *out_count)
{
    OKV_RANGE("tm_select_prefetch");
    TmImpl *t = tm_impl(m);
    if (!t) return ORCHKV_ERR_INVALID;
    return select_common(t, kSelectPrefetch, k, -1.0f, th_gpu, th_dram, out_ids, out_count, k);
}

int tm_get_threshold_state(const tiered_manager_t *m, float *hot, float *warm, uint64_t *up,
                           uint64_t *down)
{
    TmImpl *t = tm_impl(m);
    if (!t) return ORCHKV_ERR_INVALID;
    std::lock_guard<std::mutex> g(t->mu);
    if (hot) *hot = t->th_hot;
    if (warm) *warm = t->th_warm;
    if (up) *up = t->adj_up;
    if (down) *down = t->adj_down;
    return ORCHKV_OK;
}

}  // extern "C"
