/*
 * orchkv_oracle.c — CPU restatement of the scheduling + migration path.
 *
 * TEST INFRASTRUCTURE ONLY (see orchkv_oracle.h).  Built by oracle/Makefile
 * into oracle/liborchkv_oracle.so with -ffp-contract=off.
 */
#include "orchkv_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------
 * Tracker + classifier
 * ------------------------------------------------------------------------ */

static uint32_t pow2_at_least(uint32_t v)
{
    /* capacity rounding: max(v, 64) up to a power of two
     * (src/scheduler/attention_tracker.c:6-15,46) */
    uint32_t c = 64;
    if (v < 64) v = 64;
    while (c < v) c <<= 1;
    return c;
}

void oc_build_decay_table(float *table, float tau)
{
    /* src/scheduler/hotcold_classifier.c:27-34: tau clamped to >= 1,
     * inverse taken once in float, entries expf(-(float)k * inv). */
    if (tau < 1.0f) tau = 1.0f;
    float inv = 1.0f / tau;
    for (int k = 0; k < OC_DECAY_TABLE; k++)
        table[k] = expf(-(float)k * inv);
}

int oc_sched_init(oc_sched_t *s, uint32_t capacity, float lambda,
                  float alpha, float beta, float gamma, float tau,
                  float th_hot, float th_warm)
{
    memset(s, 0, sizeof(*s));
    if (capacity == 0) return -2;
    s->cap  = pow2_at_least(capacity);
    s->mask = s->cap - 1;
    /* lambda outside (0,1) falls back to 0.9 (attention_tracker.c:54-55) */
    s->lambda = (lambda > 0.0f && lambda < 1.0f) ? lambda : 0.9f;
    size_t n = s->cap;
    s->sum = calloc(n, 4); s->max = calloc(n, 4); s->ema = calloc(n, 4);
    s->hits = calloc(n, 4); s->last = calloc(n, 8); s->t_active = calloc(n, 1);
    s->hot = calloc(n, 4); s->heat = calloc(n, 1); s->c_flags = calloc(n, 1);
    s->c_active = calloc(n, 1);
    if (!s->sum || !s->max || !s->ema || !s->hits || !s->last || !s->t_active ||
        !s->hot || !s->heat || !s->c_flags || !s->c_active) {
        oc_sched_free(s);
        return -1;
    }
    s->alpha = alpha; s->beta = beta; s->gamma = gamma; s->tau = tau;
    s->th_hot = th_hot; s->th_warm = th_warm;
    oc_build_decay_table(s->table, tau);
    return 0;
}

void oc_sched_free(oc_sched_t *s)
{
    free(s->sum); free(s->max); free(s->ema); free(s->hits); free(s->last);
    free(s->t_active); free(s->hot); free(s->heat); free(s->c_flags);
    free(s->c_active);
    memset(s, 0, sizeof(*s));
}

void oc_register(oc_sched_t *s, uint64_t id, uint8_t flags)
{
    uint32_t i = (uint32_t)(id & s->mask);
    /* tracker slot zeroed + active, last = "never" (attention_tracker.c:179-191) */
    s->sum[i] = 0.0f; s->max[i] = 0.0f; s->ema[i] = 0.0f; s->hits[i] = 0;
    s->last[i] = OC_STEP_NEVER; s->t_active[i] = 1;
    /* classifier slot (hotcold_classifier.c:104-116): sink flag 0x08 -> HOT(0)
     * else COLD(2), hotness 0 */
    s->hot[i] = 0.0f;
    s->heat[i] = (flags & 0x08) ? 0 : 2;
    s->c_flags[i] = flags;
    s->c_active[i] = 1;
}

void oc_unregister(oc_sched_t *s, uint64_t id)
{
    uint32_t i = (uint32_t)(id & s->mask);
    s->sum[i] = 0.0f; s->max[i] = 0.0f; s->ema[i] = 0.0f; s->hits[i] = 0;
    s->last[i] = 0; s->t_active[i] = 0;
    s->hot[i] = 0.0f; s->heat[i] = 0; s->c_flags[i] = 0; s->c_active[i] = 0;
}

void oc_update(oc_sched_t *s, uint64_t id, float w)
{
    /* attention_tracker.c:75-92 with update_slot :27-33 */
    uint32_t i = (uint32_t)(id & s->mask);
    if (!s->t_active[i]) return;
    s->sum[i] = s->sum[i] + w;
    if (w > s->max[i]) s->max[i] = w;
    s->last[i] = s->step;
}

void oc_update_batch(oc_sched_t *s, const uint64_t *ids, const float *w, uint32_t n)
{
    for (uint32_t j = 0; j < n; j++) oc_update(s, ids[j], w[j]);
}

void oc_step_done(oc_sched_t *s)
{
    /* attention_tracker.c:120-150: one_minus formed once in float; hit slots
     * blend (lambda*ema) + (one_minus*sum), idle slots scale by lambda. */
    float lam = s->lambda;
    float om = 1.0f - lam;
    for (uint32_t i = 0; i < s->cap; i++) {
        if (!s->t_active[i]) continue;
        if (s->last[i] == s->step) {
            float a = lam * s->ema[i];
            float b = om * s->sum[i];
            s->ema[i] = a + b;
            s->hits[i] = s->hits[i] + 1;
        } else {
            s->ema[i] = s->ema[i] * lam;
        }
        s->sum[i] = 0.0f;
        s->max[i] = 0.0f;
    }
    s->step++;
}

float oc_hotness_one(const oc_sched_t *s, uint32_t i, uint64_t step)
{
    /* hotcold_classifier.c:69-83 with recency :36-42, frequency :44-49 */
    uint64_t last = s->last[i];
    uint64_t gap = (last == OC_STEP_NEVER) ? step : (step > last ? step - last : 0);
    float rec = gap >= OC_DECAY_TABLE ? 0.0f : s->table[(uint32_t)gap];
    float freq;
    if (step == 0) {
        freq = 0.0f;
    } else {
        freq = (float)s->hits[i] / (float)step;
        if (freq > 1.0f) freq = 1.0f;
    }
    float t0 = s->alpha * s->ema[i];
    float t1 = s->beta * rec;
    float t2 = s->gamma * freq;
    return (t0 + t1) + t2;
}

void oc_update_all(oc_sched_t *s)
{
    /* hotcold_classifier.c:161-185 with classify :51-63 */
    for (uint32_t i = 0; i < s->cap; i++) {
        if (!s->c_active[i] || !s->t_active[i]) continue;
        float h = oc_hotness_one(s, i, s->step);
        uint8_t lvl;
        if (s->c_flags[i] & 0x08)      lvl = 0;
        else if (h >= s->th_hot)       lvl = 0;
        else if (h >= s->th_warm)      lvl = 1;
        else                           lvl = 2;
        s->hot[i] = h;
        s->heat[i] = lvl;
    }
}

void oc_set_thresholds(oc_sched_t *s, float th_hot, float th_warm)
{
    s->th_hot = th_hot; s->th_warm = th_warm;
}

void oc_set_weights(oc_sched_t *s, float a, float b, float g)
{
    s->alpha = a; s->beta = b; s->gamma = g;
}

/* ------------------------------------------------------------------------
 * Adaptive threshold — src/scheduler/adaptive_threshold.c:82-149
 * ------------------------------------------------------------------------ */

static float clampf(float v, float lo, float hi)
{
    if (v < lo) return lo;
    if (v > hi) return hi;
    return v;
}

int oc_athresh_update(oc_athresh_t *a, float gpu, float dram)
{
    int changed = 0;
    float st = a->step;
    if (gpu > a->gpu_hwm) {
        float nh = clampf(a->th_hot + st, a->min_hot, a->max_hot);
        if (nh != a->th_hot) { a->th_hot = nh; a->up++; changed = 1; }
    } else if (gpu < a->gpu_lwm) {
        float nh = clampf(a->th_hot - st, a->min_hot, a->max_hot);
        if (nh != a->th_hot) { a->th_hot = nh; a->down++; changed = 1; }
    }
    if (dram > a->dram_hwm) {
        float nw = clampf(a->th_warm + st, a->min_warm, a->max_warm);
        if (nw != a->th_warm) { a->th_warm = nw; a->up++; changed = 1; }
    } else if (dram < a->dram_lwm) {
        float nw = clampf(a->th_warm - st, a->min_warm, a->max_warm);
        if (nw != a->th_warm) { a->th_warm = nw; a->down++; changed = 1; }
    }
    return changed;
}

/* ------------------------------------------------------------------------
 * Selection
 * ------------------------------------------------------------------------ */

uint32_t oc_orderable(float f)
{
    uint32_t u;
    if (f != f) return 0xFFFFFFFEu;          /* NaN after every number */
    if (f == 0.0f) f = 0.0f;                  /* fold -0.0 onto +0.0 */
    memcpy(&u, &f, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

typedef struct { uint32_t key, idx; } kv_pair;

static int cmp_pair(const void *a, const void *b)
{
    const kv_pair *x = a, *y = b;
    if (x->key != y->key) return x->key < y->key ? -1 : 1;
    return x->idx < y->idx ? -1 : (x->idx > y->idx);
}

static int cmp_u32(const void *a, const void *b)
{
    uint32_t x = *(const uint32_t *)a, y = *(const uint32_t *)b;
    return x < y ? -1 : (x > y);
}

static uint32_t take_k(kv_pair *v, uint32_t m, uint32_t k, uint32_t *out)
{
    qsort(v, m, sizeof(kv_pair), cmp_pair);
    uint32_t c = k < m ? k : m;
    for (uint32_t j = 0; j < c; j++) out[j] = v[j].idx;
    qsort(out, c, 4, cmp_u32);
    return c;
}

uint32_t oc_select_coldest(const float *hot, const uint8_t *eligible,
                           uint32_t n, uint32_t k, uint32_t *out)
{
    kv_pair *v = malloc((size_t)(n ? n : 1) * sizeof(kv_pair));
    uint32_t m = 0;
    for (uint32_t i = 0; i < n; i++)
        if (eligible[i]) { v[m].key = oc_orderable(hot[i]); v[m].idx = i; m++; }
    uint32_t c = take_k(v, m, k, out);
    free(v);
    return c;
}

uint32_t oc_select_prefetch(const float *ema, const uint8_t *active,
                            const uint8_t *tier, uint32_t n,
                            float th_gpu, float th_dram, uint32_t k,
                            uint32_t *out)
{
    kv_pair *v = malloc((size_t)(n ? n : 1) * sizeof(kv_pair));
    uint32_t m = 0;
    for (uint32_t i = 0; i < n; i++) {
        if (!active[i]) continue;
        if (tier[i] == 0 || tier[i] == 4) continue;
        float e = ema[i], prio;
        if (e >= th_gpu)                        prio = e;
        else if (e >= th_dram && tier[i] != 1)  prio = e * 0.5f;
        else continue;
        v[m].key = ~oc_orderable(prio);   /* descending priority */
        v[m].idx = i;
        m++;
    }
    uint32_t c = take_k(v, m, k, out);
    free(v);
    return c;
}

/* ------------------------------------------------------------------------
 * Scoring reduction
 * ------------------------------------------------------------------------ */

void oc_score_blocks(const float *probs, uint32_t R, uint32_t Hq, uint32_t Hkv,
                     uint32_t T, uint32_t tpb, const uint32_t *lens, float *out)
{
    uint32_t G = Hq / Hkv;
    uint32_t nb = (T + tpb - 1) / tpb;
    for (uint32_t r = 0; r < R; r++) {
        uint32_t len = lens ? lens[r] : T;
        if (len > T) len = T;
        for (uint32_t h = 0; h < Hkv; h++) {
            for (uint32_t b = 0; b < nb; b++) {
                float acc = 0.0f;
                uint32_t t0 = b * tpb, t1 = t0 + tpb;
                if (t1 > len) t1 = len;
                for (uint32_t g = 0; g < G; g++) {
                    const float *row = probs + ((size_t)r * Hq + (size_t)h * G + g) * T;
                    for (uint32_t t = t0; t < t1; t++) acc = acc + row[t];
                }
                out[((size_t)r * Hkv + h) * nb + b] = acc;
            }
        }
    }
}

/* ------------------------------------------------------------------------
 * Pools and batched migration
 * ------------------------------------------------------------------------ */

int oc_pool_init(oc_pool_t *p, uint32_t total)
{
    p->total = total;
    p->stack = malloc((size_t)(total ? total : 1) * 4);
    if (!p->stack) return -1;
    for (uint32_t i = 0; i < total; i++) p->stack[i] = total - 1 - i;
    p->top = total;
    return 0;
}

void oc_pool_free(oc_pool_t *p) { free(p->stack); p->stack = NULL; p->top = 0; }

int oc_pool_pop(oc_pool_t *p, uint32_t *idx)
{
    if (p->top == 0) return -4;               /* ORCHKV_ERR_TIER_FULL */
    *idx = p->stack[--p->top];
    return 0;
}

void oc_pool_push(oc_pool_t *p, uint32_t idx) { p->stack[p->top++] = idx; }

uint32_t oc_evict_batch(oc_pool_t *gpu, oc_pool_t *dram, uint32_t *loc,
                        uint8_t *state, const uint8_t *flags,
                        const uint32_t *handles, uint32_t n,
                        const uint8_t *gpu_base, uint8_t *dram_base,
                        size_t slab, uint32_t *n_skipped)
{
    uint32_t done = 0, skipped = 0;
    for (uint32_t j = 0; j < n; j++) {
        uint32_t h = handles[j];
        uint32_t w = loc[h];
        if (OC_LOC_TIER(w) != 0 || (flags && (flags[h] & 0x01))) { skipped++; continue; }
        uint32_t d;
        if (oc_pool_pop(dram, &d) != 0) { skipped++; continue; }
        uint32_t g = OC_LOC_SLAB(w);
        memcpy(dram_base + (size_t)d * slab, gpu_base + (size_t)g * slab, slab);
        loc[h] = OC_LOC(1, d);
        state[h] = 3;                          /* KV_STATE_WARM */
        oc_pool_push(gpu, g);
        done++;
    }
    if (n_skipped) *n_skipped = skipped;
    return done;
}

uint32_t oc_promote_batch(oc_pool_t *gpu, oc_pool_t *dram, uint32_t *loc,
                          uint8_t *state, const uint32_t *handles, uint32_t n,
                          uint8_t *gpu_base, const uint8_t *dram_base,
                          size_t slab, uint32_t *n_skipped)
{
    uint32_t done = 0, skipped = 0;
    for (uint32_t j = 0; j < n; j++) {
        uint32_t h = handles[j];
        uint32_t w = loc[h];
        if (OC_LOC_TIER(w) != 1) { skipped++; continue; }
        uint32_t g;
        if (oc_pool_pop(gpu, &g) != 0) { skipped++; continue; }
        uint32_t d = OC_LOC_SLAB(w);
        memcpy(gpu_base + (size_t)g * slab, dram_base + (size_t)d * slab, slab);
        loc[h] = OC_LOC(0, g);
        state[h] = 2;                          /* KV_STATE_HOT */
        oc_pool_push(dram, d);
        done++;
    }
    if (n_skipped) *n_skipped = skipped;
    return done;
}
