// pool_kernels.cu — data-plane kernels: per-block (compat) operations,
// paged append (K6), prefill, batched migration gather/scatter (K4/K5), block
// id tables and request teardown.
//
// Every kernel that pops or pushes a free stack reproduces the order in which
// the reference's per-block host loops pop and push
// (src/tiered_store/gpu_tier.cu:65-93, src/tiered_store/dram_tier.cu:70-98),
// so a batched call leaves pools, free stacks and block locations exactly as
// the equivalent sequence of per-block calls would.
#include "pool.h"

namespace okv {

namespace {

constexpr int kTileN = 1024;       // list entries per tile in batched migration

// ---- attached-scheduler hooks ----------------------------------------------

__device__ __forceinline__ void sched_register(const PoolDev &p, uint32_t id, uint8_t flags)
{
    if (!p.attached) return;
    const SchedDev &d = p.sd;
    const uint32_t s = id & d.mask;
    d.sum[s] = 0.f; d.mx[s] = 0.f; d.ema[s] = 0.f; d.hits[s] = 0;
    d.last[s] = kStepNever; d.tact[s] = 1;
    d.hot[s] = 0.f;
    d.heat[s] = (flags & KV_FLAG_ATTN_SINK) ? 0 : 2;
    d.cflags[s] = flags; d.cact[s] = 1;
    d.bflags[s] = flags; d.tier[s] = TIER_GPU_HBM; d.bstate[s] = KV_STATE_HOT;
}

__device__ __forceinline__ void sched_move(const PoolDev &p, uint32_t id, uint8_t tier,
                                           uint8_t state)
{
    if (!p.attached) return;
    const uint32_t s = id & p.sd.mask;
    p.sd.tier[s] = tier;
    p.sd.bstate[s] = state;
}

__device__ __forceinline__ void sched_unregister(const PoolDev &p, uint32_t id)
{
    if (!p.attached) return;
    const SchedDev &d = p.sd;
    const uint32_t s = id & d.mask;
    d.sum[s] = 0.f; d.mx[s] = 0.f; d.ema[s] = 0.f; d.hits[s] = 0;
    d.last[s] = 0; d.tact[s] = 0;
    d.hot[s] = 0.f; d.heat[s] = 0; d.cflags[s] = 0; d.cact[s] = 0;
    d.bflags[s] = 0; d.tier[s] = TIER_NONE; d.bstate[s] = 0;
}

// ---- cooperative copies ----------------------------------------------------

// Copy `bytes` with `nt` cooperating threads (index `t`).  16-byte vectors when
// both ends and the length allow it, 4-byte words or bytes otherwise.
__device__ __forceinline__ void coop_copy(char *dst, const char *src, unsigned long long bytes,
                                          unsigned t, unsigned nt)
{
    const uintptr_t a = (uintptr_t)dst | (uintptr_t)src | (uintptr_t)bytes;
    if ((a & 15) == 0) {
        const uint4 *s = reinterpret_cast<const uint4 *>(src);
        uint4 *d = reinterpret_cast<uint4 *>(dst);
        const unsigned long long n = bytes >> 4;
        unsigned long long i = t;
        for (; i + 3 * (unsigned long long)nt < n; i += 4 * (unsigned long long)nt) {
            uint4 v0 = s[i], v1 = s[i + nt], v2 = s[i + 2 * nt], v3 = s[i + 3 * nt];
            d[i] = v0; d[i + nt] = v1; d[i + 2 * nt] = v2; d[i + 3 * nt] = v3;
        }
        for (; i < n; i += nt) d[i] = s[i];
    } else if ((a & 3) == 0) {
        const uint32_t *s = reinterpret_cast<const uint32_t *>(src);
        uint32_t *d = reinterpret_cast<uint32_t *>(dst);
        for (unsigned long long i = t; i < (bytes >> 2); i += nt) d[i] = s[i];
    } else {
        for (unsigned long long i = t; i < bytes; i += nt) dst[i] = src[i];
    }
}

// ---------------------------------------------------------------------------
// Per-block operations (one CTA): the reference's orchkv_evict_to_dram /
// orchkv_promote_to_gpu / orchkv_get_kv_block (src/api/orchkv_api.cu:321-428)
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(256)
compat_op_kernel(PoolDev p, ReqDev r, int op, uint32_t l, uint32_t h, uint32_t bi,
                 uint32_t arg, uint32_t arg2, CompatResult *res)
{
    __shared__ int rc, dir;
    __shared__ uint32_t id, src, dst;
    if (threadIdx.x == 0) {
        rc = ORCHKV_OK;
        dir = -1;
        id = kNoBlock;
        if (l >= r.L || h >= r.H) {
            rc = ORCHKV_ERR_NOT_FOUND;
        } else {
            const uint32_t tok = req_tok(r)[l];
            const uint32_t nb = (tok + p.tpb - 1) / p.tpb;
            if (bi >= nb || bi >= r.mbph) rc = ORCHKV_ERR_NOT_FOUND;
            else id = req_table(r)[((size_t)l * r.H + h) * r.mbph + bi];
            if (rc == ORCHKV_OK && id >= p.max_blocks) rc = ORCHKV_ERR_NOT_FOUND;
        }
        if (rc == ORCHKV_OK) {
            const uint32_t w = p.loc[id];
            const uint32_t tier = loc_tier(w);
            PoolCounters *c = p.ctr;
            if (op == OP_EVICT) {
                if (tier != TIER_GPU_HBM) rc = ORCHKV_ERR_STATE;
                else if (p.flags[id] & KV_FLAG_PIN) rc = ORCHKV_ERR_LOCKED;
                else if (c->d_top == 0) rc = ORCHKV_ERR_TIER_FULL;
                else { src = loc_slab(w); dst = p.d_stack[--c->d_top]; dir = 0; }
                if (dir == 0 && (!OKV_IN(p.chk, src, p.g_total) || !OKV_IN(p.chk, dst, p.d_total))) {
                    rc = ORCHKV_ERR_CUDA;
                    dir = -1;
                }
            } else if (op == OP_PROMOTE || op == OP_GET) {
                if (tier == TIER_HOST_DRAM) {
                    if (c->g_top == 0) rc = ORCHKV_ERR_TIER_FULL;
                    else { src = loc_slab(w); dst = p.g_stack[--c->g_top]; dir = 1; }
                    if (dir == 1 && (!OKV_IN(p.chk, src, p.d_total) || !OKV_IN(p.chk, dst, p.g_total))) {
                        rc = ORCHKV_ERR_CUDA;
                        dir = -1;
                    }
                } else if (op == OP_PROMOTE || tier != TIER_GPU_HBM) {
                    rc = ORCHKV_ERR_STATE;
                }
            } else if (op == OP_SET_FLAGS) {
                p.flags[id] = (uint8_t)arg;
                if (p.attached) p.sd.bflags[id & p.sd.mask] = (uint8_t)arg;
            } else if (op == OP_DRAM_POP) {
                if (c->d_top == 0) rc = ORCHKV_ERR_TIER_FULL;
                else res->aux = p.d_stack[--c->d_top];
                if (rc == ORCHKV_OK && !OKV_IN(p.chk, res->aux, p.d_total)) rc = ORCHKV_ERR_CUDA;
            } else if (op == OP_SET_LOC) {
                const uint8_t st = (uint8_t)(arg2 & 0xFF);
                const uint32_t push = arg2 >> 8;
                p.loc[id] = arg;
                p.state[id] = st;
                if (push && OKV_IN(p.chk, c->d_top, p.d_total) && OKV_IN(p.chk, push - 1, p.d_total))
                    p.d_stack[c->d_top++] = push - 1;
                sched_move(p, id, (uint8_t)loc_tier(arg), st);
            }
        }
    }
    __syncthreads();
    if (dir == 0)
        coop_copy(p.dram_base + dst * p.slab, p.gpu_base + src * p.slab, p.slab, threadIdx.x, blockDim.x);
    else if (dir == 1)
        coop_copy(p.gpu_base + dst * p.slab, p.dram_base + src * p.slab, p.slab, threadIdx.x, blockDim.x);
    __syncthreads();
    if (threadIdx.x == 0) {
        PoolCounters *c = p.ctr;
        if (dir == 0) {
            p.loc[id] = make_loc(TIER_HOST_DRAM, dst);
            p.state[id] = KV_STATE_WARM;
            if (OKV_IN(p.chk, c->g_top, p.g_total)) p.g_stack[c->g_top++] = src;
            c->transfers_d2h++;
            c->bytes_d2h += p.slab;
            sched_move(p, id, TIER_HOST_DRAM, KV_STATE_WARM);
        } else if (dir == 1) {
            p.loc[id] = make_loc(TIER_GPU_HBM, dst);
            p.state[id] = KV_STATE_HOT;
            if (OKV_IN(p.chk, c->d_top, p.d_total)) p.d_stack[c->d_top++] = src;
            c->transfers_h2d++;
            c->bytes_h2d += p.slab;
            sched_move(p, id, TIER_GPU_HBM, KV_STATE_HOT);
        }
        res->rc = rc;
        res->id = id;
        if (id != kNoBlock && id < p.max_blocks) {
            const uint32_t w = p.loc[id];
            res->loc = w;
            res->state = p.state[id];
            res->flags = p.flags[id];
            if (loc_tier(w) == TIER_GPU_HBM && OKV_IN(p.chk, loc_slab(w), p.g_total)) {
                res->k_ptr = (unsigned long long)(p.gpu_base + (unsigned long long)loc_slab(w) * p.slab);
                res->v_ptr = res->k_ptr + p.half;
            } else {
                res->k_ptr = res->v_ptr = 0;
            }
            const uint32_t tok = req_tok(r)[l];
            const uint32_t last = (tok + p.tpb - 1) / p.tpb - 1;
            res->tok = bi < last ? p.tpb : tok - last * p.tpb;
        }
    }
}

// ---------------------------------------------------------------------------
// orchkv_append_token (src/api/orchkv_api.cu:263-317 with
// kv_request_alloc_blocks_for_layer, src/core/kv_request.c:128-211), one CTA.
// ---------------------------------------------------------------------------

constexpr int kMaxHeads = 256;

__global__ void __launch_bounds__(256)
append_one_kernel(PoolDev p, ReqDev r, uint32_t l, const char *k, const char *v,
                  CompatResult *res)
{
    __shared__ int rc;
    __shared__ uint32_t n_ok, slot;
    __shared__ uint32_t slab_of[kMaxHeads];
    if (threadIdx.x == 0) {
        rc = ORCHKV_OK;
        n_ok = 0;
        PoolCounters *c = p.ctr;
        uint32_t *tokp = req_tok(r) + l;
        const uint32_t tok = *tokp;
        const bool need_new = (tok % p.tpb) == 0;
        const uint32_t b = tok / p.tpb;
        if (need_new && (c->id_top < r.H || c->g_top < r.H || b >= r.mbph)) {
            rc = ORCHKV_ERR_TIER_FULL;
        } else {
            *tokp = tok + 1;
            slot = tok % p.tpb;
            uint32_t *tab = req_table(r) + (size_t)l * r.H * r.mbph;
            if (need_new) {
                // block ids in head order, then one slab per head in head order
                for (uint32_t hh = 0; hh < r.H; hh++) {
                    const uint32_t id = p.id_stack[--c->id_top];
                    tab[(size_t)hh * r.mbph + b] = id;
                    if (!OKV_IN(p.chk, id, p.max_blocks)) { rc = ORCHKV_ERR_CUDA; continue; }
                    p.loc[id] = make_loc(TIER_NONE, 0);
                    p.state[id] = KV_STATE_FREE;
                    p.flags[id] = 0;
                }
                for (uint32_t hh = 0; hh < r.H; hh++) {
                    const uint32_t id = tab[(size_t)hh * r.mbph + b];
                    const uint32_t g = p.g_stack[--c->g_top];
                    if (!OKV_IN(p.chk, id, p.max_blocks) || !OKV_IN(p.chk, g, p.g_total)) {
                        rc = ORCHKV_ERR_CUDA;
                        continue;
                    }
                    p.loc[id] = make_loc(TIER_GPU_HBM, g);
                    p.state[id] = KV_STATE_HOT;
                    c->live_blocks++;
                    sched_register(p, id, 0);
                }
            }
            for (uint32_t hh = 0; rc == ORCHKV_OK && hh < r.H; hh++) {
                const uint32_t id = tab[(size_t)hh * r.mbph + b];
                if (!OKV_IN(p.chk, id, p.max_blocks)) { rc = ORCHKV_ERR_CUDA; break; }
                const uint32_t w = p.loc[id];
                if (loc_tier(w) != TIER_GPU_HBM) { rc = ORCHKV_ERR_STATE; break; }
                if (!OKV_IN(p.chk, loc_slab(w), p.g_total)) { rc = ORCHKV_ERR_CUDA; break; }
                slab_of[hh] = loc_slab(w);
                n_ok = hh + 1;
            }
            if (k) { c->transfers_h2d += n_ok; c->bytes_h2d += (unsigned long long)n_ok * p.row; }
            if (v) { c->transfers_h2d += n_ok; c->bytes_h2d += (unsigned long long)n_ok * p.row; }
            if (rc == ORCHKV_OK && l == 0) r.region[0] += 1;
        }
    }
    __syncthreads();
    const unsigned warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (uint32_t hh = warp; hh < n_ok; hh += nw) {
        char *dst = p.gpu_base + (unsigned long long)slab_of[hh] * p.slab + (unsigned long long)slot * p.row;
        if (k) coop_copy(dst, k + (size_t)hh * p.row, p.row, lane, 32);
        if (v) coop_copy(dst + p.half, v + (size_t)hh * p.row, p.row, lane, 32);
    }
    if (threadIdx.x == 0) res->rc = rc;
}

// ---------------------------------------------------------------------------
// orchkv_prefill (src/api/orchkv_api.cu:204-255)
// ---------------------------------------------------------------------------

__global__ void prefill_plan_kernel(PoolDev p, ReqDev r, uint32_t l, uint32_t seq,
                                    int has_k, int has_v, uint32_t *scratch,
                                    CompatResult *res)
{
    PoolCounters *c = p.ctr;
    uint32_t *tokp = req_tok(r) + l;
    const uint32_t tok = *tokp;
    const uint32_t total = tok + seq;
    const uint32_t needed = (total + p.tpb - 1) / p.tpb;
    const uint32_t have = (tok + p.tpb - 1) / p.tpb;
    scratch[0] = 0;        // new blocks per head
    scratch[1] = have;
    scratch[2] = total;
    int rc = ORCHKV_OK;
    if (needed > have) {
        const uint32_t nn = needed - have;
        if (needed > r.mbph || c->id_top < nn * r.H || c->g_top < nn * r.H) {
            rc = ORCHKV_ERR_TIER_FULL;
        } else {
            // The per-block pops happen in prefill_copy_kernel from these
            // saved tops: ids go block-major then head (kv_request.c:177-204),
            // slabs head-major then block (orchkv_api.cu:219-226).
            scratch[3] = c->id_top;
            scratch[4] = c->g_top;
            c->id_top -= nn * r.H;
            c->g_top -= nn * r.H;
            c->live_blocks += nn * r.H;
            for (uint32_t j = 0; j < nn; j++) {
                const uint32_t ts = (have + j) * p.tpb;
                if (ts >= seq) continue;
                const uint32_t cnt = total - ts < p.tpb ? total - ts : p.tpb;
                const unsigned long long bytes = (unsigned long long)cnt * p.row * r.H;
                if (has_k) { c->transfers_h2d += r.H; c->bytes_h2d += bytes; }
                if (has_v) { c->transfers_h2d += r.H; c->bytes_h2d += bytes; }
            }
            scratch[0] = nn;
        }
    }
    if (rc == ORCHKV_OK) {
        *tokp = total;
        if (l == 0) r.region[0] += seq;
    }
    res->rc = rc;
}

__global__ void __launch_bounds__(256)
prefill_copy_kernel(PoolDev p, ReqDev r, uint32_t l, const char *k, const char *v,
                    uint32_t seq, const uint32_t *scratch)
{
    const uint32_t nn = scratch[0], have = scratch[1], total = scratch[2];
    const uint32_t id_top = scratch[3], g_top = scratch[4];
    const uint32_t n_items = nn * r.H;
    const unsigned warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const unsigned lane = threadIdx.x & 31;
    const unsigned nwarps = (gridDim.x * blockDim.x) >> 5;
    uint32_t *tab = req_table(r) + (size_t)l * r.H * r.mbph;
    for (uint32_t it = warp; it < n_items; it += nwarps) {
        const uint32_t hh = it / nn, j = it % nn;
        const uint32_t id = p.id_stack[id_top - 1 - (j * r.H + hh)];
        const uint32_t g = p.g_stack[g_top - 1 - it];
        if (!OKV_IN(p.chk, id, p.max_blocks) || !OKV_IN(p.chk, g, p.g_total)) continue;
        if (lane == 0) {
            tab[(size_t)hh * r.mbph + have + j] = id;
            p.flags[id] = 0;
            p.loc[id] = make_loc(TIER_GPU_HBM, g);
            p.state[id] = KV_STATE_HOT;
            sched_register(p, id, 0);
        }
        const uint32_t ts = (have + j) * p.tpb;
        if (ts >= seq) continue;             // source offset beyond the buffer
        uint32_t cnt = total - ts < p.tpb ? total - ts : p.tpb;
        if (cnt > seq - ts) cnt = seq - ts;  // stay inside this head's rows
        char *dst = p.gpu_base + (unsigned long long)g * p.slab;
        const size_t off = ((size_t)hh * seq + ts) * p.row;
        const unsigned long long bytes = (unsigned long long)cnt * p.row;
        if (k) coop_copy(dst, k + off, bytes, lane, 32);
        if (v) coop_copy(dst + p.half, v + off, bytes, lane, 32);
    }
}

// ---------------------------------------------------------------------------
// Batched append over (request, layer) pairs: plan (one CTA) + write kernel.
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(1024)
append_plan_kernel(PoolDev p, uint32_t *const *regions, uint32_t n, uint32_t L, uint32_t H,
                   uint32_t mbph, int has_k, int has_v, uint32_t *scratch)
{
    __shared__ uint32_t tmp[33];
    __shared__ uint32_t carry, bad_state, bad_width;
    const uint32_t P = n * L;
    if (threadIdx.x == 0) { carry = 0; bad_state = 0; bad_width = 0; }
    __syncthreads();
    for (uint32_t base = 0; base < P; base += blockDim.x) {
        const uint32_t pr = base + threadIdx.x;
        uint32_t need = 0;
        if (pr < P) {
            const uint32_t i = pr / L, l = pr % L;
            const uint32_t *reg = regions[i];
            const uint32_t tok = reg[1 + l];
            need = (tok % p.tpb) == 0;
            if (tok / p.tpb >= mbph) atomicOr(&bad_width, 1u);
            if (!need) {
                const uint32_t *tab = reg + 1 + L + (size_t)l * H * mbph;
                const uint32_t b = (tok - 1) / p.tpb;
                for (uint32_t hh = 0; hh < H; hh++) {
                    const uint32_t id = tab[(size_t)hh * mbph + b];
                    if (!OKV_IN(p.chk, id, p.max_blocks) || loc_tier(p.loc[id]) != TIER_GPU_HBM)
                        atomicOr(&bad_state, 1u);
                }
            }
            scratch[2 * pr] = tok;
        }
        uint32_t total;
        const uint32_t ex = block_excl_scan(need, tmp, &total);
        if (pr < P) scratch[2 * pr + 1] = need ? carry + ex : kNoBlock;
        __syncthreads();
        if (threadIdx.x == 0) carry += total;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        PoolCounters *c = p.ctr;
        const uint32_t need_slabs = carry * H;
        uint32_t err = ORCHKV_OK;
        if (bad_state) err = (uint32_t)ORCHKV_ERR_STATE;
        else if (bad_width || c->g_top < need_slabs || c->id_top < need_slabs)
            err = (uint32_t)ORCHKV_ERR_TIER_FULL;
        scratch[2 * P] = err;
        scratch[2 * P + 1] = c->g_top;
        scratch[2 * P + 2] = c->id_top;
        if (err == ORCHKV_OK) {
            c->g_top -= need_slabs;
            c->id_top -= need_slabs;
            c->live_blocks += need_slabs;
            const unsigned long long rows = (unsigned long long)P * H;
            if (has_k) { c->transfers_h2d += rows; c->bytes_h2d += rows * p.row; }
            if (has_v) { c->transfers_h2d += rows; c->bytes_h2d += rows * p.row; }
        } else {
            c->err = err;
        }
    }
}

__global__ void __launch_bounds__(256)
append_write_kernel(PoolDev p, uint32_t *const *regions, uint32_t n, uint32_t L, uint32_t H,
                    uint32_t mbph, const char *k, const char *v, const uint32_t *scratch)
{
    const uint32_t P = n * L;
    if (scratch[2 * P] != ORCHKV_OK) return;
    const unsigned long long warp =
        ((unsigned long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const unsigned lane = threadIdx.x & 31;
    if (warp >= (unsigned long long)P * H) return;
    const uint32_t pr = (uint32_t)(warp / H), hh = (uint32_t)(warp % H);
    const uint32_t i = pr / L, l = pr % L;
    uint32_t *reg = regions[i];
    const uint32_t tok = scratch[2 * pr], ord = scratch[2 * pr + 1];
    const uint32_t b = tok / p.tpb, slot = tok % p.tpb;
    uint32_t *tab = reg + 1 + L + (size_t)l * H * mbph;
    uint32_t g;
    if (ord != kNoBlock) {
        const uint32_t j = ord * H + hh;
        const uint32_t id = p.id_stack[scratch[2 * P + 2] - 1 - j];
        g = p.g_stack[scratch[2 * P + 1] - 1 - j];
        if (!OKV_IN(p.chk, id, p.max_blocks)) return;
        if (lane == 0) {
            tab[(size_t)hh * mbph + b] = id;
            p.loc[id] = make_loc(TIER_GPU_HBM, g);
            p.state[id] = KV_STATE_HOT;
            p.flags[id] = 0;
            sched_register(p, id, 0);
        }
    } else {
        const uint32_t id = tab[(size_t)hh * mbph + b];
        if (!OKV_IN(p.chk, id, p.max_blocks)) return;
        g = loc_slab(p.loc[id]);
    }
    if (!OKV_IN(p.chk, g, p.g_total)) return;
    char *dst = p.gpu_base + (unsigned long long)g * p.slab + (unsigned long long)slot * p.row;
    const size_t src = ((size_t)pr * H + hh) * p.row;
    if (k) coop_copy(dst, k + src, p.row, lane, 32);
    if (v) coop_copy(dst + p.half, v + src, p.row, lane, 32);
    if (hh == 0 && lane == 0) {
        reg[1 + l] = tok + 1;
        if (l == 0) reg[0] += 1;
    }
}

// ---------------------------------------------------------------------------
// Batched migration: validity count per tile, tile scan + pool bookkeeping,
// per-entry plan (metadata + free-stack pushes), then the slab copy.
// ---------------------------------------------------------------------------

// An entry moves only if it is the first occurrence of its id in the list
// (a repeat finds the block already on the destination tier, as the
// per-block loop would) and the block is on the source tier.
__device__ __forceinline__ bool mig_valid(const PoolDev &p, int dir, uint32_t id, uint32_t e)
{
    if (id >= p.max_blocks || p.first[id] != e) return false;
    const uint32_t w = p.loc[id];
    if (dir == 0) return loc_tier(w) == TIER_GPU_HBM && !(p.flags[id] & KV_FLAG_PIN);
    return loc_tier(w) == TIER_HOST_DRAM;
}

__device__ __forceinline__ uint32_t list_len(const uint32_t *count, uint32_t max_n)
{
    if (!count) return max_n;
    const uint32_t c = *count;
    return c < max_n ? c : max_n;
}

__global__ void __launch_bounds__(256)
mig_count_kernel(PoolDev p, int dir, const uint32_t *ids, const uint32_t *count,
                 uint32_t max_n, uint32_t *tile_cnt)
{
    __shared__ uint32_t tmp[33];
    const uint32_t n = list_len(count, max_n);
    const uint32_t base = blockIdx.x * kTileN;
    uint32_t c = 0;
    for (uint32_t j = threadIdx.x; j < kTileN; j += blockDim.x) {
        const uint32_t e = base + j;
        if (e < n && mig_valid(p, dir, ids[e], e)) c++;
    }
    uint32_t tot;
    block_excl_scan(c, tmp, &tot);
    if (threadIdx.x == 0) tile_cnt[blockIdx.x] = tot;
}

__global__ void __launch_bounds__(1024)
mig_scan_kernel(PoolDev p, int dir, const uint32_t *count, uint32_t max_n, uint32_t tiles,
                uint32_t *tile_cnt, uint32_t *meta, uint32_t *result)
{
    __shared__ uint32_t tmp[33];
    __shared__ uint32_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (uint32_t b0 = 0; b0 < tiles; b0 += blockDim.x) {
        const uint32_t t = b0 + threadIdx.x;
        const uint32_t c = t < tiles ? tile_cnt[t] : 0;
        uint32_t tot;
        const uint32_t ex = block_excl_scan(c, tmp, &tot);
        if (t < tiles) tile_cnt[t] = carry + ex;   // becomes the tile base
        __syncthreads();
        if (threadIdx.x == 0) carry += tot;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        PoolCounters *c = p.ctr;
        const uint32_t n = list_len(count, max_n);
        const uint32_t valid = carry;
        uint32_t *dst_top = dir == 0 ? &c->d_top : &c->g_top;
        uint32_t *src_top = dir == 0 ? &c->g_top : &c->d_top;
        const uint32_t avail = *dst_top;
        uint32_t done = valid < avail ? valid : avail;
        // repeated ids count once (mig_valid); the pushes stay bounded by
        // the source stack's free room all the same
        const uint32_t src_room = (dir == 0 ? p.g_total : p.d_total) - *src_top;
        if (done > src_room) done = src_room;
        meta[0] = done;
        meta[1] = *dst_top;
        meta[2] = *src_top;
        *dst_top -= done;
        *src_top += done;
        if (dir == 0) { c->transfers_d2h += done; c->bytes_d2h += (unsigned long long)done * p.slab; }
        else          { c->transfers_h2d += done; c->bytes_h2d += (unsigned long long)done * p.slab; }
        c->last_done = done;
        c->last_skipped = n - done;
        if (result) { result[0] = done; result[1] = n - done; }
    }
}

__global__ void __launch_bounds__(256)
mig_plan_kernel(PoolDev p, int dir, const uint32_t *ids, const uint32_t *count,
                uint32_t max_n, const uint32_t *tile_base, const uint32_t *meta,
                uint32_t *plan_src, uint32_t *plan_dst, uint32_t *plan_id)
{
    __shared__ uint32_t tmp[33];
    const uint32_t n = list_len(count, max_n);
    const uint32_t done = meta[0], dst_top = meta[1], src_top = meta[2];
    const uint32_t base = blockIdx.x * kTileN;
    // 4 consecutive entries per thread keeps the list order inside the tile
    const uint32_t e0 = base + threadIdx.x * 4;
    bool val[4];
    uint32_t idv[4], c = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t e = e0 + j;
        idv[j] = e < n ? ids[e] : kNoBlock;
        val[j] = e < n && mig_valid(p, dir, idv[j], e);
        c += val[j];
    }
    uint32_t o = tile_base[blockIdx.x] + block_excl_scan(c, tmp, nullptr);
    uint32_t *dstk = dir == 0 ? p.d_stack : p.g_stack;
    uint32_t *srck = dir == 0 ? p.g_stack : p.d_stack;
    const uint32_t dst_tier = dir == 0 ? TIER_HOST_DRAM : TIER_GPU_HBM;
    const uint8_t new_state = dir == 0 ? KV_STATE_WARM : KV_STATE_HOT;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        if (!val[j]) continue;
        if (o < done) {
            const uint32_t id = idv[j];
            const uint32_t s = loc_slab(p.loc[id]);
            const uint32_t d = dstk[dst_top - 1 - o];
            const uint32_t src_n = dir == 0 ? p.g_total : p.d_total;
            const uint32_t dst_n = dir == 0 ? p.d_total : p.g_total;
            if (!OKV_IN(p.chk, s, src_n) || !OKV_IN(p.chk, d, dst_n) ||
                !OKV_IN(p.chk, src_top + o, src_n)) {
                plan_src[o] = plan_dst[o] = kNoBlock;   // the copy kernels skip the entry
                plan_id[o] = id;
                o++;
                continue;
            }
            srck[src_top + o] = s;
            p.loc[id] = make_loc(dst_tier, d);
            p.state[id] = new_state;
            sched_move(p, id, (uint8_t)dst_tier, new_state);
            plan_src[o] = s;
            plan_dst[o] = d;
            plan_id[o] = id;
        }
        o++;
    }
}

// One warp per slab; 16-byte lanes, eight vectors in flight per lane.
__global__ void __launch_bounds__(256)
mig_copy_kernel(const char *src_base, char *dst_base, unsigned long long slab,
                const uint32_t *plan_src, const uint32_t *plan_dst, const uint32_t *meta,
                Bounds bd, uint32_t src_n, uint32_t dst_n)
{
    const uint32_t done = meta[0];
    const unsigned lane = threadIdx.x & 31;
    const unsigned long long nvec = slab >> 4;
    const unsigned long long warp0 = ((unsigned long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const unsigned long long nwarps = ((unsigned long long)gridDim.x * blockDim.x) >> 5;
    for (unsigned long long w = warp0; w < done; w += nwarps) {
        if (!OKV_IN(bd.chk, plan_src[w], src_n) || !OKV_IN(bd.chk, plan_dst[w], dst_n)) continue;
        const uint4 *s = reinterpret_cast<const uint4 *>(src_base + plan_src[w] * slab);
        uint4 *d = reinterpret_cast<uint4 *>(dst_base + plan_dst[w] * slab);
        unsigned long long i = lane;
        for (; i + 7 * 32 < nvec; i += 8 * 32) {
            uint4 v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v[u] = s[i + u * 32];
#pragma unroll
            for (int u = 0; u < 8; u++) d[i + u * 32] = v[u];
        }
        for (; i < nvec; i += 32) d[i] = s[i];
    }
}

// ---- sorted assignment of a staged evict's DRAM slabs ---------------------
// The batch popped `done` distinct slabs of the DRAM pool (bounded by d_total),
// so a byte map + scan sorts them in O(d_total).  Entry o of the victim list
// then gets the o-th smallest popped slab, and the copy engine drains the
// staging buffer run by run (maximal runs of consecutive slabs).

__global__ void mig_mark_kernel(const uint32_t *plan_dst, const uint32_t *meta, uint8_t *flags,
                                Bounds bd)
{
    const uint32_t done = meta[0];
    for (uint32_t o = blockIdx.x * blockDim.x + threadIdx.x; o < done; o += gridDim.x * blockDim.x)
        if (OKV_IN(bd.chk, plan_dst[o], bd.d_total)) flags[plan_dst[o]] = 1;
}

// Per-tile count of set bytes in flags[0 .. n) (n capped at *n_dev if given).
__global__ void __launch_bounds__(256)
mig_flag_count_kernel(const uint8_t *flags, uint32_t n, const uint32_t *n_dev,
                      uint32_t *tile_cnt)
{
    __shared__ uint32_t tmp[33];
    if (n_dev && *n_dev < n) n = *n_dev;
    const uint32_t base = blockIdx.x * kTileN + threadIdx.x * 4;
    uint32_t c = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) c += (base + j < n) ? flags[base + j] : 0u;
    uint32_t tot;
    block_excl_scan(c, tmp, &tot);
    if (threadIdx.x == 0) tile_cnt[blockIdx.x] = tot;
}

// Exclusive scan of the tile counts in place; the total goes to *total if given.
__global__ void __launch_bounds__(1024)
mig_tile_scan_kernel(uint32_t *tile_cnt, uint32_t tiles, uint32_t *total)
{
    __shared__ uint32_t tmp[33];
    __shared__ uint32_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (uint32_t b0 = 0; b0 < tiles; b0 += blockDim.x) {
        const uint32_t t = b0 + threadIdx.x;
        const uint32_t c = t < tiles ? tile_cnt[t] : 0;
        uint32_t tot;
        const uint32_t ex = block_excl_scan(c, tmp, &tot);
        if (t < tiles) tile_cnt[t] = carry + ex;
        __syncthreads();
        if (threadIdx.x == 0) carry += tot;
        __syncthreads();
    }
    if (total && threadIdx.x == 0) *total = carry;
}

__global__ void __launch_bounds__(256)
mig_flag_write_kernel(const uint8_t *flags, uint32_t n, const uint32_t *tile_base,
                      uint32_t *sorted)
{
    __shared__ uint32_t tmp[33];
    const uint32_t base = blockIdx.x * kTileN + threadIdx.x * 4;
    uint8_t f[4];
    uint32_t c = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        f[j] = (base + j < n) ? flags[base + j] : 0;
        c += f[j];
    }
    uint32_t pos = tile_base[blockIdx.x] + block_excl_scan(c, tmp, nullptr);
#pragma unroll
    for (int j = 0; j < 4; j++)
        if (f[j]) sorted[pos++] = base + j;
}

__global__ void mig_assign_kernel(PoolDev p, const uint32_t *meta, const uint32_t *sorted,
                                  const uint32_t *plan_id, uint32_t *plan_dst, uint8_t *run_flag)
{
    const uint32_t done = meta[0];
    for (uint32_t o = blockIdx.x * blockDim.x + threadIdx.x; o < done; o += gridDim.x * blockDim.x) {
        const uint32_t d = sorted[o];
        plan_dst[o] = d;
        if (OKV_IN(p.chk, plan_id[o], p.max_blocks) && OKV_IN(p.chk, d, p.d_total))
            p.loc[plan_id[o]] = make_loc(TIER_HOST_DRAM, d);
        run_flag[o] = (o == 0 || sorted[o - 1] + 1 != d) ? 1 : 0;
    }
}

// List the run starts in order: run_o[r] = list position, run_d[r] = its
// first DRAM slab, for run_flag[o] set, o < meta[0].  Tiles of kTileN list
// entries, placed by the scanned tile counts; only the first max_runs runs are
// written (meta[6], the total, may be larger).
__global__ void __launch_bounds__(256)
mig_run_write_kernel(const uint8_t *run_flag, const uint32_t *meta, const uint32_t *tile_base,
                     const uint32_t *sorted, uint32_t *run_o, uint32_t *run_d,
                     uint32_t max_runs)
{
    __shared__ uint32_t tmp[33];
    const uint32_t n = meta[0];
    const uint32_t base = blockIdx.x * kTileN + threadIdx.x * 4;
    uint8_t f[4];
    uint32_t c = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        f[j] = (base + j < n) ? run_flag[base + j] : 0;
        c += f[j];
    }
    uint32_t pos = tile_base[blockIdx.x] + block_excl_scan(c, tmp, nullptr);
#pragma unroll
    for (int j = 0; j < 4; j++)
        if (f[j]) {
            if (pos < max_runs) { run_o[pos] = base + j; run_d[pos] = sorted[base + j]; }
            pos++;
        }
}

// Length of the run of consecutive DRAM slabs that list position o belongs
// to.  run_o holds the ascending list positions where runs start (run_o[0] is
// 0); n_runs of them, the last run ending at done.
__device__ __forceinline__ uint32_t run_len_at(const uint32_t *run_o, uint32_t n_runs,
                                               uint32_t done, uint32_t o)
{
    uint32_t lo = 0, hi = n_runs;          // last q with run_o[q] <= o
    while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (__ldg(run_o + mid) <= o) lo = mid; else hi = mid;
    }
    const uint32_t end = lo + 1 < n_runs ? __ldg(run_o + lo + 1) : done;
    return end - __ldg(run_o + lo);
}

__device__ __forceinline__ void copy_slab_warp(const char *src, char *dst,
                                               unsigned long long nvec, unsigned lane)
{
    const uint4 *s = reinterpret_cast<const uint4 *>(src);
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    unsigned long long i = lane;
    for (; i + 7 * 32 < nvec; i += 8 * 32) {
        uint4 v[8];
#pragma unroll
        for (int u = 0; u < 8; u++) v[u] = s[i + u * 32];
#pragma unroll
        for (int u = 0; u < 8; u++) d[i + u * 32] = v[u];
    }
    for (; i < nvec; i += 32) d[i] = s[i];
}

// Pack list entries [pos0, pos0 + n) into the staging buffer, in list order
// (entry w at staging + w * slab).  With min_len > 0 only entries whose DRAM
// run is at least min_len slabs long are packed (the copy engine drains
// those); the rest are left to mig_drain_short_kernel.
__global__ void __launch_bounds__(256)
mig_pack_kernel(const char *src_base, char *staging, unsigned long long slab,
                const uint32_t *plan_src, uint32_t pos0, uint32_t n, const uint32_t *run_o,
                const uint32_t *meta, uint32_t min_len, Bounds bd)
{
    const unsigned lane = threadIdx.x & 31;
    const unsigned long long nvec = slab >> 4;
    const unsigned long long warp0 = ((unsigned long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const unsigned long long nwarps = ((unsigned long long)gridDim.x * blockDim.x) >> 5;
    const uint32_t done = min_len ? meta[0] : 0, n_runs = min_len ? meta[6] : 0;
    for (unsigned long long w = warp0; w < n; w += nwarps) {
        const uint32_t o = pos0 + (uint32_t)w;
        if (min_len && run_len_at(run_o, n_runs, done, o) < min_len) continue;
        if (!OKV_IN(bd.chk, plan_src[o], bd.g_total)) continue;
        copy_slab_warp(src_base + plan_src[o] * slab, staging + w * slab, nvec, lane);
    }
}

// Entries of [pos0, pos0 + n) whose DRAM run is shorter than min_len go
// straight from their GPU slab to their DRAM slab over the host link
// (mapped pinned memory): runs that short would cost the copy engine more in
// per-copy overhead than in transfer time.
// With `staged` set, entry w is read from staged + w * slab (its packed copy)
// instead of its GPU slab, which a concurrent promote may already reuse.
__global__ void __launch_bounds__(256)
mig_drain_short_kernel(const char *src_base, char *dram_base, unsigned long long slab,
                       const uint32_t *plan_src, const uint32_t *plan_dst, uint32_t pos0,
                       uint32_t n, const uint32_t *run_o, const uint32_t *meta, uint32_t min_len,
                       const char *staged, Bounds bd)
{
    const unsigned lane = threadIdx.x & 31;
    const unsigned long long nvec = slab >> 4;
    const unsigned long long warp0 = ((unsigned long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const unsigned long long nwarps = ((unsigned long long)gridDim.x * blockDim.x) >> 5;
    const uint32_t done = meta[0], n_runs = meta[6];
    for (unsigned long long w = warp0; w < n; w += nwarps) {
        const uint32_t o = pos0 + (uint32_t)w;
        if (run_len_at(run_o, n_runs, done, o) >= min_len) continue;
        if ((!staged && !OKV_IN(bd.chk, plan_src[o], bd.g_total)) ||
            !OKV_IN(bd.chk, plan_dst[o], bd.d_total))
            continue;
        const char *src = staged ? staged + w * slab : src_base + plan_src[o] * slab;
        copy_slab_warp(src, dram_base + plan_dst[o] * slab, nvec, lane);
    }
}

// ---- staged promote --------------------------------------------------------
// The promoted blocks' DRAM slabs are sorted (byte map over the DRAM pool);
// sorted position j holds slab sorted[j], which list position pos_of[slab]
// promotes into GPU slab plan_dst[pos_of[slab]].  Runs of consecutive slabs
// are copied host-to-device by the copy engine into a staging ring and
// scattered by mig_unpack_kernel; short runs are read zero-copy.

__global__ void mig_src_mark_kernel(const uint32_t *plan_src, const uint32_t *meta,
                                    uint8_t *flags, uint32_t *pos_of, Bounds bd)
{
    const uint32_t done = meta[0];
    for (uint32_t o = blockIdx.x * blockDim.x + threadIdx.x; o < done; o += gridDim.x * blockDim.x) {
        if (!OKV_IN(bd.chk, plan_src[o], bd.d_total)) continue;
        flags[plan_src[o]] = 1;
        pos_of[plan_src[o]] = o;
    }
}

__global__ void mig_runflag_kernel(const uint32_t *meta, const uint32_t *sorted, uint8_t *run_flag)
{
    const uint32_t done = meta[0];
    for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < done; j += gridDim.x * blockDim.x)
        run_flag[j] = (j == 0 || sorted[j - 1] + 1 != sorted[j]) ? 1 : 0;
}

// Sorted positions [j0, j0 + n) in DRAM runs of >= min_len slabs: staging
// entry (j - j0) goes to its block's GPU slab.
__global__ void __launch_bounds__(256)
mig_unpack_kernel(const char *staging, char *gpu_base, unsigned long long slab,
                  const uint32_t *sorted, const uint32_t *pos_of, const uint32_t *plan_dst,
                  uint32_t j0, uint32_t n, const uint32_t *run_o, const uint32_t *meta,
                  uint32_t min_len, Bounds bd)
{
    const unsigned lane = threadIdx.x & 31;
    const unsigned long long nvec = slab >> 4;
    const unsigned long long warp0 = ((unsigned long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const unsigned long long nwarps = ((unsigned long long)gridDim.x * blockDim.x) >> 5;
    const uint32_t done = meta[0], n_runs = meta[6];
    for (unsigned long long w = warp0; w < n; w += nwarps) {
        const uint32_t j = j0 + (uint32_t)w;
        if (min_len && run_len_at(run_o, n_runs, done, j) < min_len) continue;
        if (!OKV_IN(bd.chk, sorted[j], bd.d_total) || !OKV_IN(bd.chk, pos_of[sorted[j]], done))
            continue;
        const uint32_t d = plan_dst[pos_of[sorted[j]]];
        if (!OKV_IN(bd.chk, d, bd.g_total)) continue;
        copy_slab_warp(staging + w * slab, gpu_base + d * slab, nvec, lane);
    }
}

// Sorted positions in DRAM runs shorter than min_len: read over the host link
// (mapped pinned memory) straight into their GPU slabs.
__global__ void __launch_bounds__(256)
mig_promote_short_kernel(const char *dram_base, char *gpu_base, unsigned long long slab,
                         const uint32_t *sorted, const uint32_t *pos_of, const uint32_t *plan_dst,
                         const uint32_t *run_o, const uint32_t *meta, uint32_t min_len,
                         Bounds bd)
{
    const unsigned lane = threadIdx.x & 31;
    const unsigned long long nvec = slab >> 4;
    const unsigned long long warp0 = ((unsigned long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const unsigned long long nwarps = ((unsigned long long)gridDim.x * blockDim.x) >> 5;
    const uint32_t done = meta[0], n_runs = meta[6];
    for (unsigned long long w = warp0; w < done; w += nwarps) {
        const uint32_t j = (uint32_t)w;
        if (run_len_at(run_o, n_runs, done, j) >= min_len) continue;
        const uint32_t s = sorted[j];
        if (!OKV_IN(bd.chk, s, bd.d_total) || !OKV_IN(bd.chk, pos_of[s], done) ||
            !OKV_IN(bd.chk, plan_dst[pos_of[s]], bd.g_total))
            continue;
        copy_slab_warp(dram_base + s * slab, gpu_base + plan_dst[pos_of[s]] * slab, nvec, lane);
    }
}

// Promote sources that are among the DRAM slabs an evict of the same call
// just popped (evict_flags, its byte map): the promote must then wait for
// the evict's bytes to land.  Counted into *conflicts.
__global__ void mig_conflict_kernel(const uint32_t *plan_src, const uint32_t *meta,
                                    const uint8_t *evict_flags, uint32_t *conflicts, Bounds bd)
{
    const uint32_t done = meta[0];
    uint32_t c = 0;
    for (uint32_t o = blockIdx.x * blockDim.x + threadIdx.x; o < done; o += gridDim.x * blockDim.x)
        if (OKV_IN(bd.chk, plan_src[o], bd.d_total)) c += evict_flags[plan_src[o]];
    c = __reduce_add_sync(0xFFFFFFFFu, c);
    if ((threadIdx.x & 31) == 0 && c) atomicAdd(conflicts, c);
}

// ---------------------------------------------------------------------------
// Block-id table for the scoring kernel
// ---------------------------------------------------------------------------

__global__ void id_table_kernel(PoolDev p, uint32_t *const *regions, uint32_t n, uint32_t L,
                                uint32_t H, uint32_t mbph, uint32_t nb, uint32_t *out)
{
    const unsigned long long total = (unsigned long long)n * L * H * nb;
    for (unsigned long long e = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x;
         e < total; e += (unsigned long long)gridDim.x * blockDim.x) {
        const uint32_t b = (uint32_t)(e % nb);
        const unsigned long long rh = e / nb;
        const uint32_t hh = (uint32_t)(rh % H);
        const unsigned long long pr = rh / H;
        const uint32_t i = (uint32_t)(pr / L), l = (uint32_t)(pr % L);
        const uint32_t *reg = regions[i];
        const uint32_t tok = reg[1 + l];
        const uint32_t nbl = (tok + p.tpb - 1) / p.tpb;
        out[e] = (b < nbl && b < mbph) ? reg[1 + L + ((size_t)l * H + hh) * mbph + b] : kNoBlock;
    }
}

// ---------------------------------------------------------------------------
// Request teardown (src/api/orchkv_api.cu:149-183): free slabs and ids in
// (layer, head, block) order.  One CTA, contiguous chunks per thread.
// ---------------------------------------------------------------------------

// Request teardown (src/api/orchkv_api.cu:149-183): every existing block of
// the request, in table order (layer, head, block), returns its slab to the
// stack of its tier and its id to the id stack.  Tiles of kTileN table
// entries: count per tile, scan the three counts, then write in order.
__device__ __forceinline__ bool req_entry(const PoolDev &p, const ReqDev &r, size_t e, size_t E,
                                          uint32_t *id)
{
    if (e >= E) return false;
    const uint32_t bi = (uint32_t)(e % r.mbph);
    const uint32_t l = (uint32_t)(e / ((size_t)r.H * r.mbph));
    if (bi >= (req_tok(r)[l] + p.tpb - 1) / p.tpb) return false;
    *id = req_table(r)[e];
    return *id < p.max_blocks;
}

__global__ void __launch_bounds__(256)
req_free_count_kernel(PoolDev p, ReqDev r, uint32_t *tile_cnt)
{
    __shared__ uint32_t tmp[33];
    const size_t E = (size_t)r.L * r.H * r.mbph;
    const size_t e0 = (size_t)blockIdx.x * kTileN + threadIdx.x * 4;
    uint32_t ng = 0, nd = 0, ni = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        uint32_t id;
        if (!req_entry(p, r, e0 + j, E, &id)) continue;
        ni++;
        const uint32_t t = loc_tier(p.loc[id]);
        ng += t == TIER_GPU_HBM;
        nd += t == TIER_HOST_DRAM;
    }
    uint32_t tg, td, ti;
    block_excl_scan(ng, tmp, &tg);
    block_excl_scan(nd, tmp, &td);
    block_excl_scan(ni, tmp, &ti);
    if (threadIdx.x == 0) {
        tile_cnt[3 * blockIdx.x + 0] = tg;
        tile_cnt[3 * blockIdx.x + 1] = td;
        tile_cnt[3 * blockIdx.x + 2] = ti;
    }
}

// One CTA: exclusive scan of the per-tile counts into stack positions (old
// top + offset), then the stack tops move past the pushes.
__global__ void __launch_bounds__(1024)
req_free_scan_kernel(PoolDev p, uint32_t *tile_cnt, uint32_t tiles)
{
    __shared__ uint32_t tmp[33];
    __shared__ uint32_t carry[3];
    PoolCounters *c = p.ctr;
    if (threadIdx.x == 0) { carry[0] = c->g_top; carry[1] = c->d_top; carry[2] = c->id_top; }
    __syncthreads();
    for (uint32_t b0 = 0; b0 < tiles; b0 += blockDim.x) {
        const uint32_t t = b0 + threadIdx.x;
        for (int k = 0; k < 3; k++) {
            const uint32_t v = t < tiles ? tile_cnt[3 * t + k] : 0;
            uint32_t tot;
            const uint32_t ex = block_excl_scan(v, tmp, &tot);
            if (t < tiles) tile_cnt[3 * t + k] = carry[k] + ex;
            __syncthreads();
            if (threadIdx.x == 0) carry[k] += tot;
            __syncthreads();
        }
    }
    if (threadIdx.x == 0) {
        c->live_blocks -= carry[2] - c->id_top;
        c->g_top = carry[0];
        c->d_top = carry[1];
        c->id_top = carry[2];
    }
}

__global__ void __launch_bounds__(256)
req_free_write_kernel(PoolDev p, ReqDev r, const uint32_t *tile_pos)
{
    __shared__ uint32_t tmp[33];
    const size_t E = (size_t)r.L * r.H * r.mbph;
    const size_t e0 = (size_t)blockIdx.x * kTileN + threadIdx.x * 4;
    uint32_t ids[4], ws[4];
    bool ok[4];
    uint32_t ng = 0, nd = 0, ni = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        ok[j] = req_entry(p, r, e0 + j, E, &ids[j]);
        ws[j] = ok[j] ? p.loc[ids[j]] : 0;
        ni += ok[j];
        ng += ok[j] && loc_tier(ws[j]) == TIER_GPU_HBM;
        nd += ok[j] && loc_tier(ws[j]) == TIER_HOST_DRAM;
    }
    uint32_t og = tile_pos[3 * blockIdx.x + 0] + block_excl_scan(ng, tmp, nullptr);
    uint32_t od = tile_pos[3 * blockIdx.x + 1] + block_excl_scan(nd, tmp, nullptr);
    uint32_t oi = tile_pos[3 * blockIdx.x + 2] + block_excl_scan(ni, tmp, nullptr);
#pragma unroll
    for (int j = 0; j < 4; j++) {
        if (!ok[j]) continue;
        const uint32_t id = ids[j], w = ws[j];
        if (loc_tier(w) == TIER_GPU_HBM) {
            if (OKV_IN(p.chk, og, p.g_total)) p.g_stack[og] = loc_slab(w);
            og++;
        } else if (loc_tier(w) == TIER_HOST_DRAM) {
            if (OKV_IN(p.chk, od, p.d_total)) p.d_stack[od] = loc_slab(w);
            od++;
        }
        if (OKV_IN(p.chk, oi, p.max_blocks)) p.id_stack[oi] = id;
        oi++;
        p.loc[id] = make_loc(TIER_NONE, 0);
        p.state[id] = KV_STATE_EVICTED;
        p.flags[id] = 0;
        sched_unregister(p, id);
    }
}

unsigned copy_grid(uint32_t items, int per_cta)
{
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    unsigned g = (items + per_cta - 1) / per_cta;
    const unsigned cap = (unsigned)sms * 16;
    if (g > cap) g = cap;
    return g ? g : 1;
}

}  // namespace

int launch_compat_op(const PoolDev &p, const ReqDev &r, int op, uint32_t l, uint32_t h,
                     uint32_t bi, uint32_t arg, uint32_t arg2, CompatResult *res,
                     cudaStream_t s)
{
    compat_op_kernel<<<1, 256, 0, s>>>(p, r, op, l, h, bi, arg, arg2, res); note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

int launch_append_one(const PoolDev &p, const ReqDev &r, uint32_t l, const char *k,
                      const char *v, CompatResult *res, cudaStream_t s)
{
    if (r.H > (uint32_t)kMaxHeads) return ORCHKV_ERR_INVALID;
    append_one_kernel<<<1, 256, 0, s>>>(p, r, l, k, v, res); note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

int launch_prefill(const PoolDev &p, const ReqDev &r, uint32_t l, const char *k,
                   const char *v, uint32_t seq_len, uint32_t *scratch, CompatResult *res,
                   cudaStream_t s)
{
    prefill_plan_kernel<<<1, 1, 0, s>>>(p, r, l, seq_len, k != nullptr, v != nullptr,
                                        scratch, res); note_launches(1);
    const uint32_t items = ((seq_len + p.tpb - 1) / p.tpb + 1) * r.H;
    prefill_copy_kernel<<<copy_grid(items, 8), 256, 0, s>>>(p, r, l, k, v, seq_len, scratch); note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

int launch_append_batch(const PoolDev &p, uint32_t *const *regions, uint32_t n, uint32_t L,
                        uint32_t H, uint32_t mbph, const char *k, const char *v,
                        uint32_t *scratch, cudaStream_t s)
{
    append_plan_kernel<<<1, 1024, 0, s>>>(p, regions, n, L, H, mbph, k != nullptr,
                                          v != nullptr, scratch); note_launches(1);
    const unsigned long long warps = (unsigned long long)n * L * H;
    append_write_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>(p, regions, n, L, H, mbph,
                                                                     k, v, scratch); note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

// ---- batched storage moves ---------------------------------------------------

// (layer, head, block) triples of one request -> block id, location word and
// flags (kNoBlock / ~0 / 0 where the triple names no existing block).
__global__ void lhb_lookup_kernel(PoolDev p, ReqDev r, const uint32_t *lhb, uint32_t n,
                                  uint32_t *out)
{
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const uint32_t l = lhb[3 * i], h = lhb[3 * i + 1], bi = lhb[3 * i + 2];
        uint32_t id = kNoBlock, w = 0xFFFFFFFFu, f = 0;
        if (l < r.L && h < r.H && bi < r.mbph && bi < (req_tok(r)[l] + p.tpb - 1) / p.tpb) {
            const uint32_t x = req_table(r)[((size_t)l * r.H + h) * r.mbph + bi];
            if (x < p.max_blocks) { id = x; w = p.loc[x]; f = p.flags[x]; }
        }
        out[3 * i] = id;
        out[3 * i + 1] = w;
        out[3 * i + 2] = f;
    }
}

// Commit n storage moves in list order.  dir 0 (DRAM -> storage): block ->
// TIER_NVM, COLD, its DRAM slab pushed onto the DRAM stack in list order.
// dir 1 (storage -> DRAM): block -> DRAM slab d_stack[top-1-j] (WARM),
// popped.  dir 2 (GPU -> storage through one DRAM slab, as consecutive
// orchkv_evict_cold calls leave it): block -> TIER_NVM, COLD, its GPU slab
// pushed onto the GPU stack in list order, counted as a device-to-host
// transfer; the DRAM stack ends where it began.
__global__ void __launch_bounds__(1024)
storage_commit_kernel(PoolDev p, const uint32_t *ids, const uint32_t *slabs, uint32_t n, int dir)
{
    PoolCounters *c = p.ctr;
    const uint32_t top = dir == 2 ? c->g_top : c->d_top;
    for (uint32_t j = threadIdx.x; j < n; j += blockDim.x) {
        const uint32_t id = ids[j];
        if (!OKV_IN(p.chk, id, p.max_blocks)) continue;
        if (dir == 1) {
            if (!OKV_IN(p.chk, p.d_stack[top - 1 - j], p.d_total)) continue;
            p.loc[id] = make_loc(TIER_HOST_DRAM, p.d_stack[top - 1 - j]);
            p.state[id] = KV_STATE_WARM;
            sched_move(p, id, (uint8_t)TIER_HOST_DRAM, KV_STATE_WARM);
            continue;
        }
        if (dir == 0) {
            if (OKV_IN(p.chk, top + j, p.d_total)) p.d_stack[top + j] = slabs[j];
        } else if (OKV_IN(p.chk, top + j, p.g_total)) {
            p.g_stack[top + j] = slabs[j];
        }
        p.loc[id] = make_loc(TIER_NVM, 0);
        p.state[id] = KV_STATE_COLD;
        sched_move(p, id, (uint8_t)TIER_NVM, KV_STATE_COLD);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (dir == 0) c->d_top = top + n;
        else if (dir == 1) c->d_top = top - n;
        else {
            c->g_top = top + n;
            c->transfers_d2h += n;
            c->bytes_d2h += (unsigned long long)n * p.slab;
        }
    }
}

// First list position of every id of a batch (p.first), and its reset.
__global__ void mig_first_kernel(PoolDev p, const uint32_t *ids, const uint32_t *count,
                                 uint32_t max_n, int reset)
{
    const uint32_t n = list_len(count, max_n);
    for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < n; e += gridDim.x * blockDim.x) {
        const uint32_t id = ids[e];
        if (id >= p.max_blocks) continue;
        if (reset) p.first[id] = 0xFFFFFFFFu;
        else atomicMin(&p.first[id], e);
    }
}

MigPlan launch_migrate_plan(const PoolDev &p, int dir, const uint32_t *ids,
                            const uint32_t *count, uint32_t max_n, uint32_t *result,
                            uint32_t *scratch, cudaStream_t s)
{
    MigPlan mp;
    mp.tiles = (max_n + kTileN - 1) / kTileN;
    mp.meta = scratch;                         // [16]
    uint32_t *tile_cnt = scratch + 16;         // [tiles]
    mp.plan_src = tile_cnt + mp.tiles;         // [max_n]
    mp.plan_dst = mp.plan_src + max_n;         // [max_n]
    mp.plan_id = mp.plan_dst + max_n;          // [max_n]
    mp.max_n = max_n;
    mp.rc = ORCHKV_OK;
    if (max_n == 0) {                           // nothing listed: {0 done, 0 skipped}
        if (result && cudaMemsetAsync(result, 0, 2 * sizeof(uint32_t), s) != cudaSuccess)
            mp.rc = ORCHKV_ERR_CUDA;
        return mp;
    }
    const unsigned g = copy_grid(max_n, 256);
    mig_first_kernel<<<g, 256, 0, s>>>(p, ids, count, max_n, 0); note_launches(1);
    mig_count_kernel<<<mp.tiles, 256, 0, s>>>(p, dir, ids, count, max_n, tile_cnt); note_launches(1);
    mig_scan_kernel<<<1, 1024, 0, s>>>(p, dir, count, max_n, mp.tiles, tile_cnt, mp.meta, result); note_launches(1);
    mig_plan_kernel<<<mp.tiles, 256, 0, s>>>(p, dir, ids, count, max_n, tile_cnt, mp.meta,
                                             mp.plan_src, mp.plan_dst, mp.plan_id); note_launches(1);
    mig_first_kernel<<<g, 256, 0, s>>>(p, ids, count, max_n, 1); note_launches(1);
    if (cudaGetLastError() != cudaSuccess) mp.rc = ORCHKV_ERR_CUDA;
    return mp;
}

int launch_migrate_zero_copy(const PoolDev &p, int dir, const MigPlan &mp, cudaStream_t s)
{
    if (mp.max_n == 0) return ORCHKV_OK;
    const char *src_base = dir == 0 ? p.gpu_base : p.dram_base;
    char *dst_base = dir == 0 ? p.dram_base : p.gpu_base;
    mig_copy_kernel<<<copy_grid(mp.max_n, 8), 256, 0, s>>>(
        src_base, dst_base, p.slab, mp.plan_src, mp.plan_dst, mp.meta, bounds_of(p),
        dir == 0 ? p.g_total : p.d_total, dir == 0 ? p.d_total : p.g_total);
    note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

int launch_sorted_assign(const PoolDev &p, const MigPlan &mp, const SortScratch &ss,
                         cudaStream_t s)
{
    OKV_CUDA_TRY(cudaMemsetAsync(ss.flags, 0, p.d_total, s));
    const unsigned g = copy_grid(mp.max_n, 256);
    const uint32_t tiles = (p.d_total + kTileN - 1) / kTileN;
    mig_mark_kernel<<<g, 256, 0, s>>>(mp.plan_dst, mp.meta, ss.flags, bounds_of(p));
    mig_flag_count_kernel<<<tiles, 256, 0, s>>>(ss.flags, p.d_total, nullptr, ss.tile_cnt);
    mig_tile_scan_kernel<<<1, 1024, 0, s>>>(ss.tile_cnt, tiles, nullptr);
    mig_flag_write_kernel<<<tiles, 256, 0, s>>>(ss.flags, p.d_total, ss.tile_cnt, ss.sorted);
    mig_assign_kernel<<<g, 256, 0, s>>>(p, mp.meta, ss.sorted, mp.plan_id, mp.plan_dst,
                                        ss.run_flag);
    // runs of consecutive slabs among list positions [0, done), done <= min(max_n, d_total)
    const uint32_t span = mp.max_n < p.d_total ? mp.max_n : p.d_total;
    const uint32_t rtiles = (span + kTileN - 1) / kTileN;
    if (rtiles) {
        mig_flag_count_kernel<<<rtiles, 256, 0, s>>>(ss.run_flag, span, mp.meta, ss.tile_cnt);
        mig_tile_scan_kernel<<<1, 1024, 0, s>>>(ss.tile_cnt, rtiles, mp.meta + 6);
        mig_run_write_kernel<<<rtiles, 256, 0, s>>>(ss.run_flag, mp.meta, ss.tile_cnt, ss.sorted,
                                                    ss.run_o, ss.run_d, ss.max_runs);
        note_launches(3);
    } else {
        OKV_CUDA_TRY(cudaMemsetAsync(mp.meta + 6, 0, 4, s));
    }
    note_launches(5);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

int launch_pack(const PoolDev &p, const MigPlan &mp, char *staging, uint32_t pos0, uint32_t n,
                const SortScratch &ss, uint32_t min_len, cudaStream_t s)
{
    if (n == 0) return ORCHKV_OK;
    mig_pack_kernel<<<copy_grid(n, 8), 256, 0, s>>>(p.gpu_base, staging, p.slab, mp.plan_src,
                                                     pos0, n, ss.run_o, mp.meta, min_len,
                                                     bounds_of(p));
    note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

int launch_drain_short(const PoolDev &p, const MigPlan &mp, uint32_t pos0, uint32_t n,
                       const SortScratch &ss, uint32_t min_len, const char *staged,
                       cudaStream_t s)
{
    if (n == 0 || min_len == 0) return ORCHKV_OK;
    mig_drain_short_kernel<<<copy_grid(n, 8), 256, 0, s>>>(p.gpu_base, p.dram_base, p.slab,
                                                            mp.plan_src, mp.plan_dst, pos0, n,
                                                            ss.run_o, mp.meta, min_len, staged,
                                                            bounds_of(p));
    note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

int launch_sorted_sources(const PoolDev &p, const MigPlan &mp, const SortScratch &ss,
                          cudaStream_t s)
{
    if (!ss.pos_of) return ORCHKV_ERR_INVALID;
    OKV_CUDA_TRY(cudaMemsetAsync(ss.flags, 0, p.d_total, s));
    const unsigned g = copy_grid(mp.max_n, 256);
    const uint32_t tiles = (p.d_total + kTileN - 1) / kTileN;
    mig_src_mark_kernel<<<g, 256, 0, s>>>(mp.plan_src, mp.meta, ss.flags, ss.pos_of,
                                          bounds_of(p));
    mig_flag_count_kernel<<<tiles, 256, 0, s>>>(ss.flags, p.d_total, nullptr, ss.tile_cnt);
    mig_tile_scan_kernel<<<1, 1024, 0, s>>>(ss.tile_cnt, tiles, nullptr);
    mig_flag_write_kernel<<<tiles, 256, 0, s>>>(ss.flags, p.d_total, ss.tile_cnt, ss.sorted);
    mig_runflag_kernel<<<g, 256, 0, s>>>(mp.meta, ss.sorted, ss.run_flag);
    note_launches(5);
    const uint32_t span = mp.max_n < p.d_total ? mp.max_n : p.d_total;
    const uint32_t rtiles = (span + kTileN - 1) / kTileN;
    if (rtiles) {
        mig_flag_count_kernel<<<rtiles, 256, 0, s>>>(ss.run_flag, span, mp.meta, ss.tile_cnt);
        mig_tile_scan_kernel<<<1, 1024, 0, s>>>(ss.tile_cnt, rtiles, mp.meta + 6);
        mig_run_write_kernel<<<rtiles, 256, 0, s>>>(ss.run_flag, mp.meta, ss.tile_cnt, ss.sorted,
                                                    ss.run_o, ss.run_d, ss.max_runs);
        note_launches(3);
    } else {
        OKV_CUDA_TRY(cudaMemsetAsync(mp.meta + 6, 0, 4, s));
    }
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

int launch_unpack(const PoolDev &p, const MigPlan &mp, const SortScratch &ss,
                  const char *staging, uint32_t j0, uint32_t n, uint32_t min_len, cudaStream_t s)
{
    if (n == 0) return ORCHKV_OK;
    mig_unpack_kernel<<<copy_grid(n, 8), 256, 0, s>>>(staging, p.gpu_base, p.slab, ss.sorted,
                                                       ss.pos_of, mp.plan_dst, j0, n, ss.run_o,
                                                       mp.meta, min_len, bounds_of(p));
    note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

int launch_promote_short(const PoolDev &p, const MigPlan &mp, const SortScratch &ss,
                         uint32_t min_len, cudaStream_t s)
{
    if (min_len == 0) return ORCHKV_OK;
    mig_promote_short_kernel<<<copy_grid(mp.max_n, 8), 256, 0, s>>>(
        p.dram_base, p.gpu_base, p.slab, ss.sorted, ss.pos_of, mp.plan_dst, ss.run_o, mp.meta,
        min_len, bounds_of(p));
    note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

int launch_conflicts(const PoolDev &p, const MigPlan &promote, const SortScratch &evict_ss,
                     uint32_t *conflicts, cudaStream_t s)
{
    OKV_CUDA_TRY(cudaMemsetAsync(conflicts, 0, 4, s));
    mig_conflict_kernel<<<copy_grid(promote.max_n, 256), 256, 0, s>>>(
        promote.plan_src, promote.meta, evict_ss.flags, conflicts, bounds_of(p));
    note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

__global__ void check_inject_kernel(uint32_t *chk, uint32_t line)
{
    in_bounds(chk, 1, 0, line);
}

int launch_check_inject(const PoolDev &p, uint32_t line, cudaStream_t s)
{
    if (!kCheckedBuild || !p.chk) return ORCHKV_ERR_INVALID;
    check_inject_kernel<<<1, 1, 0, s>>>(p.chk, line);
    note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

int launch_migrate_batch(const PoolDev &p, int dir, const uint32_t *ids,
                         const uint32_t *count, uint32_t max_n, uint32_t *result,
                         uint32_t *scratch, cudaStream_t s)
{
    MigPlan mp = launch_migrate_plan(p, dir, ids, count, max_n, result, scratch, s);
    if (mp.rc) return mp.rc;
    return launch_migrate_zero_copy(p, dir, mp, s);
}

int launch_id_table(const PoolDev &p, uint32_t *const *regions, uint32_t n, uint32_t L,
                    uint32_t H, uint32_t mbph, uint32_t row_len, uint32_t *out,
                    cudaStream_t s)
{
    const uint32_t nb = (row_len + p.tpb - 1) / p.tpb;
    const unsigned long long total = (unsigned long long)n * L * H * nb;
    unsigned g = (unsigned)((total + 255) / 256);
    if (g > 148 * 16) g = 148 * 16;
    if (g == 0) g = 1;
    id_table_kernel<<<g, 256, 0, s>>>(p, regions, n, L, H, mbph, nb, out); note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

int launch_lhb_lookup(const PoolDev &p, const ReqDev &r, const uint32_t *lhb, uint32_t n,
                      uint32_t *out, cudaStream_t s)
{
    if (n == 0) return ORCHKV_OK;
    lhb_lookup_kernel<<<copy_grid(n, 256), 256, 0, s>>>(p, r, lhb, n, out); note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

int launch_storage_commit(const PoolDev &p, const uint32_t *ids, const uint32_t *slabs,
                          uint32_t n, int dir, cudaStream_t s)
{
    if (n == 0) return ORCHKV_OK;
    storage_commit_kernel<<<1, 1024, 0, s>>>(p, ids, slabs, n, dir); note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

int launch_request_free(const PoolDev &p, const ReqDev &r, uint32_t *scratch, cudaStream_t s)
{
    const size_t E = (size_t)r.L * r.H * r.mbph;
    const uint32_t tiles = (uint32_t)((E + kTileN - 1) / kTileN);
    if (tiles == 0) return ORCHKV_OK;
    req_free_count_kernel<<<tiles, 256, 0, s>>>(p, r, scratch);
    req_free_scan_kernel<<<1, 1024, 0, s>>>(p, scratch, tiles);
    req_free_write_kernel<<<tiles, 256, 0, s>>>(p, r, scratch);
    note_launches(3);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

}  // namespace okv
